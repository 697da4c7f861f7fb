"""Two-dimensional incompressible flow on the periodic box [0, 2 pi)^2, the consumer of the pruned
real 2D transforms (the reference's python/spectral/flow package, params and gpu modules):

    d omega / dt + u . grad omega = nu lap omega - alpha omega + f
    u = (d psi / dy, -d psi / dx),   lap psi = -omega

with Kolmogorov forcing f(y) = -A k_f cos(k_f y).

    flow.params   Flow (the physical parameters) and Grid (the spectral grid)
    flow.gpu      the batched float32 GPU solver on this library's transforms
"""

from .params import Flow, Grid

__all__ = ["Flow", "Grid"]
