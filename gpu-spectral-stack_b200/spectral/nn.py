"""SpectralConv2d: the Fourier-neural-operator spectral convolution layer on this library's
kernels, with a hand-derived backward.

The reference plans this layer (docs/ROADMAP.md:71-76, tasks 3.4-3.6) on top of its pruned
transforms but has no implementation. Forward, for real fields u of shape (b, c_in, n1, n2):

    X = rfft2_truncated(u, m1, m2)            # (b, c_in, 2 m1, m2): rows 0..m1-1, n1-m1..n1-1
    Y = mode_contract(X, W)                   # Y[b, o, k] = sum_i X[b, i, k] W[i, o, k]
    y = irfft2_from_modes(Y, (n1, n2))        # (b, c_out, n1, n2)

Backward (gradients in torch's convention for complex tensors, dL/dRe + i dL/dIm):

* Through the inverse: y is real-linear in Y, y = (1 / n1 n2) Re sum_k w(k2) Y[k] e^{+i theta_k}
  with w = 1 on the columns k2 = 0 and n2/2 (stored once) and 2 elsewhere (their conjugate
  twins are implied), so dL/dY = w / (n1 n2) * rfft2_truncated(dL/dy).
* Through the contraction (complex-linear per mode): dL/dX[b, i] = sum_o dL/dY[b, o] conj(W[i, o])
  and dL/dW[i, o] = sum_b conj(X[b, i]) dL/dY[b, o]: the same contraction kernel on transposed,
  conjugated operands.
* Through the forward transform: u is real, dL/du = Re sum_k dL/dX[k] e^{+i theta_k}
  = n1 n2 * irfft2_from_modes(dL/dX / w).

Every transform and contraction runs on this library's CUDA kernels; torch supplies only the
transposes, conjugations and per-column weights.
"""

from __future__ import annotations

import math

import torch

from .ops import irfft2_from_modes, mode_contract, rfft2_truncated


def _column_weights(m2: int, n2: int, device) -> torch.Tensor:
    """w(k2) for the kept columns k2 = 0 .. m2-1: 1 where the column is its own conjugate twin
    (k2 = 0, and k2 = n2/2 when kept), 2 elsewhere."""
    w = torch.full((m2,), 2.0, dtype=torch.float32, device=device)
    w[0] = 1.0
    if m2 > n2 // 2:
        w[n2 // 2] = 1.0
    return w


class _SpectralConv2dFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u: torch.Tensor, weight: torch.Tensor, m1: int, m2: int, impl: str) -> torch.Tensor:
        n1, n2 = u.shape[-2], u.shape[-1]
        modes = rfft2_truncated(u, m1, m2, impl=impl)
        out = irfft2_from_modes(mode_contract(modes, weight), (n1, n2), impl=impl)
        ctx.save_for_backward(modes, weight)
        ctx.dims = (n1, n2, m1, m2)
        ctx.impl = impl
        return out

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        modes, weight = ctx.saved_tensors
        n1, n2, m1, m2 = ctx.dims
        impl = ctx.impl
        w = _column_weights(m2, n2, grad.device)
        grad_out_modes = rfft2_truncated(grad.contiguous(), m1, m2, impl=impl) * (w / (n1 * n2))
        grad_u = grad_w = None
        if ctx.needs_input_grad[1]:
            # dL/dW[i, o] = sum_b conj(X[b, i]) dL/dY[b, o]: batch -> i, channels in -> b.
            xt = torch.conj_physical(modes).transpose(0, 1).contiguous()
            grad_w = mode_contract(xt, grad_out_modes)
        if ctx.needs_input_grad[0]:
            # dL/dX[b, i] = sum_o dL/dY[b, o] conj(W[i, o]): channels in <-> out swapped.
            wt = torch.conj_physical(weight).transpose(0, 1).contiguous()
            grad_modes = mode_contract(grad_out_modes, wt)
            grad_u = irfft2_from_modes(grad_modes / w, (n1, n2), impl=impl) * float(n1 * n2)
        return grad_u, grad_w, None, None, None


def spectral_conv2d(u: torch.Tensor, weight: torch.Tensor, m1: int, m2: int, *,
                    impl: str = "stockham_r8") -> torch.Tensor:
    """y = irfft2_from_modes(mode_contract(rfft2_truncated(u, m1, m2), weight), u's spatial shape).

    u: (b, c_in, n1, n2) float32 CUDA tensor; weight: (c_in, c_out, 2 m1, m2) complex64.
    Differentiable in u and weight."""
    if u.dim() != 4 or weight.dim() != 4:
        raise ValueError("spectral_conv2d: u must be (b, c_in, n1, n2) and weight (c_in, c_out, 2 m1, m2)")
    if weight.shape[0] != u.shape[1] or weight.shape[2] != 2 * m1 or weight.shape[3] != m2:
        raise ValueError(f"spectral_conv2d: weight shape {tuple(weight.shape)} does not match "
                         f"c_in = {u.shape[1]}, m1 = {m1}, m2 = {m2}")
    return _SpectralConv2dFunction.apply(u, weight, m1, m2, impl)


class SpectralConv2d(torch.nn.Module):
    """The FNO spectral convolution: keeps the 2 m1 x m2 lowest modes of each input channel's
    rfft2, mixes channels per mode with a learned complex weight, and transforms back.

    Weights start iid with real and imaginary parts N(0, 1 / (c_in c_out)), the initialisation
    of the reference's benchmark configuration."""

    def __init__(self, in_channels: int, out_channels: int, m1: int, m2: int, *,
                 impl: str = "stockham_r8", device=None):
        super().__init__()
        self.in_channels, self.out_channels, self.m1, self.m2, self.impl = in_channels, out_channels, m1, m2, impl
        std = 1.0 / math.sqrt(in_channels * out_channels)
        shape = (in_channels, out_channels, 2 * m1, m2)
        real = torch.randn(shape, device=device) * std
        imag = torch.randn(shape, device=device) * std
        self.weight = torch.nn.Parameter(torch.complex(real, imag))

    def forward(self, u: torch.Tensor) -> torch.Tensor:
        return spectral_conv2d(u, self.weight, self.m1, self.m2, impl=self.impl)

    def extra_repr(self) -> str:
        return f"{self.in_channels}, {self.out_channels}, m1={self.m1}, m2={self.m2}, impl={self.impl!r}"
