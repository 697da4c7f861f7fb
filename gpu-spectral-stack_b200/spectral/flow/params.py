"""Physical parameters of the 2D vorticity equation and the wavenumbers of its spectral grid:
the same classes, fields, defaults and functions as the reference's
python/spectral/flow/params.py (params.py:15-104), which every solver shares.

Fields are real arrays (..., n, n) of values at x_j = 2 pi j / n (last axis) and y_i = 2 pi i / n
(the axis before it); spectra are in the rfft2 layout (..., n, n // 2 + 1), rows ky = 0, 1, ...,
n/2 - 1, -n/2, ..., -1 and columns kx = 0 .. n/2.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

import numpy as np


@dataclass(frozen=True)
class Flow:
    """The equation's parameters. viscosity may be one value per trajectory (an array of shape
    (batch,)) wherever a solver takes a batch."""

    viscosity: float = 1e-3  # nu
    drag: float = 0.1  # alpha: linear friction
    forcing_amplitude: float = 1.0  # A
    forcing_wavenumber: int = 4  # k_f

    def as_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class Grid:
    """Wavenumbers of an n x n grid in the rfft2 layout and the 2/3-rule dealiasing mask."""

    n: int

    def __post_init__(self):
        if self.n < 4 or self.n & (self.n - 1):
            raise ValueError(f"n must be a power of two of at least 4, got {self.n}")

    @property
    def kx(self) -> np.ndarray:
        """(1, n // 2 + 1): 0, 1, ..., n / 2."""
        return np.arange(self.n // 2 + 1, dtype=np.float64)[None, :]

    @property
    def ky(self) -> np.ndarray:
        """(n, 1): 0, 1, ..., n/2 - 1, -n/2, ..., -1."""
        k = np.arange(self.n, dtype=np.float64)
        return np.where(k < self.n // 2, k, k - self.n)[:, None]

    @property
    def k2(self) -> np.ndarray:
        return self.kx**2 + self.ky**2

    @property
    def inverse_k2(self) -> np.ndarray:
        """1 / |k|^2, and 0 for the mean mode (the streamfunction has no mean)."""
        k2 = self.k2
        return np.divide(1.0, k2, out=np.zeros_like(k2), where=k2 > 0)

    @property
    def dealias(self) -> np.ndarray:
        """Modes the 2/3 rule keeps: |kx| and |ky| at most n / 3."""
        kmax = self.n / 3.0
        return (np.abs(self.kx) <= kmax) & (np.abs(self.ky) <= kmax)

    @property
    def y(self) -> np.ndarray:
        return (2.0 * np.pi * np.arange(self.n) / self.n)[:, None]

    @property
    def x(self) -> np.ndarray:
        return (2.0 * np.pi * np.arange(self.n) / self.n)[None, :]


def forcing(grid: Grid, flow: Flow) -> np.ndarray:
    """Kolmogorov forcing f(y) = -A k_f cos(k_f y), shape (n, n)."""
    k = flow.forcing_wavenumber
    return np.repeat(-flow.forcing_amplitude * k * np.cos(k * grid.y), grid.n, axis=1)


def forcing_velocity(grid: Grid, flow: Flow) -> np.ndarray:
    """The body force's x-component A sin(k_f y), whose curl is forcing(); shape (n, n)."""
    return np.repeat(flow.forcing_amplitude * np.sin(flow.forcing_wavenumber * grid.y), grid.n, axis=1)


def laminar_kolmogorov(grid: Grid, flow: Flow) -> np.ndarray:
    """The steady laminar shear flow omega = f / (nu k_f^2 + alpha), a fixed point of the
    equation (its nonlinear term vanishes)."""
    nu = float(np.asarray(flow.viscosity))
    return forcing(grid, flow) / (nu * flow.forcing_wavenumber**2 + flow.drag)


def taylor_green(grid: Grid, t: float, viscosity: float, drag: float) -> np.ndarray:
    """The unforced Taylor-Green vortex 2 sin x sin y exp(-(2 nu + alpha) t), an exact solution."""
    return 2.0 * np.sin(grid.x) * np.sin(grid.y) * np.exp(-(2.0 * viscosity + drag) * t)
