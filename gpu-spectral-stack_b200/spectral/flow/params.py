"""The vorticity equation's parameters and the wavenumbers of its spectral grid.

The public names and fields are those of the reference's python/spectral/flow/params.py
(params.py:15-104), which its solvers and scripts share: Flow, Grid (kx, ky, k2, inverse_k2,
dealias, x, y), forcing, forcing_velocity, laminar_kolmogorov and taylor_green.

Layout: a field is a real array (..., n, n) sampled at y_i = 2 pi i / n (rows) and x_j = 2 pi j / n
(columns); its spectrum is in the rfft2 layout (..., n, n // 2 + 1), rows ky = 0 .. n/2 - 1,
-n/2 .. -1 and columns kx = 0 .. n/2. Wavenumbers are integers stored as float64.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from functools import cached_property

import numpy as np


@dataclass(frozen=True)
class Flow:
    """nu, alpha, A and k_f of  d omega / dt + u . grad omega = nu lap omega - alpha omega + f,
    f = -A k_f cos(k_f y). A solver that advances a batch takes one viscosity per trajectory (an
    array of shape (batch,)) as well as a single value."""

    viscosity: float = 1e-3
    drag: float = 0.1
    forcing_amplitude: float = 1.0
    forcing_wavenumber: int = 4

    def as_dict(self) -> dict:
        return asdict(self)


def _signed(n: int) -> np.ndarray:
    """0, 1, ..., n/2 - 1, -n/2, ..., -1: the signed wavenumber of each of n FFT bins."""
    k = np.arange(n, dtype=np.int64)
    k[n // 2 :] -= n
    return k


@dataclass(frozen=True)
class Grid:
    """The spectral grid of an n x n periodic box (n a power of two, at least 4): the rfft2
    layout's wavenumbers, |k|^2 and its inverse, the 2/3-rule mask, and the sample points. Each
    array is built on first use and kept."""

    n: int

    def __post_init__(self):
        if self.n < 4 or self.n & (self.n - 1):
            raise ValueError(f"n must be a power of two of at least 4, got {self.n}")

    @cached_property
    def _k_int(self) -> tuple[np.ndarray, np.ndarray]:
        """(ky (n, 1), kx (1, n/2 + 1)) as integers."""
        return _signed(self.n)[:, None], np.arange(self.n // 2 + 1, dtype=np.int64)[None, :]

    @cached_property
    def kx(self) -> np.ndarray:
        """(1, n // 2 + 1): 0 .. n/2."""
        return self._k_int[1].astype(np.float64)

    @cached_property
    def ky(self) -> np.ndarray:
        """(n, 1): 0 .. n/2 - 1, -n/2 .. -1."""
        return self._k_int[0].astype(np.float64)

    @cached_property
    def k2(self) -> np.ndarray:
        """(n, n // 2 + 1): kx^2 + ky^2."""
        ky, kx = self._k_int
        return (kx * kx + ky * ky).astype(np.float64)

    @cached_property
    def inverse_k2(self) -> np.ndarray:
        """1 / |k|^2, with 0 at k = 0 (the streamfunction has no mean)."""
        k2 = self.k2
        zero = k2 == 0
        return np.where(zero, 0.0, 1.0 / np.where(zero, 1.0, k2))

    @cached_property
    def dealias(self) -> np.ndarray:
        """The modes the 2/3 rule keeps, |kx| <= n/3 and |ky| <= n/3, tested exactly in integers
        (3 |k| <= n): a quadratic product of fields inside this set aliases only onto modes
        outside it."""
        ky, kx = self._k_int
        return (3 * np.abs(kx) <= self.n) & (3 * np.abs(ky) <= self.n)

    @cached_property
    def _points(self) -> np.ndarray:
        return 2.0 * np.pi * np.arange(self.n) / self.n

    @property
    def y(self) -> np.ndarray:
        """(n, 1): the rows' coordinates."""
        return self._points[:, None]

    @property
    def x(self) -> np.ndarray:
        """(1, n): the columns' coordinates."""
        return self._points[None, :]


def _shear(grid: Grid, profile: np.ndarray) -> np.ndarray:
    """The (n, n) field that equals profile[i] along row i (a function of y only)."""
    return np.ascontiguousarray(np.broadcast_to(profile.reshape(grid.n, 1), (grid.n, grid.n)))


def forcing(grid: Grid, flow: Flow) -> np.ndarray:
    """The Kolmogorov forcing f = -A k_f cos(k_f y) on the grid, (n, n)."""
    k = flow.forcing_wavenumber
    return _shear(grid, -(flow.forcing_amplitude * k) * np.cos(k * grid.y))


def forcing_velocity(grid: Grid, flow: Flow) -> np.ndarray:
    """The body force along x, A sin(k_f y), (n, n): forcing() is its curl."""
    return _shear(grid, flow.forcing_amplitude * np.sin(flow.forcing_wavenumber * grid.y))


def laminar_kolmogorov(grid: Grid, flow: Flow) -> np.ndarray:
    """The laminar fixed point: a shear flow has no nonlinear term, so the steady state solves
    (nu k_f^2 + alpha) omega = f."""
    damping = float(np.asarray(flow.viscosity)) * flow.forcing_wavenumber**2 + flow.drag
    return forcing(grid, flow) / damping


def taylor_green(grid: Grid, t: float, viscosity: float, drag: float) -> np.ndarray:
    """The unforced Taylor-Green vortex 2 sin x sin y e^(-(2 nu + alpha) t): its streamfunction is
    proportional to omega, so advection vanishes and this decay is exact."""
    return 2.0 * np.sin(grid.x) * np.sin(grid.y) * np.exp(-(2.0 * viscosity + drag) * t)
