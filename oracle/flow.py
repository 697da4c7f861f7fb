"""Float64 Navier-Stokes solver in vorticity form: the check for spectral.flow's GPU solver.
TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

A restatement of the reference's python/spectral/flow/reference.py (Solver, to_spectral,
simulate, diagnostics, budget_rates: reference.py:32-157) on its own grid helpers
(params.py:29-104), in numpy float64. Pseudo-spectral: the state is omega_hat (rfft2 layout,
projected onto the 2/3-rule modes); u . grad omega is formed from four inverse transforms and
brought back with one forward transform, then masked. Time stepping, IMEX Crank-Nicolson / Heun
with L = -nu |k|^2 - alpha:

    w*  = [(1 + dt/2 L) w + dt F(w)] / (1 - dt/2 L)
    w'  = [(1 + dt/2 L) w + dt/2 (F(w) + F(w*))] / (1 - dt/2 L),   F = f_hat - N_hat
"""

from __future__ import annotations

import numpy as np


def wavenumbers(n: int) -> tuple[np.ndarray, np.ndarray]:
    """(kx (1, n/2 + 1), ky (n, 1)) of the rfft2 layout (params.py:39-47)."""
    kx = np.arange(n // 2 + 1, dtype=np.float64)[None, :]
    k = np.arange(n, dtype=np.float64)
    ky = np.where(k < n // 2, k, k - n)[:, None]
    return kx, ky


def dealias(n: int) -> np.ndarray:
    """|kx|, |ky| <= n / 3 (params.py:62-68)."""
    kx, ky = wavenumbers(n)
    return (np.abs(kx) <= n / 3.0) & (np.abs(ky) <= n / 3.0)


def grid_y(n: int) -> np.ndarray:
    return (2.0 * np.pi * np.arange(n) / n)[:, None]


def grid_x(n: int) -> np.ndarray:
    return (2.0 * np.pi * np.arange(n) / n)[None, :]


def forcing(n: int, amplitude: float = 1.0, wavenumber: int = 4) -> np.ndarray:
    """-A k_f cos(k_f y) on the n x n grid (params.py:81-85)."""
    return np.broadcast_to(-amplitude * wavenumber * np.cos(wavenumber * grid_y(n)), (n, n)).copy()


def forcing_velocity(n: int, amplitude: float = 1.0, wavenumber: int = 4) -> np.ndarray:
    return np.broadcast_to(amplitude * np.sin(wavenumber * grid_y(n)), (n, n)).copy()


def taylor_green(n: int, t: float, viscosity: float, drag: float) -> np.ndarray:
    return 2.0 * np.sin(grid_x(n)) * np.sin(grid_y(n)) * np.exp(-(2.0 * viscosity + drag) * t)


def rfft2(x) -> np.ndarray:
    return np.fft.rfft2(np.asarray(x, dtype=np.float64), axes=(-2, -1))


def irfft2(x, n: int) -> np.ndarray:
    return np.fft.irfft2(x, s=(n, n), axes=(-2, -1))


class Solver:
    """Operators for one grid and one parameter set (reference.py:46-88). viscosity: a float or
    one value per trajectory."""

    def __init__(self, n: int, dt: float, viscosity=1e-3, drag: float = 0.1, amplitude: float = 1.0,
                 wavenumber: int = 4):
        self.n, self.dt = n, dt
        kx, ky = wavenumbers(n)
        k2 = kx**2 + ky**2
        self.ikx, self.iky = 1j * kx, 1j * ky
        self.inverse_k2 = np.divide(1.0, k2, out=np.zeros_like(k2), where=k2 > 0)
        self.mask = dealias(n)
        self.forcing_hat = rfft2(forcing(n, amplitude, wavenumber)) * self.mask
        nu = np.asarray(viscosity, dtype=np.float64)
        nu = nu[..., None, None] if nu.ndim else nu
        linear = -nu * k2 - drag
        self.explicit = 1.0 + 0.5 * dt * linear
        self.implicit = 1.0 / (1.0 - 0.5 * dt * linear)

    def velocity_hat(self, w_hat):
        psi_hat = w_hat * self.inverse_k2
        return self.iky * psi_hat, -self.ikx * psi_hat

    def nonlinear_hat(self, w_hat) -> np.ndarray:
        n = self.n
        u_hat, v_hat = self.velocity_hat(w_hat)
        u, v = irfft2(u_hat, n), irfft2(v_hat, n)
        wx, wy = irfft2(self.ikx * w_hat, n), irfft2(self.iky * w_hat, n)
        return rfft2(u * wx + v * wy) * self.mask

    def tendency(self, w_hat) -> np.ndarray:
        return self.forcing_hat - self.nonlinear_hat(w_hat)

    def step(self, w_hat) -> np.ndarray:
        f0 = self.tendency(w_hat)
        predicted = (self.explicit * w_hat + self.dt * f0) * self.implicit
        f1 = self.tendency(predicted)
        return (self.explicit * w_hat + 0.5 * self.dt * (f0 + f1)) * self.implicit


def to_spectral(w, n: int) -> np.ndarray:
    return rfft2(w) * dealias(n)


def simulate(w0, dt: float, steps: int, record_every: int = 1, **flow) -> np.ndarray:
    """(frames, ..., n, n): frame k after k * record_every steps, frame 0 the dealiased initial
    condition (reference.py:96-111)."""
    if steps < 0 or record_every < 1:
        raise ValueError("need steps >= 0 and record_every >= 1")
    n = np.shape(w0)[-1]
    solver = Solver(n, dt, **flow)
    w_hat = to_spectral(w0, n)
    frames = [irfft2(w_hat, n)]
    for k in range(1, steps + 1):
        w_hat = solver.step(w_hat)
        if k % record_every == 0:
            frames.append(irfft2(w_hat, n))
    return np.stack(frames)


def diagnostics(w, viscosity=1e-3, drag: float = 0.1, amplitude: float = 1.0, wavenumber: int = 4) -> dict:
    """Domain averages (reference.py:117-148): energy, enstrophy, palinstrophy, energy_input,
    enstrophy_input."""
    n = np.shape(w)[-1]
    solver = Solver(n, 1.0, viscosity, drag, amplitude, wavenumber)
    w_hat = to_spectral(w, n)
    u_hat, v_hat = solver.velocity_hat(w_hat)
    u, v = irfft2(u_hat, n), irfft2(v_hat, n)
    wx, wy = irfft2(solver.ikx * w_hat, n), irfft2(solver.iky * w_hat, n)
    wp = irfft2(w_hat, n)

    def mean(a):
        return a.mean(axis=(-2, -1))

    return {
        "energy": 0.5 * mean(u**2 + v**2),
        "enstrophy": 0.5 * mean(wp**2),
        "palinstrophy": 0.5 * mean(wx**2 + wy**2),
        "energy_input": mean(u * forcing_velocity(n, amplitude, wavenumber)),
        "enstrophy_input": mean(wp * forcing(n, amplitude, wavenumber)),
    }


def budget_rates(w, viscosity=1e-3, drag: float = 0.1, amplitude: float = 1.0, wavenumber: int = 4):
    """(dE/dt, dZ/dt) from the exact budgets of the dealiased system (reference.py:151-157)."""
    d = diagnostics(w, viscosity, drag, amplitude, wavenumber)
    nu = np.asarray(viscosity, dtype=np.float64)
    de = d["energy_input"] - 2 * nu * d["enstrophy"] - 2 * drag * d["energy"]
    dz = d["enstrophy_input"] - 2 * nu * d["palinstrophy"] - 2 * drag * d["enstrophy"]
    return de, dz


def smooth_random_field(rng: np.random.Generator, n: int, batch: tuple = ()) -> np.ndarray:
    """A zero-mean random vorticity field with its energy below wavenumber about 6, unit
    standard deviation (the reference tests' initial condition, test_flow_reference.py:12-19)."""
    kx, ky = wavenumbers(n)
    filtered = rfft2(rng.standard_normal((*batch, n, n))) * np.exp(-(kx**2 + ky**2) / 18.0)
    filtered[..., 0, 0] = 0
    w = irfft2(filtered, n)
    return w / w.std(axis=(-2, -1), keepdims=True)
