"""Batched float32 pseudo-spectral solver for 2D Navier-Stokes in vorticity form on this library's
transforms: the API of the reference's python/spectral/flow/gpu.py (Spectral, GpuSolver:
gpu.py:28-146), with the same discretization as its float64 solver (flow/reference.py):
rfft2 layout, 2/3-rule dealiasing, IMEX Crank-Nicolson / Heun.

    d omega / dt + u . grad omega = nu lap omega - alpha omega + f,  u = (psi_y, -psi_x),
    lap psi = -omega

pruned=True keeps the state on the modes the 2/3 rule keeps only, in the layout of
spectral.rfft2_truncated: rows ky = 0 .. m-1 and -m .. -1, columns kx = 0 .. m-1, m = n/3 + 1
(the row ky = -m lies outside the 2/3 set and stays masked).

Each step evaluates the tendency F = f_hat - N_hat twice. One evaluation: the four spectra
(u, v, d omega/dx, d omega/dy) come from one broadcast product of omega_hat with a precomputed
(4, ...) table of i k / |k|^2 and i k factors; one batched inverse transform of the four; the
product u omega_x + v omega_y (two fused multiply-adds); one forward transform; the mask and the
forcing. With graphs=True (the default on CUDA) a whole step is captured once per state shape
as a CUDA graph and replayed, so a step costs one launch from the host instead of about thirty.

For the pruned layout with a stockham implementation (16 <= n <= 512) a step is instead two
stages of three fused kernels each (torch.ops.spectral.flow_stage, csrc/flow.cu): the derived
spectra and the inverse column transforms; the four real row transforms, the product and the
forward row transform; the forward column transforms with the mask, forcing and update. The
physical fields then stay on chip, and the corrector updates the state in place.
"""

from __future__ import annotations

from collections.abc import Iterator

import numpy as np
import torch

from .. import ops
from .params import Flow, Grid, forcing


class Spectral:
    """A forward / inverse real 2D transform pair and the wavenumbers of its layout."""

    def __init__(self, n: int, fft_impl: str, pruned: bool, device: torch.device | str):
        if fft_impl != "cufft" and fft_impl not in ops.FFT_IMPLS:
            raise ValueError(f"unknown fft_impl '{fft_impl}' (available: cufft, {', '.join(ops.FFT_IMPLS)})")
        self.n, self.fft_impl, self.pruned = n, fft_impl, pruned
        grid = Grid(n)
        ky, kx = grid.ky[:, 0], grid.kx[0]
        if pruned:
            self.m = n // 3 + 1
            ky = np.concatenate([ky[: self.m], ky[n - self.m :]])
            kx = kx[: self.m]
        self.ky = torch.as_tensor(ky, dtype=torch.float32, device=device)[:, None]
        self.kx = torch.as_tensor(kx, dtype=torch.float32, device=device)[None, :]
        self.mask = ((self.kx.abs() <= n / 3) & (self.ky.abs() <= n / 3)).to(torch.float32)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Real (..., n, n) float32 -> complex64 spectrum in this layout."""
        n = self.n
        if self.fft_impl == "cufft":
            full = torch.fft.rfft2(x)
            if not self.pruned:
                return full
            m = self.m
            return torch.cat([full[..., :m, :m], full[..., n - m :, :m]], dim=-2)
        if self.pruned:
            return ops.rfft2_truncated(x, self.m, self.m, impl=self.fft_impl)
        return ops.rfft2(x, impl=self.fft_impl)

    def inverse(self, x_hat: torch.Tensor) -> torch.Tensor:
        """Complex64 spectrum in this layout -> real (..., n, n) float32."""
        n = self.n
        if self.fft_impl == "cufft":
            if self.pruned:
                m = self.m
                full = x_hat.new_zeros((*x_hat.shape[:-2], n, n // 2 + 1))
                full[..., :m, :m] = x_hat[..., :m, :]
                full[..., n - m :, :m] = x_hat[..., m:, :]
                x_hat = full
            return torch.fft.irfft2(x_hat, s=(n, n))
        if self.pruned:
            return ops.irfft2_from_modes(x_hat, (n, n), impl=self.fft_impl)
        return ops.irfft2(x_hat, n, impl=self.fft_impl)


class GpuSolver:
    """Advances a batch of vorticity fields. viscosity: a float, or one value per trajectory."""

    def __init__(
        self,
        n: int,
        flow: Flow,
        dt: float,
        *,
        fft_impl: str = "stockham_r8",
        pruned: bool = False,
        device: torch.device | str = "cuda",
        graphs: bool = True,
    ):
        self.n, self.flow, self.dt = n, flow, dt
        self.spectral = s = Spectral(n, fft_impl, pruned, device)
        self.device = torch.device(device)
        self.graphs = graphs and self.device.type == "cuda"
        self.ikx = (1j * s.kx).to(torch.complex64)
        self.iky = (1j * s.ky).to(torch.complex64)
        k2 = s.kx**2 + s.ky**2
        self.inverse_k2 = torch.where(k2 > 0, 1.0 / k2.clamp(min=1.0), torch.zeros_like(k2))
        # omega_hat -> (u, v, omega_x, omega_y) spectra: i ky / |k|^2, -i kx / |k|^2, i kx, i ky.
        shape = self.inverse_k2.shape
        self.derive = torch.stack(
            [self.iky * self.inverse_k2, -self.ikx * self.inverse_k2, self.ikx.expand(shape), self.iky.expand(shape)]
        ).contiguous()

        f = torch.as_tensor(forcing(Grid(n), flow), dtype=torch.float32, device=device)
        self.forcing_hat = s.forward(f) * s.mask

        nu = torch.as_tensor(np.asarray(flow.viscosity), dtype=torch.float32, device=device)
        nu = nu[..., None, None] if nu.dim() else nu
        linear = -nu * k2 - flow.drag
        self.explicit = (1.0 + 0.5 * dt * linear).to(torch.complex64)
        self.implicit = (1.0 / (1.0 - 0.5 * dt * linear)).to(torch.complex64)
        self._graph_cache: dict[tuple, tuple] = {}

        # The fused stages (pruned layout, stockham implementations): real factors, contiguous.
        self.fused = (pruned and fft_impl.startswith("stockham") and 16 <= n <= 512
                      and self.device.type == "cuda")
        if self.fused:
            self._mask = s.mask.expand(self.inverse_k2.shape).contiguous()
            self._forcing = self.forcing_hat.contiguous()
            self._explicit = (1.0 + 0.5 * dt * linear).to(torch.float32).contiguous()
            self._implicit = (1.0 / (1.0 - 0.5 * dt * linear)).to(torch.float32).contiguous()

    def to_spectral(self, w: torch.Tensor) -> torch.Tensor:
        """omega_hat of physical vorticity (..., n, n), projected onto the dealiased modes."""
        return self.spectral.forward(w.to(torch.float32).contiguous()) * self.spectral.mask

    def to_physical(self, w_hat: torch.Tensor) -> torch.Tensor:
        return self.spectral.inverse(w_hat)

    def tendency(self, w_hat: torch.Tensor) -> torch.Tensor:
        """f_hat - N_hat, N = u . grad omega, dealiased."""
        fields_hat = self.derive.view(4, *([1] * (w_hat.dim() - 2)), *self.derive.shape[-2:]) * w_hat
        u, v, wx, wy = self.spectral.inverse(fields_hat)  # one batched inverse transform
        nonlinear = torch.addcmul(u * wx, v, wy)
        return self.forcing_hat - self.spectral.forward(nonlinear) * self.spectral.mask

    def _stage(self, x, w, f0, out, stage: int) -> None:
        m = self.spectral.m
        batch = w.numel() // (2 * m * m)
        work = torch.empty(5 * batch * self.n * m, dtype=torch.complex64, device=w.device)
        torch.ops.spectral.flow_stage.default(
            x, w, f0, out, self.derive, self._forcing, self._mask, self._explicit, self._implicit, work,
            self.n, m, self.dt, stage, self.spectral.fft_impl)

    def _step_fused(self, w_hat: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One step by the fused stages; out=w_hat updates the state in place."""
        w = w_hat.contiguous()
        f0 = torch.empty_like(w)
        predicted = torch.empty_like(w)
        out = torch.empty_like(w) if out is None else out
        self._stage(w, w, f0, predicted, 0)
        self._stage(predicted, w, f0, out, 1)
        return out

    def _step_eager(self, w_hat: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self._step_fused(w_hat)
        f0 = self.tendency(w_hat)
        held = self.explicit * w_hat
        predicted = (held + self.dt * f0) * self.implicit
        f1 = self.tendency(predicted)
        return (held + (0.5 * self.dt) * (f0 + f1)) * self.implicit

    def _graph(self, w_hat: torch.Tensor):
        """(graph, state): replaying `graph` advances `state` (a static buffer) by one step in
        place. Captured on first use for a shape, after one eager warm-up step (which also
        creates every twiddle table the transforms need)."""
        key = (tuple(w_hat.shape), w_hat.device)
        if key not in self._graph_cache:
            state = w_hat.detach().clone()
            side = torch.cuda.Stream(device=w_hat.device)
            side.wait_stream(torch.cuda.current_stream(w_hat.device))
            with torch.cuda.stream(side):
                self._step_eager(state)  # warm-up outside the capture
            torch.cuda.current_stream(w_hat.device).wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                if self.fused:
                    self._step_fused(state, out=state)
                else:
                    state.copy_(self._step_eager(state))
            self._graph_cache[key] = (graph, state)
        return self._graph_cache[key]

    def step(self, w_hat: torch.Tensor) -> torch.Tensor:
        if not (self.graphs and w_hat.is_cuda):
            return self._step_eager(w_hat)
        graph, state = self._graph(w_hat)
        state.copy_(w_hat)
        graph.replay()
        return state.clone()

    def frames(self, w0: torch.Tensor, steps: int, record_every: int = 1) -> Iterator[torch.Tensor]:
        """Yields physical vorticity (..., n, n) every record_every steps, starting with the
        dealiased initial condition."""
        if steps < 0 or record_every < 1:
            raise ValueError("need steps >= 0 and record_every >= 1")
        w_hat = self.to_spectral(w0)
        yield self.to_physical(w_hat)
        if not (self.graphs and w_hat.is_cuda) or steps == 0:
            for k in range(1, steps + 1):
                w_hat = self._step_eager(w_hat)
                if k % record_every == 0:
                    yield self.to_physical(w_hat)
            return
        graph, state = self._graph(w_hat)
        state.copy_(w_hat)
        for k in range(1, steps + 1):
            graph.replay()
            if k % record_every == 0:
                yield self.to_physical(state)

    def simulate(self, w0: torch.Tensor, steps: int, record_every: int = 1) -> torch.Tensor:
        """All frames, stacked: (frames, ..., n, n)."""
        return torch.stack(list(self.frames(w0, steps, record_every)))
