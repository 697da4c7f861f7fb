"""Batched float32 pseudo-spectral solver of the 2D vorticity equation on this library's
transforms. The public API is that of the reference's python/spectral/flow/gpu.py (Spectral,
GpuSolver: gpu.py:28-146), with the discretization of its float64 solver
(flow/reference.py): the rfft2 layout, the 2/3-rule dealiasing, and the IMEX step that treats
the linear terms by Crank-Nicolson and the rest by Heun's method,

    d omega / dt + u . grad omega = nu lap omega - alpha omega + f,   u = (psi_y, -psi_x),
    lap psi = -omega.

pruned=True keeps the spectrum on the dealiased modes only, in spectral.rfft2_truncated's layout:
rows ky = 0 .. m-1 and -m .. -1, columns kx = 0 .. m-1, m = n/3 + 1 (the row ky = -m is outside
the 2/3 set and stays masked).

How a step runs, from the fastest path down:
  - pruned, a stockham implementation, 16 <= n <= 512 on CUDA: two stages of three fused kernels
    (torch.ops.spectral.flow_stage, csrc/flow.cu) in which the physical fields never leave the
    chip;
  - otherwise composed from batched transforms: the four spectra u, v, omega_x, omega_y are one
    product of omega_hat with a (4, rows, cols) table of derivative factors, one inverse transform
    of the four, the advection u omega_x + v omega_y, one forward transform, mask and forcing.
With graphs=True (the default on CUDA) a step is captured once per state shape as a CUDA graph
and replayed: one launch from the host per step.
"""

from __future__ import annotations

from collections.abc import Iterator

import numpy as np
import torch

from .. import ops
from .params import Flow, Grid, forcing


class Spectral:
    """The forward and inverse real 2D transforms of an n x n field in the full or the pruned
    layout, and that layout's wavenumbers (ky: (rows, 1), kx: (1, cols)) and 2/3-rule mask."""

    def __init__(self, n: int, fft_impl: str, pruned: bool, device: torch.device | str):
        if fft_impl != "cufft" and fft_impl not in ops.FFT_IMPLS:
            raise ValueError(f"unknown fft_impl '{fft_impl}' (available: cufft, {', '.join(ops.FFT_IMPLS)})")
        self.n, self.fft_impl, self.pruned = n, fft_impl, pruned
        ky_all = np.concatenate([np.arange(n // 2), np.arange(-(n // 2), 0)])  # rfft2 row order
        if pruned:
            self.m = n // 3 + 1
            rows = np.concatenate([np.arange(self.m), np.arange(n - self.m, n)])
            cols = np.arange(self.m)
        else:
            rows, cols = np.arange(n), np.arange(n // 2 + 1)
        self._rows = torch.as_tensor(rows, dtype=torch.int64, device=device)
        ky, kx = ky_all[rows], cols
        self.ky = torch.as_tensor(ky, dtype=torch.float32, device=device)[:, None]
        self.kx = torch.as_tensor(kx, dtype=torch.float32, device=device)[None, :]
        keep = (3 * np.abs(ky)[:, None] <= n) & (3 * np.abs(kx)[None, :] <= n)  # 2/3 rule, exact
        self.mask = torch.as_tensor(keep, dtype=torch.float32, device=device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Real (..., n, n) float32 -> complex64 spectrum in this layout."""
        if self.fft_impl != "cufft":
            if self.pruned:
                return ops.rfft2_truncated(x, self.m, self.m, impl=self.fft_impl)
            return ops.rfft2(x, impl=self.fft_impl)
        full = torch.fft.rfft2(x)
        if not self.pruned:
            return full
        return full.index_select(-2, self._rows)[..., : self.m]

    def inverse(self, x_hat: torch.Tensor) -> torch.Tensor:
        """Complex64 spectrum in this layout -> real (..., n, n) float32."""
        n = self.n
        if self.fft_impl != "cufft":
            if self.pruned:
                return ops.irfft2_from_modes(x_hat, (n, n), impl=self.fft_impl)
            return ops.irfft2(x_hat, n, impl=self.fft_impl)
        if self.pruned:
            full = x_hat.new_zeros(*x_hat.shape[:-2], n, n // 2 + 1)
            full[..., : self.m].index_copy_(-2, self._rows, x_hat)
            x_hat = full
        return torch.fft.irfft2(x_hat, s=(n, n))


class GpuSolver:
    """Advances a batch of vorticity spectra by dt per step. flow.viscosity: one value, or an
    array with one value per trajectory (the batch is then the leading dimension)."""

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

        k2 = s.kx * s.kx + s.ky * s.ky
        inv_k2 = torch.where(k2 == 0, torch.zeros_like(k2), 1.0 / torch.where(k2 == 0, torch.ones_like(k2), k2))
        i_kx = torch.complex(torch.zeros_like(s.kx), s.kx).expand_as(k2)
        i_ky = torch.complex(torch.zeros_like(s.ky), s.ky).expand_as(k2)
        # omega_hat times these gives the spectra of u = psi_y, v = -psi_x, omega_x, omega_y
        # (psi_hat = omega_hat / |k|^2).
        self.derive = torch.stack([i_ky * inv_k2, -i_kx * inv_k2, i_kx, i_ky]).contiguous()

        self.forcing_hat = s.forward(torch.as_tensor(forcing(Grid(n), flow), dtype=torch.float32, device=device))
        self.forcing_hat = self.forcing_hat * s.mask

        # Crank-Nicolson factors of the linear term L = -nu |k|^2 - alpha, per trajectory when
        # the viscosity is: the state advances as (E w + dt F) I with E = 1 + dt L / 2 and
        # I = 1 / (1 - dt L / 2).
        nu = torch.as_tensor(np.asarray(flow.viscosity), dtype=torch.float32, device=device)
        linear = -(nu.reshape(*nu.shape, 1, 1) if nu.dim() else nu) * k2 - flow.drag
        self._explicit_real = (1.0 + 0.5 * dt * linear).contiguous()
        self._implicit_real = (1.0 / (1.0 - 0.5 * dt * linear)).contiguous()
        self.explicit = self._explicit_real.to(torch.complex64)
        self.implicit = self._implicit_real.to(torch.complex64)
        self._graphs: dict[tuple, tuple] = {}

        self.fused = pruned and fft_impl.startswith("stockham") and 16 <= n <= 512 and self.device.type == "cuda"
        if self.fused:
            self._mask = s.mask.expand(k2.shape).contiguous()
            self._forcing = self.forcing_hat.contiguous()

    # --- physical <-> spectral ------------------------------------------------------------

    def to_spectral(self, w: torch.Tensor) -> torch.Tensor:
        """The dealiased spectrum of physical vorticity (..., n, n)."""
        return self.spectral.forward(w.to(torch.float32).contiguous()) * self.spectral.mask

    def to_physical(self, w_hat: torch.Tensor) -> torch.Tensor:
        return self.spectral.inverse(w_hat)

    # --- the composed step ------------------------------------------------------------------

    def tendency(self, w_hat: torch.Tensor) -> torch.Tensor:
        """F(omega_hat) = f_hat - mask * FFT(u omega_x + v omega_y)."""
        planes = self.derive.view(4, *([1] * (w_hat.dim() - 2)), *self.derive.shape[1:])
        u, v, wx, wy = self.spectral.inverse(planes * w_hat)  # one batched inverse of four fields
        advection = torch.addcmul(u * wx, v, wy)
        return self.forcing_hat - self.spectral.forward(advection) * self.spectral.mask

    def _advance(self, w_hat: torch.Tensor, increment: torch.Tensor) -> torch.Tensor:
        """(E w_hat + increment) I: the Crank-Nicolson update around an explicit increment."""
        return torch.addcmul(increment, self.explicit, w_hat) * self.implicit

    def _step_composed(self, w_hat: torch.Tensor) -> torch.Tensor:
        # Heun: a predictor with the tendency at the start, a corrector with the mean of the
        # tendencies at the start and at the predicted state.
        f_start = self.tendency(w_hat)
        predicted = self._advance(w_hat, self.dt * f_start)
        f_end = self.tendency(predicted)
        return self._advance(w_hat, (0.5 * self.dt) * (f_start + f_end))

    # --- the fused stages ---------------------------------------------------------------------

    def _stage(self, x, w, f0, out, stage: int) -> None:
        m = self.spectral.m
        batch = w.numel() // (2 * m * m)
        work = torch.empty(5 * batch * self.n * m, dtype=torch.complex64, device=w.device)
        torch.ops.spectral.flow_stage.default(
            x, w, f0, out, self.derive, self._forcing, self._mask, self._explicit_real, self._implicit_real, work,
            self.n, m, self.dt, stage, self.spectral.fft_impl)

    def _step_fused(self, w_hat: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """One step by the fused stages; out = w_hat updates the state in place (the corrector
        reads each value of w before it writes it)."""
        w = w_hat.contiguous()
        f0, predicted = torch.empty_like(w), torch.empty_like(w)
        out = torch.empty_like(w) if out is None else out
        self._stage(w, w, f0, predicted, 0)
        self._stage(predicted, w, f0, out, 1)
        return out

    def _step_eager(self, w_hat: torch.Tensor) -> torch.Tensor:
        return self._step_fused(w_hat) if self.fused else self._step_composed(w_hat)

    # --- CUDA graphs ------------------------------------------------------------------------------

    def _graph(self, w_hat: torch.Tensor):
        """(graph, state) for w_hat's shape: replaying graph advances the static buffer state by
        one step in place. Captured at first use, after an eager warm-up step on a side stream
        that also builds every twiddle table the transforms need."""
        key = (tuple(w_hat.shape), w_hat.device)
        cached = self._graphs.get(key)
        if cached is not None:
            return cached
        state = w_hat.detach().clone()
        current = torch.cuda.current_stream(w_hat.device)
        side = torch.cuda.Stream(device=w_hat.device)
        side.wait_stream(current)
        with torch.cuda.stream(side):
            self._step_eager(state)
        current.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            if self.fused:
                self._step_fused(state, out=state)
            else:
                state.copy_(self._step_composed(state))
        self._graphs[key] = (graph, state)
        return graph, state

    def _use_graphs(self, w_hat: torch.Tensor) -> bool:
        return self.graphs and w_hat.is_cuda

    # --- public stepping --------------------------------------------------------------------------

    def step(self, w_hat: torch.Tensor) -> torch.Tensor:
        """The spectrum one step later (a new tensor)."""
        if not self._use_graphs(w_hat):
            return self._step_eager(w_hat)
        graph, state = self._graph(w_hat)
        state.copy_(w_hat)
        graph.replay()
        return state.clone()

    def frames(self, w0: torch.Tensor, steps: int, record_every: int = 1) -> Iterator[torch.Tensor]:
        """Physical vorticity (..., n, n): the dealiased initial condition, then every
        record_every-th of `steps` steps, one frame at a time."""
        if steps < 0 or record_every < 1:
            raise ValueError("need steps >= 0 and record_every >= 1")
        w_hat = self.to_spectral(w0)
        yield self.to_physical(w_hat)
        if steps == 0:
            return
        if self._use_graphs(w_hat):
            graph, state = self._graph(w_hat)
            state.copy_(w_hat)
            advance, current = graph.replay, lambda: state
        else:
            holder = [w_hat]

            def advance() -> None:
                holder[0] = self._step_eager(holder[0])

            current = lambda: holder[0]  # noqa: E731
        for k in range(1, steps + 1):
            advance()
            if k % record_every == 0:
                yield self.to_physical(current())

    def simulate(self, w0: torch.Tensor, steps: int, record_every: int = 1) -> torch.Tensor:
        """All frames stacked: (frames, ..., n, n)."""
        return torch.stack(list(self.frames(w0, steps, record_every)))
