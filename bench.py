"""Benchmark of the batched-FFT hot path: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload real|c2c|rfft2|pruned|slab|spectrum|fir|flow|fft1d] [--fft-impl stockham_r8]

The headline workload is the one the metric is quoted on (configs[1] of BASELINE.json): a step
is rfft then irfft of 4096 rows of 4096 float32 samples, iid U[-1, 1] from a seed, 2^24 points
per GPU. `value` is the effective bandwidth of the whole job, algorithmic bytes / time, with the
reference's byte convention (4 n + 8 (n/2 + 1) bytes per real row and direction): the inputs are
resident on the device when timing starts, every launch goes through the C ABI
(include/spectral_b200.h), and the time is device time from CUDA events, the maximum over ranks.

L2 hygiene: 4 rotating buffer sets of 192 MiB each (768 MiB, 6x the 126 MB L2). Step k
transforms set k mod 4 forward and, for the inverse, reads the spectrum of set (k + 2) mod 4,
written two steps (and 384 MiB of traffic) earlier, so no kernel reads what the previous kernel
just wrote.

Multi-GPU (torchrun, one rank per GPU): every rank transforms its own 2^24 points (weak
scaling, batch sharding with no communication); a barrier and a synchronize bracket the timed
steps, and the slowest rank's time counts.

Also on the line: `roofline` (the dominant kernel's achieved bytes / its average CUDA-event
duration against the measured HBM copy peak, and against a copy of the same size measured in the
run, `size_matched_copy`: a 4 GB copy reaches the peak, a copy of one launch's bytes does not),
`e2e` (the same metric through the public torch
API with host buffers: pinned host -> device, both transforms, device -> host, every step),
`cpu_baseline` (the float64 oracle, numpy's pocketfft as in the reference's CPU path, on the
host's cores), `clocks` (SM clock and throttle reasons, sampled through NVML during the timed steps) and `gpu_launches`.

--impl reference times the reference's CPU implementation of the path (the oracle port) on all
host cores, with the same workload, metric and unit.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gpu-spectral-stack_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "Effective FFT GB/s (% of B200 HBM peak) at 2^24 pts/GPU, 1/2/4/8 GPUs"
UNIT = "GB/s"
SETS = 4
MIN_ROUNDS = 5           # timed rounds of K steps at least (the reference's default)
MAX_ROUNDS = 400
ROUND_TARGET_MS = 40.0   # rounds enough for ~20 NVML clock samples under load
SPREAD_WARN = 0.05       # (max - min) / median of the rounds above this gets a warning


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["real", "c2c", "rfft2", "pruned", "slab", "spectrum", "fir", "flow",
                                          "fft1d"],
                   default="real")
    p.add_argument("--fft-impl", default="stockham_r8", help="registry name (spectral.FFT_IMPLS)")
    p.add_argument("--columns", default="strided", help="rfft2 workload: strided or transpose")
    p.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                   help="slab workload on 2+ GPUs: row kernel stores into the peers' memory, or an NCCL all-to-all")
    p.add_argument("--layout", choices=["columns", "natural"], default="columns",
                   help="slab workload: leave the column slab (one exchange) or return natural rows (two)")
    p.add_argument("--rounds", type=int, default=0,
                   help="timed rounds of K steps (0: enough for ~40 ms of timed work, at least 5)")
    p.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    p.add_argument("--sweep", action="store_true",
                   help="time every operation x implementation x size at 2^24 points per call and write the "
                        "reference's CSV (spectral.benchmark) instead of the JSON line")
    p.add_argument("--sweep-out", default="", help="--sweep: CSV path (default: standard output)")
    p.add_argument("--sweep-ops", default="all", help="--sweep: comma-separated operations, or all")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    p.add_argument("--method", choices=["auto", "fp32", "tensor"], default="auto",
                   help="pruned workload: the pruned transforms' row method (spectral_rfft2_modes_method); "
                        "auto is what spectral_rfft2_modes uses")
    return p.parse_args()


# --- workloads -----------------------------------------------------------------------------------
#
# Each workload describes one step on one GPU: the synthetic inputs (seeded, BASELINE.json's
# shapes and distributions), the launches of a step through the C ABI with their algorithmic
# bytes, the same step through the public torch API, and a CPU sample for the oracle.


class Real:
    """rfft then irfft, n = 4096, batch = 4096, float32 U[-1, 1]."""

    name = "rfft+irfft n=4096 batch=4096 f32 U[-1,1] (configs[1])"

    def __init__(self, impl: str, batch: int = 4096, n: int = 4096):
        self.impl, self.batch, self.n = impl, batch, n
        self.w = n // 2 + 1
        self.bytes_per_call = batch * (4 * n + 8 * self.w)  # 134,250,496 at the headline size

    def host_input(self, seed: int) -> np.ndarray:
        rng = np.random.default_rng(seed)
        return rng.uniform(-1.0, 1.0, (self.batch, self.n)).astype(np.float32)

    def device_sets(self, torch, seed: int):
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            s = torch.empty(self.batch, self.w, dtype=torch.complex64, device="cuda")
            y = torch.empty_like(x)
            sets.append((x, s, y))
        return sets

    def kernels(self) -> list[tuple[str, int]]:
        return [("rfft", self.bytes_per_call), ("irfft", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 2  # one fused kernel per direction

    def launch(self, native, sets, k: int, stream: int, which: int) -> None:
        x, s, _ = sets[k % SETS]
        _, s_old, y = sets[(k + 2) % SETS]
        imp = self.impl.encode()
        if which == 0:
            native.call("spectral_r2c", imp, x.data_ptr(), s.data_ptr(), self.n, self.batch, None, stream)
        else:
            native.call("spectral_c2r", imp, s_old.data_ptr(), y.data_ptr(), self.n, self.batch, None, stream)

    def api_step(self, spectral, x_dev):
        return spectral.irfft(spectral.rfft(x_dev, impl=self.impl), self.n, impl=self.impl)

    def io_bytes(self) -> tuple[int, int]:
        return self.batch * self.n * 4, self.batch * self.n * 4

    def cpu_step(self, ref, x: np.ndarray) -> None:
        ref.irfft(ref.rfft(x), self.n)

    def cpu_rows_bytes(self, rows: int) -> int:
        return 2 * rows * (4 * self.n + 8 * self.w)

    def parity(self, sets) -> dict:
        """Set 0 after the timed steps: its spectrum (rfft of x) and its y (irfft of that
        spectrum), on a sample of rows, against the oracle applied to the same inputs."""
        from oracle import reference as ref

        x, s, y = sets[0]
        rows = sample_rows(self.batch)
        xh, sh, yh = (t[rows].cpu().numpy() for t in (x, s, y))
        return parity_line(self.n, [("rfft", sh, ref.rfft(xh)), ("irfft", yh, ref.irfft(sh, self.n))],
                           len(rows))


class C2c:
    """fft_c2c forward then inverse, n = 1024, batch = 16384, complex64 N(0, 1)."""

    name = "fft_c2c fwd+inv n=1024 batch=16384 c64 N(0,1) (configs[0])"

    def __init__(self, impl: str, batch: int = 16384, n: int = 1024):
        self.impl, self.batch, self.n = impl, batch, n
        self.bytes_per_call = 16 * batch * n

    def host_input(self, seed: int) -> np.ndarray:
        rng = np.random.default_rng(seed)
        return (rng.standard_normal((self.batch, self.n)) + 1j * rng.standard_normal((self.batch, self.n))).astype(np.complex64)

    def device_sets(self, torch, seed: int):
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            sets.append((x, torch.empty_like(x), torch.empty_like(x)))
        return sets

    def kernels(self):
        return [("fft_fwd", self.bytes_per_call), ("fft_inv", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 2

    def launch(self, native, sets, k, stream, which):
        x, f, _ = sets[k % SETS]
        _, f_old, y = sets[(k + 2) % SETS]
        imp = self.impl.encode()
        if which == 0:
            native.call("spectral_c2c", imp, x.data_ptr(), f.data_ptr(), self.n, self.batch, 0, stream)
        else:
            native.call("spectral_c2c", imp, f_old.data_ptr(), y.data_ptr(), self.n, self.batch, 1, stream)

    def api_step(self, spectral, x_dev):
        return spectral.fft_c2c(spectral.fft_c2c(x_dev, impl=self.impl), inverse=True, impl=self.impl)

    def io_bytes(self):
        return self.batch * self.n * 8, self.batch * self.n * 8

    def cpu_step(self, ref, x):
        ref.ifft(ref.fft(x))

    def cpu_rows_bytes(self, rows):
        return 2 * 16 * rows * self.n

    def parity(self, sets) -> dict:
        from oracle import reference as ref

        x, f, y = sets[0]
        rows = sample_rows(self.batch)
        xh, fh, yh = (t[rows].cpu().numpy() for t in (x, f, y))
        return parity_line(self.n, [("fft", fh, ref.fft(xh)), ("ifft", yh, ref.ifft(fh))], len(rows))


class Rfft2:
    """rfft2 then irfft2 of 256 fields of 256 x 256 float32 N(0, 1)."""

    def __init__(self, impl: str, columns: str, batch: int = 256, n1: int = 256, n2: int = 256):
        self.impl, self.batch, self.n1, self.n2, self.columns = impl, batch, n1, n2, columns
        self.w = n2 // 2 + 1
        self.bytes_per_call = batch * (4 * n1 * n2 + 8 * n1 * self.w)
        self.name = f"rfft2+irfft2 256 x 256x256 f32 N(0,1) columns={columns} (configs[2])"
        self.method = 1 if columns == "strided" else 0

    def host_input(self, seed):
        rng = np.random.default_rng(seed)
        return rng.standard_normal((self.batch, self.n1, self.n2)).astype(np.float32)

    def device_sets(self, torch, seed):
        from spectral import native

        imp = self.impl.encode()
        wf = native.workspace("spectral_fft2_r2c_workspace", imp, self.method, self.n1, self.n2, self.batch)
        wi = native.workspace("spectral_fft2_c2r_workspace", imp, self.method, self.n1, self.n2, self.batch)
        self.work = torch.empty(max(wf, wi, 1), dtype=torch.complex64, device="cuda")
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            s = torch.empty(self.batch, self.n1, self.w, dtype=torch.complex64, device="cuda")
            sets.append((x, s, torch.empty_like(x)))
        return sets

    def kernels(self):
        return [("rfft2", self.bytes_per_call), ("irfft2", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 4 if self.method == 1 else 8  # rows + columns, or rows, transpose, rows, transpose

    def launch(self, native, sets, k, stream, which):
        x, s, _ = sets[k % SETS]
        _, s_old, y = sets[(k + 2) % SETS]
        imp = self.impl.encode()
        if which == 0:
            native.call("spectral_fft2_r2c", imp, self.method, x.data_ptr(), s.data_ptr(), self.n1,
                        self.n2, self.batch, self.work.data_ptr(), stream)
        else:
            native.call("spectral_fft2_c2r", imp, self.method, s_old.data_ptr(), y.data_ptr(), self.n1,
                        self.n2, self.batch, self.work.data_ptr(), stream)

    def api_step(self, spectral, x_dev):
        s = spectral.rfft2(x_dev, impl=self.impl, columns=self.columns)
        return spectral.irfft2(s, self.n2, impl=self.impl, columns=self.columns)

    def io_bytes(self):
        return self.batch * self.n1 * self.n2 * 4, self.batch * self.n1 * self.n2 * 4

    def cpu_step(self, ref, x):
        ref.irfft2(ref.rfft2(x), (self.n1, self.n2))

    def parity(self, sets) -> dict:
        from oracle import reference as ref

        x, s, y = sets[0]
        rows = sample_rows(self.batch, 16)
        xh, sh, yh = (t[rows].cpu().numpy() for t in (x, s, y))
        n = self.n1 * self.n2
        return parity_line(n, [("rfft2", sh, ref.rfft2(xh)), ("irfft2", yh, ref.irfft2(sh, (self.n1, self.n2)))],
                           len(rows), axes=(-2, -1))

    def cpu_rows_bytes(self, rows):
        return 2 * rows * (4 * self.n1 * self.n2 + 8 * self.n1 * self.w)


class Pruned:
    """the FNO layer, 64 samples x 64 channels of 128 x 128 float32 N(0, 1):
    rfft2_truncated (m1 = m2 = 16), per-mode contraction 64 -> 64 (W iid N(0, 1/4096) per part),
    irfft2_from_modes."""

    name = "FNO layer: rfft2_truncated + mode_contract + irfft2_from_modes, 64x64x128x128 f32 (configs[3])"

    METHODS = {"auto": 0, "fp32": 1, "tensor": 2}  # SPECTRAL_MODES_*

    def __init__(self, impl: str, samples: int = 64, channels: int = 64, n: int = 128, m: int = 16,
                 method: str = "auto"):
        self.impl, self.samples, self.channels, self.n, self.m = impl, samples, channels, n, m
        self.method = method
        self.fields = samples * channels
        self.bytes_per_call = self.fields * (4 * n * n + 16 * m * m)
        modes = 2 * m * m
        self.contract_bytes = 8 * modes * (2 * self.fields + channels * channels)

    def host_input(self, seed):
        rng = np.random.default_rng(seed)
        return rng.standard_normal((self.samples, self.channels, self.n, self.n)).astype(np.float32)

    def device_sets(self, torch, seed):
        from spectral import native

        rng = np.random.default_rng(seed + 100)
        shape = (self.channels, self.channels, 2 * self.m, self.m)
        wv = (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)) / 64.0
        self.weights = torch.from_numpy(wv.astype(np.complex64)).cuda()
        imp = self.impl.encode()
        a = native.workspace("spectral_rfft2_modes_workspace", imp, self.n, self.n, self.m, self.m, self.fields)
        b = native.workspace("spectral_irfft2_modes_workspace", imp, self.n, self.n, self.m, self.m, self.fields)
        self.work = torch.empty(max(a, b, 1), dtype=torch.complex64, device="cuda")
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            modes = torch.empty(self.samples, self.channels, 2 * self.m, self.m, dtype=torch.complex64, device="cuda")
            mixed = torch.empty_like(modes)
            sets.append((x, modes, mixed, torch.empty_like(x)))
        return sets

    def kernels(self):
        return [("rfft2_modes", self.bytes_per_call), ("mode_contract", self.contract_bytes),
                ("irfft2_modes", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 3  # the pruned forward, the contraction, the pruned inverse: one kernel each

    def launch(self, native, sets, k, stream, which):
        x, modes, mixed, _ = sets[k % SETS]
        _, _, mixed_old, y = sets[(k + 2) % SETS]
        imp = self.impl.encode()
        method = self.METHODS[self.method]
        if which == 0:
            native.call("spectral_rfft2_modes_method", imp, x.data_ptr(), modes.data_ptr(), self.n, self.n,
                        self.m, self.m, self.fields, method, self.work.data_ptr(), stream)
        elif which == 1:
            native.call("spectral_mode_contract", modes.data_ptr(), self.weights.data_ptr(),
                        mixed.data_ptr(), self.samples, self.channels, self.channels, 2 * self.m * self.m, stream)
        else:
            native.call("spectral_irfft2_modes_method", imp, mixed_old.data_ptr(), y.data_ptr(), self.n, self.n,
                        self.m, self.m, self.fields, method, self.work.data_ptr(), stream)

    def api_step(self, spectral, x_dev):
        modes = spectral.rfft2_truncated(x_dev, self.m, self.m, impl=self.impl)
        mixed = spectral.mode_contract(modes, self.weights)
        return spectral.irfft2_from_modes(mixed, (self.n, self.n), impl=self.impl)

    def io_bytes(self):
        return self.fields * self.n * self.n * 4, self.fields * self.n * self.n * 4

    def cpu_step(self, ref, x):
        modes = ref.rfft2_truncate(x, self.m, self.m)
        ref.irfft2_from_modes(modes, (self.n, self.n))

    def parity(self, sets) -> dict:
        """Set 0: its modes (rfft2_truncated of x), its contraction and its output (the inverse of
        the contraction), on a sample of samples, each stage against the oracle applied to that
        stage's own input."""
        from oracle import reference as ref
        from oracle.policy import relative_error

        x, modes, mixed, y = sets[0]
        rows = sample_rows(self.samples, 4)
        xh, mh, ch, yh = (t[rows].cpu().numpy() for t in (x, modes, mixed, y))
        n = self.n * self.n
        line = parity_line(n, [("rfft2_truncated", mh, ref.rfft2_truncate(xh, self.m, self.m)),
                               ("irfft2_from_modes", yh, ref.irfft2_from_modes(ch, (self.n, self.n)))],
                           len(rows), axes=(-2, -1))
        expected = ref.mode_contract(mh, self.weights.cpu().numpy())
        err = float(np.max(relative_error(ch.reshape(*ch.shape[:2], -1), expected.reshape(*ch.shape[:2], -1), (-1,))))
        ctol = 2 * float(np.finfo(np.float32).eps) * (math.log2(self.channels) + 1)
        line["stages"]["mode_contract"] = {"max_rel_err": err, "tol": ctol}
        line["ok"] = line["ok"] and err <= ctol
        return line

    def cpu_rows_bytes(self, rows):  # rows = samples
        return 2 * rows * self.channels * (4 * self.n * self.n + 16 * self.m * self.m)


class Spectrum:
    """The windowed spectrum (the reference's rf.spectrum): 16 complex64 signals of 2^20 N(0, 1)
    samples (2^24 points), frames of 1024 with the Hann window; one fused kernel (framing and
    window in the load). Bytes: 8 read + 8 written per sample."""

    name = "rf.spectrum nfft=1024 hann, 16 x 2^20 c64 N(0,1)"

    def __init__(self, impl: str, rows: int = 16, n: int = 1 << 20, nfft: int = 1024):
        self.impl, self.rows, self.n, self.nfft = impl, rows, n, nfft
        self.bytes_per_call = 16 * rows * n

    def host_input(self, seed):
        rng = np.random.default_rng(seed)
        shape = (self.rows, self.n)
        return ((rng.standard_normal(shape) + 1j * rng.standard_normal(shape)) / np.sqrt(2.0)).astype(np.complex64)

    def device_sets(self, torch, seed):
        from spectral import rf

        self.window = rf.window("hann", self.nfft, device="cuda")
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            sets.append((x, torch.empty(self.rows, self.n // self.nfft, self.nfft, dtype=torch.complex64, device="cuda")))
        return sets

    def kernels(self):
        return [("spectrum", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 1

    def launch(self, native, sets, k, stream, which):
        x, y = sets[k % SETS]
        native.call("spectral_spectrum", self.impl.encode(), x.data_ptr(), self.window.data_ptr(), y.data_ptr(),
                    self.n, self.nfft, self.rows, stream)

    def api_step(self, spectral, x_dev):
        from spectral import rf

        return rf.spectrum(x_dev, self.nfft, window_name="hann", fft_impl=self.impl)

    def io_bytes(self):
        return 8 * self.rows * self.n, 8 * self.rows * self.n

    def cpu_step(self, ref, x):
        from oracle import rf as orf

        orf.spectrum(x, self.nfft, "hann")

    def cpu_rows_bytes(self, rows):
        return 16 * rows * self.n


class Fir:
    """FIR filtering by overlap-save (the reference's rf.fir): 16 complex64 signals of 2^20 N(0, 1)
    samples (2^24 points), 255 real taps, blocks of 1024 (default_nfft); one fused kernel (both
    transforms and the product on chip). Bytes: 8 read + 8 written per sample (the overlap's
    re-read, 254 of every 1024 samples, is not counted)."""

    name = "rf.fir 255 taps nfft=1024 overlap-save, 16 x 2^20 c64 N(0,1)"

    def __init__(self, impl: str, rows: int = 16, n: int = 1 << 20, taps: int = 255):
        self.impl, self.rows, self.n, self.m = impl, rows, n, taps
        self.nfft = 1024
        self.bytes_per_call = 16 * rows * n

    host_input = Spectrum.host_input

    def device_sets(self, torch, seed):
        from spectral import rf

        rng = np.random.default_rng(seed + 100)
        self.taps = torch.from_numpy((rng.standard_normal(self.m) / np.sqrt(self.m)).astype(np.float32)).cuda()
        self.h = rf.taps_spectrum(self.taps, self.nfft, fft_impl=self.impl, device="cuda")
        sets = []
        for i in range(SETS):
            x = torch.from_numpy(self.host_input(seed + i)).cuda()
            sets.append((x, torch.empty_like(x)))
        return sets

    def kernels(self):
        return [("fir", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 1

    def launch(self, native, sets, k, stream, which):
        x, y = sets[k % SETS]
        native.call("spectral_fir", self.impl.encode(), x.data_ptr(), self.h.data_ptr(), y.data_ptr(),
                    self.n, self.nfft, self.m, self.rows, stream)

    def api_step(self, spectral, x_dev):
        from spectral import rf

        return rf.fir(x_dev, self.taps, nfft=self.nfft, fft_impl=self.impl)

    def io_bytes(self):
        return 8 * self.rows * self.n, 8 * self.rows * self.n

    def cpu_step(self, ref, x):
        from oracle import rf as orf

        rng = np.random.default_rng(1)
        orf.fir_overlap_save(x, rng.standard_normal(self.m) / np.sqrt(self.m), self.nfft)

    def cpu_rows_bytes(self, rows):
        return 16 * rows * self.n


class Slab:
    """one 16384 x 16384 complex64 field, N(0, 1) parts, slab-decomposed by rows over
    the ranks: row transforms, an NCCL all-to-all, column transforms (spectral.distributed).
    Strong scaling: the field is fixed, each rank holds n / R rows. Bytes: 16 per point of the
    field (the reference's convention), 4 GiB per transform."""

    def __init__(self, impl: str, n: int = 16384):
        self.impl, self.n = impl, n
        self.name = f"fft2 slab {n}x{n} c64 N(0,1), rows -> all-to-all -> columns (configs[4])"
        self.bytes_per_call = 16 * n * n

    def host_input(self, seed: int) -> np.ndarray:  # CPU sample: a few rows
        rng = np.random.default_rng(seed)
        rows = 64
        return (rng.standard_normal((rows, self.n)) + 1j * rng.standard_normal((rows, self.n))).astype(np.complex64)

    def kernels(self):
        return [("fft2_slab", self.bytes_per_call)]

    def launches_per_step(self) -> int:
        return 3 if self.n > 4096 else 2  # rows, then one or two column passes

    def cpu_step(self, ref, x):
        ref.fft(x)

    def cpu_rows_bytes(self, rows):
        return 16 * rows * self.n


def run_slab(args) -> None:
    """configs[4] on the process group: strong scaling of one 16384^2 transform."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from spectral import native
    from spectral.distributed import PeerSlab, fft2_slab

    wl = Slab(args.fft_impl)
    n = wl.n
    rows = n // world
    g = torch.Generator(device="cuda").manual_seed(4000 + rank)
    xs = [torch.complex(torch.randn(rows, n, device="cuda", generator=g),
                        torch.randn(rows, n, device="cuda", generator=g)) for _ in range(2)]
    stream = torch.cuda.current_stream()
    natural = args.layout == "natural"
    peer = PeerSlab(n, natural=natural) if world > 1 and args.exchange == "peer" else None
    if peer is not None:
        transform = peer.forward_natural if natural else peer.forward
    else:
        def transform(x):
            return fft2_slab(x, layout=args.layout)
    for k in range(args.warmup):
        transform(xs[k % 2])
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k in range(args.steps):
            transform(xs[k % 2])
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([start.elapsed_time(stop)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    faults = native.device_faults()
    if peer is not None:
        peer.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_source = hbm_peak()
    value = wl.bytes_per_call * args.steps / (max_ms * 1e-3) / 1e9
    step_s = max_ms / args.steps * 1e-3
    # The bound: two passes (rows, columns) over the rank's slab, each reading and writing it,
    # against the all-to-all's bytes leaving each GPU at the measured 770 GB/s per direction.
    # The natural layout adds a relayout pass and a second exchange.
    slab_bytes = 8 * n * n / world
    passes, exchanges = (3, 2) if args.layout == "natural" and world > 1 else (2, 1)
    hbm_s = passes * 2 * slab_bytes / (peak * 1e9)
    link_s = exchanges * slab_bytes * (world - 1) / world / 770e9
    bound_s = max(hbm_s, link_s)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": wl.name, "ranks": world, "rows_per_rank": rows, "layout": args.layout,
                   "exchange": ("none (1 rank)" if world == 1 else
                                "row kernel stores into the peers' buffers over NVLink (CUDA IPC), one all-reduce barrier"
                                if peer is not None else "torch.distributed all_to_all_single (NCCL)")},
        "roofline": {"bound": "hbm" if hbm_s >= link_s else "nvlink",
                     "achieved_step_ms": round(step_s * 1e3, 4), "bound_step_ms": round(bound_s * 1e3, 4),
                     "frac": round(bound_s / step_s, 4),
                     "note": "bound = max(2 passes x read+write of the 2 GiB/R slab at the measured HBM copy peak, "
                             "(R-1)/R of the slab over NVLink at 770 GB/s per direction)",
                     "hbm_peak_gbs": peak, "peak_source": peak_source},
        "cpu_baseline": None, "e2e": None, "gpu_launches": args.steps * wl.launches_per_step(),
        "clocks": clocks.summary(), "device_faults": faults, "impl": "ours",
    }
    print(json.dumps(line), flush=True)


# --- the Navier-Stokes consumer ------------------------------------------------------------------

FLOW_METRIC = "Navier-Stokes solver trajectory-steps/s, n=128 pruned, batch 256 (throughput.json)"
FLOW_UNIT = "trajectory-steps/s"
FLOW_PUBLISHED = 108682.0  # the reference's docs/results/throughput.json, stockham_r8 pruned, RTX 5080 Laptop


def flow_setup(batch: int, n: int, seed: int):
    """The throughput configuration of the reference's dataset params: n = 128, dt = 0.0025,
    viscosity U[1e-3, 5e-3] per trajectory, drag 0.1, Kolmogorov forcing A = 1, k_f = 4; initial
    vorticity smooth random fields of rms 5."""
    rng = np.random.default_rng(seed)
    nus = rng.uniform(1e-3, 5e-3, batch)
    kx = np.arange(n // 2 + 1)[None, :]
    k = np.arange(n)
    ky = np.where(k < n // 2, k, k - n)[:, None]
    spec = np.fft.rfft2(rng.standard_normal((batch, n, n))) * np.exp(-(kx**2 + ky**2) / 18.0)
    spec[..., 0, 0] = 0
    w0 = np.fft.irfft2(spec, s=(n, n))
    w0 = (5.0 * w0 / w0.std(axis=(-2, -1), keepdims=True)).astype(np.float32)
    return nus, w0


def run_flow(args) -> None:
    import torch

    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "unavailable": "no CUDA device visible"}))
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from spectral.flow import Flow
    from spectral.flow.gpu import GpuSolver

    batch, n, dt = 256, 128, 0.0025
    nus, w0 = flow_setup(batch, n, seed=1000 * rank + 1)
    solver = GpuSolver(n, Flow(viscosity=nus, drag=0.1), dt, fft_impl=args.fft_impl, pruned=True)
    w_hat = solver.to_spectral(torch.from_numpy(w0).cuda())
    graph, state = solver._graph(w_hat)
    state.copy_(w_hat)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    # Timed: K steps, each its own event pair, with a write of 2x the L2 between steps (outside
    # the events), so every step starts from HBM like a step of a long run with other work.
    flush = torch.empty(2 * 126 * 2**20 // 4, dtype=torch.float32, device="cuda")
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        for a, b in events:
            flush.fill_(1.0)
            a.record(stream)
            graph.replay()
            b.record(stream)
        torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in events]
    total_ms = sum(step_ms)
    # Back to back (the solver's own loop): no flush between steps.
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    s1.record(stream)
    torch.cuda.synchronize()
    b2b_ms = s0.elapsed_time(s1)
    t = torch.tensor([total_ms, b2b_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, b2b_ms = (float(v) for v in t.tolist())
    value = world * batch * args.steps / (total_ms * 1e-3)

    # Roofline of one stage (the step is two): the three fused kernels against HBM, with the
    # bytes they move through global memory (the Y and Z intermediates included, though at this
    # size they stay in the L2), timed alone with events.
    roofline = None
    if solver.fused:
        m = solver.spectral.m
        f0 = torch.empty_like(state)
        scratch = torch.empty_like(state)
        reps = 50
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        solver._stage(state, state, f0, scratch, 0)
        k0.record(stream)
        for _ in range(reps):
            solver._stage(state, state, f0, scratch, 0)
        k1.record(stream)
        torch.cuda.synchronize()
        stage_ms = k0.elapsed_time(k1) / reps
        plane = 2 * m * m * 8  # bytes of one state
        inter = n * m * 8      # bytes of one field's column-transformed intermediate
        stage_bytes = batch * (plane + 4 * inter        # derive: the state in, Y out
                               + 4 * inter + inter      # product: Y in, Z out
                               + inter + 3 * plane)     # update: Z and the state in, f0 and out
        peak, peak_source = hbm_peak()
        achieved = stage_bytes / (stage_ms * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": ncu_traffic("flow_stage", "flow"),
                    "kernel": "flow_stage", "kernels": "derive columns + product rows + update columns",
                    "peak_source": f"{peak_source} (MEASURED_PEAKS.json hbm_gbs, copy)",
                    "per_launch_us": round(1000 * stage_ms, 2), "bytes_per_launch": stage_bytes,
                    "note": "latency/FP32-bound: the intermediates are L2-resident at this size"}

    # End to end through the public API: pinned host vorticity in, to_spectral, 40 steps (one
    # recorded frame of the reference's dataset params), to_physical, the frame back to the host.
    e2e = None
    if not args.no_e2e:
        host_in = torch.from_numpy(w0).pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()
        record_every = 40

        def interval():
            frames = solver.frames(host_in.cuda(non_blocking=True), record_every, record_every)
            next(frames)
            host_out.copy_(next(frames), non_blocking=True)

        interval()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps_e = 5
        e0.record(stream)
        for _ in range(reps_e):
            interval()
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / reps_e
        e2e = {"value": round(world * batch * record_every / (e_ms * 1e-3), 1), "unit": FLOW_UNIT,
               "h2d_bytes_per_step": host_in.numel() * 4, "d2h_bytes_per_step": host_out.numel() * 4,
               "steps": reps_e, "path": "GpuSolver.frames: host vorticity in, 40 steps, frame out",
               "step": "one recorded frame interval (40 solver steps) of the reference's dataset params"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = flow_cpu(threads=os.cpu_count() or 1, trajectories=8, steps=4)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": FLOW_METRIC, "value": round(value, 1), "unit": FLOW_UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / world / FLOW_PUBLISHED, 2),
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "Navier-Stokes GpuSolver.step, 256 trajectories of 128x128, pruned (m=43), dt=0.0025, "
                               "nu U[1e-3,5e-3], drag 0.1, Kolmogorov k_f=4", "fft_impl": args.fft_impl,
                   "graph": "one CUDA graph per step", "l2": "2x L2 written between timed steps (outside the events)",
                   "back_to_back_trajectory_steps_per_s": round(world * batch * args.steps / (b2b_ms * 1e-3), 1),
                   "published_baseline": "108,682 trajectory-steps/s, stockham_r8 pruned, RTX 5080 Laptop GPU"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        # Per step: two stages of three fused kernels (the composed path is not counted).
        "gpu_launches": args.steps * 6 if solver.fused else None, "clocks": clocks.summary(), "impl": "ours",
    }
    print(json.dumps(line), flush=True)


def flow_cpu(threads: int, trajectories: int, steps: int) -> dict:
    """The reference's CPU solver (its float64 numpy flow/reference.py, restated as oracle/flow.py)
    on `trajectories` of the workload's trajectories for `steps` steps, spread over `threads`."""
    from oracle import flow as oflow

    nus, w0 = flow_setup(trajectories, 128, seed=5)
    chunks = [np.arange(trajectories)[i::threads] for i in range(min(threads, trajectories))]

    def work(idx):
        solver = oflow.Solver(128, 0.0025, viscosity=nus[idx], drag=0.1)
        w = oflow.to_spectral(w0[idx], 128)
        for _ in range(steps):
            w = solver.step(w)

    with ThreadPoolExecutor(max_workers=len(chunks)) as pool:
        list(pool.map(work, chunks))  # warm-up
        t0 = time.perf_counter()
        list(pool.map(work, chunks))
        t = time.perf_counter() - t0
    return {"value": round(trajectories * steps / t, 2), "unit": FLOW_UNIT, "cores": len(chunks), "kind": "port",
            "sample": f"{trajectories} trajectories x {steps} steps of the workload, float64 numpy solver"}


def run_flow_reference(args) -> None:
    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = os.cpu_count() or 1
    per = []
    for _ in range(max(1, args.steps)):
        per.append(flow_cpu(threads, trajectories=min(64, 2 * threads), steps=2)["value"])
    value = statistics.median(per)
    line = {"impl": "reference", "metric": FLOW_METRIC, "value": value, "unit": FLOW_UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": "Navier-Stokes step, 128x128, the reference's float64 numpy solver"},
            "cpu_baseline": {"value": value, "unit": FLOW_UNIT, "cores": threads, "kind": "port",
                             "sample": "min(64, 2 x cores) trajectories x 2 steps per measurement"},
            "e2e": {"value": value, "unit": FLOW_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_fft1d(args) -> None:
    """One 2^24-point complex signal held by the ranks in contiguous chunks, transformed by
    spectral.distributed.fft_slab (four-step over the ranks, three all-to-alls): strong scaling.
    Bytes: 16 per point of the signal (the reference's convention), 256 MiB per transform."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    from spectral.distributed import fft_slab

    n = 1 << 24
    chunk = n // world
    g = torch.Generator(device="cuda").manual_seed(6000 + rank)
    xs = [torch.complex(torch.randn(chunk, device="cuda", generator=g), torch.randn(chunk, device="cuda", generator=g))
          for _ in range(2)]
    stream = torch.cuda.current_stream()
    for k in range(args.warmup):
        fft_slab(xs[k % 2])
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k in range(args.steps):
            fft_slab(xs[k % 2])
        stop.record(stream)
        torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(stop)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
    if rank != 0:
        return
    max_ms = float(t.item())
    peak, peak_source = hbm_peak()
    value = 16 * n * args.steps / (max_ms * 1e-3) / 1e9
    # Bound: about six passes over the rank's chunk (pack, columns, unpack, rows, pack, transpose),
    # each reading and writing it, against three exchanges of (R-1)/R of it over NVLink.
    chunk_bytes = 8 * n / world
    hbm_s = 6 * 2 * chunk_bytes / (peak * 1e9)
    link_s = 3 * chunk_bytes * (world - 1) / world / 770e9
    bound_s = max(hbm_s, link_s)
    step_s = max_ms / args.steps * 1e-3
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "1D c64 transform of one 2^24-point signal in contiguous chunks over the ranks "
                               "(spectral.distributed.fft_slab)", "ranks": world},
        "roofline": {"bound": "hbm" if hbm_s >= link_s else "nvlink", "achieved_s": round(step_s, 6),
                     "bound_s": round(bound_s, 6), "frac": round(bound_s / step_s, 4),
                     "peak_source": f"{peak_source} HBM {peak} GB/s; NVLink 770 GB/s per direction (measured)"},
        # Per transform: relayout, twiddled columns, relayout, rows, relayout, transpose (the
        # all-to-alls are NCCL's).
        "cpu_baseline": None, "e2e": None, "gpu_launches": args.steps * 6, "clocks": clocks.summary(), "impl": "ours",
    }
    print(json.dumps(line), flush=True)


def make_workload(args):
    if args.workload == "real":
        return Real(args.fft_impl)
    if args.workload == "c2c":
        return C2c(args.fft_impl)
    if args.workload == "rfft2":
        return Rfft2(args.fft_impl, args.columns)
    if args.workload == "slab":
        return Slab(args.fft_impl)
    if args.workload == "spectrum":
        return Spectrum(args.fft_impl)
    if args.workload == "fir":
        return Fir(args.fft_impl)
    if args.workload == "fft1d":  # the reference arm: one 2^24-point transform and its inverse
        wl = C2c(args.fft_impl, batch=1, n=1 << 24)
        wl.name = "fft_c2c fwd+inv of one 2^24-point c64 signal"
        return wl
    return Pruned(args.fft_impl, method=args.method)


# --- parity of the timed outputs ------------------------------------------------------------------


def sample_rows(count: int, want: int = 64) -> list[int]:
    """`want` indices spread evenly over `count` rows (first and last included)."""
    if count <= want:
        return list(range(count))
    return sorted({round(i * (count - 1) / (want - 1)) for i in range(want)})


def parity_line(n: int, stages, rows: int, axes=(-1,)) -> dict:
    """Worst relative L2 error per transform of each stage against the oracle, with the
    tolerance 2 eps log2 N of oracle/policy.py."""
    from oracle.policy import fft_tolerance, relative_error

    tol = fft_tolerance(n)
    out = {}
    for name, actual, expected in stages:
        out[name] = {"max_rel_err": float(np.max(relative_error(actual, expected, axes))), "tol": tol}
    worst = max(v["max_rel_err"] for v in out.values())
    return {"max_rel_err": worst, "tol": tol, "rows": rows, "ok": all(v["max_rel_err"] <= v["tol"] for v in out.values()),
            "stages": out, "checked": "the timed steps' outputs of buffer set 0 against the float64 oracle"}


# --- peaks, clocks, profiles ---------------------------------------------------------------------


def hbm_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return 6650.0, "fallback"


def ncu_traffic(kernel: str, workload: str) -> float | None:
    """DRAM bytes per launch of `kernel` from a committed ncu summary, or None. The summaries
    under profiles/ carry a line `traffic <workload> <kernel> <bytes per launch>`."""
    for path in sorted((ROOT / "profiles").glob("*.md")):
        for line in path.read_text().splitlines():
            parts = line.strip().strip("`").split()
            if len(parts) == 4 and parts[0] == "traffic" and parts[1] == workload and parts[2] == kernel:
                try:
                    return float(parts[3])
                except ValueError:
                    return None
    return None


def size_matched_copy(nbytes: int, stream) -> float:
    """GB/s of a plain device-to-device copy (torch copy_) whose read + write traffic is `nbytes`,
    the dominant kernel's algorithmic bytes per launch: 4 rotating buffer pairs, 20 back-to-back
    copies per round, the median of 7 rounds after 6 warm-up copies. Copy bandwidth grows with
    the size of the copy (the measured peak is a 4 GB copy), so this is the ceiling for a kernel
    that moves this many bytes per launch."""
    import torch

    n = max(1, nbytes // 8)  # float32 elements per buffer: n * 4 bytes read and written
    pairs = [(torch.empty(n, device="cuda").fill_(1.0), torch.empty(n, device="cuda")) for _ in range(4)]
    with torch.cuda.stream(stream):
        for k in range(6):
            pairs[k % 4][1].copy_(pairs[k % 4][0])
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        ev[0].record(stream)
        for r in range(7):
            for k in range(20):
                pairs[k % 4][1].copy_(pairs[k % 4][0])
            ev[r + 1].record(stream)
    ev[-1].synchronize()
    ms = statistics.median(a.elapsed_time(b) / 20 for a, b in zip(ev, ev[1:]))
    del pairs
    return 8 * n / (ms * 1e-3) / 1e9


def fp32_ceiling(native, stream) -> float:
    """The GPU's FP32 ceiling in TFLOP/s: the faster of the scalar-FFMA and packed-FFMA2 forms of
    spectral_fp32_ceiling, each the median of 5 timed launches after 2 warm-up launches."""
    import ctypes

    import torch

    sink = torch.zeros(1, dtype=torch.float32, device="cuda")
    best = 0.0
    for packed in (0, 1):
        flops = ctypes.c_double(0.0)
        times = []
        for i in range(7):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            native.call("spectral_fp32_ceiling", sink.data_ptr(), 2048, packed, stream.cuda_stream,
                        ctypes.byref(flops))
            b.record(stream)
            b.synchronize()
            if i >= 2:
                times.append(a.elapsed_time(b))
        best = max(best, flops.value / (statistics.median(times) * 1e-3) / 1e12)
    return best


class ClockSampler:
    """Samples one GPU's SM clock and clock-event (throttle) reasons through NVML, every
    millisecond on a background thread, while the timed steps run. A timed region of a few
    milliseconds still gets samples; nvidia-smi's -lms loop could not flush a pipe that short."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        self._nvml = pynvml
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            self._handle = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)

    def sample(self) -> None:
        if self._handle is None:
            return
        n = self._nvml
        try:
            mhz = n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM)
            reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
        except Exception:
            return
        self.samples.append((mhz, reasons))

    def _loop(self) -> None:
        while not self._stop.wait(0.001):
            self.sample()

    def __enter__(self):
        try:
            self._open()
        except Exception:
            self._handle = None
            return self
        self.sample()
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()
        if self._nvml is not None:
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self) -> dict | None:
        if not self.samples:
            return None
        sm = [m for m, _ in self.samples]
        reasons = set()
        for name, const, bit in self.REASONS:
            mask = getattr(self._nvml, const, bit)
            if any(r & mask for _, r in self.samples):
                reasons.add(name)
        loaded = [m for m in sm if m > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": "NVML, 1 ms"}


# --- CPU legs ------------------------------------------------------------------------------------


def cpu_time(wl, rows: int, threads: int, reps: int) -> tuple[float, int]:
    """Seconds per pass of the oracle over `rows` rows (fields, samples) split over `threads`
    threads (pocketfft releases the GIL), best of `reps`; and the bytes of one pass."""
    from oracle import reference as ref

    x = wl.host_input(12345)[:rows]
    shards = np.array_split(x, threads)
    best = math.inf
    with ThreadPoolExecutor(max_workers=threads) as pool:
        for _ in range(reps):
            t0 = time.perf_counter()
            list(pool.map(lambda s: wl.cpu_step(ref, s), shards))
            best = min(best, time.perf_counter() - t0)
    return best, wl.cpu_rows_bytes(rows)


def cpu_sample_rows(wl) -> int:
    if isinstance(wl, (Pruned, Spectrum, Fir)):
        return 4
    if isinstance(wl, Rfft2):
        return 64
    return min(1024, getattr(wl, "batch", 1024))  # never more rows than the workload has


def run_reference(args) -> None:
    """The reference arm: the reference's CPU implementation of the path (float64 numpy
    pocketfft, restated as oracle/reference.py) on every host core, same workload and metric."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = make_workload(args)
    threads = os.cpu_count() or 1
    rows = cpu_sample_rows(wl)
    for _ in range(max(0, args.warmup)):
        cpu_time(wl, rows, threads, 1)
    per_step = []
    for _ in range(args.steps):
        t, nbytes = cpu_time(wl, rows, threads, 1)
        per_step.append(t)
    t = statistics.median(per_step)
    value = nbytes / t / 1e9
    sample = f"{rows} of the workload's rows per step ({nbytes / 2**20:.0f} MiB of algorithmic bytes), median of {args.steps} steps"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * t, 3), "higher_is_better": True,
        "scaling": "strong" if args.workload in ("slab", "fft1d") else "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": wl.name, "path": "numpy.fft (pocketfft) float64, the reference's python/spectral/reference.py"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --- our arm -------------------------------------------------------------------------------------


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "unavailable": "no CUDA device visible"}))
        return
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    import spectral
    from spectral import native

    wl = make_workload(args)
    peak, peak_source = hbm_peak()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    sets = wl.device_sets(torch, seed=1000 * rank + 1)
    kernels = wl.kernels()

    def step(k: int, events=None) -> None:
        for which in range(len(kernels)):
            if events is not None:
                events[k][which].record(stream)
            wl.launch(native, sets, k, sp, which)
        if events is not None:
            events[k][len(kernels)].record(stream)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()

    # Rounds: the K timed steps are measured as a round, repeated back to back (the reference's
    # protocol: median of rounds, min and max beside it, a warning above 5 % spread; its
    # csrc/common/bench.cpp:48-81). Enough rounds run for the clock sampler to see the GPU
    # under load at least ~20 times (about 40 ms of timed work), and at least 5. Every rank runs
    # the same number of rounds; each round's time is the slowest rank's.
    probe = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    probe[0].record(stream)
    for k in range(args.steps):
        step(k)
    probe[1].record(stream)
    torch.cuda.synchronize()
    est_round_ms = max(probe[0].elapsed_time(probe[1]), 1e-3)
    rounds = int(min(MAX_ROUNDS, max(MIN_ROUNDS, math.ceil(ROUND_TARGET_MS / est_round_ms))))
    if args.rounds > 0:
        rounds = args.rounds
    if world > 1:
        r = torch.tensor([rounds], dtype=torch.int64, device="cuda")
        dist.all_reduce(r, op=dist.ReduceOp.MAX)
        rounds = int(r.item())
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(rounds + 1)]

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # The timed region holds the steps alone: an event recorded between two kernels costs a few
    # microseconds of its own (it breaks the back-to-back launch of the next kernel), so events
    # sit only between rounds.
    with ClockSampler(local) as clocks:
        marks[0].record(stream)
        for r in range(rounds):
            for k in range(args.steps):
                step(r * args.steps + k)
            marks[r + 1].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    round_ms = torch.tensor([marks[r].elapsed_time(marks[r + 1]) for r in range(rounds)],
                            dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(round_ms, op=dist.ReduceOp.MAX)
    round_ms = round_ms.cpu().tolist()
    max_ms = statistics.median(round_ms)  # the median round, slowest rank per round
    spread = (max(round_ms) - min(round_ms)) / max_ms
    if spread > SPREAD_WARN and rank == 0:
        print(f"warning: rounds spread {100 * spread:.1f} % (min {min(round_ms):.4f} ms, max "
              f"{max(round_ms):.4f} ms per {args.steps} steps)", file=sys.stderr)

    # Per-kernel times for the roofline, from a separate pass with an event around every launch.
    pk = min(args.steps, 100)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(kernels) + 1)] for _ in range(pk)]
    for k in range(pk):
        step(k, ev)
    torch.cuda.synchronize()
    per_kernel_ms = [statistics.mean(ev[k][j].elapsed_time(ev[k][j + 1]) for k in range(pk))
                     for j in range(len(kernels))]
    bytes_per_step = sum(b for _, b in kernels)
    value = world * bytes_per_step * args.steps / (max_ms * 1e-3) / 1e9
    timing = {"rounds": rounds, "steps_per_round": args.steps, "statistic": "median round",
              "round_ms_median": round(max_ms, 5), "round_ms_min": round(min(round_ms), 5),
              "round_ms_max": round(max(round_ms), 5), "spread": round(spread, 4),
              "spread_warning": spread > SPREAD_WARN,
              "value_min": round(world * bytes_per_step * args.steps / (max(round_ms) * 1e-3) / 1e9, 3),
              "value_max": round(world * bytes_per_step * args.steps / (min(round_ms) * 1e-3) / 1e9, 3)}

    # The dominant kernel: the largest share of device time. Its average launch duration inside
    # the timed region is the region's time per step times its share, the shares taken from the
    # event-bracketed pass (an event between two launches costs each a few microseconds, so the
    # bracketed durations themselves overstate every kernel's time; both are on the line).
    dom = max(range(len(kernels)), key=lambda j: per_kernel_ms[j])
    dom_name, dom_bytes = kernels[dom]
    step_ms = max_ms / args.steps
    in_step_ms = [step_ms * ms / sum(per_kernel_ms) for ms in per_kernel_ms]
    achieved = dom_bytes / (in_step_ms[dom] * 1e-3) / 1e9
    traffic = ncu_traffic(dom_name, args.workload)
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": dom_name,
                "peak_source": f"{peak_source} (MEASURED_PEAKS.json hbm_gbs, copy)",
                "per_kernel_in_step_us": {n: round(1000 * ms, 2) for (n, _), ms in zip(kernels, in_step_ms)},
                "per_kernel_us": {n: round(1000 * ms, 2) for (n, _), ms in zip(kernels, per_kernel_ms)},
                "per_kernel_note": "per_kernel_us: each launch bracketed by its own events (a separate pass)"}
    copy_gbs = size_matched_copy(dom_bytes, stream)
    roofline["size_matched_copy"] = {
        "gbs": round(copy_gbs, 1), "frac": round(achieved / copy_gbs, 4),
        "how": "torch copy_ moving the dominant kernel's bytes per launch (read + write), 4 rotating "
               "buffer pairs, median of 7 rounds of 20 back-to-back copies; measured in this run"}

    # End to end through the public torch API: host -> device, the step, device -> host.
    e2e = None
    if not args.no_e2e:
        h2d, d2h = wl.io_bytes()
        hosts = [torch.from_numpy(wl.host_input(7000 + i)).pin_memory() for i in range(2)]
        outs = [torch.empty_like(h).pin_memory() for h in hosts]
        # Two streams, steps alternating between them, as a user pipelines a stream of batches:
        # step k + 1's host -> device copy runs beside step k's transforms and device -> host copy
        # (PCIe is full duplex). Every step still copies its input in and its result out.
        lanes = [torch.cuda.Stream(), torch.cuda.Stream()]

        def e2e_step(k: int) -> None:
            with torch.cuda.stream(lanes[k % 2]):
                result = wl.api_step(spectral, hosts[k % 2].cuda(non_blocking=True))
                outs[k % 2].view(result.shape).copy_(result, non_blocking=True)

        for k in range(4):
            e2e_step(k)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e_start = torch.cuda.Event(enable_timing=True)
        e_stop = torch.cuda.Event(enable_timing=True)
        e_steps = max(3, min(args.steps, 20))
        e_start.record(stream)
        for lane in lanes:
            lane.wait_event(e_start)
        for k in range(e_steps):
            e2e_step(k)
        for lane in lanes:
            stream.wait_stream(lane)
        e_stop.record(stream)
        torch.cuda.synchronize()
        et = torch.tensor([e_start.elapsed_time(e_stop)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": round(world * bytes_per_step * e_steps / (float(et.item()) * 1e-3) / 1e9, 3),
               "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "steps": e_steps, "path": "spectral.* torch ops -> C ABI, pinned host buffers",
               "pipeline": "2 streams, steps alternating: copies of neighbouring steps overlap"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        rows = cpu_sample_rows(wl)
        cpu_time(wl, rows, threads, 1)
        t_cpu, nbytes = cpu_time(wl, rows, threads, 3)
        # numpy's FFT is single-threaded: one core is the reference's CPU path as a user runs it.
        rows1 = max(1, rows // max(1, threads))
        t_one, bytes_one = cpu_time(wl, rows1, 1, 3)
        cpu = {"value": round(nbytes / t_cpu / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"oracle (numpy pocketfft float64) on {rows} rows of the workload, best of 3, {threads} threads",
               "one_core": {"value": round(bytes_one / t_one / 1e9, 3), "unit": UNIT,
                            "sample": f"{rows1} rows, best of 3, 1 thread"}}

    # The outputs the timed steps left in buffer set 0, against the oracle on a row sample (rank
    # 0; every rank's kernels are the same).
    parity = wl.parity(sets) if rank == 0 and hasattr(wl, "parity") else None
    if parity is not None and not parity["ok"]:
        print(f"error: timed outputs outside tolerance: {json.dumps(parity)}", file=sys.stderr)

    # The contraction runs on the tensor cores (split TF32) where its shape fits: its own line
    # gives its time against the HBM floor of its bytes, and its useful FLOP rate against the
    # measured FP32 ceiling (spectral_fp32_ceiling), the rate an FP32 kernel could at most reach.
    contraction = None
    if isinstance(wl, Pruned):
        ceiling = fp32_ceiling(native, stream)
        j = [n for n, _ in kernels].index("mode_contract")
        us = in_step_ms[j] * 1e3
        flops = 8.0 * wl.samples * wl.channels * wl.channels * 2 * wl.m * wl.m
        tf = flops / (us * 1e-6) / 1e12
        gbs = wl.contract_bytes / (us * 1e-6) / 1e9
        contraction = {"kernel": "mode_contract", "method": "tensor cores, split TF32 (tcgen05)",
                       "us_in_step": round(us, 2), "bytes": wl.contract_bytes,
                       "hbm": {"achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4)},
                       "useful_flops": flops, "useful_tflops": round(tf, 2),
                       "fp32_ceiling_tflops": round(ceiling, 2), "vs_fp32_ceiling": round(tf / ceiling, 4),
                       "fp32_ceiling_source": "measured in this run (spectral_fp32_ceiling)"}

    faults = native.device_faults()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": wl.name, "fft_impl": args.fft_impl, "points_per_gpu": 1 << 24,
                   "parallelism": f"batch-sharded x{world}, no communication",
                   "l2": "4 rotating buffer sets (6x L2); inverse reads a spectrum written 2 steps earlier",
                   "pct_hbm_peak": round(100 * value / world / peak, 2),
                   **({"pruned_method": args.method} if args.workload == "pruned" else {})},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": rounds * args.steps * wl.launches_per_step(),
        "clocks": clocks.summary(), "timing": timing, "parity": parity, "device_faults": faults,
        "impl": "ours",
    }
    if contraction is not None:
        line["contraction"] = contraction
    print(json.dumps(line), flush=True)

# --- the sweep: every operation x implementation x size ----------------------------------------

SWEEP_OPS = ("fft_c2c", "fft_r2c", "fft_c2r", "fft2_c2c", "fft2_r2c", "fft2_c2r", "rfft2_modes", "irfft2_modes",
             "scale")
SWEEP_POINTS = 1 << 24


def run_sweep(args) -> None:
    """The reference's spectral_bench sweep (its csrc/tools/spectral_bench.cpp:509-575) on this
    library: for each operation, implementation and power-of-two size 2 .. 4096 (2D: n x n
    arrays), batch = 2^24 / points per transform; time_cuda's median of 5 rounds of 20 calls, 4
    rotating buffer sets of 2^24 points each (twice the 126 MB L2 per set); one CSV row each,
    columns of spectral.benchmark. Rows whose rounds spread by more than 5 % are listed on
    standard error."""
    import torch

    import spectral
    from spectral import benchmark as bm
    from spectral import native

    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "unavailable": "no CUDA device visible"}))
        return
    ops = SWEEP_OPS if args.sweep_ops == "all" else tuple(args.sweep_ops.split(","))
    unknown = set(ops) - set(SWEEP_OPS)
    if unknown:
        raise SystemExit(f"--sweep-ops: unknown operations {sorted(unknown)}; choose from {SWEEP_OPS}")
    peak, peak_source = hbm_peak()
    stream = torch.cuda.current_stream().cuda_stream
    gen = torch.Generator(device="cuda").manual_seed(0)
    sets = [(torch.randn(SWEEP_POINTS, dtype=torch.complex64, device="cuda", generator=gen),
             torch.empty(SWEEP_POINTS + 4096, dtype=torch.complex64, device="cuda")) for _ in range(SETS)]
    work_holder = [torch.empty(1, dtype=torch.complex64, device="cuda")]

    def work_for(fn: str, *args) -> int:
        """A workspace of at least the size the library reports for this call (spectral_*_workspace):
        the library can check only that the pointer is not null, not the buffer's length."""
        need = native.workspace(fn, *args)
        if work_holder[0].numel() < need:
            work_holder[0] = torch.empty(need, dtype=torch.complex64, device="cuda")
        return work_holder[0].data_ptr()
    impls = [n for n in spectral.FFT_IMPLS]
    sizes = [1 << k for k in range(1, 13)]
    results = []

    def timed(op, impl, n, batch, flops_bytes, launch):
        try:
            t = bm.time_cuda(launch, arg_sets=[(x.data_ptr(), y.data_ptr()) for x, y in sets])
        except ValueError as e:  # the implementation does not take this shape
            print(f"skipped {op} {impl} n={n}: {e}", file=sys.stderr)
            return
        flops, nbytes = flops_bytes
        results.append(bm.Result(op, impl, n, batch, t, flops, nbytes))
        if t.spread > SPREAD_WARN:
            print(f"warning: {op} {impl} n={n} batch={batch}: rounds spread {100 * t.spread:.1f} %", file=sys.stderr)

    def limits(impl):
        import ctypes

        v = [ctypes.c_int(0) for _ in range(6)]
        native.call("spectral_impl_limits", impl.encode(), *[ctypes.byref(a) for a in v])
        return [a.value for a in v]  # max_n, max_c2c_n, max_real_n, has_columns, has_pruned, needs_work

    for op in ops:
        for impl in impls:
            imp = impl.encode()
            max_n, max_c2c, max_real, has_columns, _, _ = limits(impl)
            if op == "scale":
                if impl == impls[0]:
                    timed("scale", "ours", SWEEP_POINTS, 1, (2.0 * SWEEP_POINTS, 16.0 * SWEEP_POINTS),
                          lambda x, y: native.call("spectral_scale", x, y, SWEEP_POINTS, 0.5, stream))
                continue
            for n in sizes:
                if op == "fft_c2c" and n <= max_c2c:
                    for inv in (0,):
                        b = SWEEP_POINTS // n
                        timed(op, impl, n, b, bm.fft_c2c_work(n, b),
                              lambda x, y, n=n, b=b: native.call("spectral_c2c", imp, x, y, n, b, inv, stream))
                elif op in ("fft_r2c", "fft_c2r") and n <= max_real:
                    b = SWEEP_POINTS // n
                    fn = "spectral_r2c" if op == "fft_r2c" else "spectral_c2r"
                    wp = work_for("spectral_real_workspace", imp, n, b)
                    timed(op, impl, n, b, bm.fft_real_work(n, b),
                          lambda x, y, n=n, b=b, fn=fn, wp=wp: native.call(fn, imp, x, y, n, b, wp, stream))
                elif op.startswith("fft2_") and n <= max_n and n * n <= SWEEP_POINTS:
                    b = SWEEP_POINTS // (n * n)
                    for method, cname in ((1, "strided"), (0, "transpose")):
                        if method == 1 and not has_columns:
                            continue
                        name = f"{impl}/{cname}"
                        wp = work_for(f"spectral_{op}_workspace", imp, method, n, n, b)
                        if op == "fft2_c2c":
                            fb = bm.fft_c2c_work(n * n, b)
                            call = lambda x, y, n=n, b=b, m=method, wp=wp: native.call(
                                "spectral_fft2_c2c", imp, m, x, y, n, n, b, 0, wp, stream)
                        elif op == "fft2_r2c":
                            fb = bm.fft2_real_work(n, n, b)
                            call = lambda x, y, n=n, b=b, m=method, wp=wp: native.call(
                                "spectral_fft2_r2c", imp, m, x, y, n, n, b, wp, stream)
                        else:
                            fb = bm.fft2_real_work(n, n, b)
                            call = lambda x, y, n=n, b=b, m=method, wp=wp: native.call(
                                "spectral_fft2_c2r", imp, m, x, y, n, n, b, wp, stream)
                        timed(op, name, n, b, fb, call)
                elif op in ("rfft2_modes", "irfft2_modes") and 2 <= n <= max_n and n * n <= SWEEP_POINTS:
                    b = SWEEP_POINTS // (n * n)
                    m = max(1, n // 8)
                    fn = "spectral_rfft2_modes" if op == "rfft2_modes" else "spectral_irfft2_modes"
                    wp = work_for(f"{fn}_workspace", imp, n, n, m, m, b)
                    timed(op, impl, n, b, bm.pruned_work(n, n, m, m, b),
                          lambda x, y, n=n, b=b, m=m, fn=fn, wp=wp: native.call(fn, imp, x, y, n, n, m, m, b, wp, stream))
    prop = torch.cuda.get_device_properties(0)
    comments = [f"device: {prop.name}, {prop.multi_processor_count} SMs",
                f"torch {torch.__version__}, CUDA {torch.version.cuda}",
                "timing: 3 warm-up calls, then the median over 5 rounds of 20 calls (4 rotating buffer sets of "
                "2^24 points); times are per call",
                f"hbm peak {peak} GB/s ({peak_source}); batch = 2^24 / points per transform"]
    text = bm.format_csv(results, comments, gpus=1, hbm_peak_gbs=peak, peak_source=peak_source,
                         cpu_cores=os.cpu_count() or "")
    if args.sweep_out:
        Path(args.sweep_out).write_text(text)
        print(json.dumps({"sweep": args.sweep_out, "rows": len(results)}), flush=True)
    else:
        sys.stdout.write(text)


def main() -> None:
    args = parse()
    if args.sweep:
        run_sweep(args)
        return
    if args.workload == "flow":
        (run_flow_reference if args.impl == "reference" else run_flow)(args)
    elif args.workload == "fft1d" and args.impl == "ours":
        run_fft1d(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.workload == "slab":
        run_slab(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
