"""Timing GPU work from Python, the bytes-moved convention, and comparing result files.

The same helpers as the reference's python/spectral/benchmark.py (time_cuda, fft_c2c_work,
fft_real_work, format_csv, read_results, compare; benchmark.py:43-120 there), with two changes
for B200:

- time_cuda can rotate through several argument sets, so that no launch finds its input in
  the 126 MB L2 left behind by the previous one. The reference reuses one buffer pair, which on
  its 64 MB-L2 laptop part let its FFT rows report more than its own copy peak.
- The CSV gains the columns gpus, pct_hbm_peak, peak_source and cpu_cores.

Bytes follow the reference's convention (csrc/common/bench.cpp:93-136): 16 B per complex point
(read + write), 4 n + 8 (n/2 + 1) B per real row, 4 n1 n2 + 8 n1 (n2/2 + 1) B per real 2D field,
4 n1 n2 + 16 m1 m2 B per pruned field.
"""

from __future__ import annotations

import csv
import math
import statistics
from collections.abc import Callable, Iterable, Sequence
from dataclasses import dataclass
from pathlib import Path

CSV_COLUMNS = [
    "op", "impl", "n", "batch", "time_ms", "min_ms", "max_ms", "gflops", "gbps",
    "gpus", "pct_hbm_peak", "peak_source", "cpu_cores",
]

Key = tuple[str, str, int, int]  # (op, impl, n, batch)


@dataclass(frozen=True)
class Timing:
    median_ms: float  # all three per call
    min_ms: float
    max_ms: float

    @property
    def spread(self) -> float:
        """(max - min) / median: above 0.05 the rounds disagree enough to warn."""
        return (self.max_ms - self.min_ms) / self.median_ms if self.median_ms > 0 else 0.0


@dataclass(frozen=True)
class Result:
    op: str
    impl: str
    n: int
    batch: int
    timing: Timing
    flops: float
    nbytes: float


def time_cuda(
    fn: Callable[..., object],
    *,
    warmup: int = 3,
    rounds: int = 5,
    iters: int = 20,
    arg_sets: Sequence[tuple] | None = None,
) -> Timing:
    """Median, minimum and maximum time per call of `fn`, which must enqueue its GPU work on the
    current stream. With `arg_sets`, call i runs fn(*arg_sets[i % len(arg_sets)])."""
    import torch

    if warmup < 0 or rounds < 1 or iters < 1:
        raise ValueError("need warmup >= 0, rounds >= 1, iters >= 1")
    sets = list(arg_sets) if arg_sets else [()]
    calls = 0

    def step() -> None:
        nonlocal calls
        fn(*sets[calls % len(sets)])
        calls += 1

    for _ in range(warmup):
        step()
    stream = torch.cuda.current_stream()
    per_call = []
    for _ in range(rounds):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(iters):
            step()
        stop.record(stream)
        stop.synchronize()
        per_call.append(start.elapsed_time(stop) / iters)
    return Timing(statistics.median(per_call), min(per_call), max(per_call))


def fft_c2c_work(n: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` complex transforms of n points: 5 n log2 n flops per
    transform, 16 bytes per point."""
    points = n * batch
    return 5.0 * points * math.log2(n) if n > 1 else 0.0, 16.0 * points


def fft_real_work(n: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` real transforms of n points, either direction:
    2.5 n log2 n flops, n float32 plus n/2 + 1 complex64 values per row."""
    return 2.5 * n * batch * math.log2(n), batch * (4.0 * n + 8.0 * (n // 2 + 1))


def fft2_real_work(n1: int, n2: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` real 2D transforms of n1 x n2, either direction."""
    return (
        2.5 * n1 * n2 * batch * math.log2(n1 * n2),
        batch * (4.0 * n1 * n2 + 8.0 * n1 * (n2 // 2 + 1)),
    )


def pruned_work(n1: int, n2: int, m1: int, m2: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` pruned real 2D transforms keeping (2 m1) x m2 modes, either
    direction: the full transform's flops, 4 n1 n2 + 16 m1 m2 bytes per field."""
    return 2.5 * n1 * n2 * batch * math.log2(n1 * n2), batch * (4.0 * n1 * n2 + 16.0 * m1 * m2)


def format_csv(
    results: Iterable[Result],
    comments: Iterable[str],
    *,
    gpus: int = 1,
    hbm_peak_gbs: float | None = None,
    peak_source: str = "",
    cpu_cores: int | str = "",
) -> str:
    lines = [f"# {c}" for c in comments]
    lines.append(",".join(CSV_COLUMNS))
    for r in results:
        t = r.timing
        gbps = r.nbytes / (t.median_ms * 1e6)
        pct = f"{100.0 * gbps / hbm_peak_gbs:.1f}" if hbm_peak_gbs else ""
        lines.append(
            f"{r.op},{r.impl},{r.n},{r.batch},{t.median_ms:.6f},{t.min_ms:.6f},{t.max_ms:.6f},"
            f"{r.flops / (t.median_ms * 1e6):.1f},{gbps:.1f},{gpus},{pct},{peak_source},{cpu_cores}"
        )
    return "\n".join(lines) + "\n"


def read_results(path: Path) -> dict[Key, float]:
    """Median time in ms for each (op, impl, n, batch) of a results CSV; '#' lines skipped."""
    with Path(path).open(newline="") as f:
        lines = [line for line in f if not line.startswith("#")]
    return {
        (row["op"], row["impl"], int(row["n"]), int(row["batch"])): float(row["time_ms"])
        for row in csv.DictReader(lines)
    }


def compare(
    old: dict[Key, float], new: dict[Key, float], threshold: float
) -> tuple[list[str], bool]:
    """A report line per row, and whether any row present in both got slower than
    old * (1 + threshold). Rows in only one of them are listed and never fail."""
    lines = [f"{'op':<10} {'impl':<12} {'n':>7} {'batch':>9} {'old ms':>10} {'new ms':>10} ratio"]
    regressed = False
    for key in sorted(old.keys() & new.keys()):
        ratio = new[key] / old[key]
        flag = ""
        if ratio > 1 + threshold:
            flag, regressed = "  SLOWER", True
        elif ratio < 1 - threshold:
            flag = "  faster"
        op, impl, n, batch = key
        lines.append(
            f"{op:<10} {impl:<12} {n:>7} {batch:>9} {old[key]:>10.4f} {new[key]:>10.4f} "
            f"{ratio:5.2f}x{flag}"
        )
    lines += [f"only in old: {key}" for key in sorted(old.keys() - new.keys())]
    lines += [f"only in new: {key}" for key in sorted(new.keys() - old.keys())]
    return lines, regressed
