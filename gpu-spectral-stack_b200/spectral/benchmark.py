"""Benchmark helpers: device timing, the bytes-moved convention, and results files.

The public names are those of the reference's python/spectral/benchmark.py (time_cuda,
fft_c2c_work, fft_real_work, format_csv, read_results, compare, Timing, Result), so scripts
written against it keep working; the implementation here is this library's own.

Timing. time_cuda enqueues every timed round back to back on the current stream, with one CUDA
event between consecutive rounds, and synchronizes once at the end: the GPU never idles between
rounds waiting for the host. It reports the median, minimum and maximum time per call over the
rounds. With `arg_sets` the calls rotate through several argument tuples, so that on a GPU whose
L2 (126 MB on B200) holds a whole buffer set, no call finds its input left in L2 by the one
before it.

Work. Bytes follow the reference's convention (its csrc/common/bench.cpp:93-136): 16 bytes per
complex point (one read, one write), 4 n + 8 (n/2 + 1) bytes per real row, 4 n1 n2 + 8 n1
(n2/2 + 1) bytes per real 2D field, 4 n1 n2 + 16 m1 m2 bytes per pruned field; flops are
5 N log2 N per complex transform and half that for real ones.

Files. The CSV holds the reference's nine columns (op, impl, n, batch, time_ms, min_ms, max_ms,
gflops, gbps) followed by four of this library's (gpus, pct_hbm_peak, peak_source, cpu_cores);
lines starting with '#' are comments.
"""

from __future__ import annotations

import csv
import io
import math
import statistics
from collections.abc import Callable, Iterable, Iterator, Sequence
from dataclasses import dataclass
from pathlib import Path

REFERENCE_COLUMNS = ("op", "impl", "n", "batch", "time_ms", "min_ms", "max_ms", "gflops", "gbps")
CSV_COLUMNS = [*REFERENCE_COLUMNS, "gpus", "pct_hbm_peak", "peak_source", "cpu_cores"]

Key = tuple[str, str, int, int]  # (op, impl, n, batch)


@dataclass(frozen=True)
class Timing:
    """Milliseconds per call: the median round and the extreme rounds."""

    median_ms: float
    min_ms: float
    max_ms: float

    @property
    def spread(self) -> float:
        """(max - min) / median; above 0.05 the rounds disagree enough to warn about."""
        if self.median_ms <= 0:
            return 0.0
        return (self.max_ms - self.min_ms) / self.median_ms


@dataclass(frozen=True)
class Result:
    op: str
    impl: str
    n: int
    batch: int
    timing: Timing
    flops: float
    nbytes: float

    def gflops(self) -> float:
        return self.flops / (self.timing.median_ms * 1e6)

    def gbps(self) -> float:
        return self.nbytes / (self.timing.median_ms * 1e6)


def time_cuda(
    fn: Callable[..., object],
    *,
    warmup: int = 3,
    rounds: int = 5,
    iters: int = 20,
    arg_sets: Sequence[tuple] | None = None,
) -> Timing:
    """Time per call of `fn`, which must enqueue its GPU work on the current stream. Call k runs
    fn(*arg_sets[k % len(arg_sets)]) (fn() without arg_sets)."""
    import torch

    if warmup < 0 or rounds < 1 or iters < 1:
        raise ValueError("need warmup >= 0, rounds >= 1, iters >= 1")
    sets = list(arg_sets) if arg_sets else [()]
    calls = iter(range(warmup + rounds * iters))

    def call() -> None:
        fn(*sets[next(calls) % len(sets)])

    for _ in range(warmup):
        call()
    stream = torch.cuda.current_stream()
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(rounds + 1)]
    marks[0].record(stream)
    for r in range(rounds):
        for _ in range(iters):
            call()
        marks[r + 1].record(stream)
    marks[-1].synchronize()
    per_call = sorted(a.elapsed_time(b) / iters for a, b in zip(marks, marks[1:]))
    return Timing(statistics.median(per_call), per_call[0], per_call[-1])


def fft_c2c_work(n: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` complex transforms of n points."""
    points = n * batch
    return (5.0 * points * math.log2(n) if n > 1 else 0.0), 16.0 * points


def fft_real_work(n: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` real transforms of n points, either direction."""
    return 2.5 * n * batch * math.log2(n), batch * (4.0 * n + 8.0 * (n // 2 + 1))


def fft2_real_work(n1: int, n2: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` real 2D transforms of n1 x n2, either direction."""
    points = n1 * n2
    return 2.5 * points * batch * math.log2(points), batch * (4.0 * points + 8.0 * n1 * (n2 // 2 + 1))


def pruned_work(n1: int, n2: int, m1: int, m2: int, batch: int) -> tuple[float, float]:
    """(flops, bytes) of `batch` pruned real 2D transforms keeping (2 m1) x m2 modes, either
    direction: the full transform's flops; only the kept modes cross HBM on the complex side."""
    flops, _ = fft2_real_work(n1, n2, batch)
    return flops, batch * (4.0 * n1 * n2 + 16.0 * m1 * m2)


def _row(r: Result, gpus: int, hbm_peak_gbs: float | None, peak_source: str, cpu_cores) -> list[str]:
    t = r.timing
    gbps = r.gbps()
    pct = f"{100.0 * gbps / hbm_peak_gbs:.1f}" if hbm_peak_gbs else ""
    return [r.op, r.impl, str(r.n), str(r.batch), f"{t.median_ms:.6f}", f"{t.min_ms:.6f}", f"{t.max_ms:.6f}",
            f"{r.gflops():.1f}", f"{gbps:.1f}", str(gpus), pct, peak_source, str(cpu_cores)]


def format_csv(
    results: Iterable[Result],
    comments: Iterable[str],
    *,
    gpus: int = 1,
    hbm_peak_gbs: float | None = None,
    peak_source: str = "",
    cpu_cores: int | str = "",
) -> str:
    """The results as CSV text, comment lines first."""
    buf = io.StringIO()
    for c in comments:
        buf.write(f"# {c}\n")
    writer = csv.writer(buf, lineterminator="\n")
    writer.writerow(CSV_COLUMNS)
    writer.writerows(_row(r, gpus, hbm_peak_gbs, peak_source, cpu_cores) for r in results)
    return buf.getvalue()


def _data_lines(path: Path) -> Iterator[str]:
    with Path(path).open(newline="") as f:
        yield from (line for line in f if not line.lstrip().startswith("#"))


def read_results(path: Path) -> dict[Key, float]:
    """Median milliseconds per (op, impl, n, batch) of a results file (this library's or the
    reference's nine-column CSV)."""
    table: dict[Key, float] = {}
    for rec in csv.DictReader(_data_lines(path)):
        table[(rec["op"], rec["impl"], int(rec["n"]), int(rec["batch"]))] = float(rec["time_ms"])
    return table


def compare(old: dict[Key, float], new: dict[Key, float], threshold: float) -> tuple[list[str], bool]:
    """A report line per row and whether any row present in both files got slower than
    old (1 + threshold). Rows in only one file are listed and never count as a regression."""
    header = f"{'op':<12} {'impl':<22} {'n':>7} {'batch':>9} {'old ms':>10} {'new ms':>10} ratio"
    lines = [header]
    regressed = False
    for key in sorted(old.keys() & new.keys()):
        ratio = new[key] / old[key]
        verdict = "SLOWER" if ratio > 1 + threshold else "faster" if ratio < 1 - threshold else ""
        regressed = regressed or verdict == "SLOWER"
        op, impl, n, batch = key
        line = f"{op:<12} {impl:<22} {n:>7} {batch:>9} {old[key]:>10.4f} {new[key]:>10.4f} {ratio:5.2f}x"
        lines.append(f"{line}  {verdict}" if verdict else line)
    lines.extend(f"only in old: {key}" for key in sorted(old.keys() - new.keys()))
    lines.extend(f"only in new: {key}" for key in sorted(new.keys() - old.keys()))
    return lines, regressed
