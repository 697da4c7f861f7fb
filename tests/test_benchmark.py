"""The benchmarking helpers: the bytes convention, comparison, CSV reading, and (on a GPU) that
time_cuda measures real kernel time (the reference's tests/test_benchmark.py)."""

import pytest
import torch

import spectral
from spectral.benchmark import (
    compare,
    fft2_real_work,
    fft_c2c_work,
    fft_real_work,
    format_csv,
    pruned_work,
    read_results,
    time_cuda,
)


def test_fft_work_follows_the_5_n_log2_n_convention():
    flops, nbytes = fft_c2c_work(1024, 3)
    assert flops == 5 * 1024 * 10 * 3
    assert nbytes == 16 * 1024 * 3


def test_real_fft_work_counts_both_sides():
    flops, nbytes = fft_real_work(1024, 3)
    assert flops == fft_c2c_work(1024, 3)[0] / 2
    assert nbytes == 3 * (4 * 1024 + 8 * 513)


def test_headline_configuration_bytes():
    # The figures the bench's roofline uses: 2^24 points per call.
    assert fft_c2c_work(1024, 16384)[1] == 268_435_456
    assert fft_real_work(4096, 4096)[1] == 134_250_496
    assert fft2_real_work(256, 256, 256)[1] == 134_742_016
    assert pruned_work(128, 128, 16, 16, 4096)[1] == 285_212_672


def test_compare_flags_only_changes_beyond_the_threshold():
    old = {("fft", "a", 64, 1): 1.0, ("fft", "b", 64, 1): 1.0, ("fft", "c", 64, 1): 1.0}
    new = {("fft", "a", 64, 1): 1.05, ("fft", "b", 64, 1): 1.2, ("fft", "c", 64, 1): 0.5}
    lines, regressed = compare(old, new, threshold=0.10)
    assert regressed
    assert [line.split()[1] for line in lines if "SLOWER" in line] == ["b"]
    assert [line.split()[1] for line in lines if "faster" in line] == ["c"]


def test_csv_round_trip(tmp_path):
    from spectral.benchmark import Result, Timing

    r = Result("fft_c2c", "stockham_r8", 1024, 16384, Timing(0.05, 0.049, 0.051), 1e9, 268435456)
    path = tmp_path / "bench.csv"
    path.write_text(format_csv([r], ["device: test"], hbm_peak_gbs=6543.4, peak_source="measured"))
    assert read_results(path) == {("fft_c2c", "stockham_r8", 1024, 16384): 0.05}
    assert ",82.0,measured," in path.read_text()  # 5368.7 GB/s of 6543.4


def test_time_cuda_rejects_a_bad_configuration():
    with pytest.raises(ValueError, match="rounds"):
        time_cuda(lambda: None, rounds=0)


@pytest.mark.gpu
def test_time_cuda_measures_real_kernel_time():
    x = torch.randn(1 << 24, dtype=torch.complex64, device="cuda")
    t = time_cuda(lambda: spectral.scale(x, 0.5))
    assert 0 < t.min_ms <= t.median_ms <= t.max_ms
    gbps = 16 * (1 << 24) / (t.median_ms * 1e6)
    assert 100 < gbps < 12000  # B200: a few TB/s; a timing bug reads as far more
