"""Radio-signal consumers (spectral.rf): periodic windows, the framed spectrum and overlap-save FIR
filtering, against the float64 oracle (oracle/rf.py), which is pinned to the reference's own
rf.py outputs (tests/golden/rf_golden.npz) and to scipy. The reference's tests/test_rf.py is the
model: every GPU check runs with cuFFT and with each implementation; the fused kernels (the
stockham names) are additionally swept over every block size and checked for ragged inputs,
empty signals, rows, complex taps, the command line and the C ABI.

The reference's recorded test signals are not used; chirp, root-raised-cosine, BPSK and QPSK
signals of the same kind are synthesised here from seeds.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import scipy.signal
import torch

from oracle import rf as orf
from oracle.policy import fft_tolerance

GOLDEN = Path(__file__).resolve().parent / "golden" / "rf_golden.npz"
SIZES = [1 << k for k in range(1, 13)]


def relative_error(actual, expected) -> float:
    actual = np.asarray(actual, dtype=np.complex128)
    expected = np.asarray(expected, dtype=np.complex128)
    return float(np.linalg.norm(actual - expected) / max(np.linalg.norm(expected), 1e-30))


def random_complex(rng, shape) -> np.ndarray:
    z = rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return (z / np.sqrt(2.0)).astype(np.complex64)


@pytest.fixture(scope="module")
def golden():
    with np.load(GOLDEN) as g:
        return {k: g[k] for k in g.files}


# --- the oracle against the reference's outputs and scipy (CPU) --------------------------------


@pytest.mark.parametrize("name", orf.WINDOWS)
@pytest.mark.parametrize("n", [1, 2, 7, 64, 1024])
def test_oracle_windows_are_the_reference_windows(golden, name, n):
    np.testing.assert_array_equal(orf.window(name, n), golden[f"window_{name}_{n}"])


@pytest.mark.parametrize("name", ["hann", "hamming", "blackman"])
@pytest.mark.parametrize("n", [1, 2, 7, 64, 1024])
def test_oracle_windows_match_scipy_periodic_windows(name, n):
    expected = scipy.signal.get_window(name, n, fftbins=True)
    np.testing.assert_allclose(orf.window(name, n), expected, rtol=0, atol=1e-7)


def test_oracle_default_block_size_is_the_reference_one(golden):
    got = [orf.default_nfft(int(m)) for m in golden["default_nfft_taps"]]
    assert got == list(golden["default_nfft"])


def test_oracle_frames_and_spectrum_are_the_reference_ones(golden):
    for key in [k for k in golden if k.startswith("frames_") and k.endswith("_x")]:
        _, n, nfft, _ = key.split("_")
        x = golden[key]
        np.testing.assert_array_equal(orf.frames(x, int(nfft)), golden[key[:-1] + "y"])
        for name in ("rect", "hann", "blackman"):
            expected = golden[f"spectrum_{n}_{nfft}_{name}"]  # torch.fft in complex64
            assert relative_error(orf.spectrum(x, int(nfft), name), expected) < 1e-6


def test_oracle_fir_is_the_reference_fir(golden):
    cases = [k[:-2] for k in golden if k.startswith("fir_") and k.endswith("_x")]
    assert len(cases) == 7
    for tag in cases:
        y = orf.fir(golden[f"{tag}_x"], golden[f"{tag}_taps"])
        assert y.shape == golden[f"{tag}_y"].shape
        assert relative_error(y, golden[f"{tag}_y"]) < 1e-5, tag  # the reference's in complex64


@pytest.mark.parametrize(("n", "m"), [(1000, 1), (5, 63), (1000, 63), (4097, 64)])
def test_oracle_fir_is_lfilter(rng, n, m):
    x = random_complex(rng, (2, n))
    taps = rng.standard_normal(m)
    expected = scipy.signal.lfilter(taps, 1.0, x.astype(np.complex128), axis=-1)
    np.testing.assert_allclose(orf.fir(x, taps), expected, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize(("n", "m", "nfft"), [(1000, 63, None), (5, 63, None), (777, 31, 64), (4097, 64, None), (10, 1, 2)])
def test_oracle_overlap_save_is_the_direct_convolution(rng, n, m, nfft):
    x = random_complex(rng, (2, n))
    taps = random_complex(rng, m)
    np.testing.assert_allclose(orf.fir_overlap_save(x, taps, nfft), orf.fir(x, taps), rtol=0, atol=1e-11)


# --- host logic (CPU) ----------------------------------------------------------------------------


def test_windows_are_the_oracle_windows():
    from spectral import rf

    for name in orf.WINDOWS:
        for n in (1, 3, 256, 4096):
            np.testing.assert_array_equal(rf.window(name, n).numpy(), orf.window(name, n))


def test_default_block_size(golden):
    from spectral import rf

    assert [rf.default_nfft(int(m)) for m in golden["default_nfft_taps"]] == list(golden["default_nfft"])
    assert rf.default_nfft(1) == 64 and rf.default_nfft(1025) == 4096 and rf.default_nfft(5000) == 8192


def test_rejects_unknown_names():
    from spectral import rf

    with pytest.raises(ValueError, match="unknown window"):
        rf.window("kaiser", 8)
    with pytest.raises(ValueError, match="unknown fft_impl"):
        rf.fft(torch.zeros(4, dtype=torch.complex64), fft_impl="fftw")
    with pytest.raises(ValueError, match="complex64 CUDA tensor"):
        rf.spectrum(torch.zeros(4, dtype=torch.complex64), 4)


def test_backends_are_cufft_and_the_registry():
    from spectral import rf

    assert rf.FFT_BACKENDS == ("cufft", "naive", "stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table")
    assert rf.FUSED_IMPLS == ("stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table")


# --- GPU: every backend, the reference's cases ---------------------------------------------------

BACKENDS = ("cufft", "naive", "stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table")
FUSED = BACKENDS[2:]


def cuda(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
@pytest.mark.parametrize("window_name", ["rect", "hann", "blackman"])
@pytest.mark.parametrize("n", [1, 1000, 4096])
def test_spectrum_matches_the_oracle(rng, fft_impl, window_name, n):
    from spectral import rf

    x = random_complex(rng, n)
    y = rf.spectrum(cuda(x), 256, window_name=window_name, fft_impl=fft_impl)
    assert y.shape == (-(-n // 256), 256)
    assert relative_error(y.cpu().numpy(), orf.spectrum(x, 256, window_name)) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", FUSED)
@pytest.mark.parametrize("nfft", SIZES)
def test_fused_spectrum_every_block_size(rng, fft_impl, nfft):
    # Ragged: 3 signals of 2.5 frames (the last frame zero-padded), Hann window; per frame within
    # the transform's tolerance of the float64 result.
    from spectral import rf

    n = 2 * nfft + nfft // 2 + (1 if nfft == 2 else 0)
    x = random_complex(rng, (3, n))
    y = rf.spectrum(cuda(x), nfft, window_name="hann", fft_impl=fft_impl).cpu().numpy()
    expected = orf.spectrum(x, nfft, "hann")
    assert y.shape == expected.shape
    err = np.linalg.norm(y - expected, axis=-1) / np.maximum(np.linalg.norm(expected, axis=-1), 1e-30)
    assert err.max() <= fft_tolerance(nfft)


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", FUSED)
def test_fused_spectrum_edge_cases(fft_impl):
    from spectral import rf

    empty = rf.spectrum(torch.zeros(0, dtype=torch.complex64, device="cuda"), 64, fft_impl=fft_impl)
    assert empty.shape == (1, 64) and torch.count_nonzero(empty) == 0
    no_rows = rf.spectrum(torch.zeros(0, 5, dtype=torch.complex64, device="cuda"), 64, fft_impl=fft_impl)
    assert no_rows.shape == (0, 1, 64)
    # Frames of a constant with the rectangular window: nfft at bin 0 of every full frame, exactly.
    ones = torch.ones(4 * 512, dtype=torch.complex64, device="cuda")
    s = rf.spectrum(ones, 512, fft_impl=fft_impl)
    assert torch.equal(s[:, 0], torch.full((4,), 512.0, dtype=torch.complex64, device="cuda"))


FIR_CASES = [(1000, 1), (5, 63), (63, 63), (1000, 63), (4097, 64), (10_000, 1025), (3000, 4096)]


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
@pytest.mark.parametrize(("n", "m"), FIR_CASES)
def test_fir_matches_the_oracle(rng, fft_impl, n, m):
    from spectral import rf

    x = random_complex(rng, n)
    taps = rng.standard_normal(m).astype(np.float32)
    y = rf.fir(cuda(x), cuda(taps), fft_impl=fft_impl)
    assert y.shape == (n,)
    assert relative_error(y.cpu().numpy(), orf.fir(x, taps)) < 2e-5


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
def test_fir_with_complex_taps_rows_and_a_chosen_block_size(rng, fft_impl):
    from spectral import rf

    x = random_complex(rng, (3, 777))
    taps = random_complex(rng, 31)
    y = rf.fir(cuda(x), cuda(taps), nfft=64, fft_impl=fft_impl)
    assert relative_error(y.cpu().numpy(), orf.fir(x, taps)) < 2e-5


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", FUSED)
@pytest.mark.parametrize("nfft", SIZES)
def test_fused_fir_every_block_size(rng, fft_impl, nfft):
    # Taps of 1, nfft / 4 + 1 and nfft (one new output per block), rows, lengths that leave the
    # last block partly empty.
    from spectral import rf

    for m in sorted({1, nfft // 4 + 1, nfft}):
        x = random_complex(rng, (2, 3 * nfft + 5))
        taps = random_complex(rng, m)
        y = rf.fir(cuda(x), cuda(taps), nfft=nfft, fft_impl=fft_impl).cpu().numpy()
        expected = orf.fir(x, taps)
        assert relative_error(y, expected) < 4 * fft_tolerance(nfft), (nfft, m)


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
def test_fir_of_zeros_is_zeros(fft_impl):
    from spectral import rf

    x = torch.zeros(500, dtype=torch.complex64, device="cuda")
    taps = torch.ones(17, device="cuda")
    assert torch.count_nonzero(rf.fir(x, taps, fft_impl=fft_impl)) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", FUSED)
def test_fused_fir_edge_cases(fft_impl):
    from spectral import rf

    empty = rf.fir(torch.zeros(0, dtype=torch.complex64, device="cuda"), torch.ones(3, device="cuda"),
                   fft_impl=fft_impl)
    assert empty.shape == (0,)
    # A strided (non-contiguous) signal is filtered like its contiguous copy.
    rng = np.random.default_rng(5)
    big = cuda(random_complex(rng, (4, 900)))
    taps = cuda(rng.standard_normal(40).astype(np.float32))
    view = big[:, ::3]
    assert torch.equal(rf.fir(view, taps, fft_impl=fft_impl), rf.fir(view.contiguous(), taps, fft_impl=fft_impl))


@pytest.mark.gpu
def test_fir_rejects_a_block_shorter_than_the_filter():
    from spectral import rf

    x = torch.zeros(100, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError, match="at least len\\(taps\\) = 65"):
        rf.fir(x, torch.ones(65, device="cuda"), nfft=64)


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", ["stockham_r8", "stockham_r8_table"])
def test_fused_fir_at_full_size_is_a_delay(fft_impl):
    # 2^24 samples (the headline's size), taps = a unit impulse at d: the output is the input
    # delayed by d, each sample within the round trip's tolerance (size-independent property).
    from spectral import rf

    n, d = 1 << 24, 37
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(n, dtype=torch.complex64, device="cuda", generator=g)
    taps = torch.zeros(128, device="cuda")
    taps[d] = 1.0
    y = rf.fir(x, taps, fft_impl=fft_impl)
    assert torch.count_nonzero(y[:d].abs() > 1e-5) == 0
    err = (y[d:] - x[:-d]).abs().max().item()
    assert err < 8 * fft_tolerance(512) * x.abs().max().item()


# --- synthetic test signals: chirp, RRC-shaped BPSK / QPSK ------------------------------------

SAMPLE_RATE = 1.0e6
SPS = 8  # samples per symbol


def chirp(n: int = 16384) -> np.ndarray:
    """Unit-amplitude linear FM from -fs/4 to +fs/4 over n samples."""
    t = np.arange(n) / SAMPLE_RATE
    f0, f1 = -SAMPLE_RATE / 4, SAMPLE_RATE / 4
    k = (f1 - f0) / (n / SAMPLE_RATE)
    return np.exp(2j * np.pi * (f0 * t + 0.5 * k * t * t)).astype(np.complex64)


def rrc(beta: float = 0.35, span: int = 8) -> np.ndarray:
    """Root-raised-cosine pulse, span * SPS + 1 taps, unit energy (the textbook closed form, with
    its limits at t = 0 and |t| = T / (4 beta))."""
    t = (np.arange(span * SPS + 1) - span * SPS / 2) / SPS  # in symbol periods
    h = np.empty_like(t)
    for i, ti in enumerate(t):
        if abs(ti) < 1e-12:
            h[i] = 1.0 + beta * (4.0 / np.pi - 1.0)
        elif abs(abs(ti) - 1.0 / (4.0 * beta)) < 1e-12:
            h[i] = (beta / np.sqrt(2.0)) * ((1 + 2 / np.pi) * np.sin(np.pi / (4 * beta))
                                            + (1 - 2 / np.pi) * np.cos(np.pi / (4 * beta)))
        else:
            num = np.sin(np.pi * ti * (1 - beta)) + 4 * beta * ti * np.cos(np.pi * ti * (1 + beta))
            h[i] = num / (np.pi * ti * (1 - (4 * beta * ti) ** 2))
    return (h / np.linalg.norm(h)).astype(np.float32)


def shaped(symbols: np.ndarray, pulse: np.ndarray, seed: int, snr_db: float = 20.0) -> np.ndarray:
    up = np.zeros(len(symbols) * SPS, dtype=np.complex128)
    up[::SPS] = symbols
    x = np.convolve(up, pulse)[: len(up)]
    rng = np.random.default_rng(seed)
    power = np.mean(np.abs(x) ** 2)
    noise = (rng.standard_normal(len(x)) + 1j * rng.standard_normal(len(x))) * np.sqrt(power / 2 * 10 ** (-snr_db / 10))
    return (x + noise).astype(np.complex64)


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
def test_chirp_spectrum_peak_follows_the_sweep(fft_impl):
    from spectral import rf

    x = chirp()
    nfft = 256
    spec = rf.spectrum(cuda(x), nfft, window_name="hann", fft_impl=fft_impl).abs().cpu().numpy()
    peaks = np.fft.fftfreq(nfft)[np.argmax(spec, axis=-1)] * SAMPLE_RATE
    centers = (np.arange(len(peaks)) + 0.5) * nfft
    expected = -SAMPLE_RATE / 4 + (SAMPLE_RATE / 2) * centers / len(x)
    assert np.max(np.abs(peaks - expected)) <= 2 * SAMPLE_RATE / nfft


@pytest.mark.gpu
@pytest.mark.parametrize("fft_impl", BACKENDS)
@pytest.mark.parametrize("scheme", ["bpsk", "qpsk"])
def test_matched_filter_recovers_the_symbols(fft_impl, scheme):
    from spectral import rf

    rng = np.random.default_rng(11 if scheme == "bpsk" else 12)
    pulse = rrc()
    if scheme == "bpsk":
        truth = rng.integers(0, 2, 512)
        symbols = 2.0 * truth - 1.0
    else:
        truth = rng.integers(0, 4, 512)  # bit 0: sign of I, bit 1: sign of Q (Gray)
        symbols = ((1 - 2 * (truth & 1)) + 1j * (1 - 2 * (truth >> 1))) / np.sqrt(2.0)
    x = shaped(symbols, pulse, seed=int(rng.integers(1 << 30)))
    y = rf.fir(cuda(x), cuda(pulse), fft_impl=fft_impl).cpu().numpy()
    samples = y[len(pulse) - 1 :: SPS]
    truth = truth[: len(samples)]
    if scheme == "bpsk":
        assert np.array_equal((samples.real > 0).astype(int), truth)
    else:
        decided = (samples.real < 0).astype(int) + 2 * (samples.imag < 0).astype(int)
        assert np.array_equal(decided, truth)


# --- command line and C ABI ----------------------------------------------------------------------


@pytest.mark.gpu
def test_command_line_fir_matches_the_api(tmp_path):
    from spectral import rf

    x = shaped(np.sign(np.random.default_rng(1).standard_normal(256)), rrc(), seed=2)
    rf.write_cf32(tmp_path / "x.cf32", x)
    rrc().astype("<f4").tofile(tmp_path / "h.f32")
    out = tmp_path / "y.cf32"
    args = ["fir", "--in", str(tmp_path / "x.cf32"), "--taps", str(tmp_path / "h.f32"), "--out", str(out)]
    assert rf.main([*args, "--fft-impl", "stockham_r8"]) == 0
    expected = rf.fir(cuda(x), cuda(rrc()), fft_impl="stockham_r8")
    np.testing.assert_array_equal(rf.read_cf32(out), expected.cpu().numpy())


@pytest.mark.gpu
def test_command_line_spectrum(tmp_path):
    from spectral import rf

    rf.write_cf32(tmp_path / "c.cf32", chirp())
    out = tmp_path / "s.cf32"
    assert rf.main(["spectrum", "--in", str(tmp_path / "c.cf32"), "--out", str(out), "--nfft", "512",
                    "--window", "hann", "--fft-impl", "stockham_r4"]) == 0
    assert rf.read_cf32(out).size == 16384


@pytest.mark.gpu
def test_c_abi_matches_the_operators(rng):
    from spectral import native, rf

    x = cuda(random_complex(rng, (2, 5000)))
    taps = cuda(random_complex(rng, 100))
    h = rf.taps_spectrum(taps, 512, fft_impl="stockham_r8", device="cuda")
    y = torch.empty_like(x)
    s = torch.cuda.current_stream().cuda_stream
    native.call("spectral_fir", b"stockham_r8", x.data_ptr(), h.data_ptr(), y.data_ptr(), 5000, 512, 100, 2,
                ctypes.c_void_p(s))
    assert torch.equal(y, rf.fir(x, taps, nfft=512, fft_impl="stockham_r8"))

    w = rf.window("hamming", 1024, device="cuda")
    spec = torch.empty(2, 5, 1024, dtype=torch.complex64, device="cuda")
    native.call("spectral_spectrum", b"stockham_r8_table", x.data_ptr(), w.data_ptr(), spec.data_ptr(), 5000,
                1024, 2, ctypes.c_void_p(s))
    assert torch.equal(spec, rf.spectrum(x, 1024, window_name="hamming", fft_impl="stockham_r8_table"))
