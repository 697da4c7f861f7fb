"""Real-to-complex and complex-to-real transforms against the float64 oracle, every
implementation (the reference's tests/test_real.py, same cases)."""

import numpy as np
import pytest
import torch

import spectral
from oracle import reference as ref
from oracle.policy import (
    BATCHES,
    assert_transform_close,
    fft_tolerance,
    random_complex,
    random_real,
)

pytestmark = pytest.mark.gpu

IMPLS = spectral.FFT_IMPLS
SIZES = [2**p for p in range(1, 14)]
ENGINES = [impl for impl in IMPLS if impl.startswith("stockham")]


def rfft(x: np.ndarray, impl: str) -> np.ndarray:
    return spectral.rfft(torch.from_numpy(x).cuda(), impl=impl).cpu().numpy()


def irfft(x: np.ndarray, n: int, impl: str) -> np.ndarray:
    return spectral.irfft(torch.from_numpy(x).cuda(), n, impl=impl).cpu().numpy()


def hermitian_spectrum(rng, batch: int, n: int) -> np.ndarray:
    return ref.rfft(random_real(rng, (batch, n))).astype(np.complex64)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", BATCHES)
@pytest.mark.parametrize("n", SIZES)
def test_rfft_matches_the_oracle(rng, impl, n, batch):
    x = random_real(rng, (batch, n))
    y = rfft(x, impl)
    assert y.shape == (batch, n // 2 + 1)
    assert_transform_close(y, ref.rfft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", BATCHES)
@pytest.mark.parametrize("n", SIZES)
def test_irfft_matches_the_oracle(rng, impl, n, batch):
    spectrum = hermitian_spectrum(rng, batch, n)
    y = irfft(spectrum, n, impl)
    assert y.shape == (batch, n)
    assert y.dtype == np.float32
    assert_transform_close(y, ref.irfft(spectrum, n), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("n", [2, 64, 8192])
def test_irfft_undoes_rfft(rng, impl, n):
    x = torch.from_numpy(random_real(rng, (3, n))).cuda()
    back = spectral.irfft(spectral.rfft(x, impl=impl), n, impl=impl)
    assert_transform_close(back, x, n, tol=2 * fft_tolerance(n))


@pytest.mark.parametrize("impl", IMPLS)
def test_irfft_of_a_non_hermitian_spectrum_matches_torch(rng, impl):
    n = 256
    spectrum = random_complex(rng, (4, n // 2 + 1))
    expected = torch.fft.irfft(torch.from_numpy(spectrum).to(torch.complex128), n).numpy()
    assert_transform_close(irfft(spectrum, n, impl), expected, n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", [255, 257, 1000])
@pytest.mark.parametrize("n", [16, 4096])
def test_batches_that_do_not_fill_the_last_block(rng, impl, batch, n):
    x = random_real(rng, (batch, n))
    assert_transform_close(rfft(x, impl), ref.rfft(x), n)
    spectrum = hermitian_spectrum(rng, batch, n)
    assert_transform_close(irfft(spectrum, n, impl), ref.irfft(spectrum, n), n)


@pytest.mark.parametrize("impl", IMPLS)
def test_constant_signal_lands_in_bin_zero(impl):
    x = np.ones((1, 128), dtype=np.float32)
    expected = np.zeros((1, 65), dtype=np.complex128)
    expected[0, 0] = 128
    np.testing.assert_allclose(rfft(x, impl), expected, rtol=0, atol=1e-4)


@pytest.mark.parametrize("impl", IMPLS)
def test_leading_dimensions_and_non_contiguous_input(rng, impl):
    x = torch.from_numpy(random_real(rng, (64, 2, 3))).cuda().permute(1, 2, 0)
    assert not x.is_contiguous()
    y = spectral.rfft(x, impl=impl)
    assert y.shape == (2, 3, 33)
    assert_transform_close(y, ref.rfft(x.cpu().numpy()), 64)
    back = spectral.irfft(y.transpose(0, 1), 64, impl=impl)
    assert back.shape == (3, 2, 64)
    assert_transform_close(back, x.transpose(0, 1), 64, tol=2 * fft_tolerance(64))


@pytest.mark.parametrize("impl", IMPLS)
def test_empty_input_gives_empty_output(impl):
    x = torch.zeros(0, 8, device="cuda")
    assert spectral.rfft(x, impl=impl).shape == (0, 5)
    empty = torch.zeros(0, 5, dtype=torch.complex64, device="cuda")
    assert spectral.irfft(empty, 8, impl=impl).shape == (0, 8)


@pytest.mark.parametrize("impl", ENGINES)
def test_repeated_runs_are_bit_identical(rng, impl):
    x = torch.from_numpy(random_real(rng, (777, 4096))).cuda()
    assert torch.equal(spectral.rfft(x, impl=impl), spectral.rfft(x, impl=impl))
    s = spectral.rfft(x, impl=impl)
    assert torch.equal(spectral.irfft(s, 4096, impl=impl), spectral.irfft(s, 4096, impl=impl))


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("n", [1, 12])
def test_rejects_sizes_that_are_not_a_power_of_two_from_2(impl, n):
    with pytest.raises(RuntimeError, match="power of two of at least 2"):
        spectral.rfft(torch.zeros(2, n, device="cuda"), impl=impl)


@pytest.mark.parametrize("impl", ENGINES)
def test_rejects_a_size_above_the_implementation_limit(impl):
    with pytest.raises(RuntimeError, match="real sizes up to 8192"):
        spectral.rfft(torch.zeros(2, 16384, device="cuda"), impl=impl)


def test_rejects_a_spectrum_of_the_wrong_length():
    x = torch.zeros(2, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="n/2 \\+ 1 = 5 inputs"):
        spectral.irfft(x, 8)


def test_rejects_wrong_dtypes():
    with pytest.raises(RuntimeError, match="float32"):
        spectral.rfft(torch.zeros(2, 8, dtype=torch.complex64, device="cuda"))
    with pytest.raises(RuntimeError, match="complex64"):
        spectral.irfft(torch.zeros(2, 5, device="cuda"), 8)


def test_odd_offset_float_views_are_accepted(rng):
    # A contiguous float32 view that starts at an odd element is 4-byte aligned; the operators
    # copy it to an aligned allocation instead of handing it to the kernels.
    flat = torch.from_numpy(random_real(rng, (3 * 256 + 1,))).cuda()
    x = flat[1:].view(3, 256)
    assert x.data_ptr() % 8 == 4
    assert_transform_close(spectral.rfft(x, impl="stockham_r8"), ref.rfft(x.cpu().numpy()), 256)
    flat2 = torch.from_numpy(random_real(rng, (2 * 32 * 32 + 1,))).cuda()
    u = flat2[1:].view(2, 32, 32)
    assert_transform_close(spectral.rfft2(u, impl="stockham_r8"), ref.rfft2(u.cpu().numpy()), 1024,
                           axes=(-2, -1))
    modes = spectral.rfft2_truncated(u, 4, 4, impl="stockham_r8")
    assert modes.shape == (2, 8, 4)

