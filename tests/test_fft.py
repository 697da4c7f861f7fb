"""Batched complex FFTs on the GPU against the float64 oracle at 2 eps log2 N, for every
implementation in the registry (the reference's tests/test_fft.py, same cases)."""

import numpy as np
import pytest
import torch

import spectral
from oracle import reference as ref
from oracle.policy import (
    BATCHES,
    POW2_SIZES,
    assert_transform_close,
    fft_tolerance,
    random_complex,
)

pytestmark = pytest.mark.gpu

IMPLS = spectral.FFT_IMPLS
SIZES = [1, *POW2_SIZES]
ENGINES = [impl for impl in IMPLS if impl.startswith("stockham")]
LARGE_SIZES = [8192, 1 << 16, 1 << 20]


def run(x: np.ndarray, *, inverse: bool = False, impl: str) -> np.ndarray:
    return spectral.fft_c2c(torch.from_numpy(x).cuda(), inverse=inverse, impl=impl).cpu().numpy()


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", BATCHES)
@pytest.mark.parametrize("n", SIZES)
def test_forward_matches_the_oracle(rng, impl, n, batch):
    x = random_complex(rng, (batch, n))
    assert_transform_close(run(x, impl=impl), ref.fft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", BATCHES)
@pytest.mark.parametrize("n", SIZES)
def test_inverse_matches_the_oracle(rng, impl, n, batch):
    x = random_complex(rng, (batch, n))
    assert_transform_close(run(x, inverse=True, impl=impl), ref.ifft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("n", [2, 64, 4096])
def test_inverse_undoes_forward(rng, impl, n):
    x = torch.from_numpy(random_complex(rng, (3, n))).cuda()
    back = spectral.fft_c2c(spectral.fft_c2c(x, impl=impl), inverse=True, impl=impl)
    assert_transform_close(back, x, n, tol=2 * fft_tolerance(n))


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", [255, 257, 1000])
@pytest.mark.parametrize("n", [8, 1024, 2048])
def test_batches_that_do_not_fill_the_last_block(rng, impl, batch, n):
    x = random_complex(rng, (batch, n))
    assert_transform_close(run(x, impl=impl), ref.fft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("n", LARGE_SIZES)
def test_large_forward_matches_the_oracle(rng, impl, n, batch):
    x = random_complex(rng, (batch, n))
    assert_transform_close(run(x, impl=impl), ref.fft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("batch", [1, 2])
@pytest.mark.parametrize("n", LARGE_SIZES)
def test_large_inverse_matches_the_oracle(rng, impl, n, batch):
    x = random_complex(rng, (batch, n))
    assert_transform_close(run(x, inverse=True, impl=impl), ref.ifft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
def test_largest_size(rng, impl):
    n = 1 << 24
    x = random_complex(rng, (1, n))
    assert_transform_close(run(x, impl=impl), ref.fft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
def test_large_single_frequency_lands_in_one_bin(impl):
    n, k0 = 1 << 20, 12345
    x = np.exp(2j * np.pi * k0 * np.arange(n) / n).astype(np.complex64)[None, :]
    expected = np.zeros((1, n), dtype=np.complex128)
    expected[0, k0] = n
    assert_transform_close(run(x, impl=impl), expected, n)


@pytest.mark.parametrize("impl", ENGINES)
def test_large_transform_on_a_side_stream(rng, impl):
    x = torch.from_numpy(random_complex(rng, (2, 1 << 16))).cuda()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        y = spectral.fft_c2c(x, impl=impl)
    side.synchronize()
    assert_transform_close(y, ref.fft(x.cpu().numpy()), 1 << 16)


@pytest.mark.parametrize("impl", IMPLS)
def test_impulse_transforms_to_all_ones(impl):
    x = np.zeros((1, 256), dtype=np.complex64)
    x[0, 0] = 1
    np.testing.assert_allclose(run(x, impl=impl), np.ones((1, 256)), rtol=0, atol=1e-6)


@pytest.mark.parametrize("impl", IMPLS)
def test_single_frequency_lands_in_one_bin(impl):
    n, k0 = 256, 5
    x = np.exp(2j * np.pi * k0 * np.arange(n) / n).astype(np.complex64)[None, :]
    expected = np.zeros((1, n), dtype=np.complex128)
    expected[0, k0] = n
    assert_transform_close(run(x, impl=impl), expected, n)


@pytest.mark.parametrize("impl", IMPLS)
def test_leading_dimensions_are_batch_dimensions(rng, impl):
    x = random_complex(rng, (2, 3, 64))
    y = run(x, impl=impl)
    assert y.shape == (2, 3, 64)
    assert_transform_close(y, ref.fft(x), 64)


@pytest.mark.parametrize("impl", IMPLS)
def test_non_contiguous_input(rng, impl):
    x = torch.from_numpy(random_complex(rng, (64, 128))).cuda().T
    assert not x.is_contiguous()
    assert_transform_close(spectral.fft_c2c(x, impl=impl), ref.fft(x.cpu().numpy()), 64)


@pytest.mark.parametrize("impl", IMPLS)
def test_empty_input_gives_empty_output(impl):
    x = torch.zeros(0, 8, dtype=torch.complex64, device="cuda")
    assert spectral.fft_c2c(x, impl=impl).shape == (0, 8)


@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize("n", [256, 1024, 2048, 4096])
def test_repeated_runs_are_bit_identical(rng, impl, n):
    # Shared-memory races show up as run-to-run differences; the engine is deterministic.
    x = torch.from_numpy(random_complex(rng, (333, n))).cuda()
    a = spectral.fft_c2c(x, impl=impl)
    b = spectral.fft_c2c(x, impl=impl)
    assert torch.equal(a, b)


@pytest.mark.parametrize("impl", IMPLS)
def test_rejects_a_size_that_is_not_a_power_of_two(impl):
    x = torch.zeros(4, 12, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="power of two"):
        spectral.fft_c2c(x, impl=impl)


@pytest.mark.parametrize("impl", ENGINES)
def test_rejects_a_size_above_the_implementation_limit(impl):
    x = torch.empty(1, 1 << 25, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="sizes up to 16777216"):
        spectral.fft_c2c(x, impl=impl)


def test_rejects_an_unknown_implementation():
    x = torch.zeros(4, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="unknown FFT implementation"):
        spectral.fft_c2c(x, impl="nope")
