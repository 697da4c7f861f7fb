"""2D transforms against the float64 oracle: every implementation with the transpose method,
the ones with a column kernel with the strided method too (the reference's tests/test_fft2.py)."""

import numpy as np
import pytest
import torch

import spectral
from oracle import reference as ref
from oracle.policy import assert_transform_close, fft_tolerance, random_complex, random_real

pytestmark = pytest.mark.gpu

AXES = (-2, -1)
ENGINES = [impl for impl in spectral.FFT_IMPLS if impl.startswith("stockham")]
METHODS = [(impl, "transpose") for impl in spectral.FFT_IMPLS] + [(impl, "strided") for impl in ENGINES]
METHOD_IDS = [f"{impl}-{cols}" for impl, cols in METHODS]

SHAPES = [(1, 8), (8, 1), (2, 2), (16, 16), (64, 32), (8, 256), (256, 8), (4096, 4), (4, 4096),
          (256, 256)]
REAL_SHAPES = [(1, 8), (8, 2), (16, 16), (64, 32), (8, 256), (256, 8), (4096, 4), (2, 8192),
               (256, 256), (128, 128)]


def cuda(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(x).cuda()


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
@pytest.mark.parametrize(("n1", "n2"), SHAPES)
def test_fft2_matches_the_oracle(rng, impl, columns, n1, n2):
    x = random_complex(rng, (3, n1, n2))
    y = spectral.fft2(cuda(x), impl=impl, columns=columns)
    assert_transform_close(y, ref.fft2(x), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
@pytest.mark.parametrize(("n1", "n2"), SHAPES)
def test_ifft2_matches_the_oracle(rng, impl, columns, n1, n2):
    x = random_complex(rng, (3, n1, n2))
    y = spectral.fft2(cuda(x), inverse=True, impl=impl, columns=columns)
    assert_transform_close(y, ref.ifft2(x), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
@pytest.mark.parametrize(("n1", "n2"), REAL_SHAPES)
def test_rfft2_matches_the_oracle(rng, impl, columns, n1, n2):
    x = random_real(rng, (3, n1, n2))
    y = spectral.rfft2(cuda(x), impl=impl, columns=columns)
    assert y.shape == (3, n1, n2 // 2 + 1)
    assert_transform_close(y, ref.rfft2(x), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
@pytest.mark.parametrize(("n1", "n2"), REAL_SHAPES)
def test_irfft2_matches_the_oracle(rng, impl, columns, n1, n2):
    spectrum = ref.rfft2(random_real(rng, (3, n1, n2))).astype(np.complex64)
    y = spectral.irfft2(cuda(spectrum), n2, impl=impl, columns=columns)
    assert y.shape == (3, n1, n2)
    assert_transform_close(y, ref.irfft2(spectrum, (n1, n2)), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
@pytest.mark.parametrize("n", [16, 256])
def test_irfft2_of_a_non_hermitian_spectrum_matches_torch(rng, impl, columns, n):
    # Columns 0 and n/2 with arbitrary imaginary parts: only their real parts after the column
    # transforms reach the output, as in numpy and torch.
    spectrum = random_complex(rng, (2, n, n // 2 + 1))
    expected = torch.fft.irfft2(torch.from_numpy(spectrum).to(torch.complex128), s=(n, n))
    y = spectral.irfft2(cuda(spectrum), n, impl=impl, columns=columns)
    assert_transform_close(y, expected.numpy(), n * n, axes=AXES)


@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize("fields", [1, 2, 75, 150, 301])
def test_many_256_x_256_fields(rng, impl, fields):
    # Field counts below, at and above one per SM pair and per SM (74 and 148 on a B200), so the
    # persistent row and column grids walk several tiles; the oracle checks the first, middle
    # and last fields.
    n = 256
    x = random_real(rng, (fields, n, n))
    s = spectral.rfft2(cuda(x), impl=impl, columns="strided")
    y = spectral.irfft2(s, n, impl=impl, columns="strided")
    idx = sorted({0, fields // 2, fields - 1})
    assert_transform_close(s[idx], ref.rfft2(x[idx]), n * n, axes=AXES)
    spectrum = s[idx].cpu().numpy()
    assert_transform_close(y[idx], ref.irfft2(spectrum, (n, n)), n * n, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
def test_round_trips(rng, impl, columns):
    x = cuda(random_complex(rng, (2, 32, 64)))
    back = spectral.fft2(spectral.fft2(x, impl=impl, columns=columns), inverse=True, impl=impl,
                         columns=columns)
    assert_transform_close(back, x, 32 * 64, axes=AXES, tol=2 * fft_tolerance(32 * 64))
    r = cuda(random_real(rng, (2, 32, 64)))
    back = spectral.irfft2(spectral.rfft2(r, impl=impl, columns=columns), 64, impl=impl)
    assert_transform_close(back, r, 32 * 64, axes=AXES, tol=2 * fft_tolerance(32 * 64))


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
def test_many_arrays_and_leading_dimensions(rng, impl, columns):
    x = random_real(rng, (2, 3, 50, 8, 16))
    y = spectral.rfft2(cuda(x), impl=impl, columns=columns)
    assert y.shape == (2, 3, 50, 8, 9)
    assert_transform_close(y, ref.rfft2(x), 128, axes=AXES)


@pytest.mark.parametrize(("impl", "columns"), METHODS, ids=METHOD_IDS)
def test_non_contiguous_input(rng, impl, columns):
    x = cuda(random_complex(rng, (16, 32, 3))).permute(2, 0, 1)
    assert not x.is_contiguous()
    y = spectral.fft2(x, impl=impl, columns=columns)
    assert_transform_close(y, ref.fft2(x.cpu().numpy()), 16 * 32, axes=AXES)


def test_auto_picks_strided_when_available(rng):
    x = cuda(random_real(rng, (4, 32, 32)))
    for impl in ENGINES:
        assert torch.equal(spectral.rfft2(x, impl=impl), spectral.rfft2(x, impl=impl, columns="strided"))
    naive = spectral.rfft2(x, impl="naive")
    assert torch.equal(naive, spectral.rfft2(x, impl="naive", columns="transpose"))


def test_empty_input_gives_empty_output():
    x = torch.zeros(0, 4, 8, device="cuda")
    assert spectral.rfft2(x).shape == (0, 4, 5)
    assert spectral.fft2(x.to(torch.complex64)).shape == (0, 4, 8)
    empty = torch.zeros(0, 4, 5, dtype=torch.complex64, device="cuda")
    assert spectral.irfft2(empty, 8).shape == (0, 4, 8)


def test_rejects_strided_without_a_column_kernel():
    x = torch.zeros(4, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="no strided column kernel"):
        spectral.fft2(x, impl="naive", columns="strided")


def test_rejects_an_unknown_column_method():
    x = torch.zeros(4, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="columns must be"):
        spectral.fft2(x, impl="naive", columns="sideways")


@pytest.mark.parametrize("impl", ENGINES)
def test_rejects_columns_longer_than_the_kernel_supports(impl):
    x = torch.zeros(8192, 2, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError, match="n1 to be a power of two up to 4096"):
        spectral.fft2(x, impl=impl)


def test_rejects_one_dimensional_input():
    with pytest.raises(RuntimeError, match="at least two dimensions"):
        spectral.rfft2(torch.zeros(8, device="cuda"))


def test_rejects_a_spectrum_of_the_wrong_width():
    x = torch.zeros(4, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="n2/2 \\+ 1 = 5 input columns"):
        spectral.irfft2(x, 8)
