"""The whole-field rfft2 / irfft2 kernel (one kernel per direction, the row spectrum kept in an
L2-resident scratch) that serves columns="strided" for fields of up to 512 KiB of row spectrum:
square and non-square fields, a non-128-byte-aligned scratch, more fields than the device holds
CTAs at once, and non-Hermitian spectra, against the float64 oracle."""

import numpy as np
import pytest
import torch

import spectral
from spectral import native
from oracle import reference as ref
from oracle.policy import assert_transform_close, fft_tolerance, random_complex, random_real

pytestmark = pytest.mark.gpu

AXES = (-2, -1)
ENGINES = [impl for impl in spectral.FFT_IMPLS if impl.startswith("stockham")]
SHAPES = [(16, 16), (16, 1024), (1024, 16), (32, 64), (64, 128), (128, 128), (128, 256),
          (256, 128), (256, 256), (512, 512), (1024, 512), (256, 1024)]


def cuda(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(x).cuda()


@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize(("n1", "n2"), SHAPES)
def test_fields_rfft2(rng, impl, n1, n2):
    x = random_real(rng, (3, n1, n2))
    y = spectral.rfft2(cuda(x), impl=impl, columns="strided")
    assert_transform_close(y, ref.rfft2(x), n1 * n2, axes=AXES)


@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize(("n1", "n2"), SHAPES)
def test_fields_irfft2(rng, impl, n1, n2):
    spectrum = ref.rfft2(random_real(rng, (3, n1, n2))).astype(np.complex64)
    y = spectral.irfft2(cuda(spectrum), n2, impl=impl, columns="strided")
    assert_transform_close(y, ref.irfft2(spectrum, (n1, n2)), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("n1", "n2"), [(16, 16), (128, 256), (256, 256)])
def test_fields_irfft2_of_a_non_hermitian_spectrum_matches_torch(rng, n1, n2):
    spectrum = random_complex(rng, (3, n1, n2 // 2 + 1))
    expected = torch.fft.irfft2(torch.from_numpy(spectrum).to(torch.complex128), s=(n1, n2))
    y = spectral.irfft2(cuda(spectrum), n2, impl="stockham_r8", columns="strided")
    assert_transform_close(y, expected.numpy(), n1 * n2, axes=AXES)


@pytest.mark.parametrize(("n1", "n2"), [(256, 256), (64, 64)])
def test_fields_many_fields_and_round_trip(rng, n1, n2):
    x = random_real(rng, (1500, n1, n2))
    y = spectral.rfft2(cuda(x), impl="stockham_r8", columns="strided")
    assert_transform_close(y, ref.rfft2(x), n1 * n2, axes=AXES)
    back = spectral.irfft2(y, n2, impl="stockham_r8", columns="strided")
    assert_transform_close(back, x, n1 * n2, axes=AXES, tol=2 * fft_tolerance(n1 * n2))


def test_fields_with_an_unaligned_scratch_through_the_c_abi(rng):
    # The kernel drops its scratch from L2 only when the scratch is whole 128-byte lines; an
    # 8-byte-offset scratch takes the path that leaves it to be written back.
    n1, n2, batch = 128, 128, 5
    x = cuda(random_real(rng, (batch, n1, n2)))
    stream = torch.cuda.current_stream().cuda_stream
    count = native.workspace("spectral_fft2_r2c_workspace", b"stockham_r8", 1, n1, n2, batch)
    work = torch.empty(count + 1, dtype=torch.complex64, device="cuda")
    y = torch.empty(batch, n1, n2 // 2 + 1, dtype=torch.complex64, device="cuda")
    native.call("spectral_fft2_r2c", b"stockham_r8", 1, x.data_ptr(), y.data_ptr(), n1, n2, batch,
                work.data_ptr() + 8, stream)
    torch.cuda.synchronize()
    assert_transform_close(y, ref.rfft2(x.cpu().numpy()), n1 * n2, axes=AXES)


def test_fields_match_the_transpose_method(rng):
    x = cuda(random_real(rng, (4, 256, 256)))
    a = spectral.rfft2(x, impl="stockham_r8", columns="strided")
    b = spectral.rfft2(x, impl="stockham_r8", columns="transpose")
    # Each is within the tolerance of the exact transform, so they agree within twice it.
    assert_transform_close(a, b.cpu().numpy().astype(np.complex128), 256 * 256, axes=AXES,
                           tol=2 * fft_tolerance(256 * 256))
