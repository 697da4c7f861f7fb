"""The C ABI called directly (ctypes, raw device pointers, an explicit stream): the boundary a
non-torch caller binds. Results must equal the torch operators' bit for bit, since both reach
the same kernels, and match the float64 oracle."""

import numpy as np
import pytest
import torch

from oracle import reference as ref
from oracle.policy import assert_transform_close, random_complex, random_real
from spectral import native

pytestmark = pytest.mark.gpu

ENGINES = ["stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table"]


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize("n", [1024, 8192])
def test_c2c_through_the_abi(rng, impl, n):
    import spectral

    x = torch.from_numpy(random_complex(rng, (16, n))).cuda()
    y = torch.empty_like(x)
    native.call("spectral_c2c", impl.encode(), x.data_ptr(), y.data_ptr(), n, 16, 0, stream())
    torch.cuda.synchronize()
    assert_transform_close(y, ref.fft(x.cpu().numpy()), n)
    assert torch.equal(y, spectral.fft_c2c(x, impl=impl))


@pytest.mark.parametrize("impl", ENGINES)
def test_real_round_trip_through_the_abi(rng, impl):
    n, batch = 4096, 64
    x = torch.from_numpy(random_real(rng, (batch, n))).cuda()
    spec = torch.empty(batch, n // 2 + 1, dtype=torch.complex64, device="cuda")
    back = torch.empty_like(x)
    native.call("spectral_r2c", impl.encode(), x.data_ptr(), spec.data_ptr(), n, batch, None, stream())
    native.call("spectral_c2r", impl.encode(), spec.data_ptr(), back.data_ptr(), n, batch, None, stream())
    torch.cuda.synchronize()
    assert_transform_close(spec, ref.rfft(x.cpu().numpy()), n)
    assert_transform_close(back, x, n, tol=2 * 2 * np.finfo(np.float32).eps * 12)


def test_naive_real_transform_needs_its_workspace(rng):
    n, batch = 64, 3
    x = torch.from_numpy(random_real(rng, (batch, n))).cuda()
    y = torch.empty(batch, n // 2 + 1, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError, match="needs a workspace"):
        native.call("spectral_r2c", b"naive", x.data_ptr(), y.data_ptr(), n, batch, None, stream())
    count = native.workspace("spectral_real_workspace", b"naive", n, batch)
    work = torch.empty(count, dtype=torch.complex64, device="cuda")
    native.call("spectral_r2c", b"naive", x.data_ptr(), y.data_ptr(), n, batch, work.data_ptr(), stream())
    torch.cuda.synchronize()
    assert_transform_close(y, ref.rfft(x.cpu().numpy()), n)


@pytest.mark.parametrize("impl", ENGINES)
def test_columns_in_place_through_the_abi(rng, impl):
    n, cols, slabs = 256, 129, 5
    x = random_complex(rng, (slabs, n, cols))
    t = torch.from_numpy(x).cuda()
    native.call("spectral_columns", impl.encode(), t.data_ptr(), t.data_ptr(), n, cols, slabs, 0, stream())
    torch.cuda.synchronize()
    expected = np.fft.fft(x.astype(np.complex128), axis=-2)
    assert_transform_close(t.cpu().numpy().swapaxes(-1, -2), expected.swapaxes(-1, -2), n)
