"""spectral_fft2_c2r_noalloc, the allocation-free complex-to-real 2D transform, called through the
C ABI. It serves callers that cannot allocate device memory (a host framework that owns every
allocation, a real-time loop that must stay out of the allocator, a binding with pointers but no
allocator): its workspace is a fixed array inside the library. It must give the results of
spectral_fft2_c2r with a caller workspace, call after call, since every call reuses that array.

This file is named to be collected last, so a run that stops at the first failure has already
run every other test."""

import numpy as np
import pytest
import torch

from oracle import reference as ref
from oracle.policy import assert_transform_close, random_real
from spectral import native

ENGINES = ["stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table"]


def test_oversized_requests_are_rejected_before_any_gpu_work():
    limit = 1 << 22
    # 64 arrays of 256 x 129 values: 2.1 Mi values fit; 256 of them (8.5 Mi) do not.
    with pytest.raises(ValueError, match="exceed the built-in scratch array"):
        native.call("spectral_fft2_c2r_noalloc", b"stockham_r8", None, None, 256, 256, 256, None)
    assert 64 * 256 * 129 <= limit


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ENGINES)
@pytest.mark.parametrize(("batch", "n1", "n2"), [(3, 64, 32), (64, 256, 256), (7, 128, 128)])
def test_noalloc_matches_the_allocating_entry_point(rng, impl, batch, n1, n2):
    stream = torch.cuda.current_stream().cuda_stream
    w = n2 // 2 + 1
    count = native.workspace("spectral_fft2_c2r_workspace", impl.encode(), 1, n1, n2, batch)
    work = torch.empty(max(count, 1), dtype=torch.complex64, device="cuda")
    for call in range(2):  # two calls in a row: the shared scratch keeps the last call's data
        spectrum = ref.rfft2(random_real(rng, (batch, n1, n2))).astype(np.complex64)
        x = torch.from_numpy(spectrum).cuda()
        expected = torch.empty(batch, n1, n2, device="cuda")
        got = torch.empty(batch, n1, n2, device="cuda")
        native.call("spectral_fft2_c2r", impl.encode(), 1, x.data_ptr(), expected.data_ptr(), n1, n2,
                    batch, work.data_ptr(), stream)
        native.call("spectral_fft2_c2r_noalloc", impl.encode(), x.data_ptr(), got.data_ptr(), n1, n2,
                    batch, stream)
        torch.cuda.synchronize()
        # Within the parity tolerance of the transform, against the allocating entry point and
        # against the float64 oracle.
        assert_transform_close(got, expected, n1 * n2, axes=(-2, -1))
        assert_transform_close(got, ref.irfft2(spectrum, (n1, n2)), n1 * n2, axes=(-2, -1))
        assert x.shape == (batch, n1, w)
