"""The torch extension: registered operators, our own scale kernel (bit-exact), launches on
PyTorch's current stream, rejections (the reference's tests/test_extension.py)."""

import pytest
import torch

import spectral


def test_operator_is_registered():
    assert hasattr(torch.ops.spectral, "scale")


def test_fft_implementations_come_from_the_registry():
    assert spectral.FFT_IMPLS[0] == "naive"
    assert {"stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table"} <= set(spectral.FFT_IMPLS)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 255, 256, 257, 1 << 20])
def test_scale_matches_torch(n):
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.randn(n, dtype=torch.complex64, device="cuda", generator=g)
    torch.testing.assert_close(spectral.scale(x, 0.5), x * 0.5, rtol=0, atol=0)


@pytest.mark.gpu
def test_scale_non_contiguous_input():
    x = torch.randn(1000, dtype=torch.complex64, device="cuda")[::2]
    assert not x.is_contiguous()
    torch.testing.assert_close(spectral.scale(x, 0.5), x * 0.5, rtol=0, atol=0)


@pytest.mark.gpu
def test_scale_on_side_stream():
    x = torch.randn(1 << 20, dtype=torch.complex64, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        y = spectral.scale(x, 0.5)
    side.synchronize()
    torch.testing.assert_close(y, x * 0.5, rtol=0, atol=0)


def test_cpu_input_is_rejected_by_the_dispatcher():
    x = torch.zeros(4, dtype=torch.complex64)
    with pytest.raises(NotImplementedError, match="CPU"):
        spectral.scale(x, 0.5)


@pytest.mark.gpu
def test_wrong_dtype_is_rejected():
    x = torch.zeros(4, dtype=torch.float32, device="cuda")
    with pytest.raises(RuntimeError, match="complex64"):
        spectral.scale(x, 0.5)


@pytest.mark.gpu
@pytest.mark.parametrize("offset", [0, 1])
@pytest.mark.parametrize("n", [2, 3, 4097, 1 << 22])
def test_scale_on_both_paths_and_in_place(offset, n):
    # offset 0: 16-byte aligned (two values per access, an odd tail on its own); offset 1: 8 bytes
    # off (the one-value kernel). In place through the C ABI too: every value is read before the
    # same thread writes it.
    from spectral import native

    g = torch.Generator(device="cuda").manual_seed(n + offset)
    base = torch.randn(n + 1, dtype=torch.complex64, device="cuda", generator=g)
    x = base[offset:offset + n]
    expected = x * 0.25
    torch.testing.assert_close(spectral.scale(x, 0.25), expected, rtol=0, atol=0)
    stream = torch.cuda.current_stream().cuda_stream
    native.call("spectral_scale", x.data_ptr(), x.data_ptr(), n, 0.25, stream)
    torch.cuda.synchronize()
    torch.testing.assert_close(x, expected, rtol=0, atol=0)
