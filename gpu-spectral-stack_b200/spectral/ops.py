"""Python entry points for the torch.ops.spectral operators.

The same functions, keyword arguments and defaults as the reference's python/spectral/ops.py
(ops.py:9-114): each forwards to a torch.ops.spectral operator, which checks its arguments and
calls the C ABI (include/spectral_b200.h) on the current CUDA stream. Conventions are numpy's and
torch's (norm="backward"): forward unnormalized, inverse divided by the number of points.
"""

import torch

from . import _C

# Every FFT implementation, in registry order, read from the C ABI: the reference's five names.
FFT_IMPLS: tuple[str, ...] = _C.fft_impls()


def scale(x: torch.Tensor, alpha: float) -> torch.Tensor:
    """alpha * x for a complex64 CUDA tensor, as a new contiguous tensor."""
    return torch.ops.spectral.scale.default(x, alpha)


def fft_c2c(x: torch.Tensor, *, inverse: bool = False, impl: str = "naive") -> torch.Tensor:
    """Batched complex FFT along the last dimension (a power of two); leading dimensions are
    batch. Like torch.fft.fft, or torch.fft.ifft with inverse=True. complex64 on a CUDA device."""
    return torch.ops.spectral.fft_c2c.default(x, inverse, impl)


def rfft(x: torch.Tensor, *, impl: str = "naive") -> torch.Tensor:
    """Batched real-to-complex FFT along the last dimension, like torch.fft.rfft: float32 with a
    power-of-two last dimension n >= 2 to complex64 with n // 2 + 1 values."""
    return torch.ops.spectral.fft_r2c.default(x, impl)


def irfft(x: torch.Tensor, n: int, *, impl: str = "naive") -> torch.Tensor:
    """Inverse of rfft divided by n, like torch.fft.irfft(x, n); the imaginary parts of the zero
    and n/2 frequencies are ignored."""
    return torch.ops.spectral.fft_c2r.default(x, n, impl)


# 2D: `columns` picks how the column transforms run. "strided" transforms them where they are,
# "transpose" goes through transposes and row transforms, "auto" is "strided" when the
# implementation has a column kernel (every one but "naive").


def fft2(
    x: torch.Tensor, *, inverse: bool = False, impl: str = "naive", columns: str = "auto"
) -> torch.Tensor:
    """Batched 2D complex FFT over the last two dimensions, like torch.fft.fft2 (or ifft2)."""
    return torch.ops.spectral.fft2_c2c.default(x, inverse, impl, columns)


def rfft2(x: torch.Tensor, *, impl: str = "naive", columns: str = "auto") -> torch.Tensor:
    """Batched 2D real-to-complex FFT, like torch.fft.rfft2: (..., n1, n2) float32 to
    (..., n1, n2 // 2 + 1) complex64."""
    return torch.ops.spectral.fft2_r2c.default(x, impl, columns)


def irfft2(x: torch.Tensor, n2: int, *, impl: str = "naive", columns: str = "auto") -> torch.Tensor:
    """Inverse of rfft2, like torch.fft.irfft2(x, s=(x.shape[-2], n2)): divides by n1 * n2."""
    return torch.ops.spectral.fft2_c2r.default(x, n2, impl, columns)


# Pruned transforms: only the low-frequency modes an FNO spectral convolution keeps, in the
# layout of the reference's spectral.reference (rfft2_truncate / irfft2_from_modes).


def fft_truncated(x: torch.Tensor, k: int, *, impl: str = "naive") -> torch.Tensor:
    """The first k outputs of fft_c2c(x): (..., n) complex64 -> (..., k)."""
    return torch.ops.spectral.fft_c2c_pruned.default(x, x.shape[-1], k, False, impl)


def ifft_from_modes(modes: torch.Tensor, n: int, *, impl: str = "naive") -> torch.Tensor:
    """Inverse FFT of n points whose first k = modes.shape[-1] inputs are `modes`, the rest
    zero: (..., k) complex64 -> (..., n), divided by n."""
    return torch.ops.spectral.fft_c2c_pruned.default(modes, n, modes.shape[-1], True, impl)


def rfft2_truncated(x: torch.Tensor, m1: int, m2: int, *, impl: str = "naive") -> torch.Tensor:
    """The low-frequency modes of rfft2(x): (..., n1, n2) float32 -> (..., 2 m1, m2) complex64;
    rows 0 .. m1-1 then n1-m1 .. n1-1, columns 0 .. m2-1."""
    return torch.ops.spectral.rfft2_modes.default(x, m1, m2, impl)


def irfft2_from_modes(
    modes: torch.Tensor, shape: tuple[int, int], *, impl: str = "naive"
) -> torch.Tensor:
    """Inverse of rfft2_truncated: (..., 2 m1, m2) complex64 -> (..., n1, n2) float32, every
    dropped mode taken as zero."""
    n1, n2 = shape
    return torch.ops.spectral.irfft2_modes.default(modes, n1, n2, impl)


def mode_contract(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """The per-mode channel contraction of an FNO spectral convolution:
    out[b, o, *m] = sum_i x[b, i, *m] * w[i, o, *m], complex64 on a CUDA device. x is
    (batch, cin, *modes), w is (cin, cout, *modes). An addition of this library: the reference
    plans this step (its ROADMAP tasks 3.3-3.6) but does not implement it."""
    return torch.ops.spectral.mode_contract.default(x, w)
