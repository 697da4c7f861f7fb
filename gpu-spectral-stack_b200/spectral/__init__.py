"""spectral: B200-native batched FFTs behind the API of gpu-spectral-stack's `spectral` package.

Importing the package loads the CUDA extension (spectral._C, a shim over libspectral_b200.so),
which registers the torch.ops.spectral operators. There is no CPU path: if the extension is not
built, the import fails and says how to build it.
"""

import torch  # noqa: F401  # libtorch must be loaded before the extension that links against it

try:
    from . import _C  # noqa: F401  # registers torch.ops.spectral
except ImportError as exc:  # pragma: no cover - exercised only on an unbuilt checkout
    raise ImportError(
        "spectral: the CUDA extension is not built (expected spectral/_C*.so and "
        "spectral/libspectral_b200.so); run `python gpu-spectral-stack_b200/build.py`"
    ) from exc

from . import nn
from .ops import (
    FFT_IMPLS,
    fft2,
    fft_c2c,
    fft_truncated,
    ifft_from_modes,
    irfft,
    irfft2,
    irfft2_from_modes,
    mode_contract,
    rfft,
    rfft2,
    rfft2_truncated,
    scale,
)

__all__ = [
    "FFT_IMPLS",
    "fft2",
    "fft_c2c",
    "fft_truncated",
    "ifft_from_modes",
    "irfft",
    "irfft2",
    "irfft2_from_modes",
    "mode_contract",
    "rfft",
    "rfft2",
    "rfft2_truncated",
    "scale",
]
