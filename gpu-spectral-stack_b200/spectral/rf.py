"""Radio signal processing on this library's transforms: periodic windows, the windowed
spectrum of back-to-back frames, and causal FIR filtering by overlap-save.

The public names, arguments, errors and command line are those of the reference's
python/spectral/rf.py (rf.py:31-212), which its callers use; the implementation is this
library's. Every operation takes a backend:

    fft_impl="stockham_r8"   (default) this library's engine; any of spectral.FFT_IMPLS works
    fft_impl="cufft"         torch.fft (cuFFT), kept as the library baseline to compare against

The reference defaults to "cufft". Here the default is the engine, so that a caller who names no
backend runs this library's kernels and no cuFFT: the results agree with cuFFT's within the
transforms' FP32 tolerance, not bit for bit.

With a stockham implementation and blocks of 2 .. 4096 points each operation is one kernel
(csrc/rf.cu, through torch.ops.spectral): `spectrum` cuts the frames, zero-pads the last one and
applies the window in the transform's load; `fir` transforms each block, multiplies it by the
taps' spectrum and transforms it back on chip, storing only the exact outputs. Other backends and
longer blocks are composed here from the library's transforms (or torch.fft for "cufft") and
strided views: no copy of the signal is made beyond one zero-extended buffer.

    python -m spectral.rf spectrum --in x.cf32 --out spec.cf32 --nfft 1024 --window hann
    python -m spectral.rf fir --in x.cf32 --taps h.f32 --out y.cf32 --fft-impl stockham_r8

Files: .cf32 is interleaved little-endian float32 I/Q (numpy complex64), .f32 raw float32.
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

from . import ops

FFT_BACKENDS: tuple[str, ...] = ("cufft", *ops.FFT_IMPLS)
WINDOWS: tuple[str, ...] = ("rect", "hann", "hamming", "blackman")
DEFAULT_FFT_IMPL = "stockham_r8"

# The implementations with the fused kernels, and the largest block those kernels hold.
FUSED_IMPLS: tuple[str, ...] = tuple(name for name in ops.FFT_IMPLS if name.startswith("stockham"))
FUSED_MAX_NFFT = 4096

# Windows as sums of cosines: w[k] = sum_j (-1)^j a_j cos(2 pi j k / n) (periodic form).
_COSINE_TERMS: dict[str, tuple[float, ...]] = {
    "rect": (1.0,),
    "hann": (0.5, 0.5),
    "hamming": (0.54, 0.46),
    "blackman": (0.42, 0.5, 0.08),
}


def _check_backend(fft_impl: str) -> None:
    if fft_impl not in FFT_BACKENDS:
        raise ValueError(f"unknown fft_impl '{fft_impl}' (available: {', '.join(FFT_BACKENDS)})")


def _check_complex(x: torch.Tensor, name: str) -> None:
    if not (x.is_cuda and x.dtype == torch.complex64):
        raise ValueError(f"{name} must be a complex64 CUDA tensor, got {x.dtype} on {x.device}")


def _fused(fft_impl: str, nfft: int) -> bool:
    return fft_impl in FUSED_IMPLS and 2 <= nfft <= FUSED_MAX_NFFT


def fft(x: torch.Tensor, *, inverse: bool = False, fft_impl: str = DEFAULT_FFT_IMPL) -> torch.Tensor:
    """Complex transform along the last dimension, the inverse divided by n, by `fft_impl`."""
    _check_backend(fft_impl)
    if fft_impl != "cufft":
        return ops.fft_c2c(x, inverse=inverse, impl=fft_impl)
    return (torch.fft.ifft if inverse else torch.fft.fft)(x)


def window(name: str, n: int, *, device: torch.device | str | None = None) -> torch.Tensor:
    """The periodic n-point window (scipy.signal.get_window's fftbins=True form) as float32,
    evaluated in float64:

    rect      1
    hann      0.5 - 0.5 cos(2 pi k / n)
    hamming   0.54 - 0.46 cos(2 pi k / n)
    blackman  0.42 - 0.5 cos(2 pi k / n) + 0.08 cos(4 pi k / n)

    A one-point window is [1] for every name, as in scipy."""
    if n < 1:
        raise ValueError(f"a window needs at least one point, got {n}")
    terms = _COSINE_TERMS.get(name)
    if terms is None:
        raise ValueError(f"unknown window '{name}' (available: {', '.join(WINDOWS)})")
    if n == 1:
        return torch.ones(1, device=device)
    angle = 2.0 * np.pi * np.arange(n) / n
    w = np.full(n, terms[0])
    for j in range(1, len(terms)):
        w = w + (-terms[j] if j % 2 else terms[j]) * np.cos(j * angle)
    return torch.from_numpy(w.astype(np.float32)).to(device)


def frames(x: torch.Tensor, nfft: int) -> torch.Tensor:
    """(..., n) -> (..., max(1, ceil(n / nfft)), nfft): back-to-back frames of x, the last one
    completed with zeros."""
    n = x.shape[-1]
    count = max(1, -(-n // nfft))
    out = x.new_zeros(*x.shape[:-1], count * nfft)
    out[..., :n] = x
    return out.view(*x.shape[:-1], count, nfft)


def spectrum(
    x: torch.Tensor, nfft: int, *, window_name: str = "rect", fft_impl: str = DEFAULT_FFT_IMPL
) -> torch.Tensor:
    """The transform of each windowed nfft-sample frame of x: complex64 (..., n) ->
    (..., frames, nfft)."""
    _check_complex(x, "x")
    _check_backend(fft_impl)
    w = window(window_name, nfft, device=x.device)
    if _fused(fft_impl, nfft):
        # One kernel; the rectangular window is all ones, so it passes none.
        return torch.ops.spectral.spectrum_frames.default(x, nfft, w if window_name != "rect" else None, fft_impl)
    return fft(frames(x, nfft) * w, fft_impl=fft_impl)


def default_nfft(num_taps: int) -> int:
    """The overlap-save block fir() picks for `num_taps` taps: the power of two nearest above four
    times the filter (at least 64), so that three quarters of each block are new output; capped at
    4096, the fused kernel's largest block, unless the filter itself is longer, which then gets the
    power of two at or above its length."""
    if num_taps < 1:
        raise ValueError("the filter needs at least one tap")
    block = 1 << max(6, (4 * num_taps - 1).bit_length())
    if block <= 4096:
        return block
    return max(4096, 1 << (num_taps - 1).bit_length())


def taps_spectrum(taps: torch.Tensor, nfft: int, *, fft_impl: str = DEFAULT_FFT_IMPL, device=None) -> torch.Tensor:
    """The nfft-point transform of `taps` (real or complex) extended with zeros: complex64."""
    h = torch.zeros(nfft, dtype=torch.complex64, device=device)
    h[: taps.numel()] = taps.to(device=device, dtype=torch.complex64)
    return fft(h, fft_impl=fft_impl)


def _overlap_save(x: torch.Tensor, h_spec: torch.Tensor, m: int, nfft: int, fft_impl: str) -> torch.Tensor:
    """Overlap-save from the library's transforms: the signal extended by m - 1 leading zeros
    (the zero initial state) and trailing zeros up to whole blocks, read as overlapping blocks of
    nfft samples at a hop of nfft - m + 1 through a strided view; each block's last nfft - m + 1
    circular-convolution outputs are the exact ones."""
    hop = nfft - m + 1
    n = x.shape[-1]
    count = max(1, -(-n // hop))
    lead = x.shape[:-1]
    rows = math.prod(lead)
    span = (count - 1) * hop + nfft
    ext = x.new_zeros(rows, span)
    ext[:, m - 1 : m - 1 + n] = x.reshape(rows, n)
    blocks = ext.as_strided((rows, count, nfft), (span, hop, 1))
    out = fft(fft(blocks.contiguous(), fft_impl=fft_impl) * h_spec, inverse=True, fft_impl=fft_impl)
    return out[..., nfft - hop :].reshape(rows, count * hop)[:, :n].reshape(*lead, n)


def fir(
    x: torch.Tensor, taps: torch.Tensor, *, nfft: int | None = None, fft_impl: str = DEFAULT_FFT_IMPL
) -> torch.Tensor:
    """Causal FIR filter y[j] = sum_k taps[k] x[j - k] with zero initial state (what
    scipy.signal.lfilter(taps, 1, x) computes), per row: complex64 (..., n) -> (..., n). taps
    may be real or complex. Computed by overlap-save in blocks of nfft samples (a power of two of
    at least len(taps); default_nfft() by default)."""
    _check_complex(x, "x")
    _check_backend(fft_impl)
    if taps.dim() != 1 or taps.numel() < 1:
        raise ValueError("taps must be a non-empty 1D tensor")
    m = taps.numel()
    block = default_nfft(m) if nfft is None else nfft
    if block < m or block & (block - 1):
        raise ValueError(f"nfft must be a power of two of at least len(taps) = {m}, got {block}")
    h_spec = taps_spectrum(taps, block, fft_impl=fft_impl, device=x.device)
    if _fused(fft_impl, block):
        return torch.ops.spectral.fir_overlap_save.default(x, h_spec, m, block, fft_impl)
    if x.numel() == 0:
        return x.new_empty(x.shape)
    return _overlap_save(x, h_spec, m, block, fft_impl)


# --- files and command line ---------------------------------------------------------------------


def read_cf32(path: Path) -> np.ndarray:
    """A .cf32 recording: interleaved little-endian float32 I/Q as complex64."""
    return np.fromfile(path, dtype=np.dtype("<c8"))


def write_cf32(path: Path, x: np.ndarray) -> None:
    np.ascontiguousarray(x, dtype=np.dtype("<c8")).tofile(path)


def read_f32(path: Path) -> np.ndarray:
    return np.fromfile(path, dtype=np.dtype("<f4"))


def _run_spectrum(args, x: torch.Tensor) -> torch.Tensor:
    return spectrum(x, args.nfft, window_name=args.window, fft_impl=args.fft_impl)


def _run_fir(args, x: torch.Tensor) -> torch.Tensor:
    taps = torch.from_numpy(read_f32(args.taps)).cuda()
    return fir(x, taps, nfft=args.nfft, fft_impl=args.fft_impl)


_COMMANDS = {
    "spectrum": ("windowed FFT of back-to-back frames", _run_spectrum),
    "fir": ("FIR filter by overlap-save", _run_fir),
}


def _parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="python -m spectral.rf",
                                     description="Spectrum and FIR filtering of .cf32 recordings on the GPU.")
    sub = parser.add_subparsers(dest="op", required=True)
    for name, (help_text, _) in _COMMANDS.items():
        p = sub.add_parser(name, help=help_text)
        p.add_argument("--in", dest="inp", type=Path, required=True)
        if name == "fir":
            p.add_argument("--taps", type=Path, required=True, help="raw float32 taps (.f32)")
        p.add_argument("--out", type=Path, required=True)
        if name == "spectrum":
            p.add_argument("--nfft", type=int, default=1024)
            p.add_argument("--window", choices=WINDOWS, default="rect")
        else:
            p.add_argument("--nfft", type=int, default=None, help="block size (default: about 4x taps)")
        p.add_argument("--fft-impl", choices=FFT_BACKENDS, default=DEFAULT_FFT_IMPL)
    return parser


def main(argv: list[str] | None = None) -> int:
    args = _parser().parse_args(argv)
    x = torch.from_numpy(read_cf32(args.inp)).cuda()
    y = _COMMANDS[args.op][1](args, x)
    write_cf32(args.out, y.reshape(-1).cpu().numpy())
    print(f"{args.op}[{args.fft_impl}]: {x.numel()} samples in, {y.numel()} out -> {args.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
