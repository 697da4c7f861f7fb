"""Float64 references for the radio-signal consumers of the transforms: periodic windows, the
framed spectrum and causal FIR filtering. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

A restatement of the semantics of the reference's python/spectral/rf.py:

    window(name, n)        rf.py:54-80   periodic window, computed in float64, returned float32
    frames(x, nfft)        rf.py:86-91   back-to-back frames, the last one zero-padded
    spectrum(x, nfft, w)   rf.py:94-102  FFT of each frame times the window
    default_nfft(m)        rf.py:108-117 overlap-save block size for m taps
    fir(x, taps)           rf.py:120-153 y[j] = sum_k taps[k] x[j - k], zero initial state

The reference computes fir by overlap-save; the restatement here is the definition (a direct
convolution truncated to the signal's length, scipy.signal.lfilter(taps, 1, x) for a row),
which is what overlap-save must reproduce, so the check does not share the algorithm it checks.
Everything is float64 / complex128.
"""

from __future__ import annotations

import math

import numpy as np

WINDOWS: tuple[str, ...] = ("rect", "hann", "hamming", "blackman")


def window(name: str, n: int) -> np.ndarray:
    """The periodic window of n points as float32 (rf.py:54-80): the cosine-sum formulas with
    phase 2 pi k / n evaluated in float64, then rounded to float32; one point gives [1]."""
    if n < 1:
        raise ValueError(f"a window needs at least one point, got {n}")
    if name not in WINDOWS:
        raise ValueError(f"unknown window '{name}' (available: {', '.join(WINDOWS)})")
    if n == 1:
        return np.ones(1, dtype=np.float32)
    phase = 2.0 * np.pi * np.arange(n) / n
    coeffs = {"rect": (1.0,), "hann": (0.5, 0.5), "hamming": (0.54, 0.46), "blackman": (0.42, 0.5, 0.08)}
    w = np.zeros(n)
    for j, a in enumerate(coeffs[name]):
        w = w + (a if j == 0 else (-a if j % 2 else a) * np.cos(j * phase))
    return w.astype(np.float32)


def frames(x, nfft: int) -> np.ndarray:
    """(..., n) -> (..., max(1, ceil(n / nfft)), nfft), zero-padded (rf.py:86-91)."""
    x = np.asarray(x)
    n = x.shape[-1]
    count = max(1, math.ceil(n / nfft))
    padded = np.zeros(x.shape[:-1] + (count * nfft,), dtype=np.complex128)
    padded[..., :n] = x
    return padded.reshape(x.shape[:-1] + (count, nfft))


def spectrum(x, nfft: int, window_name: str = "rect") -> np.ndarray:
    """np.fft.fft of each frame times the float32 window (rf.py:94-102), in complex128."""
    w = window(window_name, nfft).astype(np.float64)
    return np.fft.fft(frames(x, nfft) * w, axis=-1)


def default_nfft(num_taps: int) -> int:
    """A power of two about four times the filter length, 64 .. 4096; longer filters get the next
    power of two above their length (rf.py:108-117)."""
    if num_taps < 1:
        raise ValueError("the filter needs at least one tap")
    nfft = 1 << max(6, math.ceil(math.log2(4 * num_taps)))
    if nfft > 4096:
        nfft = max(4096, 1 << math.ceil(math.log2(num_taps)))
    return nfft


def fir(x, taps) -> np.ndarray:
    """y[..., j] = sum_k taps[k] x[..., j - k] for j < n, x zero before 0 (rf.py:120-131): the
    direct convolution of each row, truncated to its length."""
    x = np.asarray(x, dtype=np.complex128)
    taps = np.asarray(taps, dtype=np.complex128)
    n = x.shape[-1]
    rows = x.reshape(-1, n)
    out = np.empty_like(rows)
    for r in range(rows.shape[0]):
        out[r] = np.convolve(rows[r], taps)[:n]
    return out.reshape(x.shape)


def fir_overlap_save(x, taps, nfft: int | None = None) -> np.ndarray:
    """The same filter by the reference's own algorithm (rf.py:139-153) in complex128: blocks of
    nfft samples of x after len(taps) - 1 zeros, step nfft - len(taps) + 1, each transformed,
    multiplied by the spectrum of the zero-padded taps and transformed back, the first
    len(taps) - 1 outputs of each block dropped. The CPU baseline's method; fir() checks it."""
    x = np.asarray(x, dtype=np.complex128)
    taps = np.asarray(taps, dtype=np.complex128)
    m = taps.shape[0]
    nfft = default_nfft(m) if nfft is None else nfft
    step = nfft - m + 1
    n = x.shape[-1]
    blocks = max(1, math.ceil(n / step))
    padded = np.zeros(x.shape[:-1] + (m - 1 + blocks * step,), dtype=np.complex128)
    padded[..., m - 1 : m - 1 + n] = x
    idx = np.arange(blocks)[:, None] * step + np.arange(nfft)[None, :]
    h = np.fft.fft(taps, n=nfft)
    y = np.fft.ifft(np.fft.fft(padded[..., idx], axis=-1) * h, axis=-1)[..., m - 1 :]
    return y.reshape(x.shape[:-1] + (blocks * step,))[..., :n]
