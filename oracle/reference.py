"""Float64 references for every transform of the hot path. TEST INFRASTRUCTURE ONLY (see
oracle/__init__.py).

A restatement of the reference's python/spectral/reference.py. Conventions (reference.py:3-12):
transforms act on the last axis (1D) or the last two (2D), leading axes are batch; forward
transforms are unnormalized, inverse ones divide by N (N1 N2 in 2D); real transforms keep the
N // 2 + 1 non-negative frequencies of the last axis. Everything is computed in complex128 /
float64 from whatever precision the input has, so a float32 result is compared against the
exact transform of the float32 values it was computed from.

The arithmetic is numpy's bundled pocketfft (numpy.fft; numpy 2.3.5 in this image, the
reference's only numerical dependency, requirements.txt:4 and pyproject.toml:10 there), exactly
as in the reference; the O(N^2) `dft` below is the definitional check of it.
"""

from __future__ import annotations

import numpy as np


def _c128(x) -> np.ndarray:
    return np.asarray(x, dtype=np.complex128)


def _f64(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64)


def dft(x) -> np.ndarray:
    """X[k] = sum_m x[m] exp(-2 pi i k m / n), by the definition (reference.py:28-34)."""
    x = _c128(x)
    n = x.shape[-1]
    idx = np.arange(n)
    # k m mod n keeps the angle small, so the exponentials stay accurate for large n.
    kernel = np.exp(-2j * np.pi * (np.outer(idx, idx) % max(n, 1)) / max(n, 1))
    return x @ kernel


def fft(x) -> np.ndarray:  # reference.py:37-38
    return np.fft.fft(_c128(x), axis=-1)


def ifft(x) -> np.ndarray:  # reference.py:41-42
    return np.fft.ifft(_c128(x), axis=-1)


def rfft(x) -> np.ndarray:  # reference.py:45-46
    return np.fft.rfft(_f64(x), axis=-1)


def irfft(x, n: int) -> np.ndarray:
    """Inverse of rfft for n output points (reference.py:49-52): the imaginary parts of bins 0
    and n/2 are ignored, as numpy and torch do."""
    return np.fft.irfft(_c128(x), n=n, axis=-1)


def fft2(x) -> np.ndarray:  # reference.py:55-56
    return np.fft.fft2(_c128(x), axes=(-2, -1))


def ifft2(x) -> np.ndarray:  # reference.py:59-60
    return np.fft.ifft2(_c128(x), axes=(-2, -1))


def rfft2(x) -> np.ndarray:  # reference.py:63-64
    return np.fft.rfft2(_f64(x), axes=(-2, -1))


def irfft2(x, shape: tuple[int, int]) -> np.ndarray:  # reference.py:67-68
    return np.fft.irfft2(_c128(x), s=shape, axes=(-2, -1))


def fft_truncate(x, k: int) -> np.ndarray:
    """The first k outputs of fft(x) (reference.py:71-76)."""
    n = np.shape(x)[-1]
    if not 0 < k <= n:
        raise ValueError(f"k must be in [1, {n}], got {k}")
    return fft(x)[..., :k]


def ifft_from_modes(modes, n: int) -> np.ndarray:
    """Inverse FFT of n points whose first k = modes.shape[-1] inputs are `modes`, the rest zero
    (the expectation of the reference's test_pruned.py:22-25)."""
    modes = _c128(modes)
    full = np.zeros(modes.shape[:-1] + (n,), dtype=np.complex128)
    full[..., : modes.shape[-1]] = modes
    return ifft(full)


def mode_rows(n1: int, m1: int) -> np.ndarray:
    """Row indices of the kept modes along an axis of n1 frequencies: 0 .. m1-1 (positive),
    then n1-m1 .. n1-1 (negative), the layout of reference.py:79-91."""
    return np.concatenate([np.arange(m1), np.arange(n1 - m1, n1)])


def rfft2_truncate(x, m1: int, m2: int) -> np.ndarray:
    """The (2 m1) x m2 low-frequency modes of rfft2(x) (reference.py:79-91)."""
    n1, n2 = np.shape(x)[-2:]
    if not (0 < 2 * m1 <= n1 and 0 < m2 <= n2 // 2 + 1):
        raise ValueError(f"need 0 < 2*m1 <= {n1} and 0 < m2 <= {n2 // 2 + 1}, got {m1}, {m2}")
    return rfft2(x)[..., mode_rows(n1, m1), :][..., :m2]


def irfft2_from_modes(modes, shape: tuple[int, int]) -> np.ndarray:
    """Inverse of rfft2_truncate: every dropped mode zero, then irfft2 (reference.py:94-105)."""
    modes = _c128(modes)
    n1, n2 = shape
    two_m1, m2 = modes.shape[-2:]
    if two_m1 % 2 or not (0 < two_m1 <= n1 and 0 < m2 <= n2 // 2 + 1):
        raise ValueError(f"modes of shape {modes.shape[-2:]} do not fit an output of {shape}")
    full = np.zeros(modes.shape[:-2] + (n1, n2 // 2 + 1), dtype=np.complex128)
    full[..., mode_rows(n1, two_m1 // 2), :m2] = modes
    return irfft2(full, shape)


def mode_contract(x, w) -> np.ndarray:
    """out[b, o, *m] = sum_i x[b, i, *m] w[i, o, *m] in complex128: the per-mode channel
    contraction of an FNO spectral convolution. The reference has no implementation of it
    (docs/ROADMAP.md:71-76 there); this einsum is its definition."""
    x = _c128(x)
    w = _c128(w)
    return np.einsum("bi...,io...->bo...", x, w)
