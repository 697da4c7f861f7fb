"""The tolerance policy and test helpers. TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

A restatement of the reference's python/spectral/testing.py with the limit tightened 4x:

    relative L2 error of each transform  <=  2 * eps_fp32 * log2 N     (N = N1 N2 in 2D)

(the reference allows 8 eps log2 N, testing.py:26-35). The error is normwise,
||actual - expected|| / ||expected|| over each transform's axes, so near-zero bins do not
dominate, and it is checked per transform so one bad transform cannot hide in a batch. Round
trips get twice the limit, as in the reference's tests (test_fft.py:57). A wrong index, twiddle
or race gives errors of order 1, far above any of these limits.

Truncated outputs (fft_truncated, rfft2_truncated) keep a few modes of a transform. Their
absolute error is that of the full transform, but a handful of kept modes of a random input can
be arbitrarily small (one kept mode is a sum that may cancel), so dividing by their own norm
measures the input's cancellation rather than the transform. assert_truncated_close therefore
divides by the norm the kept modes have on average: the full transform's norm scaled by
sqrt(kept / total).
"""

from __future__ import annotations

import math

import numpy as np

FLOAT32_EPS = float(np.finfo(np.float32).eps)  # 2^-23
FFT_TOLERANCE_FACTOR = 2.0

POW2_SIZES = [2**p for p in range(1, 13)]  # 2 .. 4096: one CTA per transform
BATCHES = [1, 3, 64]


def fft_tolerance(n: int, eps: float = FLOAT32_EPS) -> float:
    """The largest relative L2 error allowed for one transform of n points."""
    return FFT_TOLERANCE_FACTOR * eps * max(1.0, math.log2(n))


def to_numpy(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def relative_error(actual, expected, axes: tuple[int, ...]) -> np.ndarray:
    """||actual - expected|| / ||expected|| for each transform, norms over `axes`."""
    a = to_numpy(actual).astype(np.complex128)
    e = to_numpy(expected).astype(np.complex128)
    if a.shape != e.shape:
        raise AssertionError(f"shape {a.shape} differs from the expected {e.shape}")
    num = np.sqrt(np.sum(np.abs(a - e) ** 2, axis=axes))
    den = np.sqrt(np.sum(np.abs(e) ** 2, axis=axes))
    return num / np.maximum(den, np.finfo(np.float64).tiny)


def assert_transform_close(
    actual, expected, n: int, axes: tuple[int, ...] = (-1,), tol: float | None = None
) -> float:
    """Fails if any transform of the batch exceeds the tolerance for n points; returns the
    worst error."""
    tol = fft_tolerance(n) if tol is None else tol
    err = relative_error(actual, expected, axes)
    worst = float(np.max(err)) if np.size(err) else 0.0
    if worst > tol:
        where = np.unravel_index(int(np.argmax(err)), np.shape(err)) if np.ndim(err) else ()
        raise AssertionError(
            f"relative L2 error {worst:.3e} exceeds the tolerance {tol:.3e} "
            f"(n = {n}) in transform {tuple(int(i) for i in where)}"
        )
    return worst


def assert_truncated_close(
    actual, expected, full, n: int, axes: tuple[int, ...] = (-1,), tol: float | None = None
) -> float:
    """Like assert_transform_close for the kept modes `expected` of the full transform `full`."""
    tol = fft_tolerance(n) if tol is None else tol
    a = to_numpy(actual).astype(np.complex128)
    e = to_numpy(expected).astype(np.complex128)
    f = to_numpy(full).astype(np.complex128)
    if a.shape != e.shape:
        raise AssertionError(f"shape {a.shape} differs from the expected {e.shape}")
    kept = np.prod([e.shape[ax] for ax in axes])
    total = np.prod([f.shape[ax] for ax in axes])
    num = np.sqrt(np.sum(np.abs(a - e) ** 2, axis=axes))
    den = np.sqrt(np.sum(np.abs(f) ** 2, axis=axes) * (kept / total))
    err = num / np.maximum(den, np.finfo(np.float64).tiny)
    worst = float(np.max(err)) if np.size(err) else 0.0
    if worst > tol:
        where = np.unravel_index(int(np.argmax(err)), np.shape(err)) if np.ndim(err) else ()
        raise AssertionError(
            f"relative L2 error {worst:.3e} exceeds the tolerance {tol:.3e} "
            f"(n = {n}) in transform {tuple(int(i) for i in where)}"
        )
    return worst


def random_complex(rng: np.random.Generator, shape, dtype=np.complex64) -> np.ndarray:
    """Complex Gaussian samples of unit variance (half in each part)."""
    z = rng.standard_normal(shape) + 1j * rng.standard_normal(shape)
    return (z / math.sqrt(2.0)).astype(dtype)


def random_real(rng: np.random.Generator, shape, dtype=np.float32) -> np.ndarray:
    return rng.standard_normal(shape).astype(dtype)
