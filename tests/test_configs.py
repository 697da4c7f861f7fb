"""Parity at the five benchmark configurations, at their full shapes, distributions and seeds.

Each configuration's input is drawn exactly as the benchmark describes it (seed = the
configuration's index, float64 draws cast to float32 / complex64) and every transform is checked
against the float64 oracle per transform, at 2 eps log2 N relative L2 error (N = n1 n2 in 2D),
with round trips at twice that. A stage that consumes the previous stage's GPU output is checked
against the oracle applied to that same output, so each kernel is held to its own tolerance.

The pruned forward of configuration 4 is reported both ways: against the full transform's norm
scaled to the kept modes (oracle/policy.py: assert_truncated_close) and against the kept modes'
own norm, which is how the reference's tests/test_pruned.py:38-39 normalise it.

Configuration 5 (the 16384^2 slab) is checked at full size in tests/test_slab.py (one GPU,
emulated ranks) and tests/test_multi_gpu.py (two processes).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import spectral
from oracle import reference as ref
from oracle.policy import assert_transform_close, assert_truncated_close, fft_tolerance, relative_error

pytestmark = pytest.mark.gpu

IMPL = "stockham_r8"  # the benchmark's implementation; the others share the engine
EPS32 = float(np.finfo(np.float32).eps)


def cuda(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(x).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()


def report(name: str, worst: float, tol: float) -> None:
    print(f"{name}: worst relative L2 error {worst:.3e} (tolerance {tol:.3e}, {worst / tol:.2f} of it)")


# --- configuration 1: fft_c2c forward then inverse, 16384 x 1024 complex64 N(0, 1) ---------------


def test_config1_c2c_forward_then_inverse():
    rng = np.random.default_rng(0)
    shape = (16384, 1024)
    x = (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)
    f = spectral.fft_c2c(cuda(x), impl=IMPL)
    fh = host(f)
    report("cfg1 forward", assert_transform_close(fh, ref.fft(x), 1024), fft_tolerance(1024))
    g = host(spectral.fft_c2c(f, inverse=True, impl=IMPL))
    report("cfg1 inverse", assert_transform_close(g, ref.ifft(fh), 1024), fft_tolerance(1024))
    tol = 2 * fft_tolerance(1024)
    report("cfg1 round trip", assert_transform_close(g, x, 1024, tol=tol), tol)


# --- configuration 2: rfft then irfft, 4096 x 4096 float32 U[-1, 1] (the headline) ------------


def test_config2_rfft_then_irfft():
    rng = np.random.default_rng(1)
    x = rng.uniform(-1.0, 1.0, (4096, 4096)).astype(np.float32)
    s = spectral.rfft(cuda(x), impl=IMPL)
    assert s.shape == (4096, 2049)
    sh = host(s)
    report("cfg2 rfft", assert_transform_close(sh, ref.rfft(x), 4096), fft_tolerance(4096))
    y = host(spectral.irfft(s, 4096, impl=IMPL))
    report("cfg2 irfft", assert_transform_close(y, ref.irfft(sh, 4096), 4096), fft_tolerance(4096))
    tol = 2 * fft_tolerance(4096)
    report("cfg2 round trip", assert_transform_close(y, x, 4096, tol=tol), tol)


# --- configuration 3: rfft2 then irfft2, 256 fields of 256 x 256 float32 N(0, 1) ----------------


@pytest.fixture(scope="module")
def config3_input() -> tuple[np.ndarray, np.ndarray]:
    rng = np.random.default_rng(2)
    x = rng.standard_normal((256, 256, 256)).astype(np.float32)
    return x, ref.rfft2(x)


@pytest.mark.parametrize("columns", ["strided", "transpose"])
def test_config3_rfft2_then_irfft2(config3_input, columns):
    x, expected = config3_input
    n = 256 * 256
    s = spectral.rfft2(cuda(x), impl=IMPL, columns=columns)
    assert s.shape == (256, 256, 129)
    sh = host(s)
    report(f"cfg3 rfft2 {columns}", assert_transform_close(sh, expected, n, axes=(-2, -1)), fft_tolerance(n))
    y = host(spectral.irfft2(s, 256, impl=IMPL, columns=columns))
    report(f"cfg3 irfft2 {columns}",
           assert_transform_close(y, ref.irfft2(sh, (256, 256)), n, axes=(-2, -1)), fft_tolerance(n))
    tol = 2 * fft_tolerance(n)
    report(f"cfg3 round trip {columns}", assert_transform_close(y, x, n, axes=(-2, -1), tol=tol), tol)


def test_config3_strided_and_transpose_agree(config3_input):
    # Two column methods of the same transform: both within tolerance of the oracle (above), and
    # of each other at the round-trip limit.
    x, _ = config3_input
    xd = cuda(x)
    a = host(spectral.rfft2(xd, impl=IMPL, columns="strided"))
    b = host(spectral.rfft2(xd, impl=IMPL, columns="transpose"))
    assert_transform_close(a, b, 256 * 256, axes=(-2, -1), tol=2 * fft_tolerance(256 * 256))


# --- configuration 4: the FNO layer, 64 x 64 x 128 x 128, m1 = m2 = 16 ---------------------------


def test_config4_fno_layer():
    rng = np.random.default_rng(3)
    samples, channels, n, m = 64, 64, 128, 16
    x = rng.standard_normal((samples, channels, n, n)).astype(np.float32)
    wshape = (channels, channels, 2 * m, m)
    # iid N(0, 1 / (64 * 64)) per real and imaginary part
    w = ((rng.standard_normal(wshape) + 1j * rng.standard_normal(wshape)) / 64.0).astype(np.complex64)
    nn = n * n

    modes = spectral.rfft2_truncated(cuda(x), m, m, impl=IMPL)
    assert modes.shape == (samples, channels, 2 * m, m)
    mh = host(modes)
    full = ref.rfft2(x)
    kept = full[..., ref.mode_rows(n, m), :][..., :m]
    tol = fft_tolerance(nn)
    report("cfg4 rfft2_truncated (full-norm scaled)",
           assert_truncated_close(mh, kept, full, nn, axes=(-2, -1)), tol)
    # The reference's normalisation: the kept modes' own norm, same tolerance.
    own = float(np.max(relative_error(mh, kept, (-2, -1))))
    report("cfg4 rfft2_truncated (kept modes' own norm)", own, tol)
    assert own <= tol
    del full

    mixed = spectral.mode_contract(modes, cuda(w))
    xh = host(mixed)
    expected = ref.mode_contract(mh, w)
    # A 64-term complex dot product per output in FP32: 2 eps (log2 cin + 1), per output channel.
    ctol = 2 * EPS32 * (np.log2(channels) + 1)
    cerr = np.linalg.norm((xh - expected).reshape(samples, channels, -1), axis=-1) / np.maximum(
        np.linalg.norm(expected.reshape(samples, channels, -1), axis=-1), 1e-300)
    report("cfg4 mode_contract", float(cerr.max()), ctol)
    assert cerr.max() <= ctol

    y = host(spectral.irfft2_from_modes(mixed, (n, n), impl=IMPL))
    assert y.shape == (samples, channels, n, n)
    report("cfg4 irfft2_from_modes",
           assert_transform_close(y, ref.irfft2_from_modes(xh, (n, n)), nn, axes=(-2, -1)), tol)

    # The whole layer against the float64 layer on the float32 input and weights: the three
    # stages' limits added.
    layer = ref.irfft2_from_modes(ref.mode_contract(kept, w), (n, n))
    ltol = 2 * tol + ctol
    report("cfg4 layer end to end", assert_transform_close(y, layer, nn, axes=(-2, -1), tol=ltol), ltol)
