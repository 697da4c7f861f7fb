"""The pruned 2D real transforms by method: the FP32 engine (rows and columns by FFT passes) and the
tensor-core method (the rows' kept DFT outputs as a split-TF32 GEMM on tcgen05, the columns by the
engine), each against the float64 oracle (spectral.reference.rfft2_truncate) at the FFT
tolerance, with the kept modes' own norm as the reference's tests/test_pruned.py normalises it,
and against each other."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import reference as ref
from oracle.policy import (assert_transform_close, assert_truncated_close, fft_tolerance, random_complex, random_real,
                           relative_error)
from spectral import native

AUTO, FP32, TENSOR = 0, 1, 2
N = 128


def modes_by(x: torch.Tensor, m1: int, m2: int, method: int, impl: bytes = b"stockham_r8") -> torch.Tensor:
    fields = x.shape[0]
    out = torch.empty((fields, 2 * m1, m2), dtype=torch.complex64, device=x.device)
    native.call("spectral_rfft2_modes_method", impl, x.data_ptr(), out.data_ptr(), N, N, m1, m2, fields, method,
                None, torch.cuda.current_stream().cuda_stream)
    return out


def own_norm_error(actual: np.ndarray, expected: np.ndarray) -> float:
    return float(np.max(relative_error(actual, expected, (-2, -1))))


# (fields, m1, m2): the FNO configuration's kept block, the smallest, every kept row, ragged
# counts of fields against the 148-CTA grid (one field per CTA, several per CTA, an odd share per
# column group), and m2 below the 16 the operand holds.
CASES = [(1, 16, 16), (3, 1, 1), (5, 64, 16), (149, 16, 16), (300, 5, 11), (297, 16, 7), (1024, 16, 16)]


@pytest.mark.gpu
@pytest.mark.parametrize(("fields", "m1", "m2"), CASES)
@pytest.mark.parametrize("method", [FP32, TENSOR])
def test_methods_match_the_oracle(rng, fields, m1, m2, method):
    x = random_real(rng, (fields, N, N))
    y = modes_by(torch.from_numpy(x).cuda(), m1, m2, method).cpu().numpy()
    expected = ref.rfft2_truncate(x, m1, m2)
    tol = fft_tolerance(N * N)
    err = own_norm_error(y, expected)
    assert err <= tol, (err, tol)
    assert native.device_faults(clear=False) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("impl", [b"stockham_r2", b"stockham_r4", b"stockham_r8", b"stockham_r8_table"])
def test_tensor_method_serves_every_engine_name(rng, impl):
    x = random_real(rng, (33, N, N))
    y = modes_by(torch.from_numpy(x).cuda(), 16, 16, TENSOR, impl).cpu().numpy()
    assert own_norm_error(y, ref.rfft2_truncate(x, 16, 16)) <= fft_tolerance(N * N)


@pytest.mark.gpu
def test_tensor_and_fp32_methods_agree_and_the_tensor_method_repeats_exactly(rng):
    x = torch.from_numpy(random_real(rng, (512, N, N))).cuda()
    a = modes_by(x, 16, 16, TENSOR)
    b = modes_by(x, 16, 16, TENSOR)
    c = modes_by(x, 16, 16, FP32)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert own_norm_error(a.cpu().numpy(), c.cpu().numpy().astype(np.complex128)) <= 2 * fft_tolerance(N * N)
    assert native.device_faults(clear=False) == 0


@pytest.mark.gpu
def test_structured_inputs(rng):
    # A constant field (all energy in mode (0, 0)), single cosines on kept and dropped modes, and
    # large and small magnitudes in one batch: the split keeps each field's relative error.
    n1 = np.arange(N)[:, None]
    n2 = np.arange(N)[None, :]
    fields = [np.ones((N, N)), np.cos(2 * np.pi * (3 * n1 + 5 * n2) / N), np.cos(2 * np.pi * (40 * n1 + 50 * n2) / N)
              + np.cos(2 * np.pi * (120 * n1 + 2 * n2) / N), 1e6 * rng.standard_normal((N, N)),
              1e-6 * rng.standard_normal((N, N))]
    x = np.stack(fields).astype(np.float32)
    y = modes_by(torch.from_numpy(x).cuda(), 16, 16, TENSOR).cpu().numpy()
    # Errors against each field's whole spectrum (scaled to the kept share), since the field with
    # only dropped modes has no kept energy of its own to compare with.
    assert_truncated_close(y, ref.rfft2_truncate(x, 16, 16), ref.rfft2(x), N * N, axes=(-2, -1))


def test_method_argument_checks():
    # Refused before any CUDA call: the fake (aligned) pointers never reach a kernel.
    with pytest.raises(ValueError, match="method must be"):
        native.call("spectral_rfft2_modes_method", b"stockham_r8", 4096, 8192, N, N, 16, 16, 4, 3, None, None)
    for n1, n2, m1, m2, x in [(64, 128, 16, 16, 4096), (128, 256, 16, 16, 4096), (128, 128, 16, 17, 4096),
                              (128, 128, 16, 16, 4104)]:
        with pytest.raises(ValueError, match="tensor-core method needs"):
            native.call("spectral_rfft2_modes_method", b"stockham_r8", x, 1 << 20, n1, n2, m1, m2, 4, TENSOR, None,
                        None)
    with pytest.raises(ValueError, match="tensor-core method needs"):  # no fused kernel behind "naive"
        native.call("spectral_rfft2_modes_method", b"naive", 4096, 1 << 20, N, N, 16, 16, 4, TENSOR, 1 << 24, None)


# --- the inverse ------------------------------------------------------------------------------------


def inverse_by(modes: torch.Tensor, method: int, impl: bytes = b"stockham_r8") -> torch.Tensor:
    fields, rows, m2 = modes.shape
    y = torch.empty((fields, N, N), dtype=torch.float32, device=modes.device)
    native.call("spectral_irfft2_modes_method", impl, modes.data_ptr(), y.data_ptr(), N, N, rows // 2, m2, fields,
                method, None, torch.cuda.current_stream().cuda_stream)
    return y


@pytest.mark.gpu
@pytest.mark.parametrize(("fields", "m1", "m2"), CASES)
@pytest.mark.parametrize("method", [FP32, TENSOR])
def test_inverse_methods_match_the_oracle(rng, fields, m1, m2, method):
    # Random modes, the DC column's imaginary parts included: the real inverse drops them, as
    # numpy's irfft2 does.
    modes = random_complex(rng, (fields, 2 * m1, m2))
    y = inverse_by(torch.from_numpy(modes).cuda(), method).cpu().numpy()
    assert_transform_close(y, ref.irfft2_from_modes(modes, (N, N)), N * N, axes=(-2, -1))
    assert native.device_faults(clear=False) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("impl", [b"stockham_r2", b"stockham_r4", b"stockham_r8", b"stockham_r8_table"])
def test_inverse_tensor_method_serves_every_engine_name(rng, impl):
    modes = random_complex(rng, (33, 32, 16))
    y = inverse_by(torch.from_numpy(modes).cuda(), TENSOR, impl).cpu().numpy()
    assert_transform_close(y, ref.irfft2_from_modes(modes, (N, N)), N * N, axes=(-2, -1))


@pytest.mark.gpu
def test_inverse_methods_agree_the_tensor_method_repeats_and_round_trips(rng):
    x = torch.from_numpy(random_real(rng, (512, N, N))).cuda()
    modes = modes_by(x, 16, 16, TENSOR)
    a = inverse_by(modes, TENSOR)
    b = inverse_by(modes, TENSOR)
    c = inverse_by(modes, FP32)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert_transform_close(a.cpu().numpy(), c.cpu().numpy().astype(np.float64), N * N, axes=(-2, -1),
                           tol=2 * fft_tolerance(N * N))
    # Forward of the inverse, against the oracle's: not the modes themselves, since a DC-column
    # mode whose conjugate partner was not kept (kx = -m1) comes back halved by the real inverse.
    again = modes_by(a, 16, 16, TENSOR).cpu().numpy()
    expected = ref.rfft2_truncate(ref.irfft2_from_modes(modes.cpu().numpy(), (N, N)), 16, 16)
    assert own_norm_error(again, expected) <= 2 * fft_tolerance(N * N)
    assert native.device_faults(clear=False) == 0


def test_inverse_method_argument_checks():
    with pytest.raises(ValueError, match="method must be"):
        native.call("spectral_irfft2_modes_method", b"stockham_r8", 4096, 1 << 20, N, N, 16, 16, 4, 3, None, None)
    for n1, n2, m1, m2, y in [(64, 128, 16, 16, 1 << 20), (128, 256, 16, 16, 1 << 20), (128, 128, 16, 17, 1 << 20),
                              (128, 128, 16, 16, (1 << 20) + 8)]:
        with pytest.raises(ValueError, match="tensor-core method needs"):
            native.call("spectral_irfft2_modes_method", b"stockham_r8", 4096, y, n1, n2, m1, m2, 4, TENSOR, None,
                        None)
