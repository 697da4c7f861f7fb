"""Pruned (FNO) transforms against the float64 oracle for every implementation, the mode
layout bit-exact (the reference's tests/test_pruned.py), and the per-mode contraction."""

import numpy as np
import pytest
import torch

import spectral
from oracle import reference as ref
from oracle.policy import (
    assert_transform_close,
    assert_truncated_close,
    fft_tolerance,
    random_complex,
    random_real,
)

pytestmark = pytest.mark.gpu

IMPLS = spectral.FFT_IMPLS
AXES = (-2, -1)


def cuda(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(x).cuda()


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize(("n", "k"), [(1, 1), (8, 1), (8, 3), (64, 16), (256, 255), (4096, 32)])
@pytest.mark.parametrize("batch", [1, 3, 300])
def test_fft_truncated_matches_the_oracle(rng, impl, n, k, batch):
    x = random_complex(rng, (batch, n))
    y = spectral.fft_truncated(cuda(x), k, impl=impl)
    assert y.shape == (batch, k)
    # The kept modes against the full transform's scale (oracle/policy.py explains why).
    assert_truncated_close(y, ref.fft_truncate(x, k), ref.fft(x), n)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize(("n", "k"), [(1, 1), (8, 1), (8, 3), (64, 16), (256, 255), (4096, 32)])
@pytest.mark.parametrize("batch", [1, 3, 300])
def test_ifft_from_modes_matches_the_oracle(rng, impl, n, k, batch):
    modes = random_complex(rng, (batch, k))
    y = spectral.ifft_from_modes(cuda(modes), n, impl=impl)
    assert y.shape == (batch, n)
    assert_transform_close(y, ref.ifft_from_modes(modes, n), n)


@pytest.mark.parametrize("impl", IMPLS)
def test_keeping_every_mode_is_the_full_transform(rng, impl):
    x = cuda(random_complex(rng, (5, 128)))
    assert torch.equal(spectral.fft_truncated(x, 128, impl=impl), spectral.fft_c2c(x, impl=impl))


CASES_2D = [
    (2, 2, 1, 1),
    (8, 8, 2, 3),
    (16, 16, 8, 9),
    (64, 32, 12, 12),
    (32, 128, 4, 20),
    (128, 128, 16, 16),
    (256, 256, 16, 16),
    (4096, 2, 2, 2),
    (2, 8192, 1, 64),
]


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize(("n1", "n2", "m1", "m2"), CASES_2D)
def test_rfft2_truncated_matches_the_oracle(rng, impl, n1, n2, m1, m2):
    x = random_real(rng, (3, n1, n2))
    y = spectral.rfft2_truncated(cuda(x), m1, m2, impl=impl)
    assert y.shape == (3, 2 * m1, m2)
    assert_truncated_close(y, ref.rfft2_truncate(x, m1, m2), ref.rfft2(x), n1 * n2, axes=AXES)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize(("n1", "n2", "m1", "m2"), CASES_2D)
def test_irfft2_from_modes_matches_the_oracle(rng, impl, n1, n2, m1, m2):
    modes = random_complex(rng, (3, 2 * m1, m2))
    y = spectral.irfft2_from_modes(cuda(modes), (n1, n2), impl=impl)
    assert y.shape == (3, n1, n2)
    assert_transform_close(y, ref.irfft2_from_modes(modes, (n1, n2)), n1 * n2, axes=AXES)


@pytest.mark.parametrize("impl", IMPLS)
def test_mode_layout_is_the_full_transform_gathered(rng, impl):
    # The kept modes are exactly the rows/columns of the full rfft2 the layout names: compare the
    # pruned output with the engine's own full transform gathered on the host, per mode.
    n1, n2, m1, m2 = 64, 64, 8, 8
    x = cuda(random_real(rng, (2, n1, n2)))
    modes = spectral.rfft2_truncated(x, m1, m2, impl=impl).cpu().numpy()
    full = spectral.rfft2(x, impl=impl).cpu().numpy()
    gathered = full[..., ref.mode_rows(n1, m1), :][..., :m2]
    assert_transform_close(modes, gathered, n1 * n2, axes=AXES)


@pytest.mark.parametrize("impl", IMPLS)
def test_a_band_limited_field_survives_the_round_trip(rng, impl):
    n1, n2, m1, m2 = 64, 64, 8, 8
    modes = ref.rfft2_truncate(random_real(rng, (2, n1, n2)), m1, m2)
    modes[..., m1, 0] = 0
    field = ref.irfft2_from_modes(modes, (n1, n2)).astype(np.float32)
    back = spectral.irfft2_from_modes(
        spectral.rfft2_truncated(cuda(field), m1, m2, impl=impl), (n1, n2), impl=impl
    )
    assert_transform_close(back, field, n1 * n2, axes=AXES, tol=2 * fft_tolerance(n1 * n2))


@pytest.mark.parametrize("impl", IMPLS)
def test_many_arrays_and_leading_dimensions(rng, impl):
    x = random_real(rng, (2, 70, 16, 32))
    y = spectral.rfft2_truncated(cuda(x), 4, 5, impl=impl)
    assert y.shape == (2, 70, 8, 5)
    assert_truncated_close(y, ref.rfft2_truncate(x, 4, 5), ref.rfft2(x), 512, axes=AXES)


def test_every_implementation_agrees(rng):
    x = cuda(random_real(rng, (4, 128, 128)))
    results = [spectral.rfft2_truncated(x, 12, 12, impl=impl) for impl in IMPLS]
    for r in results[1:]:
        assert_transform_close(r, results[0], 128 * 128, axes=AXES, tol=2 * fft_tolerance(2**14))


def test_rejects_modes_that_do_not_fit():
    x = torch.zeros(8, 8, device="cuda")
    with pytest.raises(RuntimeError, match="1 <= m1 <= n1/2"):
        spectral.rfft2_truncated(x, 5, 2)
    with pytest.raises(RuntimeError, match="1 <= m1 <= n1/2"):
        spectral.rfft2_truncated(x, 2, 6)
    with pytest.raises(RuntimeError, match="do not fit"):
        spectral.irfft2_from_modes(torch.zeros(3, 2, dtype=torch.complex64, device="cuda"), (8, 8))


def test_rejects_keep_out_of_range():
    x = torch.zeros(2, 8, dtype=torch.complex64, device="cuda")
    with pytest.raises(RuntimeError, match="1 <= keep <= n"):
        spectral.fft_truncated(x, 9)
    with pytest.raises(RuntimeError, match="1 <= keep <= n"):
        spectral.ifft_from_modes(x, 4)


# --- the per-mode contraction of the FNO layer --------------------------------------------------


@pytest.mark.parametrize(("batch", "cin", "cout", "modes"), [(3, 5, 7, (4, 3)), (64, 64, 64, (32, 16)),
                                                             (9, 64, 70, (32, 16)), (1, 1, 1, (1, 1)),
                                                             (16, 4, 16, (4, 8)), (32, 12, 48, (8, 8))])
def test_mode_contract_matches_the_oracle(rng, batch, cin, cout, modes):
    x = random_complex(rng, (batch, cin, *modes))
    w = (random_complex(rng, (cin, cout, *modes)) / np.sqrt(cin)).astype(np.complex64)
    y = spectral.mode_contract(cuda(x), cuda(w)).cpu().numpy()
    expected = ref.mode_contract(x, w)
    # Each output is a cin-term complex dot product in FP32: relative error per output channel
    # grows like eps sqrt(cin); 2 eps log2(cin) + 2 eps bounds it with room to spare.
    tol = 2 * np.finfo(np.float32).eps * (np.log2(max(cin, 2)) + 1)
    err = np.linalg.norm((y - expected).reshape(batch, cout, -1), axis=-1) / np.maximum(
        np.linalg.norm(expected.reshape(batch, cout, -1), axis=-1), 1e-300)
    assert err.max() <= tol, err.max()


def test_mode_contract_staged_and_direct_kernels_agree_exactly(rng):
    # Shapes that tile by 32 modes x 16 outputs x 16 samples take the shared-memory staged
    # kernel; the same data 8 bytes off a 16-byte boundary takes the direct one. Both sum the
    # channels in the same order with the same operations.
    from spectral import native

    batch, cin, cout, modes = 32, 8, 32, 64
    x = cuda(random_complex(rng, (batch, cin, modes)))
    w = cuda((random_complex(rng, (cin, cout, modes)) / np.sqrt(cin)).astype(np.complex64))
    staged = spectral.mode_contract(x, w)
    xo = torch.empty(x.numel() + 1, dtype=torch.complex64, device="cuda")
    xo[1:] = x.reshape(-1)
    direct = torch.empty_like(staged)
    native.call("spectral_mode_contract", xo.data_ptr() + 8, w.data_ptr(), direct.data_ptr(), batch,
                cin, cout, modes, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(staged, direct)

