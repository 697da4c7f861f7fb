"""Pins the oracle before any kernel is compared against it: against golden vectors made by the
reference's own python/spectral/reference.py (tests/golden/make_golden.py), against the DFT's
definition, and against the known answers of the reference's tests. Also checks the tolerance
policy. CPU only."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import policy
from oracle import reference as ref

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "reference_golden.npz")


def keys(prefix: str) -> list[str]:
    return sorted({k.rsplit("_", 1)[0] for k in GOLDEN.files if k.startswith(prefix)})


def same(actual, expected):
    # Both sides run numpy's pocketfft on the same float32 inputs: equal to the last bits up to
    # the library's own summation order; 1e-13 leaves room only for that.
    np.testing.assert_allclose(actual, expected, rtol=1e-13, atol=1e-13)


@pytest.mark.parametrize("n", [1, 2, 8, 64, 256])
def test_fft_and_ifft_match_the_reference_oracle(n):
    x = GOLDEN[f"fft_n{n}_x"]
    same(ref.fft(x), GOLDEN[f"fft_n{n}_y"])
    same(ref.ifft(x), GOLDEN[f"ifft_n{n}_y"])


@pytest.mark.parametrize("n", [3, 5, 12])
def test_dft_matches_the_reference_oracle(n):
    x = GOLDEN[f"dft_n{n}_x"]
    same(ref.dft(x), GOLDEN[f"dft_n{n}_y"])


@pytest.mark.parametrize("n", [2, 8, 64, 512])
def test_rfft_and_irfft_match_the_reference_oracle(n):
    same(ref.rfft(GOLDEN[f"rfft_n{n}_x"]), GOLDEN[f"rfft_n{n}_y"])
    same(ref.irfft(GOLDEN[f"irfft_n{n}_x"], n), GOLDEN[f"irfft_n{n}_y"])


@pytest.mark.parametrize("shape", [(8, 16), (16, 8), (32, 32)])
def test_2d_transforms_match_the_reference_oracle(shape):
    n1, n2 = shape
    t = f"{n1}x{n2}"
    same(ref.fft2(GOLDEN[f"fft2_{t}_x"]), GOLDEN[f"fft2_{t}_y"])
    same(ref.ifft2(GOLDEN[f"fft2_{t}_x"]), GOLDEN[f"ifft2_{t}_y"])
    same(ref.rfft2(GOLDEN[f"rfft2_{t}_x"]), GOLDEN[f"rfft2_{t}_y"])
    same(ref.irfft2(GOLDEN[f"irfft2_{t}_x"], shape), GOLDEN[f"irfft2_{t}_y"])


@pytest.mark.parametrize(("n", "k"), [(64, 16), (8, 3), (1, 1)])
def test_fft_truncate_matches_the_reference_oracle(n, k):
    same(ref.fft_truncate(GOLDEN[f"trunc_n{n}_k{k}_x"], k), GOLDEN[f"trunc_n{n}_k{k}_y"])


@pytest.mark.parametrize("case", [(16, 16, 3, 4), (64, 32, 12, 12), (8, 8, 4, 5), (32, 64, 8, 8)])
def test_mode_layout_matches_the_reference_oracle_bit_for_bit(case):
    n1, n2, m1, m2 = case
    tag = f"modes_{n1}x{n2}_m{m1}x{m2}"
    # The mode gather and scatter are pure index work: exactly equal, not merely close.
    np.testing.assert_array_equal(ref.rfft2_truncate(GOLDEN[f"{tag}_x"], m1, m2), GOLDEN[f"{tag}_y"])
    same(ref.irfft2_from_modes(GOLDEN[f"{tag}_modes"], (n1, n2)), GOLDEN[f"{tag}_inv"])


# --- known answers (the reference's test_reference.py:22-74, test_fft.py:144-158) ----------------


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 12, 16, 31, 64])
def test_fft_matches_the_definition(rng, n):
    x = policy.random_complex(rng, (4, n))
    np.testing.assert_allclose(ref.fft(x), ref.dft(x), rtol=0, atol=1e-10 * n)


@pytest.mark.parametrize("n", [2, 64, 4096])
def test_ifft_inverts_fft(rng, n):
    x = policy.random_complex(rng, (3, n))
    np.testing.assert_allclose(ref.ifft(ref.fft(x)), x, rtol=0, atol=1e-12)


@pytest.mark.parametrize("n", [8, 9, 64])
def test_rfft_is_the_nonnegative_half_of_fft(rng, n):
    x = policy.random_real(rng, (3, n))
    np.testing.assert_allclose(ref.rfft(x), ref.fft(x)[..., : n // 2 + 1], rtol=0, atol=1e-10)


def test_fft2_is_rows_then_columns(rng):
    x = policy.random_complex(rng, (2, 8, 16))
    np.testing.assert_allclose(ref.fft2(x), np.fft.fft(ref.fft(x), axis=-2), rtol=0, atol=1e-10)


def test_impulse_transforms_to_all_ones():
    x = np.zeros((1, 256), dtype=np.complex64)
    x[0, 0] = 1
    np.testing.assert_array_equal(ref.fft(x), np.ones((1, 256)))


def test_single_frequency_lands_in_one_bin():
    n, k0 = 256, 5
    x = np.exp(2j * np.pi * k0 * np.arange(n) / n)[None, :]
    expected = np.zeros((1, n), dtype=np.complex128)
    expected[0, k0] = n
    np.testing.assert_allclose(ref.fft(x), expected, atol=1e-9)


def test_constant_lands_in_bin_zero():
    expected = np.zeros((1, 65))
    expected[0, 0] = 128
    np.testing.assert_allclose(ref.rfft(np.ones((1, 128), dtype=np.float32)), expected, atol=1e-12)


def test_truncation_is_a_low_pass_filter():
    i, j = np.meshgrid(np.arange(32), np.arange(32), indexing="ij")
    low = np.cos(2 * np.pi * (1 * i + 2 * j) / 32)
    high = np.cos(2 * np.pi * (10 * i + 12 * j) / 32)
    modes = ref.rfft2_truncate(low + high, m1=4, m2=4)
    np.testing.assert_allclose(ref.irfft2_from_modes(modes, (32, 32)), low, rtol=0, atol=1e-12)


def test_keeping_every_mode_round_trips(rng):
    x = policy.random_real(rng, (2, 8, 8))
    modes = ref.rfft2_truncate(x, m1=4, m2=5)
    np.testing.assert_allclose(ref.irfft2_from_modes(modes, (8, 8)), x, rtol=0, atol=1e-12)


def test_ifft_from_modes_zero_fills(rng):
    modes = policy.random_complex(rng, (3, 5))
    full = np.zeros((3, 16), dtype=np.complex128)
    full[:, :5] = modes
    np.testing.assert_allclose(ref.ifft_from_modes(modes, 16), np.fft.ifft(full), atol=1e-15)


def test_mode_contract_is_a_per_mode_matrix_product(rng):
    x = policy.random_complex(rng, (3, 4, 2, 5))
    w = policy.random_complex(rng, (4, 6, 2, 5))
    out = ref.mode_contract(x, w)
    for a in range(2):
        for b in range(5):
            np.testing.assert_allclose(
                out[:, :, a, b], x[:, :, a, b].astype(np.complex128) @ w[:, :, a, b], atol=1e-12
            )


def test_rejects_modes_that_do_not_fit():
    with pytest.raises(ValueError):
        ref.rfft2_truncate(np.zeros((8, 8)), 5, 2)
    with pytest.raises(ValueError):
        ref.irfft2_from_modes(np.zeros((3, 2), dtype=np.complex64), (8, 8))


# --- the policy ---------------------------------------------------------------------------------


@pytest.mark.parametrize("n", policy.POW2_SIZES)
def test_policy_accepts_float32_rounding_of_the_exact_result(rng, n):
    x = policy.random_complex(rng, (8, n))
    exact = ref.fft(x)
    policy.assert_transform_close(exact.astype(np.complex64), exact, n)


def test_policy_rejects_one_bad_transform_in_a_batch(rng):
    n = 1024
    exact = ref.fft(policy.random_complex(rng, (64, n)))
    actual = exact.copy()
    actual[17, 5] += 10 * policy.fft_tolerance(n) * np.linalg.norm(exact[17])
    with pytest.raises(AssertionError, match=r"exceeds the tolerance .* in transform \(17,\)"):
        policy.assert_transform_close(actual, exact, n)


def test_truncated_policy_scales_by_the_full_transform(rng):
    # One kept mode that cancels to almost nothing: its own norm would make a rounding-level
    # error look huge; against the full transform's scale it is rounding-level.
    n = 8
    x = policy.random_complex(rng, (1, n)).astype(np.complex128)
    x[0, -1] -= x.sum()  # X[0] = sum(x) = 0
    full = ref.fft(x)
    kept = full[:, :1]
    noisy = kept + 1e-8
    with pytest.raises(AssertionError):
        policy.assert_transform_close(noisy, kept, n)
    policy.assert_truncated_close(noisy, kept, full, n)


def test_policy_limit_is_two_eps_per_stage():
    assert policy.fft_tolerance(4096) == pytest.approx(2 * policy.FLOAT32_EPS * 12)
    assert policy.fft_tolerance(2) == pytest.approx(2 * policy.FLOAT32_EPS)


def test_torch_cpu_fft_meets_the_policy(rng):
    # A production float32 FFT (pocketfft) passes at every size: the bar is attainable.
    for n in policy.POW2_SIZES:
        x = policy.random_complex(rng, (64, n))
        policy.assert_transform_close(torch.fft.fft(torch.from_numpy(x)), ref.fft(x), n)
        r = policy.random_real(rng, (64, n))
        policy.assert_transform_close(torch.fft.rfft(torch.from_numpy(r)), ref.rfft(r), n)
