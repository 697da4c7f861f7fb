"""The slab-decomposed 2D transform's kernels on one GPU, with R ranks emulated: every "rank"
runs spectral_slab_rows on its rows, the all-to-all is a gather done with torch, and every rank
runs spectral_slab_columns on what it received. Checked against the float64 oracle: fully for
small fields, on sampled output columns for the 16384 x 16384 field of the benchmark (a float64
matrix-vector product per sampled column, then a 1D FFT)."""

import numpy as np
import pytest
import torch

from oracle.policy import FLOAT32_EPS, assert_transform_close, fft_tolerance
from spectral.distributed import columns_kernel, rows_kernel

pytestmark = pytest.mark.gpu


def forward_emulated(x: torch.Tensor, ranks: int) -> list[torch.Tensor]:
    n = x.shape[0]
    rows = n // ranks
    chunks = [rows_kernel(x[r * rows:(r + 1) * rows].contiguous(), n, rows, ranks, False)
              for r in range(ranks)]
    out = []
    for s in range(ranks):
        received = torch.stack([chunks[r][s] for r in range(ranks)])  # (ranks, rows, w)
        out.append(columns_kernel(received.reshape(n, n // ranks), n, n // ranks, False))
    return out


def inverse_emulated(cols: list[torch.Tensor], ranks: int) -> list[torch.Tensor]:
    n = cols[0].shape[0]
    rows = n // ranks
    done = [columns_kernel(c.clone(), n, n // ranks, True) for c in cols]
    return [rows_kernel(torch.stack([done[s][r * rows:(r + 1) * rows] for s in range(ranks)]),
                        n, rows, ranks, True) for r in range(ranks)]


@pytest.mark.parametrize("ranks", [1, 2, 4])
@pytest.mark.parametrize("n", [256, 1024, 8192])
def test_slab_forward_and_inverse_match_the_oracle(rng, n, ranks):
    if n == 8192 and ranks == 4:
        pytest.skip("covered by the smaller cases and the 16384 case")
    x = (rng.standard_normal((n, n)) + 1j * rng.standard_normal((n, n))).astype(np.complex64)
    xd = torch.from_numpy(x).cuda()
    cols = forward_emulated(xd, ranks)
    full = torch.cat(cols, dim=1).cpu().numpy()
    expected = np.fft.fft2(x.astype(np.complex128))
    # One 2D transform: the whole field is a single transform of n * n points.
    assert_transform_close(full[None], expected[None], n * n, axes=(-2, -1))
    back = torch.cat(inverse_emulated(cols, ranks), dim=0)
    assert_transform_close(back.cpu().numpy()[None], x[None], n * n, axes=(-2, -1),
                           tol=2 * fft_tolerance(n * n))


def test_benchmark_field_on_eight_ranks_sampled():
    # 16384 x 16384, N(0,1) real and imaginary parts, 8 ranks of 2048 rows.
    n, ranks = 16384, 8
    g = torch.Generator(device="cuda").manual_seed(4)
    xd = torch.complex(torch.randn(n, n, device="cuda", generator=g),
                       torch.randn(n, n, device="cuda", generator=g))
    cols = forward_emulated(xd, ranks)
    x = xd.cpu().numpy()
    w = n // ranks
    for k2 in [0, 1, 5000, 16383]:
        kernel = np.exp(-2j * np.pi * (np.arange(n) * k2 % n) / n)
        expected = np.fft.fft(x.astype(np.complex128) @ kernel)     # column k2 of fft2(x)
        got = cols[k2 // w][:, k2 % w].cpu().numpy()
        err = np.linalg.norm(got - expected) / np.linalg.norm(expected)
        assert err <= 2 * FLOAT32_EPS * 28, (k2, err)


def test_rejects_bad_shapes():
    x = torch.zeros(4, 12, dtype=torch.complex64, device="cuda")
    with pytest.raises(ValueError, match="power of two"):
        rows_kernel(x, 12, 4, 3, False)


@pytest.mark.parametrize(("ranks", "w"), [(1, 8), (2, 512), (4, 1), (8, 3), (16, 64)])
def test_relayout_moves_every_block(rng, ranks, w):
    # Blocks of w x w between the two sides, both directions, odd and even w (the 16-byte and the
    # 8-byte path), exact copies.
    from spectral.distributed import relayout_kernel

    n = ranks * w
    blocks = torch.from_numpy((rng.standard_normal((ranks, w, w)) + 1j * rng.standard_normal((ranks, w, w)))
                              .astype(np.complex64)).cuda()
    rows = torch.empty((w, n), dtype=torch.complex64, device="cuda")
    relayout_kernel(blocks, rows, ranks, w, [r * w * w for r in range(ranks)], w, [r * w for r in range(ranks)], n)
    assert torch.equal(rows, blocks.permute(1, 0, 2).reshape(w, n))
    back = torch.empty_like(blocks)
    relayout_kernel(rows, back, ranks, w, [r * w for r in range(ranks)], n, [r * w * w for r in range(ranks)], w)
    assert torch.equal(back, blocks)


def test_natural_layout_on_one_rank_is_the_full_transform(rng):
    from spectral.distributed import fft2_slab

    n = 1024
    x = (rng.standard_normal((n, n)) + 1j * rng.standard_normal((n, n))).astype(np.complex64)
    y = fft2_slab(torch.from_numpy(x).cuda(), layout="natural")
    assert y.shape == (n, n)
    assert_transform_close(y.cpu().numpy()[None], np.fft.fft2(x.astype(np.complex128))[None], n * n, axes=(-2, -1))
    back = fft2_slab(y, inverse=True, layout="natural")
    assert_transform_close(back.cpu().numpy()[None], x[None], n * n, axes=(-2, -1), tol=2 * fft_tolerance(n * n))


# --- the distributed 1D transform's kernels -------------------------------------------------------


@pytest.mark.parametrize(("n1", "width", "col0", "n"), [(64, 16, 48, 4096), (4096, 8, 4088, 1 << 24), (2, 1, 1, 4)])
@pytest.mark.parametrize("inverse", [False, True])
def test_twiddle_columns_match_the_oracle(rng, n1, width, col0, n, inverse):
    from spectral.distributed import twiddle_columns_kernel

    x = (rng.standard_normal((n1, width)) + 1j * rng.standard_normal((n1, width))).astype(np.complex64)
    y = twiddle_columns_kernel(torch.from_numpy(x).cuda(), n1, width, col0, n, inverse).cpu().numpy()
    a = x.astype(np.complex128)
    ref = np.fft.ifft(a, axis=0) if inverse else np.fft.fft(a, axis=0)
    k1 = np.arange(n1)[:, None]
    j2 = (col0 + np.arange(width))[None, :]
    ref = ref * np.exp((2j if inverse else -2j) * np.pi * ((k1 * j2) % n) / n)
    assert_transform_close(y.T, ref.T, n1, tol=2 * fft_tolerance(n1))


def test_transpose_entry_point(rng):
    from spectral.distributed import transpose_kernel

    x = torch.from_numpy((rng.standard_normal((96, 40)) + 1j * rng.standard_normal((96, 40))).astype(np.complex64)).cuda()
    assert torch.equal(transpose_kernel(x), x.t().contiguous())


@pytest.mark.parametrize("n", [16, 1 << 12, 1 << 17, 1 << 24])
def test_distributed_1d_transform_on_one_rank(rng, n):
    # One rank: the four-step path of fft_slab (twiddled columns, rows, transpose) against the
    # oracle, and back.
    from spectral.distributed import fft_slab

    x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
    y = fft_slab(torch.from_numpy(x).cuda())
    assert_transform_close(y.cpu().numpy()[None], np.fft.fft(x.astype(np.complex128))[None], n)
    back = fft_slab(y, inverse=True)
    assert_transform_close(back.cpu().numpy()[None], x[None], n, tol=2 * fft_tolerance(n))
