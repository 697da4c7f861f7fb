"""The large single-field 2D complex FFT, slab-decomposed over the ranks of a process group.

An n x n complex64 field (n a power of two up to 16384) is split by rows: with R ranks, rank r
holds rows [r n/R, (r+1) n/R). The forward transform runs

    1. the rank's row transforms (spectral_slab_rows), stored as R chunks of w = n/R columns;
    2. one all-to-all of those chunks (torch.distributed, NCCL over NVLink on GPUs);
    3. the column transforms of the received n x w column slab (spectral_slab_columns),

and returns the rank's w columns of the 2D transform, as an (n, w) tensor in natural order:
element [k1, c] is X[k1, r w + c]. The inverse takes that column slab back to the rank's rows of
ifft2 (divided by n^2). The reference cannot run this case (its fft2 stops at 4096 per side and it
has no multi-GPU code); batched transforms need no communication and use the plain operators.

The kernel steps are arguments, so the index arithmetic of the decomposition can be tested on
CPU ranks (gloo) with stand-ins; the defaults are the library's CUDA kernels.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist

from . import native


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def rows_kernel(x: torch.Tensor, n: int, rows: int, ranks: int, inverse: bool) -> torch.Tensor:
    """Forward: (rows, n) -> chunks (ranks, rows, n/ranks). Inverse: chunks -> (rows, n)."""
    shape = (rows, n) if inverse else (ranks, rows, n // ranks)
    y = torch.empty(shape, dtype=torch.complex64, device=x.device)
    native.call("spectral_slab_rows", x.data_ptr(), y.data_ptr(), n, rows, ranks,
                1 if inverse else 0, _stream())
    return y


def columns_kernel(x: torch.Tensor, n: int, width: int, inverse: bool) -> torch.Tensor:
    """n-point transforms down the columns of an (n, width) matrix; x is used as scratch."""
    y = torch.empty((n, width), dtype=torch.complex64, device=x.device)
    native.call("spectral_slab_columns", x.data_ptr(), y.data_ptr(), n, width,
                1 if inverse else 0, _stream())
    return y


def _world(group) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def _exchange(send: torch.Tensor, group) -> torch.Tensor:
    ranks, _ = _world(group)
    if ranks == 1:
        return send
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send.contiguous(), group=group)
    return recv


def fft2_slab(
    x: torch.Tensor,
    *,
    inverse: bool = False,
    group=None,
    rows_fn: Callable = rows_kernel,
    columns_fn: Callable = columns_kernel,
) -> torch.Tensor:
    """Forward: x is this rank's (n / R, n) row slab; returns its (n, n / R) column slab of fft2.
    Inverse: x is the (n, n / R) column slab; returns the (n / R, n) row slab of ifft2."""
    ranks, _ = _world(group)
    if x.dtype != torch.complex64 or x.dim() != 2:
        raise ValueError("fft2_slab: x must be a 2D complex64 tensor")
    if not inverse:
        rows, n = x.shape
        if rows * ranks != n:
            raise ValueError(f"fft2_slab: {ranks} ranks of {rows} rows do not make a {n} x {n} field")
        chunks = rows_fn(x.contiguous(), n, rows, ranks, False)         # (ranks, rows, w)
        received = _exchange(chunks, group)                             # (ranks, rows, w)
        return columns_fn(received.reshape(n, n // ranks), n, n // ranks, False)
    n, w = x.shape
    if w * ranks != n:
        raise ValueError(f"fft2_slab: {ranks} ranks of {w} columns do not make a {n} x {n} field")
    cols = columns_fn(x.contiguous().clone(), n, w, True)                # (n, w) = (ranks, rows, w)
    received = _exchange(cols.reshape(ranks, n // ranks, w), group)
    return rows_fn(received, n, n // ranks, ranks, True)
