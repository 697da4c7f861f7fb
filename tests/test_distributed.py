"""The slab decomposition of the large 2D transform on CPU ranks (gloo): the chunk layout, the
all-to-all, the column slab and the natural-layout second exchange, with numpy stand-ins for the
kernels (whose layouts the GPU
tests in test_slab.py check). world_size 2 and 4, spawned processes."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N = 32


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def field() -> np.ndarray:
    rng = np.random.default_rng(5)
    return (rng.standard_normal((N, N)) + 1j * rng.standard_normal((N, N))).astype(np.complex64)


def rows_stub(x, n, rows, ranks, inverse):
    a = x.numpy().astype(np.complex128)
    if not inverse:
        y = np.fft.fft(a, axis=1).reshape(rows, ranks, n // ranks).transpose(1, 0, 2)
    else:
        y = np.fft.ifft(a.transpose(1, 0, 2).reshape(rows, n), axis=1)
    return torch.from_numpy(np.ascontiguousarray(y).astype(np.complex64))


def columns_stub(x, n, width, inverse):
    a = x.numpy().astype(np.complex128)
    y = np.fft.ifft(a, axis=0) if inverse else np.fft.fft(a, axis=0)
    return torch.from_numpy(y.astype(np.complex64))


def relayout_stub(src, dst, ranks, w, src_offsets, src_stride, dst_offsets, dst_stride, h=None):
    """The relayout kernel's contract on flat CPU tensors: block r, h (default w) rows of w values."""
    s, d = src.reshape(-1), dst.reshape(-1)
    for r in range(ranks):
        for k in range(w if h is None else h):
            a, b = src_offsets[r] + k * src_stride, dst_offsets[r] + k * dst_stride
            d[b:b + w] = s[a:a + w]


def worker(rank: int, world: int, port: int, out: dict) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "gpu-spectral-stack_b200"))
        from spectral.distributed import fft2_slab

        rows = N // world
        x = torch.from_numpy(field()[rank * rows:(rank + 1) * rows])
        cols = fft2_slab(x, rows_fn=rows_stub, columns_fn=columns_stub)
        gathered = [torch.empty_like(cols) for _ in range(world)]
        dist.all_gather(gathered, cols)
        back = fft2_slab(cols, inverse=True, rows_fn=rows_stub, columns_fn=columns_stub)
        every = [torch.empty_like(back) for _ in range(world)]
        dist.all_gather(every, back)
        # Natural layout: the second exchange returns the rank's rows of fft2, and the natural
        # inverse takes them back to the rank's rows of the field.
        stubs = dict(rows_fn=rows_stub, columns_fn=columns_stub, relayout_fn=relayout_stub)
        nat = fft2_slab(x, layout="natural", **stubs)
        nat_rows = [torch.empty_like(nat) for _ in range(world)]
        dist.all_gather(nat_rows, nat)
        nat_back = fft2_slab(nat, inverse=True, layout="natural", **stubs)
        nat_every = [torch.empty_like(nat_back) for _ in range(world)]
        dist.all_gather(nat_every, nat_back)
        if rank == 0:
            out["forward"] = torch.cat(gathered, dim=1).numpy()
            out["inverse"] = torch.cat(every, dim=0).numpy()
            out["natural"] = torch.cat(nat_rows, dim=0).numpy()
            out["natural_inverse"] = torch.cat(nat_every, dim=0).numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_slab_decomposition_on_gloo_ranks(world):
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(worker, args=(world, free_port(), out), nprocs=world, start_method="spawn")
    expected = np.fft.fft2(field().astype(np.complex128))
    np.testing.assert_allclose(out["forward"], expected, rtol=0, atol=1e-4 * np.abs(expected).max())
    np.testing.assert_allclose(out["inverse"], field(), rtol=0, atol=1e-5)
    np.testing.assert_array_equal(out["natural"], out["forward"])
    np.testing.assert_allclose(out["natural_inverse"], field(), rtol=0, atol=1e-5)


# --- the distributed 1D transform ---------------------------------------------------------------


def twiddle_stub(x, n1, width, col0, n, inverse):
    a = x.numpy().astype(np.complex128)
    y = np.fft.ifft(a, axis=0) if inverse else np.fft.fft(a, axis=0)
    k1 = np.arange(n1)[:, None]
    j2 = (col0 + np.arange(width))[None, :]
    y = y * np.exp((2j if inverse else -2j) * np.pi * (k1 * j2) / n)
    return torch.from_numpy(y.astype(np.complex64))


def rows1d_stub(x, n2, inverse):
    a = x.numpy().astype(np.complex128)
    return torch.from_numpy((np.fft.ifft(a, axis=1) if inverse else np.fft.fft(a, axis=1)).astype(np.complex64))


def transpose_stub(x):
    return x.t().contiguous()


def signal(n: int) -> np.ndarray:
    rng = np.random.default_rng(9)
    return (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)


def worker_1d(rank: int, world: int, port: int, n: int, out: dict) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "gpu-spectral-stack_b200"))
        from spectral.distributed import fft_slab

        stubs = dict(relayout_fn=relayout_stub, twiddle_fn=twiddle_stub, rows_fn=rows1d_stub,
                     transpose_fn=transpose_stub)
        chunk = n // world
        x = torch.from_numpy(signal(n)[rank * chunk:(rank + 1) * chunk])
        y = fft_slab(x, **stubs)
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        back = fft_slab(y, inverse=True, **stubs)
        bs = [torch.empty_like(back) for _ in range(world)]
        dist.all_gather(bs, back)
        if rank == 0:
            out["forward"] = torch.cat(ys).numpy()
            out["inverse"] = torch.cat(bs).numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("n", [256, 512])
def test_distributed_1d_transform_on_gloo_ranks(world, n):
    # n = 512 has a non-square view (16 x 32): the row and column blocks differ in shape.
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(worker_1d, args=(world, free_port(), n, out), nprocs=world, start_method="spawn")
    expected = np.fft.fft(signal(n).astype(np.complex128))
    np.testing.assert_allclose(out["forward"], expected, rtol=0, atol=1e-4 * np.abs(expected).max())
    np.testing.assert_allclose(out["inverse"], signal(n), rtol=0, atol=1e-5)
