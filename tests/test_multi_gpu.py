"""The slab-decomposed 2D transform across real ranks: one process per GPU, the exchange by NCCL
all-to-all and by peer memory over NVLink, every rank checking its column slab (forward) and its
row slab (inverse) against the float64 oracle. Needs two GPUs; skipped otherwise (the one-GPU emulation is tests/test_slab.py and
the index arithmetic on CPU ranks is tests/test_distributed.py)."""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, n: int) -> None:
    import torch.distributed as dist

    from oracle.policy import assert_transform_close, fft_tolerance
    from spectral.distributed import PeerSlab, fft2_slab

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        rng = np.random.default_rng(5)
        x = (rng.standard_normal((n, n)) + 1j * rng.standard_normal((n, n))).astype(np.complex64)
        rows = n // world
        w = n // world
        local = torch.from_numpy(x[rank * rows:(rank + 1) * rows]).cuda()
        cols = fft2_slab(local)
        expected = np.fft.fft2(x.astype(np.complex128))[:, rank * w:(rank + 1) * w]
        got = cols.cpu().numpy()
        # The rank's share of one n x n transform: its norm-wise error stays within the bound of
        # the whole transform.
        assert_transform_close(got[None], expected[None], n * n, axes=(-2, -1))
        back = fft2_slab(cols, inverse=True)
        assert_transform_close(back.cpu().numpy()[None], x[rank * rows:(rank + 1) * rows][None],
                               n * n, axes=(-2, -1), tol=2 * fft_tolerance(n * n))
        # The same through peer memory, twice in a row (both receive buffers), and bit for bit
        # what the all-to-all path gives: the kernels and their order are the same.
        plan = PeerSlab(n)
        for _ in range(2):
            pcols = plan.forward(local)
            assert torch.equal(pcols, cols)
            pback = plan.inverse(pcols)
            assert torch.equal(pback, back)
        plan.close()

        # Natural layout: the rank's rows of fft2 by the second all-to-all and by peer memory,
        # bit for bit the column slab's values, and back.
        start = rank * w
        expected_rows = np.fft.fft2(x.astype(np.complex128))[start:start + w]
        nat = fft2_slab(local, layout="natural")
        assert_transform_close(nat.cpu().numpy()[None], expected_rows[None], n * n, axes=(-2, -1))
        nat_back = fft2_slab(nat, inverse=True, layout="natural")
        assert_transform_close(nat_back.cpu().numpy()[None], x[rank * rows:(rank + 1) * rows][None],
                               n * n, axes=(-2, -1), tol=2 * fft_tolerance(n * n))
        gathered = [torch.empty_like(cols) for _ in range(world)]
        dist.all_gather(gathered, cols)
        assert torch.equal(nat, torch.cat(gathered, dim=1)[start:start + w])
        nplan = PeerSlab(n, natural=True)
        for _ in range(3):
            assert torch.equal(nplan.forward_natural(local), nat)
            assert torch.equal(nplan.inverse_natural(nat), nat_back)
        nplan.close()

        # The same through the C ABI on an NCCL communicator of the library's own making.
        import ctypes

        from spectral import native

        lib = native.lib()
        uid = ctypes.create_string_buffer(128)
        if rank == 0:
            native.check(lib.spectral_nccl_unique_id(uid))
        shared = [uid.raw]
        dist.broadcast_object_list(shared, src=0)
        comm = ctypes.c_void_p()
        native.check(lib.spectral_nccl_comm_init(shared[0], rank, world, ctypes.byref(comm)))
        count = ctypes.c_size_t(0)
        native.check(lib.spectral_fft2_slab_workspace(n, world, ctypes.byref(count)))
        work = torch.empty(count.value, dtype=torch.complex64, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        ccols = torch.empty_like(cols)
        native.check(lib.spectral_fft2_slab(local.data_ptr(), ccols.data_ptr(), work.data_ptr(), n, rank,
                                            world, 0, comm, stream))
        cback = torch.empty_like(back)
        native.check(lib.spectral_fft2_slab(ccols.data_ptr(), cback.data_ptr(), work.data_ptr(), n, rank,
                                            world, 1, comm, stream))
        torch.cuda.synchronize()
        assert torch.equal(ccols, cols)
        assert torch.equal(cback, back)
        native.check(lib.spectral_nccl_comm_destroy(comm))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [1024, 4096])
def test_slab_across_two_gpus(n):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.multiprocessing.spawn(_rank_main, args=(2, _free_port(), n), nprocs=2, join=True)


def _rank_main_1d(rank: int, world: int, port: int, n: int) -> None:
    import torch.distributed as dist

    from oracle.policy import assert_transform_close, fft_tolerance
    from spectral.distributed import fft_slab

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        rng = np.random.default_rng(8)
        x = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
        chunk = n // world
        mine = slice(rank * chunk, (rank + 1) * chunk)
        y = fft_slab(torch.from_numpy(x[mine]).cuda())
        expected = np.fft.fft(x.astype(np.complex128))
        # This rank's chunk of one n-point transform, against the bound for the whole transform.
        scale = np.linalg.norm(expected) / np.sqrt(world)
        err = np.linalg.norm(y.cpu().numpy() - expected[mine]) / scale
        assert err <= fft_tolerance(n), err
        back = fft_slab(y, inverse=True)
        assert_transform_close(back.cpu().numpy()[None], x[mine][None], n, tol=2 * fft_tolerance(n))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [1 << 16, 1 << 24])
def test_distributed_1d_transform_across_two_gpus(n):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    torch.multiprocessing.spawn(_rank_main_1d, args=(2, _free_port(), n), nprocs=2, join=True)
