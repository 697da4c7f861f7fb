"""Failure detection without a GPU fault.

On the GPU: every wait of this library's kernels on an asynchronous copy is bounded (tma.cuh).
spectral_probe_bounded_wait arms an mbarrier for more bytes than its one bulk copy delivers, so
the wait cannot succeed; the kernel must give up after the spin limit, record
SPECTRAL_FAULT_WAIT_TIMEOUT in the device fault word, let its real copy land, and return. The
context stays usable: the next transform is correct and records nothing.

On the host: the distributed transforms rely on the process group's timeout. A rank that never
reaches the exchange, or that leaves between steps, must make the other rank's next collective
end with an error within that timeout instead of waiting forever (gloo ranks on the CPU; the
kernels are stand-ins, as in test_distributed.py).
"""

from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

FAULT_WAIT_TIMEOUT = 1
FAULT_DRAIN_TIMEOUT = 2


# --- the bounded wait on the GPU ------------------------------------------------------------------


@pytest.mark.gpu
def test_bounded_wait_gives_up_records_the_fault_and_leaves_the_context_usable(rng):
    import spectral
    from oracle import reference as ref
    from oracle.policy import assert_transform_close, random_complex
    from spectral import native

    stream = torch.cuda.current_stream().cuda_stream
    src = torch.arange(256, dtype=torch.float32, device="cuda")  # 1 KiB
    dst = torch.zeros_like(src)
    torch.cuda.synchronize()
    assert native.device_faults(clear=True) == 0

    # A copy that completes: no fault, the staged bytes arrive.
    native.call("spectral_probe_bounded_wait", src.data_ptr(), dst.data_ptr(), 0, 1 << 20, stream)
    torch.cuda.synchronize()
    assert native.device_faults(clear=True) == 0
    assert torch.equal(dst, src)

    # 16 bytes that never come: the wait gives up after 64 polls and the kernel returns, having
    # drained its real copy (so only the timeout code, not the drain code, is recorded).
    dst.zero_()
    t0 = time.perf_counter()
    native.call("spectral_probe_bounded_wait", src.data_ptr(), dst.data_ptr(), 16, 64, stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert native.device_faults(clear=True) == FAULT_WAIT_TIMEOUT
    assert torch.equal(dst, src)
    assert native.device_faults(clear=True) == 0  # cleared

    # The context is still good: a staged transform (2048-point rows, 16-byte aligned input) is
    # correct and records nothing.
    x = random_complex(rng, (64, 2048))
    y = spectral.fft_c2c(torch.from_numpy(x).cuda(), impl="stockham_r8")
    torch.cuda.synchronize()
    assert native.device_faults(clear=False) == 0
    assert_transform_close(y.cpu().numpy(), ref.fft(x), 2048)


def test_bounded_wait_probe_rejects_bad_arguments():
    from spectral import native

    with pytest.raises(ValueError, match="must not be null"):
        native.call("spectral_probe_bounded_wait", None, None, 0, 1, None)
    with pytest.raises(ValueError, match="16-byte aligned"):
        native.call("spectral_probe_bounded_wait", 4104, 8192, 0, 1, None)
    with pytest.raises(ValueError, match="multiple of 16"):
        native.call("spectral_probe_bounded_wait", 4096, 8192, 8, 1, None)
    with pytest.raises(ValueError, match="spin_limit"):
        native.call("spectral_probe_bounded_wait", 4096, 8192, 16, 0, None)


# --- a rank that stalls or leaves, on gloo ---------------------------------------------------------

TIMEOUT_S = 3.0
N = 32


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rows_stub(x, n, rows, ranks, inverse):
    a = x.numpy().astype(np.complex128)
    y = np.fft.fft(a, axis=1).reshape(rows, ranks, n // ranks).transpose(1, 0, 2)
    return torch.from_numpy(np.ascontiguousarray(y).astype(np.complex64))


def columns_stub(x, n, width, inverse):
    return torch.from_numpy(np.fft.fft(x.numpy().astype(np.complex128), axis=0).astype(np.complex64))


def stalled_worker(rank: int, world: int, port: int, mode: str, out: dict) -> None:
    """Rank 0 runs two slab transforms; rank 1 runs the first and then stalls ("sleep": it stays
    alive but never joins the second exchange) or leaves ("exit": its process ends between the
    steps). Rank 0 records how its second transform ended and how long it took."""
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "..", "gpu-spectral-stack_b200"))
    from spectral.distributed import fft2_slab

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=TIMEOUT_S))
    rng = np.random.default_rng(rank)
    rows = N // world
    x = torch.from_numpy((rng.standard_normal((rows, N)) + 0j).astype(np.complex64))
    fft2_slab(x, rows_fn=rows_stub, columns_fn=columns_stub)  # every rank: one good step
    if rank == 1:
        if mode == "sleep":
            time.sleep(3 * TIMEOUT_S)
        os._exit(0)  # leaves without a collective in flight and without tearing the group down
    t0 = time.perf_counter()
    try:
        fft2_slab(x, rows_fn=rows_stub, columns_fn=columns_stub)
        out["outcome"] = "returned"
    except Exception as e:  # noqa: BLE001 - the error type is gloo's; its arrival is the test
        out["outcome"] = type(e).__name__
        out["message"] = str(e)[:200]
    out["elapsed"] = time.perf_counter() - t0
    os._exit(0)


@pytest.mark.parametrize("mode", ["sleep", "exit"])
def test_a_rank_that_stalls_or_leaves_ends_the_next_exchange_with_an_error(mode):
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(stalled_worker, args=(2, free_port(), mode, out), nprocs=2, start_method="spawn")
    assert out.get("outcome") not in (None, "returned"), dict(out)
    # Within the process group's timeout, plus slack for a loaded host.
    assert out["elapsed"] < TIMEOUT_S + 15.0, dict(out)
