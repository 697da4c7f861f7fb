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

import ctypes
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


class PeerSlab:
    """The slab transform with the exchange inside the row kernel, through peer memory.

    Every rank owns two n x w receive buffers allocated through CUDA IPC and maps every other
    rank's buffers into its own address space (plain NVLink loads and stores, no multicast). The
    forward row kernel stores each chunk straight into its destination rank's buffer, so no
    all-to-all pass runs; the inverse row kernel loads its chunks straight from the ranks' column
    slabs. One stream-ordered all-reduce of one value per call orders the ranks between the two
    stages. Calls alternate between the two buffers, so that barrier also keeps a rank from writing
    a buffer that another rank may still be reading from two calls before.

    Usage (every rank, same order): plan = PeerSlab(n); cols = plan.forward(rows);
    rows = plan.inverse(cols); plan.close().
    """

    def __init__(self, n: int, group=None):
        ranks, rank = _world(group)
        if n % ranks:
            raise ValueError(f"PeerSlab: {ranks} ranks do not divide n = {n}")
        self.n, self.ranks, self.rank, self.group = n, ranks, rank, group
        self.w = n // ranks
        self.rows = n // ranks
        self._flag = torch.zeros(1, device="cuda")
        self._calls = 0
        self._local: list[int] = []
        self._opened: list[int] = []
        self._peers = []
        lib = native.lib()
        nbytes = 8 * n * self.w
        for _ in range(2):
            ptr = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            native.check(lib.spectral_ipc_alloc(nbytes, ctypes.byref(ptr), handle))
            self._local.append(ptr.value)
            handles = [None] * ranks
            if ranks > 1:
                dist.all_gather_object(handles, handle.raw, group=group)
            else:
                handles[0] = handle.raw
            table = (ctypes.c_void_p * ranks)()
            for q in range(ranks):
                if q == rank:
                    table[q] = ptr.value
                else:
                    mapped = ctypes.c_void_p()
                    native.check(lib.spectral_ipc_open(handles[q], ctypes.byref(mapped)))
                    self._opened.append(mapped.value)
                    table[q] = mapped.value
            self._peers.append(table)
        self._barrier()

    def _barrier(self) -> None:
        if self.ranks > 1:
            dist.all_reduce(self._flag, group=self.group)

    def _next(self) -> int:
        b = self._calls % 2
        self._calls += 1
        return b

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: this rank's (n / R, n) rows; returns its (n, n / R) column slab of fft2."""
        if x.shape != (self.rows, self.n) or x.dtype != torch.complex64:
            raise ValueError(f"PeerSlab.forward: x must be ({self.rows}, {self.n}) complex64")
        b = self._next()
        x = x.contiguous()
        native.call("spectral_slab_rows_peer", x.data_ptr(), None, self._peers[b], self.n,
                    self.rows, self.rank, self.ranks, 0, _stream())
        self._barrier()
        out = torch.empty((self.n, self.w), dtype=torch.complex64, device=x.device)
        # The received slab is this call's scratch: nobody writes it again before two calls on.
        native.call("spectral_slab_columns", self._local[b], out.data_ptr(), self.n, self.w, 0,
                    _stream())
        return out

    def inverse(self, cols: torch.Tensor) -> torch.Tensor:
        """cols: the (n, n / R) column slab; returns this rank's (n / R, n) rows of ifft2."""
        if cols.shape != (self.n, self.w) or cols.dtype != torch.complex64:
            raise ValueError(f"PeerSlab.inverse: cols must be ({self.n}, {self.w}) complex64")
        b = self._next()
        scratch = cols.contiguous().clone()
        native.call("spectral_slab_columns", scratch.data_ptr(), self._local[b], self.n, self.w, 1,
                    _stream())
        self._barrier()
        y = torch.empty((self.rows, self.n), dtype=torch.complex64, device=cols.device)
        native.call("spectral_slab_rows_peer", None, y.data_ptr(), self._peers[b], self.n,
                    self.rows, self.rank, self.ranks, 1, _stream())
        return y

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's, after every rank is done with them."""
        torch.cuda.synchronize()
        if self.ranks > 1:
            dist.barrier(group=self.group)
        lib = native.lib()
        for p in self._opened:
            native.check(lib.spectral_ipc_close(ctypes.c_void_p(p)))
        torch.cuda.synchronize()
        if self.ranks > 1:
            dist.barrier(group=self.group)
        for p in self._local:
            native.check(lib.spectral_ipc_free(ctypes.c_void_p(p)))
        self._opened, self._local, self._peers = [], [], []

