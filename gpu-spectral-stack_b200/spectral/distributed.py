"""The large single-field 2D complex FFT, slab-decomposed over the ranks of a process group.

An n x n complex64 field (n a power of two up to 16384) is split by rows: with R ranks, rank r
holds rows [r n/R, (r+1) n/R). The forward transform runs

    1. the rank's row transforms (spectral_slab_rows), stored as R chunks of w = n/R columns;
    2. one all-to-all of those chunks (torch.distributed, NCCL over NVLink on GPUs);
    3. the column transforms of the received n x w column slab (spectral_slab_columns),

and returns the rank's w columns of the 2D transform, as an (n, w) tensor in natural order:
element [k1, c] is X[k1, r w + c]. The inverse takes that column slab back to the rank's rows of
ifft2 (divided by n^2).

layout="natural" adds the second exchange: the column slab's w x w row blocks go to the ranks
that own those output rows, and a relayout kernel (spectral_slab_relayout) assembles the rank's
rows [r w, (r+1) w) of fft2 as a (w, n) tensor, the layout of the input. The natural inverse
starts from those rows: the relayout packs the send blocks, and the exchange delivers the column
slab the plain inverse takes. The reference cannot run this case (its fft2 stops at 4096 per side and it
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


def relayout_kernel(src: torch.Tensor, dst: torch.Tensor, ranks: int, w: int, src_offsets, src_stride: int,
                    dst_offsets, dst_stride: int, h: int | None = None) -> None:
    """Copies, for each rank r, the h x w block (h = w unless given) of src at element offset
    src_offsets[r] (row stride src_stride) to dst at dst_offsets[r] (row stride dst_stride),
    complex64 on one device."""
    table = ctypes.c_void_p * ranks
    sp = table(*[src.data_ptr() + 8 * o for o in src_offsets])
    dp = table(*[dst.data_ptr() + 8 * o for o in dst_offsets])
    native.call("spectral_slab_relayout", sp, dp, ranks, w if h is None else h, w, src_stride, dst_stride,
                _stream())


def _blocks_to_rows(recv: torch.Tensor, ranks: int, w: int, relayout_fn) -> torch.Tensor:
    """(ranks, w, w) received blocks -> (w, ranks w): out[k, r w + c] = recv[r, k, c]."""
    n = ranks * w
    out = torch.empty((w, n), dtype=torch.complex64, device=recv.device)
    relayout_fn(recv, out, ranks, w, [r * w * w for r in range(ranks)], w, [r * w for r in range(ranks)], n)
    return out


def _rows_to_blocks(x: torch.Tensor, ranks: int, w: int, relayout_fn) -> torch.Tensor:
    """(w, ranks w) rows -> (ranks, w, w) send blocks: send[r, k, c] = x[k, r w + c]."""
    n = ranks * w
    send = torch.empty((ranks, w, w), dtype=torch.complex64, device=x.device)
    relayout_fn(x, send, ranks, w, [r * w for r in range(ranks)], n, [r * w * w for r in range(ranks)], w)
    return send


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
    layout: str = "columns",
    rows_fn: Callable = rows_kernel,
    columns_fn: Callable = columns_kernel,
    relayout_fn: Callable = relayout_kernel,
) -> torch.Tensor:
    """Forward: x is this rank's (n / R, n) row slab; returns its (n, n / R) column slab of fft2,
    or with layout="natural" its (n / R, n) rows of fft2. Inverse: x is the (n, n / R) column
    slab (layout="natural": the (n / R, n) rows of the spectrum); returns the (n / R, n) row slab
    of ifft2."""
    ranks, _ = _world(group)
    if x.dtype != torch.complex64 or x.dim() != 2:
        raise ValueError("fft2_slab: x must be a 2D complex64 tensor")
    if layout not in ("columns", "natural"):
        raise ValueError(f"fft2_slab: layout must be 'columns' or 'natural', got {layout!r}")
    if layout == "natural":
        w, n = x.shape
        if w * ranks != n:
            raise ValueError(f"fft2_slab: {ranks} ranks of {w} rows do not make a {n} x {n} field")
        kw = dict(group=group, rows_fn=rows_fn, columns_fn=columns_fn, relayout_fn=relayout_fn)
        if not inverse:
            cols = fft2_slab(x, **kw)                                       # (n, w) = (ranks, w, w)
            received = _exchange(cols.reshape(ranks, w, w), group)
            return _blocks_to_rows(received, ranks, w, relayout_fn)
        received = _exchange(_rows_to_blocks(x.contiguous(), ranks, w, relayout_fn), group)
        return fft2_slab(received.reshape(n, w), inverse=True, **kw)
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


# --- the 1D transform of one long signal, distributed by contiguous chunks --------------------


def twiddle_columns_kernel(x: torch.Tensor, n1: int, width: int, col0: int, n: int, inverse: bool) -> torch.Tensor:
    """n1-point transforms down the columns of an (n1, width) slab holding columns col0 .. of the
    n1 x (n / n1) view of a signal, output k1 of column j2 times W_n^(k1 j2) (conjugate and / n1
    for the inverse)."""
    y = torch.empty((n1, width), dtype=torch.complex64, device=x.device)
    native.call("spectral_slab_twiddle_columns", x.data_ptr(), y.data_ptr(), n1, width, col0, n,
                1 if inverse else 0, _stream())
    return y


def c2c_rows_kernel(x: torch.Tensor, n2: int, inverse: bool) -> torch.Tensor:
    """n2-point transforms of the rows of x (inverse divided by n2)."""
    y = torch.empty_like(x)
    native.call("spectral_c2c", b"stockham_r8", x.data_ptr(), y.data_ptr(), n2, x.numel() // n2,
                1 if inverse else 0, _stream())
    return y


def transpose_kernel(x: torch.Tensor) -> torch.Tensor:
    rows, cols = x.shape
    y = torch.empty((cols, rows), dtype=torch.complex64, device=x.device)
    native.call("spectral_transpose", x.data_ptr(), y.data_ptr(), rows, cols, 1, _stream())
    return y


def fft_slab(
    x: torch.Tensor,
    *,
    inverse: bool = False,
    group=None,
    relayout_fn: Callable = relayout_kernel,
    twiddle_fn: Callable = twiddle_columns_kernel,
    rows_fn: Callable = c2c_rows_kernel,
    transpose_fn: Callable = transpose_kernel,
) -> torch.Tensor:
    """The 1D FFT (or inverse FFT, divided by n) of one complex64 signal of n = R * len(x) points
    (a power of two up to 2^24) held by the R ranks of the group in contiguous chunks: rank r holds
    x[r n/R .. (r+1) n/R) and receives the same chunk of the transform.

    The four-step algorithm over the n1 x n2 view (n1 = 2^floor(log2(n) / 2)): the column
    transforms with the inter-step twiddles on each rank's column slab, the row transforms on its
    rows, and three all-to-alls between those layouts (in, between, out); the relayout and a
    transpose fit the blocks together (spectral_slab_twiddle_columns, spectral_c2c,
    spectral_slab_relayout, spectral_transpose)."""
    ranks, rank = _world(group)
    if x.dtype != torch.complex64 or x.dim() != 1:
        raise ValueError("fft_slab: x must be a 1D complex64 tensor (this rank's chunk)")
    n = x.numel() * ranks
    if n < 4 or n & (n - 1) or n > 1 << 24:
        raise ValueError(f"fft_slab: the signal's length must be a power of two from 4 to 2^24, got {n}")
    n1 = 1 << ((n.bit_length() - 1) // 2)
    n2 = n // n1
    if n1 % ranks:
        raise ValueError(f"fft_slab: {ranks} ranks do not divide the {n1} x {n2} view of {n} points")
    h1, w2 = n1 // ranks, n2 // ranks
    blocks = [r * h1 * w2 for r in range(ranks)]

    def rows_to_blocks(a: torch.Tensor) -> torch.Tensor:
        send = torch.empty((ranks, h1, w2), dtype=torch.complex64, device=a.device)
        relayout_fn(a, send, ranks, w2, [r * w2 for r in range(ranks)], n2, blocks, w2, h=h1)
        return send

    recv = _exchange(rows_to_blocks(x.contiguous().reshape(h1, n2)), group)            # (n1, w2) column slab
    y = twiddle_fn(recv.reshape(n1, w2), n1, w2, rank * w2, n, inverse)
    back = _exchange(y.reshape(ranks, h1, w2), group)                                  # my rows, by column block
    rows = torch.empty((h1, n2), dtype=torch.complex64, device=x.device)
    relayout_fn(back, rows, ranks, w2, blocks, w2, [r * w2 for r in range(ranks)], n2, h=h1)
    z = rows_fn(rows, n2, inverse)
    out = _exchange(rows_to_blocks(z), group)                                         # (n1, w2): Z[k1][k2 mine]
    return transpose_fn(out.reshape(n1, w2)).reshape(-1)


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

    natural=True adds the second exchange, again through peer memory: forward_natural returns the
    rank's (n / R, n) rows of fft2 and inverse_natural takes them. The column transforms write the
    column slab into a second pair of shared buffers, and the relayout kernel builds the rank's
    rows by loading its w x w block from every rank's slab over NVLink. The inverse stages the
    rows in that buffer and gathers the column slab the same way. Each direction adds one
    barrier and no separate exchange pass.
    """

    def __init__(self, n: int, group=None, natural: bool = False):
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
        self.natural = natural
        # Buffers 0, 1: the receive slabs of the row exchange; 2, 3 (natural only): the column
        # slabs (forward) and staged rows (inverse) of the second exchange.
        for _ in range(4 if natural else 2):
            self._peers.append(self._shared(8 * n * self.w))
        self._barrier()

    def _shared(self, nbytes: int):
        """Allocates one buffer per rank through CUDA IPC; returns every rank's address in this
        process (this rank's own, the others' mapped)."""
        lib = native.lib()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        native.check(lib.spectral_ipc_alloc(nbytes, ctypes.byref(ptr), handle))
        self._local.append(ptr.value)
        handles = [None] * self.ranks
        if self.ranks > 1:
            dist.all_gather_object(handles, handle.raw, group=self.group)
        else:
            handles[0] = handle.raw
        table = (ctypes.c_void_p * self.ranks)()
        for q in range(self.ranks):
            if q == self.rank:
                table[q] = ptr.value
            else:
                mapped = ctypes.c_void_p()
                native.check(lib.spectral_ipc_open(handles[q], ctypes.byref(mapped)))
                self._opened.append(mapped.value)
                table[q] = mapped.value
        return table

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
        out = torch.empty((self.n, self.w), dtype=torch.complex64, device=x.device)
        self._forward(x, b, out.data_ptr())
        return out

    def _forward(self, x: torch.Tensor, b: int, out_ptr: int) -> None:
        x = x.contiguous()
        native.call("spectral_slab_rows_peer", x.data_ptr(), None, self._peers[b], self.n,
                    self.rows, self.rank, self.ranks, 0, _stream())
        self._barrier()
        # The received slab is this call's scratch: nobody writes it again before two calls on.
        native.call("spectral_slab_columns", self._peers[b][self.rank], out_ptr, self.n, self.w, 0,
                    _stream())

    def forward_natural(self, x: torch.Tensor) -> torch.Tensor:
        """x: this rank's (n / R, n) rows; returns its (n / R, n) rows of fft2."""
        if not self.natural:
            raise ValueError("PeerSlab.forward_natural: the plan was made without natural=True")
        if x.shape != (self.rows, self.n) or x.dtype != torch.complex64:
            raise ValueError(f"PeerSlab.forward_natural: x must be ({self.rows}, {self.n}) complex64")
        b = self._next()
        slabs = self._peers[2 + b]
        self._forward(x, b, slabs[self.rank])
        self._barrier()
        out = torch.empty((self.w, self.n), dtype=torch.complex64, device=x.device)
        w = self.w
        src = (ctypes.c_void_p * self.ranks)(*[slabs[r] + 8 * self.rank * w * w for r in range(self.ranks)])
        dst = (ctypes.c_void_p * self.ranks)(*[out.data_ptr() + 8 * r * w for r in range(self.ranks)])
        native.call("spectral_slab_relayout", src, dst, self.ranks, w, w, w, self.n, _stream())
        return out

    def inverse_natural(self, x: torch.Tensor) -> torch.Tensor:
        """x: this rank's (n / R, n) rows of the spectrum; returns its (n / R, n) rows of ifft2."""
        if not self.natural:
            raise ValueError("PeerSlab.inverse_natural: the plan was made without natural=True")
        if x.shape != (self.w, self.n) or x.dtype != torch.complex64:
            raise ValueError(f"PeerSlab.inverse_natural: x must be ({self.w}, {self.n}) complex64")
        b = self._next()
        staged = self._peers[2 + b]
        x = x.contiguous()
        native.call("spectral_scale", x.data_ptr(), staged[self.rank], x.numel(), 1.0, _stream())
        self._barrier()
        w = self.w
        cols = torch.empty((self.n, w), dtype=torch.complex64, device=x.device)
        src = (ctypes.c_void_p * self.ranks)(*[staged[r] + 8 * self.rank * w for r in range(self.ranks)])
        dst = (ctypes.c_void_p * self.ranks)(*[cols.data_ptr() + 8 * r * w * w for r in range(self.ranks)])
        native.call("spectral_slab_relayout", src, dst, self.ranks, w, w, self.n, w, _stream())
        return self._inverse(cols, b)

    def inverse(self, cols: torch.Tensor) -> torch.Tensor:
        """cols: the (n, n / R) column slab; returns this rank's (n / R, n) rows of ifft2."""
        if cols.shape != (self.n, self.w) or cols.dtype != torch.complex64:
            raise ValueError(f"PeerSlab.inverse: cols must be ({self.n}, {self.w}) complex64")
        return self._inverse(cols.contiguous().clone(), self._next())

    def _inverse(self, scratch: torch.Tensor, b: int) -> torch.Tensor:
        native.call("spectral_slab_columns", scratch.data_ptr(), self._peers[b][self.rank], self.n, self.w, 1,
                    _stream())
        self._barrier()
        y = torch.empty((self.rows, self.n), dtype=torch.complex64, device=scratch.device)
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

