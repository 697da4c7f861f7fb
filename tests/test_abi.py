"""The drop-in boundary, on the CPU: the C-ABI library loads and exports exactly what
include/spectral_b200.h declares, the registry keeps the reference's names, order and limits,
and argument checks answer with the reference's messages before any GPU work. No kernels run."""

import re
from pathlib import Path

import pytest
import torch

import spectral
from spectral import native

HEADER = Path(__file__).resolve().parent.parent / "include" / "spectral_b200.h"


def declared() -> set[str]:
    return set(re.findall(r"SPECTRAL_API\s+(?:int|const char\*)\s+(spectral_\w+)", HEADER.read_text()))


def test_library_exports_every_declared_symbol():
    lib = native.lib()
    names = declared()
    assert len(names) >= 24
    for name in names:
        assert hasattr(lib, name), name


def test_ctypes_table_covers_the_header():
    assert declared() == set(native.SIGNATURES)


def test_registry_keeps_the_reference_names_and_order():
    assert native.impl_names() == (
        "naive", "stockham_r2", "stockham_r4", "stockham_r8", "stockham_r8_table"
    )
    assert spectral.FFT_IMPLS == native.impl_names()


@pytest.mark.parametrize(
    ("impl", "limits"),
    [
        ("naive", (1 << 30, 1 << 30, 1 << 30, 0, 0, 1)),
        ("stockham_r8", (4096, 1 << 24, 8192, 1, 1, 0)),
        ("stockham_r8_table", (4096, 1 << 24, 8192, 1, 1, 0)),
    ],
)
def test_registry_limits(impl, limits):
    import ctypes

    out = [ctypes.c_int(-1) for _ in range(6)]
    native.check(native.lib().spectral_impl_limits(impl.encode(), *[ctypes.byref(o) for o in out]))
    assert tuple(o.value for o in out) == limits


def test_unknown_implementation_is_rejected_by_name():
    with pytest.raises(ValueError, match="unknown FFT implementation 'nope'"):
        native.call("spectral_c2c", b"nope", 0, 0, 8, 1, 0, None)
    assert native.lib().spectral_impl_find(b"nope") == -1


@pytest.mark.parametrize(
    ("fn", "args", "message"),
    [
        ("spectral_c2c", (b"stockham_r8", 0, 0, 12, 1, 0, None), "power of two"),
        ("spectral_c2c", (b"stockham_r8", 0, 0, 1 << 25, 1, 0, None), "up to 16777216"),
        ("spectral_r2c", (b"stockham_r8", 0, 0, 16384, 1, 0, None), "power of two from 2 to 8192"),
        ("spectral_fft2_c2c", (b"stockham_r8", 1, 0, 0, 8192, 2, 1, 0, 0, None),
         "n1 to be a power of two up to 4096"),
        ("spectral_fft2_c2c", (b"naive", 1, 0, 0, 8, 8, 1, 0, 0, None),
         "no strided column kernel"),
        ("spectral_rfft2_modes", (b"stockham_r8", 0, 0, 8, 8, 5, 2, 1, 0, None),
         "1 <= m1 <= n1/2"),
        ("spectral_c2c_pruned", (b"stockham_r8", 0, 0, 8, 9, 1, 0, 0, None), "keep must be in"),
        ("spectral_c2c", (b"stockham_r8", 4096, 4096, 8, 2, 0, None), "must not overlap"),
        ("spectral_spectrum", (b"stockham_r8", 0, 0, 0, 100, 12, 1, None), "power of two from 2 to 4096"),
        ("spectral_spectrum", (b"naive", 4096, 0, 1 << 20, 100, 64, 1, None), "no fused kernel"),
        ("spectral_fir", (b"stockham_r8", 0, 0, 0, 100, 64, 65, 1, None), "at least len\\(taps\\) = 65"),
        ("spectral_fir", (b"stockham_r8", 4096, 0, 4096, 100, 64, 8, 1, None), "must not overlap"),
        ("spectral_fir", (b"stockham_r8", 4096, 0, 4104, 100, 64, 8, 1, None), "must not overlap"),
        ("spectral_spectrum", (b"stockham_r8", 4096, 0, 4096 + 8 * 50, 100, 64, 1, None), "must not overlap"),
        ("spectral_fir", (b"stockham_r8", 0, 0, 0, 100, 8192, 8, 1, None), "power of two from 2 to 4096"),
    ],
)
def test_argument_checks_use_the_reference_messages(fn, args, message):
    with pytest.raises(ValueError, match=message):
        native.call(fn, *args)


@pytest.mark.parametrize(
    ("fn", "args"),
    [
        ("spectral_r2c", (b"stockham_r8", 4100, 8192, 64, 1, 0, None)),
        ("spectral_c2r", (b"stockham_r8", 8192, 4100, 64, 1, 0, None)),
        ("spectral_fft2_r2c", (b"stockham_r8", 1, 4100, 8192, 8, 8, 1, 0, None)),
        ("spectral_rfft2_modes", (b"stockham_r8", 4100, 8192, 8, 8, 2, 2, 1, 0, None)),
        ("spectral_c2c", (b"stockham_r8", 4100, 8192, 8, 1, 0, None)),
        ("spectral_mode_contract", (4100, 8192, 16384, 1, 1, 1, 1, None)),
        ("spectral_slab_rows", (4100, 8192, 8, 8, 1, 0, None)),
        ("spectral_spectrum", (b"stockham_r8", 4100, 0, 8192, 100, 64, 1, None)),
        ("spectral_fir", (b"stockham_r8", 4096, 4100, 8192, 100, 64, 8, 1, None)),
    ],
)
def test_misaligned_arrays_are_refused_before_any_launch(fn, args):
    # The kernels read every array as 8-byte values; a 4-byte-aligned float32 pointer (a view
    # that starts at an odd element) is refused with a message instead of faulting the GPU.
    with pytest.raises(ValueError, match="8-byte aligned"):
        native.call(fn, *args)


def test_workspace_sizes_follow_the_drivers():
    # Strided 2D needs none; the transpose method two arrays; the engine's real transforms none;
    # naive's real transforms batch * n/2 complex values.
    assert native.workspace("spectral_fft2_c2c_workspace", b"stockham_r8", 1, 16, 32, 3) == 0
    assert native.workspace("spectral_fft2_c2c_workspace", b"stockham_r8", 0, 16, 32, 3) == 2 * 3 * 16 * 32
    assert native.workspace("spectral_real_workspace", b"stockham_r8", 4096, 7) == 0
    assert native.workspace("spectral_real_workspace", b"naive", 4096, 7) == 7 * 2048
    assert native.workspace("spectral_fft2_c2r_workspace", b"stockham_r8", 1, 8, 16, 2) == 2 * 8 * 9


def test_cpu_tensors_are_rejected_by_the_dispatcher():
    x = torch.zeros(4, dtype=torch.complex64)
    with pytest.raises(NotImplementedError, match="CPU"):
        spectral.scale(x, 0.5)
    with pytest.raises(NotImplementedError, match="CPU"):
        spectral.fft_c2c(x, impl="stockham_r8")


def test_every_operator_schema_is_registered():
    for op in ["scale", "fft_c2c", "fft_r2c", "fft_c2r", "fft2_c2c", "fft2_r2c", "fft2_c2r",
               "fft_c2c_pruned", "rfft2_modes", "irfft2_modes", "mode_contract", "spectrum_frames",
               "fir_overlap_save"]:
        assert hasattr(torch.ops.spectral, op), op
    schema = str(torch.ops.spectral.fft_c2c.default._schema)
    assert 'str impl="naive"' in schema and "bool inverse=False" in schema


def test_slab_relayout_argument_checks():
    import ctypes

    table = (ctypes.c_void_p * 2)(8, 16)
    with pytest.raises(ValueError, match="ranks must be from 1 to 16"):
        native.call("spectral_slab_relayout", table, table, 17, 4, 4, 4, 4, None)
    with pytest.raises(ValueError, match="row strides of at least w"):
        native.call("spectral_slab_relayout", table, table, 2, 4, 4, 3, 4, None)
    odd = (ctypes.c_void_p * 2)(8, 20)
    with pytest.raises(ValueError, match="8-byte aligned"):
        native.call("spectral_slab_relayout", odd, table, 2, 4, 4, 4, 4, None)
    with pytest.raises(ValueError, match="columns must lie in"):
        native.call("spectral_slab_twiddle_columns", 8, 16, 64, 8, 60, 4096, 0, None)
    with pytest.raises(ValueError, match="must not overlap"):
        native.call("spectral_transpose", 8, 8, 4, 4, 1, None)


@pytest.mark.parametrize(
    ("fn", "args"),
    [
        # (x, y) one value apart: a partial overlap, not the same pointer.
        ("spectral_slab_twiddle_columns", (4096, 4104, 64, 8, 0, 4096, 0, None)),
        ("spectral_transpose", (4096, 4104, 4, 4, 1, None)),
        ("spectral_slab_rows", (4096, 4104, 8, 8, 2, 0, None)),
        ("spectral_slab_rows", (4096, 4096, 8, 8, 1, 1, None)),
        ("spectral_slab_columns", (4096, 4104, 8, 8, 0, None)),
        ("spectral_slab_columns", (4096 + 8 * 63, 4096, 8, 8, 1, None)),
        # Pruned 2D transforms of 2 fields of 16 x 16, 4 x 4 modes: x is 2048 bytes, modes 512.
        ("spectral_rfft2_modes", (b"stockham_r8", 4096, 4096 + 2040, 16, 16, 2, 4, 2, None, None)),
        ("spectral_irfft2_modes", (b"stockham_r8", 4096 + 2040, 4096, 16, 16, 2, 4, 2, None, None)),
        ("spectral_rfft2_modes_method", (b"stockham_r8", 4096, 4096, 16, 16, 2, 4, 2, 1, None, None)),
    ],
)
def test_overlapping_input_and_output_ranges_are_refused(fn, args):
    # Every check runs before any CUDA call, so the fake pointers never reach a kernel.
    with pytest.raises(ValueError, match="must not overlap"):
        native.call(fn, *args)


def test_slab_relayout_refuses_a_source_block_that_overlaps_any_destination_block():
    import ctypes

    # Two 4 x 4 blocks: source block 1 (rows of stride 4 from 4096 + 128) shares its last row with
    # destination block 0 (from 4096 + 224); sources and destinations are otherwise disjoint.
    src = (ctypes.c_void_p * 2)(4096, 4096 + 128)
    dst = (ctypes.c_void_p * 2)(4096 + 224, 8192)
    with pytest.raises(ValueError, match="source block 1 overlaps destination block 0"):
        native.call("spectral_slab_relayout", src, dst, 2, 4, 4, 4, 4, None)
