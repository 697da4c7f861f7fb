"""ctypes binding of the C ABI (include/spectral_b200.h), for callers that hold raw device
pointers rather than torch tensors, and for tests that exercise the ABI directly.

`lib()` loads libspectral_b200.so from this directory and declares every entry point's argument
types. `check(status)` turns a status code into an exception: SPECTRAL_INVALID_ARGUMENT into
ValueError, anything else into RuntimeError, with the library's message. Pointers are passed as
integers (e.g. tensor.data_ptr()), streams as integers (torch.cuda.current_stream().cuda_stream).
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

LIB_PATH = Path(__file__).with_name("libspectral_b200.so")

OK = 0
INVALID_ARGUMENT = 1
CUDA_ERROR = 2
INTERNAL_ERROR = 3

COLUMNS_TRANSPOSE = 0
COLUMNS_STRIDED = 1

_p = ctypes.c_void_p
_s = ctypes.c_char_p
_i = ctypes.c_int
_ll = ctypes.c_longlong
_f = ctypes.c_float
_szp = ctypes.POINTER(ctypes.c_size_t)
_ip = ctypes.POINTER(ctypes.c_int)

# name -> (restype, argtypes), in the order of include/spectral_b200.h.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "spectral_last_error": (_s, []),
    "spectral_device_faults": (_i, [ctypes.POINTER(ctypes.c_uint), _i]),
    "spectral_probe_bounded_wait": (_i, [_p, _p, ctypes.c_uint, ctypes.c_uint, _p]),
    "spectral_impl_count": (_i, []),
    "spectral_impl_name": (_s, [_i]),
    "spectral_impl_find": (_i, [_s]),
    "spectral_impl_limits": (_i, [_s, _ip, _ip, _ip, _ip, _ip, _ip]),
    "spectral_scale": (_i, [_p, _p, ctypes.c_size_t, _f, _p]),
    "spectral_c2c": (_i, [_s, _p, _p, _i, _ll, _i, _p]),
    "spectral_r2c": (_i, [_s, _p, _p, _i, _ll, _p, _p]),
    "spectral_c2r": (_i, [_s, _p, _p, _i, _ll, _p, _p]),
    "spectral_real_workspace": (_i, [_s, _i, _ll, _szp]),
    "spectral_columns": (_i, [_s, _p, _p, _i, _i, _ll, _i, _p]),
    "spectral_fft2_c2c_workspace": (_i, [_s, _i, _i, _i, _ll, _szp]),
    "spectral_fft2_r2c_workspace": (_i, [_s, _i, _i, _i, _ll, _szp]),
    "spectral_fft2_c2r_workspace": (_i, [_s, _i, _i, _i, _ll, _szp]),
    "spectral_fft2_c2c": (_i, [_s, _i, _p, _p, _i, _i, _ll, _i, _p, _p]),
    "spectral_fft2_r2c": (_i, [_s, _i, _p, _p, _i, _i, _ll, _p, _p]),
    "spectral_fft2_c2r": (_i, [_s, _i, _p, _p, _i, _i, _ll, _p, _p]),
    "spectral_fft2_c2r_noalloc": (_i, [_s, _p, _p, _i, _i, _ll, _p]),
    "spectral_c2c_pruned_workspace": (_i, [_s, _i, _i, _ll, _szp]),
    "spectral_c2c_pruned": (_i, [_s, _p, _p, _i, _i, _ll, _i, _p, _p]),
    "spectral_rfft2_modes_workspace": (_i, [_s, _i, _i, _i, _i, _ll, _szp]),
    "spectral_irfft2_modes_workspace": (_i, [_s, _i, _i, _i, _i, _ll, _szp]),
    "spectral_rfft2_modes": (_i, [_s, _p, _p, _i, _i, _i, _i, _ll, _p, _p]),
    "spectral_rfft2_modes_method": (_i, [_s, _p, _p, _i, _i, _i, _i, _ll, _i, _p, _p]),
    "spectral_irfft2_modes": (_i, [_s, _p, _p, _i, _i, _i, _i, _ll, _p, _p]),
    "spectral_irfft2_modes_method": (_i, [_s, _p, _p, _i, _i, _i, _i, _ll, _i, _p, _p]),
    "spectral_slab_rows": (_i, [_p, _p, _i, _ll, _i, _i, _p]),
    "spectral_slab_columns": (_i, [_p, _p, _i, _i, _i, _p]),
    "spectral_slab_rows_peer": (_i, [_p, _p, ctypes.POINTER(_p), _i, _ll, _i, _i, _i, _p]),
    "spectral_slab_relayout": (_i, [ctypes.POINTER(_p), ctypes.POINTER(_p), _i, _i, _i, _ll, _ll, _p]),
    "spectral_slab_twiddle_columns": (_i, [_p, _p, _i, _i, _ll, _ll, _i, _p]),
    "spectral_transpose": (_i, [_p, _p, _i, _i, _ll, _p]),
    "spectral_fft2_slab_workspace": (_i, [_i, _i, _szp]),
    "spectral_fft2_slab": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "spectral_slab_exchange": (_i, [_p, _p, _ll, _i, _p, _p]),
    "spectral_nccl_unique_id": (_i, [_p]),
    "spectral_nccl_comm_init": (_i, [_p, _i, _i, ctypes.POINTER(_p)]),
    "spectral_nccl_comm_destroy": (_i, [_p]),
    "spectral_ipc_alloc": (_i, [ctypes.c_ulonglong, ctypes.POINTER(_p), _p]),
    "spectral_ipc_open": (_i, [_p, ctypes.POINTER(_p)]),
    "spectral_ipc_close": (_i, [_p]),
    "spectral_ipc_free": (_i, [_p]),
    "spectral_mode_contract": (_i, [_p, _p, _p, _ll, _i, _i, _ll, _p]),
    "spectral_mode_contract_method": (_i, [_p, _p, _p, _ll, _i, _i, _ll, _i, _p]),
    "spectral_fp32_ceiling": (_i, [_p, _i, _i, _p, ctypes.POINTER(ctypes.c_double)]),
    "spectral_spectrum": (_i, [_s, _p, _p, _p, _ll, _i, _ll, _p]),
    "spectral_fir": (_i, [_s, _p, _p, _p, _ll, _i, _i, _ll, _p]),
    "spectral_flow_workspace": (_i, [_i, _i, _ll, _szp]),
    "spectral_flow_stage": (_i, [_s, _p, _p, _p, _p, _p, _p, _p, _p, _p, _ll, _p, _i, _i, _ll, _f, _i, _p]),
}


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    """The loaded library, every entry point declared. Raises OSError if it is not built."""
    if not LIB_PATH.exists():
        raise OSError(
            f"{LIB_PATH} is not built; run `python gpu-spectral-stack_b200/build.py`"
        )
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return handle


def last_error() -> str:
    return (lib().spectral_last_error() or b"").decode()


def check(status: int) -> None:
    """Raises for a non-zero status, as the torch operators do."""
    if status == OK:
        return
    message = last_error()
    if status == INVALID_ARGUMENT:
        raise ValueError(message)
    raise RuntimeError(message)


def device_faults(clear: bool = True) -> int:
    """Fault codes kernels recorded on the current device (0: none); see spectral_device_faults."""
    value = ctypes.c_uint(0)
    check(lib().spectral_device_faults(ctypes.byref(value), 1 if clear else 0))
    return value.value


def impl_names() -> tuple[str, ...]:
    handle = lib()
    return tuple(handle.spectral_impl_name(i).decode() for i in range(handle.spectral_impl_count()))


def workspace(fn: str, *args) -> int:
    """Complex values of workspace that `fn` (a spectral_*_workspace name) reports."""
    count = ctypes.c_size_t(0)
    check(getattr(lib(), fn)(*args, ctypes.byref(count)))
    return count.value


def call(fn: str, *args) -> None:
    """Calls entry point `fn` and raises on a non-zero status."""
    check(getattr(lib(), fn)(*args))


def enc(name: str) -> bytes:
    return name.encode()
