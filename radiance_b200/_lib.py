"""ctypes binding of the C ABI in ``include/radiance_nvfp4.h``.

The library is the only implementation of the NVFP4 path: if it cannot be loaded every op raises
(there is no CPU, Triton or eager-torch fallback).  Device pointers go in as plain integers and
the stream is torch's current CUDA stream, so the calls are ordered with the surrounding torch
work and can be captured in a CUDA graph.
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

# name -> (restype, argtypes); mirrors include/radiance_nvfp4.h
SIGNATURES: dict[str, tuple] = {
    "rb_nvfp4_last_error": (ctypes.c_char_p, []),
    "rb_nvfp4_abi_version": (_int, []),
    "rb_nvfp4_device_status": (_int, [_int]),
    "rb_nvfp4_set_sm_budget": (_int, [_int]),
    "rb_nvfp4_global_scale": (_int, [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "rb_nvfp4_global_scale_noalloc": (_int, [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p]),
    "rb_nvfp4_quantize": (
        _int,
        [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_quantize_auto_scale": (
        _int,
        [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_gemm": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _int,
         _c_void_p, _int, _i64, _c_void_p],
    ),
    "rb_nvfp4_gemm_allgather": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _int,
         _c_void_p, _int, _i64, ctypes.POINTER(_c_void_p), _int, _c_void_p],
    ),
    "rb_nvfp4_gemm_swiglu": (
        _int,
        [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p, _int,
         _c_void_p, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_update_global_scale": (
        _int, [_c_void_p, _int, _c_void_p, _int, _i64, ctypes.c_float, _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_global_scale_colsum_workspace": (ctypes.c_size_t, [_int, _i64, _i64]),
    "rb_nvfp4_global_scale_colsum": (_int, [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _c_void_p, _c_void_p,
                                            _c_void_p]),
    "rb_nvfp4_global_scale_grouped": (
        _int, [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _int, _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_quantize_grouped": (
        _int,
        [_c_void_p, _int, _i64, _i64, _i64, _c_void_p, _int, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
         _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_gemm_grouped": (
        _int,
        [_c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _c_void_p, _int, _c_void_p, _c_void_p,
         _c_void_p, _int, _i64, _i64, _c_void_p],
    ),
    "rb_nvfp4_selftest_division": (_int, [_c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p]),
    "rb_nvfp4_selftest_scale": (_int, [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "rb_nvfp4_selftest_silu": (_int, [_c_void_p, _c_void_p]),
    "rb_nvfp4_swiglu_backward": (
        _int, [_c_void_p, _i64, _c_void_p, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_swiglu_forward_strided": (
        _int, [_c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_swiglu_backward_strided": (
        _int, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _c_void_p, _c_void_p, _i64, _i64,
               _c_void_p, _c_void_p, _c_void_p],
    ),
    "rb_nvfp4_selftest_wait_timeout": (_int, [_int, ctypes.c_longlong, _c_void_p, _c_void_p]),
    "rb_peer_alloc": (_int, [ctypes.c_size_t, ctypes.POINTER(_c_void_p)]),
    "rb_peer_free": (_int, [_c_void_p]),
    "rb_peer_handle": (_int, [_c_void_p, ctypes.c_char_p]),
    "rb_peer_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_c_void_p)]),
    "rb_peer_close": (_int, [_c_void_p]),
}

RB_PEER_HANDLE_BYTES = 64

ABI_VERSION = 7

RB_DTYPE_BF16 = 0
RB_DTYPE_F32 = 1
RB_OUT_BF16 = 0
RB_OUT_F32 = 1

_ERRORS = {1: ValueError, 2: ValueError, 3: RuntimeError, 4: RuntimeError}

_lock = threading.Lock()
_lib = None


class LibraryNotAvailable(RuntimeError):
    pass


def load(path: str | None = None):
    """Load (once) and return the CUDA library; raise LibraryNotAvailable if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = path or os.environ.get("RADIANCE_B200_LIB", LIB_PATH)
        if not os.path.exists(path):
            raise LibraryNotAvailable(
                f"radiance_b200 CUDA library not found at {path}; build it with `python -m radiance_b200.build` "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.rb_nvfp4_abi_version() != ABI_VERSION:
            raise LibraryNotAvailable(f"{path} has ABI {lib.rb_nvfp4_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _lib.rb_nvfp4_last_error().decode(errors="replace") if _lib is not None else ""
        raise _ERRORS.get(rc, RuntimeError)(f"{what}: {msg}")


def set_sm_budget(sms: int) -> int:
    """Size this library's kernel grids for `sms` SMs of the current device (0 = all); returns the
    previous budget.  Leaves SMs free for kernels of other streams (an overlapped collective)."""
    return int(load().rb_nvfp4_set_sm_budget(int(sms)))


def device_status(clear: bool = True) -> int:
    """First device-side error code recorded since the last clear (synchronises)."""
    return load().rb_nvfp4_device_status(1 if clear else 0)
