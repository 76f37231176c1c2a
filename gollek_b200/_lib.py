"""Loads libgollek_kernels.so and declares the C ABI of include/gollek_kernels.h.

There is no CPU fallback: if the library cannot be loaded, every call into it raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH, build, stale

# dtype codes (GOLLEK_DTYPE_*)
F32, BF16, F16, I8, I4 = 0, 1, 2, 3, 4

# status codes (GOLLEK_ERR_*) and device status bits (GOLLEK_STATUS_*)
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED = -2
ERR_BAD_BLOCK_ID = -3
ERR_TIMEOUT = -4
ERR_NO_DEVICE = -5
ERR_WORKSPACE = -6
ERR_BAD_POSITION = -7
STATUS_BAD_BLOCK_ID = 0x1
STATUS_TIMEOUT = 0x2
STATUS_BAD_POSITION = 0x4

_c_int, _c_float, _c_ll, _c_size, _vp = (ctypes.c_int, ctypes.c_float, ctypes.c_longlong,
                                         ctypes.c_size_t, ctypes.c_void_p)

# name -> (restype, argtypes), in header order
SIGNATURES = {
    "paged_attention_launch": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int,
                                        _c_int, _c_int, _c_float]),
    "gollek_cuda_device_count": (_c_int, []),
    "gollek_cuda_device_name": (_c_int, [ctypes.c_char_p, _c_int]),
    "gollek_paged_attention_v2": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int,
                                           _c_int, _c_int, _c_int, _c_int, _c_int, _c_ll, _c_int,
                                           _c_int, _c_ll, _c_ll, _c_ll, _c_float, _c_float, _c_int,
                                           _vp, _c_size, _vp]),
    "gollek_paged_attention_workspace_size": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "gollek_paged_attention_prefill": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int,
                                                _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                                _c_int, _c_ll, _c_int, _c_int, _c_ll, _c_ll, _c_ll,
                                                _c_float, _c_float, _c_int, _c_int, _vp, _c_size,
                                                _vp]),
    "gollek_paged_attention_prefill_workspace_size": (_c_size, [_c_int, _c_int, _c_int, _c_int,
                                                                _c_int]),
    "gollek_paged_attention_v2_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_int,
                                                   _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                                   _c_ll, _c_int, _c_int, _c_ll, _c_ll, _c_ll,
                                                   _c_float, _c_float, _c_int, _vp]),
    "gollek_kv_append": (_c_int, [_vp, _vp, _c_int, _vp, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp,
                                  _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_ll, _c_ll, _c_ll,
                                  _c_ll, _vp]),
    "gollek_kv_migrate": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_ll,
                                   _c_ll, _c_ll, _c_int, _vp]),
    "gollek_kv_block_checksum": (_c_int, [_vp, _vp, _c_int, _c_int, _c_ll, _c_ll, _vp, _vp]),
    "gollek_enable_peer_access": (_c_int, [_c_int, _c_int]),
    "gollek_ipc_get_handle": (_c_int, [_vp, _vp, ctypes.POINTER(_c_ll)]),
    "gollek_ipc_open_handle": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "gollek_ipc_close_handle": (_c_int, [_vp]),
    "gollek_device_status": (_c_int, [_c_int, _c_int, ctypes.POINTER(ctypes.c_uint)]),
    "gollek_last_error_string": (ctypes.c_char_p, []),
    "gollek_version": (ctypes.c_char_p, []),
}

_lock = threading.Lock()
_lib = None


class GollekError(RuntimeError):
    """A non-zero status from libgollek_kernels.so."""

    def __init__(self, code: int, message: str):
        super().__init__(f"gollek status {code}: {message}")
        self.code = code


def load(path: str | None = None, build_if_missing: bool = True):
    """Loads (building first if the sources are newer) and returns the CDLL."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if path is None and build_if_missing and stale():
            build()
        if not os.path.exists(p):
            raise OSError(f"libgollek_kernels.so not found at {p}")
        lib = ctypes.CDLL(p)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().gollek_last_error_string()
        raise GollekError(rc, msg.decode() if msg else "")
