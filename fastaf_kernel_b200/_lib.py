"""ctypes binding of libgdn_b200.so (the C ABI in include/gdn_b200.h).

There is no fallback: if the CUDA library is missing or cannot be loaded, every
entry point raises.  Build it with ``python -m fastaf_kernel_b200.build`` (or
``__graft_entry__.build()``).
"""

from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

GDN_OK = 0
GDN_ERR_INVALID_ARGUMENT = -1
GDN_ERR_UNSUPPORTED = -2
GDN_ERR_CUDA = -3
GDN_ERR_DEVICE_TIMEOUT = -4

GDN_DTYPE_F32 = 0
GDN_DTYPE_BF16 = 1

GDN_PREFILL_AUTO = 0
GDN_PREFILL_CHUNKED = 1
GDN_PREFILL_RECURRENT = 2
GDN_PREFILL_TCGEN05 = 3

GDN_FLAG_QK_L2NORM = 1

# Every symbol include/gdn_b200.h declares.
EXPORTED_SYMBOLS = ("gdn_prefill", "gdn_prefill_ex", "gdn_prefill_ws", "gdn_prefill_workspace_size",
                    "gdn_prefill_resolve", "gdn_prefill_tc_launches", "gdn_prefill_noalloc", "gdn_prefill_flags",
                    "gdn_prefill_gated", "gdn_prefill_strided", "gdn_decode_strided",
                    "gdn_decode", "gdn_decode_flags", "gdn_output_gate", "gdn_device_status",
                    "gdn_set_wait_limit_ns", "gdn_last_error", "gdn_version")

_lock = threading.Lock()
_lib = None


class GdnError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


def library_path() -> str:
    return os.environ.get("GDN_B200_LIB", LIB_PATH)


def load() -> ctypes.CDLL:
    """Load libgdn_b200.so once and declare the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"libgdn_b200.so not found at {path}; the CUDA library must be built "
                "(python -m fastaf_kernel_b200.build) -- there is no CPU fallback")
        lib = ctypes.CDLL(path)
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        prefill_args = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i32, i32, i32, f32,
                        i32, i32, vp, vp]
        lib.gdn_prefill.argtypes = prefill_args + [vp]
        lib.gdn_prefill.restype = i32
        lib.gdn_prefill_ex.argtypes = prefill_args + [i32, vp]
        lib.gdn_prefill_ex.restype = i32
        lib.gdn_prefill_ws.argtypes = prefill_args + [i32, vp, ctypes.c_size_t, vp]
        lib.gdn_prefill_ws.restype = i32
        lib.gdn_prefill_noalloc.argtypes = prefill_args + [vp]
        lib.gdn_prefill_noalloc.restype = i32
        lib.gdn_prefill_resolve.argtypes = [i64, i64, i32]
        lib.gdn_prefill_resolve.restype = i32
        lib.gdn_prefill_tc_launches.argtypes = [i64, i32, i32, i32]
        lib.gdn_prefill_tc_launches.restype = i32
        lib.gdn_prefill_workspace_size.argtypes = [i64, i64, i32]
        lib.gdn_prefill_workspace_size.restype = ctypes.c_size_t
        lib.gdn_decode.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, f32,
                                   i32, i32, vp, vp, vp]
        lib.gdn_decode.restype = i32
        lib.gdn_decode_flags.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, f32,
                                         i32, i32, vp, vp, i32, vp]
        lib.gdn_decode_flags.restype = i32
        lib.gdn_prefill_strided.argtypes = prefill_args + [i64, i64, i32, i32, vp]
        lib.gdn_prefill_strided.restype = i32
        lib.gdn_decode_strided.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i64, i32, i32, i32, f32,
                                           i32, i32, vp, vp, i64, i64, i32, vp]
        lib.gdn_decode_strided.restype = i32
        lib.gdn_prefill_flags.argtypes = prefill_args + [i32, i32, vp]
        lib.gdn_prefill_flags.restype = i32
        lib.gdn_prefill_gated.argtypes = prefill_args + [vp, vp, i32, f32, i32, i32, vp]
        lib.gdn_prefill_gated.restype = i32
        lib.gdn_output_gate.argtypes = [vp, vp, vp, i32, i64, i32, f32, vp]
        lib.gdn_output_gate.restype = i32
        lib.gdn_device_status.argtypes = [vp]
        lib.gdn_device_status.restype = i32
        lib.gdn_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
        lib.gdn_set_wait_limit_ns.restype = ctypes.c_uint64
        lib.gdn_last_error.argtypes = []
        lib.gdn_last_error.restype = ctypes.c_char_p
        lib.gdn_version.argtypes = []
        lib.gdn_version.restype = ctypes.c_char_p
        _lib = lib
        return lib


def check(status: int) -> None:
    if status != GDN_OK:
        msg = load().gdn_last_error().decode(errors="replace")
        if status == GDN_ERR_INVALID_ARGUMENT:
            raise ValueError(msg)
        if status == GDN_ERR_UNSUPPORTED:
            raise NotImplementedError(msg)
        raise GdnError(status, msg)


def version() -> str:
    return load().gdn_version().decode()
