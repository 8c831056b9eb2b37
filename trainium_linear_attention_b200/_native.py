"""ctypes binding of ``libla_attention.so`` (the C ABI in ``include/la_attention.h``).

This is the reference-side binding a Python caller adds: plain pointers,
sizes and a ``cudaStream_t``; no torch types cross the boundary.  Loading is
lazy and fails loudly: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libla_attention.so"

LA_OK = 0
LA_ERR_INVALID_ARGUMENT = 1
LA_ERR_UNSUPPORTED = 2
LA_ERR_CUDA = 3
LA_ERR_WORKSPACE = 4
LA_ERR_NO_DEVICE = 5
LA_ERR_DEVICE_TIMEOUT = 6

LA_DTYPE_FLOAT32 = 0
LA_DTYPE_BFLOAT16 = 1

LA_CHUNKED_NORMALIZE = 1
LA_CHUNKED_REUSE_SEGMENTS = 2
LA_CHUNKED_IDENTITY = 4

#: every symbol declared in include/la_attention.h
EXPORTED_SYMBOLS = (
    "la_status_string",
    "la_abi_version",
    "la_take_device_error",
    "la_launch_count",
    "la_based_feature_dim",
    "la_based_parallel_fwd",
    "la_based_chunked_plan",
    "la_based_chunked_workspace_size",
    "la_based_chunked_fwd",
    "la_based_chunked_fwd_noalloc",
    "la_based_chunked_state",
    "la_sliding_window_fwd",
    "la_based_layer_fwd",
)

_lock = threading.Lock()
_lib = None

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t


class LaError(RuntimeError):
    """A non-zero status returned by the native library."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


def _declare(lib) -> None:
    lib.la_status_string.argtypes = [_int]
    lib.la_status_string.restype = ctypes.c_char_p
    lib.la_abi_version.argtypes = []
    lib.la_abi_version.restype = _int
    lib.la_take_device_error.argtypes = [_p]
    lib.la_take_device_error.restype = _int
    lib.la_launch_count.argtypes = []
    lib.la_launch_count.restype = ctypes.c_uint64
    lib.la_based_feature_dim.argtypes = [_i64]
    lib.la_based_feature_dim.restype = _i64
    lib.la_based_parallel_fwd.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _f, _p]
    lib.la_based_parallel_fwd.restype = _int
    lib.la_based_chunked_plan.argtypes = [_i64, _i64, _i64, _i64, _int, _int,
                                          ctypes.POINTER(_int), ctypes.POINTER(_sz)]
    lib.la_based_chunked_plan.restype = _int
    lib.la_based_chunked_workspace_size.argtypes = [_i64, _i64, _i64, _i64, _int]
    lib.la_based_chunked_workspace_size.restype = _sz
    lib.la_based_chunked_fwd.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int,
                                         _i64, _f, ctypes.c_uint, _p, _p, _p, _sz, _int, _p]
    lib.la_based_chunked_fwd.restype = _int
    lib.la_based_chunked_fwd_noalloc.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                                 _int, _i64, _f, ctypes.c_uint, _p, _p, _int, _p]
    lib.la_based_chunked_fwd_noalloc.restype = _int
    lib.la_based_chunked_state.argtypes = [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int,
                                           _p, _sz, _int, _p]
    lib.la_based_chunked_state.restype = _int
    lib.la_sliding_window_fwd.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _int, _i64, _p]
    lib.la_sliding_window_fwd.restype = _int
    lib.la_based_layer_fwd.argtypes = [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _int, _i64,
                                       _f, _p, _sz, _int, _p]
    lib.la_based_layer_fwd.restype = _int


def lib():
    """The loaded native library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = Path(os.environ.get("LA_ATTENTION_LIB", LIB_PATH))
                if not path.exists():
                    raise RuntimeError(
                        f"native library {path} is missing; build it with "
                        "`python -m trainium_linear_attention_b200.build`")
                handle = ctypes.CDLL(str(path))
                _declare(handle)
                _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().la_status_string(int(status)).decode()


def check(status: int, where: str) -> None:
    if status != LA_OK:
        raise LaError(status, where)
