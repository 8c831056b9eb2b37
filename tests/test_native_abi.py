"""The C-ABI library loads, exports every symbol the header declares, and its
host-side logic (status codes, planning, argument checks) behaves -- all
without a GPU (no compute call reaches a kernel here)."""

import ctypes
import re
from pathlib import Path

import pytest

from trainium_linear_attention_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "la_attention.h"


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(la_[a-z0-9_]+)\s*\(", text)))


def test_header_matches_binding_table():
    assert header_functions() == sorted(N.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = N.lib()
    for name in header_functions():
        assert hasattr(lib, name), name
    # the exported dynamic symbols, read back through dlsym
    handle = ctypes.CDLL(str(N.LIB_PATH))
    for name in header_functions():
        assert ctypes.cast(getattr(handle, name), ctypes.c_void_p).value


def test_status_strings():
    assert N.status_string(N.LA_OK) == "ok"
    for code in range(1, 7):
        assert N.status_string(code) not in ("ok", "unknown status")
    assert N.status_string(99) == "unknown status"


def test_feature_dim_and_version():
    lib = N.lib()
    assert lib.la_abi_version() == 1
    assert lib.la_based_feature_dim(16) == 153
    assert lib.la_based_feature_dim(64) == 2145
    assert lib.la_based_feature_dim(0) == 0


def test_workspace_size_math():
    lib = N.lib()
    F, dv = 153, 64
    # one segment never needs a workspace
    assert lib.la_based_chunked_workspace_size(128, 32768, 16, 64, 1) == 0
    ws = lib.la_based_chunked_workspace_size(16, 32768, 16, 64, 8)
    assert ws >= 16 * 8 * F * (dv + 1) * 4 and ws % 256 == 0
    # segments beyond what the sequence can hold collapse (tiles of 128 tokens)
    assert lib.la_based_chunked_workspace_size(4, 200, 16, 64, 8) == \
        lib.la_based_chunked_workspace_size(4, 200, 16, 64, 2)


def test_plan_with_explicit_segments_needs_no_device():
    g = ctypes.c_int(0)
    ws = ctypes.c_size_t(0)
    st = N.lib().la_based_chunked_plan(16, 32768, 16, 64, N.LA_DTYPE_BFLOAT16, 8,
                                       ctypes.byref(g), ctypes.byref(ws))
    assert st == N.LA_OK and g.value == 8 and ws.value > 0
    st = N.lib().la_based_chunked_plan(16, 100, 16, 64, N.LA_DTYPE_BFLOAT16, 8,
                                       ctypes.byref(g), ctypes.byref(ws))
    assert st == N.LA_OK and g.value == 1 and ws.value == 0


@pytest.mark.parametrize("args,code", [
    ((-1, 4, 16, 16, 64), N.LA_ERR_INVALID_ARGUMENT),   # negative batch
    ((1, 4, 16, 0, 64), N.LA_ERR_INVALID_ARGUMENT),     # d_qk = 0
])
def test_parallel_rejects_bad_sizes(args, code):
    p = ctypes.c_void_p(16)
    st = N.lib().la_based_parallel_fwd(p, p, p, p, *args, N.LA_DTYPE_FLOAT32, 1e-6, None)
    assert st == code


def test_bad_dtype_and_null_pointers():
    lib = N.lib()
    p = ctypes.c_void_p(16)
    assert lib.la_based_parallel_fwd(p, p, p, p, 1, 1, 8, 16, 64, 7, 1e-6, None) == \
        N.LA_ERR_INVALID_ARGUMENT
    assert lib.la_based_parallel_fwd(None, p, p, p, 1, 1, 8, 16, 64, 0, 1e-6, None) == \
        N.LA_ERR_INVALID_ARGUMENT
    assert lib.la_sliding_window_fwd(p, p, p, p, 1, 1, 8, 64, 1, 0, None) == \
        N.LA_ERR_INVALID_ARGUMENT  # window 0
    assert lib.la_based_chunked_fwd(p, p, p, p, 1, 1, 8, 16, 64, 1, 0, 1e-6, 1, None, None, None,
                                    0, 0, None) == N.LA_ERR_INVALID_ARGUMENT  # chunk 0
    assert lib.la_based_chunked_fwd(p, p, p, p, 1, 1, 8, 16, 64, 1, 64, 1e-6, 0x80, None, None,
                                    None, 0, 0, None) == N.LA_ERR_INVALID_ARGUMENT  # bad flag


def test_empty_problems_are_ok_without_launch():
    lib = N.lib()
    assert lib.la_based_parallel_fwd(None, None, None, None, 0, 4, 16, 16, 64, 1, 1e-6, None) == N.LA_OK
    assert lib.la_sliding_window_fwd(None, None, None, None, 2, 2, 0, 64, 1, 64, None) == N.LA_OK


def test_no_device_is_reported_not_faked():
    """Without a GPU a real request must fail with a status, never run on the CPU."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = ctypes.c_void_p(16)
    st = N.lib().la_based_parallel_fwd(p, p, p, p, 1, 1, 8, 16, 64, 1, 1e-6, None)
    assert st == N.LA_ERR_NO_DEVICE


def test_identity_flag_is_numerator_only():
    """LA_CHUNKED_IDENTITY with LA_CHUNKED_NORMALIZE is rejected before any
    device work (the identity map has no normalised form in the reference)."""
    p = ctypes.c_void_p(256)
    flags = N.LA_CHUNKED_IDENTITY | N.LA_CHUNKED_NORMALIZE
    assert N.lib().la_based_chunked_fwd(p, p, p, p, 1, 1, 8, 16, 64, 1, 64, 1e-6, flags, None,
                                        None, None, 0, 0, None) == N.LA_ERR_INVALID_ARGUMENT
