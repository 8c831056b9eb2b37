"""The allocation-free chunked entry point (la_based_chunked_fwd_noalloc).

Callers that cannot allocate device memory -- a plugin whose host framework
owns all device memory and offers no allocation hook, or latency-critical
code that must not call cudaMalloc -- use this variant, which takes its
segment scratch from a fixed array inside the library.  It is checked here
through the C ABI against the regular entry point (which is given a
workspace allocated by the caller) on two calls in a row, with the scratch
actually in use (several segments per head).  This file sorts last so that a
run stopping at the first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from trainium_linear_attention_b200 import _native as N
from trainium_linear_attention_b200 import ops

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-2
SCRATCH_BYTES = 8 << 20


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _noalloc(q, k, v, out, segments, normalize=True):
    b, h, t, d = q.shape
    flags = N.LA_CHUNKED_NORMALIZE if normalize else 0
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return N.lib().la_based_chunked_fwd_noalloc(
        _p(q), _p(k), _p(v), _p(out), b, h, t, d, v.shape[-1], N.LA_DTYPE_BFLOAT16, 64, 1e-6,
        flags, None, None, segments, stream)


def _inputs(b, h, t, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda d: (torch.randn(b, h, t, d, generator=g) * 0.5).to(torch.bfloat16).cuda()
    return mk(16), mk(16), mk(64)


def test_noalloc_matches_regular_entry_point_twice():
    """Two calls in a row with different inputs of the same shape and segment
    count: each must equal the regular entry point bit for bit (both run the
    same kernels), so a call that read the previous call's segment states
    from the shared scratch would fail here."""
    segments = 4
    g, ws = ops.chunked_plan(8, 4096, 16, 64, torch.bfloat16, segments)
    assert g == segments and 0 < ws <= SCRATCH_BYTES  # the scratch is really used
    for seed in (21, 22):
        q, k, v = _inputs(1, 8, 4096, seed=seed)
        want = ops.based_chunked(q, k, v, segments=segments)  # caller-allocated workspace
        out = torch.empty_like(v)
        assert _noalloc(q, k, v, out, segments) == N.LA_OK
        torch.cuda.synchronize()
        assert torch.equal(out, want)
        oracle = O.based_attn_reduced(*(x.float().cpu().numpy().astype(np.float64)
                                        for x in (q, k, v)))
        assert O.rel_l2(out.float().cpu().numpy(), oracle) <= TOL_BF16
    num = torch.empty_like(v)
    assert _noalloc(q, k, v, num, segments, normalize=False) == N.LA_OK
    want_num = ops.based_chunked(q, k, v, segments=segments, normalize=False)
    torch.cuda.synchronize()
    assert torch.equal(num, want_num)


def test_noalloc_rejects_requests_beyond_its_scratch():
    # 128 heads x 8 segments of 153 x 65 fp32 states = 40.7 MB > 8 MiB
    q, k, v = (torch.empty((8, 16, 8192, d), dtype=torch.bfloat16, device="cuda")
               for d in (16, 16, 64))
    out = torch.empty_like(v)
    assert _noalloc(q, k, v, out, segments=8) == N.LA_ERR_WORKSPACE
    flags = N.LA_CHUNKED_NORMALIZE | N.LA_CHUNKED_REUSE_SEGMENTS
    st = N.lib().la_based_chunked_fwd_noalloc(_p(q), _p(k), _p(v), _p(out), 8, 16, 8192, 16, 64,
                                              N.LA_DTYPE_BFLOAT16, 64, 1e-6, flags, None, None, 8,
                                              None)
    assert st == N.LA_ERR_INVALID_ARGUMENT


def test_noalloc_lead_main_split():
    """segments=0 at 96 heads: the library's lead/main split, one seed state
    per head in the scratch."""
    q, k, v = _inputs(6, 16, 4096, seed=23)
    want = ops.based_chunked(q, k, v)
    out = torch.empty_like(v)
    assert _noalloc(q, k, v, out, 0) == N.LA_OK
    torch.cuda.synchronize()
    assert torch.equal(out, want)
