"""The full BASED layer: linear attention plus sliding-window softmax attention.

The reference states the composition at kernels/nki_attention_sliding.py:4-5
("final_output = linear_attention(Q,K,V) + sliding_window_softmax(Q,K,V)")
and ships its two halves as separate kernels and benchmarks; its module
wrapper (benchmarks/based_attention_benchmark.py:24-69) projects q, k, v and
calls one attention function.

* ``ref_based_layer(q, k, v, window_size=64, eps=1e-6)`` -- the composition of
  the reference's two PyTorch formulas (kernels/pytorch_attention.py:27-42
  and benchmarks/sliding_attention_benchmark.py:32-56), for comparisons only.
* ``based_layer(q, k, v, window_size=64, chunk_size=64, eps=1e-6)`` -- both
  terms on sm_100a (window <= 129): for bf16, d_qk = 16, d_v = 64 the chunked
  tensor-core kernel followed by the sliding-window kernel, which adds its
  term to the first one's output; other shapes in one pass over q, k, v on
  CUDA cores.
"""

from __future__ import annotations

from .. import ops
from .pytorch_attention import ref_based_attn
from .sliding_attention import ref_sliding_window_attn


def ref_based_layer(q, k, v, window_size=64, eps=1e-6):
    """based(q, k, v) + sliding_window(q, k, v) with the reference formulas."""
    return ref_based_attn(q, k, v, eps=eps) + ref_sliding_window_attn(q, k, v, window_size)


def based_layer(q, k, v, window_size=64, chunk_size=64, eps=1e-6):
    """Full BASED layer on the sm_100a kernel.

    q, k: (b, h, t, d_qk); v: (b, h, t, d_v).  Returns (b, h, t, d_v) in
    q.dtype.  ``chunk_size`` is accepted for the chunked API's signature; the
    result does not depend on it."""
    if int(chunk_size) < 1:
        raise ValueError("chunk_size must be >= 1")
    return ops.based_layer(q, k, v, window_size=window_size, eps=eps)
