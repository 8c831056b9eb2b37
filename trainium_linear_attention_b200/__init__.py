"""B200 (sm_100a) BASED linear attention and sliding-window attention.

Hand-written tcgen05 / TMEM / TMA CUDA kernels behind the C ABI of
``include/la_attention.h`` (``lib/libla_attention.so``), with the Python API
of the reference's ``kernels/pytorch_attention.py`` in
:mod:`trainium_linear_attention_b200.kernels`.
"""

from .kernels.pytorch_attention import (  # noqa: F401
    ref_based_attn, solution_nki, solution, trace_solution, TracedSolution)
from .kernels.chunked_attention import (  # noqa: F401
    chunked_nki_numerator, based_chunked, based_chunked_state, taylor_feature_map,
    chunked_identity_numerator, ref_identity_numerator, based_chunked_host)
from .kernels.sliding_attention import nki_sliding_window_attn, ref_sliding_window_attn  # noqa: F401
from .kernels.based_layer import based_layer, ref_based_layer  # noqa: F401
from .kernels.based_module import (  # noqa: F401
    TrainiumBasedLinearAttention, TrainiumBasedLinearAttentionNKI)
from ._native import LaError  # noqa: F401

__all__ = [
    "ref_based_attn", "solution_nki", "solution", "trace_solution", "TracedSolution",
    "chunked_nki_numerator", "based_chunked",
    "based_chunked_state", "taylor_feature_map", "chunked_identity_numerator",
    "ref_identity_numerator", "based_chunked_host", "nki_sliding_window_attn",
    "ref_sliding_window_attn", "based_layer", "ref_based_layer",
    "TrainiumBasedLinearAttention", "TrainiumBasedLinearAttentionNKI", "LaError",
]
