"""Same names as the reference's benchmarks/chunked_attention_benchmark.py."""
from ..kernels.chunked_attention import (  # noqa: F401
    taylor_feature_map, ref_based_attn, ref_based_numerator, ref_identity_numerator,
    chunked_nki_numerator, chunked_identity_numerator, based_chunked)
