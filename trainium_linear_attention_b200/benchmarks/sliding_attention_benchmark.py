"""Same names as the reference's benchmarks/sliding_attention_benchmark.py."""
from ..kernels.sliding_attention import ref_sliding_window_attn, nki_sliding_window_attn  # noqa: F401
