"""Same names as the reference's benchmarks/based_attention_benchmark.py."""
from ..kernels.based_module import (  # noqa: F401
    TrainiumBasedLinearAttention, TrainiumBasedLinearAttentionNKI)
