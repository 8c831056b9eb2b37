"""CPU oracle for the BASED / sliding-window attention hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg
of ``bench.py`` may use it, and only as the checker (or as the timed CPU
reference arm), never as the thing measured on the GPU.

The functions restate the reference repository's own algorithms in numpy
(float64 by default).  Each function cites the reference file:line it
follows.  The restatement is pinned against golden vectors produced by the
reference's own PyTorch functions (``tests/golden/make_golden.py``).
"""

from .based_oracle import (  # noqa: F401
    based_attn_reduced,
    taylor_feature_map,
    taylor_feature_map_full,
    based_attn_features,
    based_numerator_features,
    based_chunked,
    chunked_state,
    kernel_feature_map_k,
    kernel_feature_map_q,
    sliding_window_attn,
    identity_numerator,
    identity_chunked,
    based_layer,
    feature_dim,
    rel_l2,
)
