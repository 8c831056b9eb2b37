"""BASED attention modules: q, k, v, o projections around one attention call.

Same classes, constructor arguments and forward as the reference's module
wrappers (benchmarks/based_attention_benchmark.py:24-69):

* ``TrainiumBasedLinearAttention(dim, heads=8, eps=1e-6)`` -- the reference
  path: ``ref_based_attn`` in plain PyTorch between the projections (for
  comparisons; it materialises the (t, t) score matrix).
* ``TrainiumBasedLinearAttentionNKI(dim, heads=8, eps=1e-6, window_size=None)``
  -- the kernel path: ``solution_nki`` (the parallel BASED kernel) as in the
  reference; ``attention="auto"`` uses ``solution`` instead (parallel or
  chunked by the measured crossover), and ``window_size`` adds the
  sliding-window term (the full BASED layer, ``based_layer``).

The projections are ``nn.Linear`` layers without bias (cuBLAS GEMMs); the
attention runs on the library's sm_100a kernels, which fail loudly when the
CUDA library is missing.  Head layout as the reference: ``(b, t, dim)`` ->
``(b, heads, t, dim // heads)`` and back.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .based_layer import based_layer
from .pytorch_attention import ref_based_attn, solution, solution_nki


class _Projections(nn.Module):
    def __init__(self, dim: int, heads: int, eps: float):
        super().__init__()
        assert dim % heads == 0
        self.num_heads = heads
        self.head_dim = dim // heads
        self.eps = eps
        self.q_proj = nn.Linear(dim, dim, bias=False)
        self.k_proj = nn.Linear(dim, dim, bias=False)
        self.v_proj = nn.Linear(dim, dim, bias=False)
        self.o_proj = nn.Linear(dim, dim, bias=False)

    def _heads(self, proj: nn.Linear, x: torch.Tensor) -> torch.Tensor:
        b, t, _ = x.size()
        return proj(x).view(b, t, self.num_heads, self.head_dim).transpose(1, 2)

    def _attend(self, q, k, v):
        raise NotImplementedError

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        b, t, _ = hidden_states.size()
        q = self._heads(self.q_proj, hidden_states)
        k = self._heads(self.k_proj, hidden_states)
        v = self._heads(self.v_proj, hidden_states)
        y = self._attend(q, k, v)
        y = y.transpose(1, 2).reshape(b, t, -1)
        return self.o_proj(y.to(hidden_states.dtype))


class TrainiumBasedLinearAttention(_Projections):
    """BASED attention module, reference path (``ref_based_attn``)."""

    def __init__(self, dim: int, heads: int = 8, eps: float = 1e-6):
        super().__init__(dim, heads, eps)

    def _attend(self, q, k, v):
        return ref_based_attn(q, k, v, eps=self.eps)


class TrainiumBasedLinearAttentionNKI(_Projections):
    """BASED attention module on the sm_100a kernels.

    ``attention``: "parallel" (``solution_nki``, the reference's call) or
    "auto" (``solution``).  ``window_size``: if set, the full BASED layer
    (linear attention + sliding-window softmax over the last ``window_size``
    keys) replaces the linear attention.
    """

    def __init__(self, dim: int, heads: int = 8, eps: float = 1e-6,
                 window_size: int | None = None, attention: str = "parallel"):
        super().__init__(dim, heads, eps)
        if attention not in ("parallel", "auto"):
            raise ValueError("attention must be 'parallel' or 'auto'")
        if window_size is not None and int(window_size) < 1:
            raise ValueError("window_size must be >= 1")
        self.window_size = window_size
        self.attention = attention

    def _attend(self, q, k, v):
        if self.window_size is not None:
            return based_layer(q, k, v, window_size=self.window_size, eps=self.eps)
        if self.attention == "auto":
            return solution(q, k, v, eps=self.eps)
        return solution_nki(q, k, v, eps=self.eps)
