"""Sliding-window causal softmax attention: the reference's host API.

Counterparts of benchmarks/sliding_attention_benchmark.py:

* ``ref_sliding_window_attn(q, k, v, window_size=64, eps=1e-6)`` (:32-56):
  the reference formula in plain PyTorch, for comparisons only.
* ``nki_sliding_window_attn(q, k, v, window_size=64, block_size=64)``
  (:59-99): the sm_100a band kernel.  The mask is computed from indices, no
  padding copies are made and any ``window_size >= 1`` works (the reference
  asserts window <= 66 at block 64).  ``block_size`` is the reference's tiling
  parameter; it is validated but the kernel uses its own tile.
"""

from __future__ import annotations

import math

import torch

from .. import ops


def ref_sliding_window_attn(q, k, v, window_size=64, eps=1e-6):
    """Reference causal sliding-window softmax attention (fp32, cast to q.dtype)."""
    b, h, t, d = q.shape
    scale = 1.0 / math.sqrt(d)
    scores = torch.matmul(q.float() * scale, k.float().transpose(-2, -1))
    row = torch.arange(t, device=q.device).unsqueeze(1)
    col = torch.arange(t, device=q.device).unsqueeze(0)
    mask = (col <= row) & (col >= row - window_size + 1)
    scores = scores.masked_fill(~mask.unsqueeze(0).unsqueeze(0), float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v.float()).to(q.dtype)


def nki_sliding_window_attn(q, k, v, window_size=64, block_size=64):
    """Sliding-window softmax attention on the sm_100a kernel.

    q, k, v: (b, h, t, d).  Returns (b, h, t, d) in q.dtype.
    """
    if int(block_size) < 1:
        raise ValueError("block_size must be >= 1")
    return ops.sliding_window(q, k, v, window_size=window_size)
