"""Chunked recurrent BASED attention: the reference's chunked host API.

Counterparts of the functions in the reference's
benchmarks/chunked_attention_benchmark.py:

* ``taylor_feature_map(x)`` (:34-53) and ``ref_based_attn`` /
  ``ref_based_numerator`` (:55-76): the reference formulas in plain PyTorch,
  for comparisons only; no CUDA path calls them.
* ``chunked_nki_numerator(q, k, v, chunk_size=64)`` (:96-126): numerator-only
  output of the sm_100a chunked kernel, in q.dtype.  The features are expanded
  on chip (never written to HBM) and d_v may differ from d_qk.
* ``based_chunked(q, k, v, chunk_size=64, eps=1e-6)``: the normalised output
  (the reference's chunked kernel has no normaliser).
* ``based_chunked_host(q, k, v, ...)``: the same on pinned host tensors, with
  the copies overlapped with the kernels per group of heads.
* ``based_chunked_state(k, v)``: total per-head state, the quantity the
  sequence-parallel mode exchanges between GPUs.
* ``ref_identity_numerator(q, k, v)`` (:79-93): the identity-feature-map
  numerator formula in plain PyTorch, for comparisons only, and
  ``chunked_identity_numerator(q, k, v, chunk_size=64)``: the same quantity
  from the chunked kernel with phi(x) = x (the recurrence of the reference's
  old/identity_linear_attn_nki_CHUNKED.py:26-63).
"""

from __future__ import annotations

import math

import torch

from .. import ops


def _flatten_diag_outer_product_off1(x):
    z = torch.einsum("...i,...j->...ij", x, x)
    n = z.size(-1)
    tri_i, tri_j = torch.triu_indices(n, n, 1, device=x.device)
    diag_idx = torch.arange(n, device=x.device, dtype=torch.long)
    return z[..., tri_i, tri_j], z[..., diag_idx, diag_idx]


def taylor_feature_map(x):
    """BASED Taylor feature map, width 1 + d + d + d(d-1)/2 (153 at d = 16)."""
    d = x.shape[-1]
    r2 = math.sqrt(2.0)
    rd = math.sqrt(d)
    rrd = math.sqrt(rd)
    x2_1, x2_2 = _flatten_diag_outer_product_off1(x)
    return torch.cat([torch.ones_like(x[..., 0:1]), x / rrd, x2_2 / (rd * r2), x2_1 / rd], dim=-1)


def ref_based_attn(q, k, v, eps=1e-6):
    """Dense normalised reference over Taylor features (fp32, cast to q.dtype)."""
    q_phi = taylor_feature_map(q.float())
    k_phi = taylor_feature_map(k.float())
    scores = torch.matmul(q_phi, k_phi.transpose(-2, -1))
    t = q.shape[-2]
    masked = scores * torch.tril(torch.ones(t, t, device=q.device, dtype=scores.dtype))
    den = masked.sum(dim=-1, keepdim=True) + eps
    return (torch.matmul(masked, v.float()) / den).to(q.dtype)


def ref_based_numerator(q, k, v):
    """Dense numerator-only reference over Taylor features."""
    q_phi = taylor_feature_map(q.float())
    k_phi = taylor_feature_map(k.float())
    scores = torch.matmul(q_phi, k_phi.transpose(-2, -1))
    t = q.shape[-2]
    masked = scores * torch.tril(torch.ones(t, t, device=q.device, dtype=scores.dtype))
    return torch.matmul(masked, v.float()).to(q.dtype)


def ref_identity_numerator(q, k, v):
    """Dense identity-feature-map numerator: tril((q / sqrt(d)) k^T) v, in q.dtype."""
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d)
    scores = torch.matmul(q * scale, k.transpose(-2, -1))
    t = q.shape[-2]
    mask = torch.tril(torch.ones(t, t, device=q.device, dtype=q.dtype))
    return torch.matmul(scores * mask, v)


def chunked_identity_numerator(q, k, v, chunk_size=64):
    """Chunked identity-feature-map linear attention (numerator) on the sm_100a kernels.

    q, k: (b, h, t, d_qk); v: (b, h, t, d_v).  Returns (b, h, t, d_v) in q.dtype.
    """
    return ops.based_chunked(q, k, v, chunk_size=chunk_size, normalize=False,
                             feature_map="identity")


def chunked_nki_numerator(q, k, v, chunk_size=64):
    """Numerator-only chunked BASED on the sm_100a kernel.

    q, k: (b, h, t, d_qk); v: (b, h, t, d_v).  Returns (b, h, t, d_v) in q.dtype.
    """
    return ops.based_chunked(q, k, v, chunk_size=chunk_size, normalize=False)


def based_chunked(q, k, v, chunk_size=64, eps=1e-6):
    """Normalised chunked BASED attention on the sm_100a kernel."""
    return ops.based_chunked(q, k, v, chunk_size=chunk_size, eps=eps, normalize=True)


def based_chunked_host(q, k, v, chunk_size=64, eps=1e-6, head_groups=8, out=None):
    """Normalised chunked BASED attention on pinned host tensors, with the
    host<->device copies of head groups overlapped with the kernels (see
    ``ops.based_chunked_host``); the result is in ``out`` once the current
    CUDA stream has reached the end of the call."""
    return ops.based_chunked_host(q, k, v, chunk_size=chunk_size, eps=eps, normalize=True,
                                  head_groups=head_groups, out=out)


def based_chunked_state(k, v):
    """fp32 (b*h, F, d_v + 1) state sum_j phi_k(k_j) [v_j, 1]^T of every head."""
    return ops.based_chunked_state(k, v)
