"""numpy restatement of the reference's three attention paths (CPU oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Parity is pinned by
``tests/test_oracle_golden.py`` against vectors produced by the reference's
own PyTorch functions (``tests/golden/make_golden.py``).

Conventions shared with the CUDA kernels (all arrays are ``(b, h, t, d)``):

* ``scale = 1/sqrt(d_qk)`` where ``d_qk`` is q's last dim;
* causal masking includes the diagonal;
* ``eps`` is added to the denominator after the masked sum;
* the sliding window of token ``i`` is ``[i - W + 1, i]`` (W tokens incl. self).
"""

from __future__ import annotations

import math

import numpy as np


def rel_l2(y, y_ref) -> float:
    """||y - y_ref||_2 / ||y_ref||_2 over the whole tensor (float64)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    den = np.linalg.norm(y_ref.ravel())
    num = np.linalg.norm((y - y_ref).ravel())
    return float(num / den) if den > 0 else float(num)


def feature_dim(d_qk: int) -> int:
    """Width of the packed symmetric Taylor feature map: 1 + d + d(d+1)/2.

    153 for d=16, 2145 for d=64 (benchmarks/chunked_attention_benchmark.py:23-53).
    """
    return 1 + d_qk + d_qk * (d_qk + 1) // 2


# ---------------------------------------------------------------------------
# Parallel (quadratic) form
# ---------------------------------------------------------------------------

def based_attn_reduced(q, k, v, eps: float = 1e-6, dtype=np.float64, block: int = 1024):
    """BASED causal attention in the reduced scalar form.

    Follows kernels/pytorch_attention.py:27-42:
      s = (q * 1/sqrt(d)) @ k^T ; poly = 1 + s + s^2/2 ; masked = poly * tril
      den = masked.sum(-1) + eps ; out = masked @ v / den
    Computed in ``dtype`` (float64 by default).  Query rows are processed in
    blocks of ``block`` so the t x t matrix is never materialised whole; this
    is a memory optimisation only -- each row's sums are the same.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    d = q.shape[-1]
    t = q.shape[-2]
    scale = dtype(1.0 / math.sqrt(d)) if dtype is not np.float64 else 1.0 / math.sqrt(d)
    out = np.empty(q.shape[:-1] + (v.shape[-1],), dtype=dtype)
    qs = q * scale
    for r0 in range(0, t, block):
        r1 = min(t, r0 + block)
        s = np.matmul(qs[..., r0:r1, :], np.swapaxes(k[..., :r1, :], -1, -2))
        poly = 1.0 + s + 0.5 * s * s
        rows = np.arange(r0, r1)[:, None]
        cols = np.arange(r1)[None, :]
        poly = np.where(cols <= rows, poly, 0.0).astype(dtype, copy=False)
        den = poly.sum(axis=-1, keepdims=True) + eps
        out[..., r0:r1, :] = np.matmul(poly, v[..., :r1, :]) / den
    return out


# ---------------------------------------------------------------------------
# Feature maps
# ---------------------------------------------------------------------------

def taylor_feature_map(x):
    """The reference's packed Taylor feature map (width 1 + 2d + d(d-1)/2).

    Follows benchmarks/chunked_attention_benchmark.py:23-53:
      [1, x / d^(1/4), diag(x x^T) / (sqrt(d) sqrt(2)), strict-upper(x x^T) / sqrt(d)]
    with the strict upper triangle in ``torch.triu_indices(d, d, 1)`` order
    (row-major over i < j).
    """
    x = np.asarray(x)
    d = x.shape[-1]
    rd = math.sqrt(d)
    rrd = math.sqrt(rd)
    r2 = math.sqrt(2.0)
    iu, ju = np.triu_indices(d, 1)
    outer = x[..., :, None] * x[..., None, :]
    diag = outer[..., np.arange(d), np.arange(d)]
    off = outer[..., iu, ju]
    ones = np.ones(x.shape[:-1] + (1,), dtype=x.dtype)
    return np.concatenate([ones, x / rrd, diag / (rd * r2), off / rd], axis=-1)


def taylor_feature_map_full(x):
    """Full-vec form [1, x / d^(1/4), vec(x (x) x) / sqrt(2d)], width 1 + d + d^2.

    273 wide at d=16.  phi(q).phi(k) = 1 + s + s^2/2, identical to the packed
    map above (the 2x weight of an off-diagonal pair comes from counting
    (i,j) and (j,i) separately).
    """
    x = np.asarray(x)
    d = x.shape[-1]
    outer = (x[..., :, None] * x[..., None, :]).reshape(x.shape[:-1] + (d * d,))
    ones = np.ones(x.shape[:-1] + (1,), dtype=x.dtype)
    return np.concatenate([ones, x / math.sqrt(math.sqrt(d)), outer / math.sqrt(2.0 * d)], axis=-1)


def _pairs(d: int):
    """(i, j) with i <= j in row-major order: the kernels' quadratic features."""
    ii, jj = np.triu_indices(d, 0)
    return ii, jj


def kernel_feature_map_k(x):
    """Key-side feature basis used by the CUDA kernels and the public state.

    phi_k(k) = [1, k_0..k_{d-1}, k_i k_j for i <= j (row-major)], unscaled.
    Paired with :func:`kernel_feature_map_q`, phi_q(q).phi_k(k) = 1 + s + s^2/2
    exactly as the reference's symmetric map (chunked_attention_benchmark.py:34-53);
    the scale factors are all moved to the query side (powers of two at d=16).
    """
    x = np.asarray(x)
    d = x.shape[-1]
    ii, jj = _pairs(d)
    ones = np.ones(x.shape[:-1] + (1,), dtype=x.dtype)
    return np.concatenate([ones, x, x[..., ii] * x[..., jj]], axis=-1)


def kernel_feature_map_q(x):
    """Query-side partner of :func:`kernel_feature_map_k`.

    phi_q(q) = [1, q_i / sqrt(d), q_i q_j * w_ij] with w_ii = 1/(2d), w_ij = 1/d (i < j).
    """
    x = np.asarray(x)
    d = x.shape[-1]
    ii, jj = _pairs(d)
    w = np.where(ii == jj, 1.0 / (2.0 * d), 1.0 / d).astype(x.dtype)
    ones = np.ones(x.shape[:-1] + (1,), dtype=x.dtype)
    return np.concatenate([ones, x / math.sqrt(d), x[..., ii] * x[..., jj] * w], axis=-1)


def based_attn_features(q, k, v, eps: float = 1e-6, dtype=np.float64):
    """Dense normalised reference over explicit Taylor features.

    Follows benchmarks/chunked_attention_benchmark.py:55-65 (computed in
    ``dtype``; the reference uses float32 and casts the result to q.dtype).
    """
    qf = taylor_feature_map(np.asarray(q, dtype=dtype))
    kf = taylor_feature_map(np.asarray(k, dtype=dtype))
    s = np.matmul(qf, np.swapaxes(kf, -1, -2))
    t = s.shape[-1]
    s = s * np.tril(np.ones((t, t), dtype=dtype))
    den = s.sum(axis=-1, keepdims=True) + eps
    return np.matmul(s, np.asarray(v, dtype=dtype)) / den


def based_numerator_features(q, k, v, dtype=np.float64):
    """Dense numerator-only reference (benchmarks/chunked_attention_benchmark.py:68-76)."""
    qf = taylor_feature_map(np.asarray(q, dtype=dtype))
    kf = taylor_feature_map(np.asarray(k, dtype=dtype))
    s = np.matmul(qf, np.swapaxes(kf, -1, -2))
    t = s.shape[-1]
    s = s * np.tril(np.ones((t, t), dtype=dtype))
    return np.matmul(s, np.asarray(v, dtype=dtype))


# ---------------------------------------------------------------------------
# Chunked recurrent form
# ---------------------------------------------------------------------------

def chunked_state(k, v, dtype=np.float64):
    """Total KV state of a token range in the kernels' basis.

    Returns ``(..., F, d_v + 1)``: ``S[f, e] = sum_j phi_k(k_j)[f] v_j[e]`` and
    ``S[f, d_v] = sum_j phi_k(k_j)[f]`` (the normaliser column).  This is the
    state the reference's chunked kernel carries across chunks
    (kernels/nki_attention_chunked.py:100-102, ``S_f += K_f^T @ V``) with the
    normaliser added as one extra value column.
    """
    kf = kernel_feature_map_k(np.asarray(k, dtype=dtype))
    v = np.asarray(v, dtype=dtype)
    v_aug = np.concatenate([v, np.ones(v.shape[:-1] + (1,), dtype=dtype)], axis=-1)
    return np.matmul(np.swapaxes(kf, -1, -2), v_aug)


def based_chunked(q, k, v, chunk: int = 64, eps: float = 1e-6, normalize: bool = True,
                  init_state=None, return_state: bool = False, dtype=np.float64):
    """Chunked recurrent BASED attention.

    Follows the per-chunk recurrence of kernels/nki_attention_chunked.py:71-109:
      acc_o  = phi(Q_c) @ S          (state before the update, :94-95)
      scores = phi(Q_c) @ phi(K_c)^T (:97-98)
      S     += phi(K_c)^T @ V_c      (:100-102)
      acc_o += tril(scores) @ V_c    (:104-107)
    extended with the normaliser the reference omits (den = phi(q).z + the
    masked row sum + eps, z carried as the last state column).  The feature
    map is the reference's Taylor map (benchmarks/chunked_attention_benchmark.py:34-53)
    in the equivalent query/key-split basis of :func:`kernel_feature_map_k`.

    ``init_state`` (``(..., F, d_v+1)``) seeds the recurrence, as the
    sequence-parallel mode does with the prefix of earlier ranks.  With
    ``normalize=False`` the numerator alone is returned (the reference
    kernel's output, chunked_attention_benchmark.py:96-126).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    lead = q.shape[:-2]
    t = q.shape[-2]
    dv = v.shape[-1]
    F = feature_dim(q.shape[-1])
    if init_state is None:
        S = np.zeros(lead + (F, dv + 1), dtype=dtype)
    else:
        S = np.array(init_state, dtype=dtype, copy=True)
    out = np.empty(lead + (t, dv), dtype=dtype)
    v_aug = np.concatenate([v, np.ones(v.shape[:-1] + (1,), dtype=dtype)], axis=-1)
    for c0 in range(0, t, chunk):
        c1 = min(t, c0 + chunk)
        qf = kernel_feature_map_q(q[..., c0:c1, :])
        kf = kernel_feature_map_k(k[..., c0:c1, :])
        va = v_aug[..., c0:c1, :]
        acc = np.matmul(qf, S)
        scores = np.matmul(qf, np.swapaxes(kf, -1, -2))
        n = c1 - c0
        scores = scores * np.tril(np.ones((n, n), dtype=dtype))
        acc = acc + np.matmul(scores, va)
        S = S + np.matmul(np.swapaxes(kf, -1, -2), va)
        if normalize:
            out[..., c0:c1, :] = acc[..., :dv] / (acc[..., dv:] + eps)
        else:
            out[..., c0:c1, :] = acc[..., :dv]
    if return_state:
        return out, S
    return out


def identity_numerator(q, k, v, dtype=np.float64):
    """Dense identity-feature-map numerator, tril((q / sqrt(d)) k^T) v.

    Follows benchmarks/chunked_attention_benchmark.py:81-93
    (``ref_identity_numerator``: scale, mask, multiply by v; no feature map).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    d = q.shape[-1]
    t = q.shape[-2]
    s = np.matmul(q / math.sqrt(d), np.swapaxes(k, -1, -2))
    s = s * np.tril(np.ones((t, t), dtype=dtype))
    return np.matmul(s, v)


def identity_chunked(q, k, v, chunk: int = 64, init_state=None, return_state: bool = False,
                     dtype=np.float64):
    """Chunked identity-feature-map numerator.

    The recurrence of old/identity_linear_attn_nki_CHUNKED.py:38-59 (the
    reference's chunked identity kernel: acc = Q_c S; acc += tril(Q_c K_c^T) V_c;
    S += K_c^T V_c) with Q pre-scaled by 1/sqrt(d) as its caller does.  The
    state is ``(..., d_qk, d_v + 1)`` with sum k as the last column, the
    layout of the kernels' identity state.
    """
    q = np.asarray(q, dtype=dtype) / math.sqrt(q.shape[-1])
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    lead = q.shape[:-2]
    t = q.shape[-2]
    d, dv = k.shape[-1], v.shape[-1]
    S = (np.zeros(lead + (d, dv + 1), dtype=dtype) if init_state is None
         else np.array(init_state, dtype=dtype, copy=True))
    v_aug = np.concatenate([v, np.ones(v.shape[:-1] + (1,), dtype=dtype)], axis=-1)
    out = np.empty(lead + (t, dv), dtype=dtype)
    for c0 in range(0, t, chunk):
        c1 = min(t, c0 + chunk)
        qc, kc, va = q[..., c0:c1, :], k[..., c0:c1, :], v_aug[..., c0:c1, :]
        n = c1 - c0
        acc = np.matmul(qc, S) + np.matmul(
            np.matmul(qc, np.swapaxes(kc, -1, -2)) * np.tril(np.ones((n, n), dtype=dtype)), va)
        S = S + np.matmul(np.swapaxes(kc, -1, -2), va)
        out[..., c0:c1, :] = acc[..., :dv]
    if return_state:
        return out, S
    return out


# ---------------------------------------------------------------------------
# Sliding-window softmax
# ---------------------------------------------------------------------------

def sliding_window_attn(q, k, v, window: int = 64, dtype=np.float64):
    """Causal sliding-window softmax attention.

    Follows benchmarks/sliding_attention_benchmark.py:32-56: scores =
    (q / sqrt(d)) k^T, valid iff ``col <= row and col >= row - W + 1``,
    invalid scores are -inf, softmax over keys, times v.  Only the W-wide band
    is evaluated (the other scores are -inf and contribute exactly zero).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    d = q.shape[-1]
    t = q.shape[-2]
    W = max(1, min(int(window), t))
    pad = W - 1
    kp = np.concatenate([np.zeros(k.shape[:-2] + (pad, d), dtype=dtype), k], axis=-2)
    vp = np.concatenate([np.zeros(v.shape[:-2] + (pad, v.shape[-1]), dtype=dtype), v], axis=-2)
    # window w of query i covers padded rows i .. i + W - 1 == keys i - W + 1 .. i
    kw = np.lib.stride_tricks.sliding_window_view(kp, W, axis=-2)  # (..., t, d, W)
    vw = np.lib.stride_tricks.sliding_window_view(vp, W, axis=-2)  # (..., t, dv, W)
    s = np.einsum("...td,...tdw->...tw", q / math.sqrt(d), kw)
    key_idx = np.arange(t)[:, None] - (W - 1) + np.arange(W)[None, :]
    s = np.where(key_idx >= 0, s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.einsum("...tw,...tew->...te", p, vw)


def based_layer(q, k, v, window: int = 64, eps: float = 1e-6, dtype=np.float64):
    """The full BASED layer: BASED attention + sliding-window softmax attention.

    The composition stated at kernels/nki_attention_sliding.py:4-5, each half
    as restated above (kernels/pytorch_attention.py:27-42 and
    benchmarks/sliding_attention_benchmark.py:32-56).
    """
    return (based_attn_reduced(q, k, v, eps=eps, dtype=dtype)
            + sliding_window_attn(q, k, v, window, dtype=dtype))
