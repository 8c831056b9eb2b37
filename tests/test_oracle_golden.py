"""Pin the CPU oracle to the reference's own outputs (golden.npz) and check
the algebraic identities the kernels rely on.  CPU only."""

import numpy as np
import pytest

import oracle as O

PAR_CASES = ["c1", "par_odd", "par_n1", "par_d8"]
SLIDE_CASES = ["slide_w64", "slide_w16_odd", "slide_w1", "slide_wbig", "slide_w100"]


@pytest.mark.parametrize("case", PAR_CASES)
def test_reduced_form_matches_reference(golden, case):
    """oracle.based_attn_reduced vs kernels/pytorch_attention.py:27 ref_based_attn."""
    q, k, v = golden[f"{case}.q"], golden[f"{case}.k"], golden[f"{case}.v"]
    y = O.based_attn_reduced(q, k, v)
    assert O.rel_l2(y, golden[f"{case}.out"]) < 1e-6


@pytest.mark.parametrize("d", [16, 8, 4])
def test_feature_map_matches_reference(golden, d):
    """oracle.taylor_feature_map vs benchmarks/chunked_attention_benchmark.py:34."""
    x = golden[f"feat_d{d}.x"].astype(np.float64)
    phi = O.taylor_feature_map(x)
    assert phi.shape[-1] == 1 + 2 * d + d * (d - 1) // 2 == O.feature_dim(d)
    np.testing.assert_allclose(phi, golden[f"feat_d{d}.phi"], rtol=1e-6, atol=1e-7)


def test_feature_widths():
    assert O.feature_dim(16) == 153
    assert O.feature_dim(64) == 2145
    x = np.zeros((1, 16))
    assert O.taylor_feature_map_full(x).shape[-1] == 273


def test_dense_feature_refs_match_reference(golden):
    q, k, v = golden["dense.q"], golden["dense.k"], golden["dense.v"]
    assert O.rel_l2(O.based_attn_features(q, k, v), golden["dense.out"]) < 1e-6
    assert O.rel_l2(O.based_numerator_features(q, k, v), golden["dense.num"]) < 1e-6


@pytest.mark.parametrize("chunk", [1, 7, 64, 128, 1000])
def test_chunked_recurrence_matches_dense(golden, chunk):
    """The chunked restatement (nki_attention_chunked.py:71-109 + normaliser)
    equals the dense reference for any chunk size."""
    q, k, v = golden["dense.q"], golden["dense.k"], golden["dense.v"]
    assert O.rel_l2(O.based_chunked(q, k, v, chunk=chunk), golden["dense.out"]) < 1e-6
    num = O.based_chunked(q, k, v, chunk=chunk, normalize=False)
    assert O.rel_l2(num, golden["dense.num"]) < 1e-6


def test_chunked_matches_reduced_c1(golden):
    q, k, v = golden["c1.q"], golden["c1.k"], golden["c1.v"]
    assert O.rel_l2(O.based_chunked(q, k, v, chunk=64), golden["c1.out"]) < 1e-6


def test_feature_forms_agree():
    """273-wide full-vec, 153-wide packed and the kernels' q/k-split basis give
    the same kernel value 1 + s + s^2/2."""
    rng = np.random.default_rng(0)
    x, y = rng.standard_normal((7, 16)), rng.standard_normal((9, 16))
    s = x @ y.T / 4.0
    want = 1 + s + s * s / 2
    np.testing.assert_allclose(O.taylor_feature_map(x) @ O.taylor_feature_map(y).T, want, rtol=1e-12)
    np.testing.assert_allclose(O.taylor_feature_map_full(x) @ O.taylor_feature_map_full(y).T, want,
                               rtol=1e-12)
    np.testing.assert_allclose(O.kernel_feature_map_q(x) @ O.kernel_feature_map_k(y).T, want,
                               rtol=1e-12)


def test_state_is_additive_and_seeds_recurrence():
    """State of a concatenation is the sum of the parts; seeding the second
    half with the first half's state reproduces the whole -- the identity the
    segmented and sequence-parallel modes rely on."""
    rng = np.random.default_rng(1)
    q, k = rng.standard_normal((2, 3, 300, 16)) * 0.5, rng.standard_normal((2, 3, 300, 16)) * 0.5
    v = rng.standard_normal((2, 3, 300, 64)) * 0.5
    full, s_full = O.based_chunked(q, k, v, return_state=True)
    s1 = O.chunked_state(k[..., :130, :], v[..., :130, :])
    s2 = O.chunked_state(k[..., 130:, :], v[..., 130:, :])
    np.testing.assert_allclose(s1 + s2, s_full, rtol=1e-10, atol=1e-10)
    second = O.based_chunked(q[..., 130:, :], k[..., 130:, :], v[..., 130:, :], init_state=s1)
    assert O.rel_l2(second, full[..., 130:, :]) < 1e-12


@pytest.mark.parametrize("case", SLIDE_CASES)
def test_sliding_matches_reference(golden, case):
    """oracle.sliding_window_attn vs benchmarks/sliding_attention_benchmark.py:32."""
    q, k, v = golden[f"{case}.q"], golden[f"{case}.k"], golden[f"{case}.v"]
    y = O.sliding_window_attn(q, k, v, int(golden[f"{case}.window"]))
    assert O.rel_l2(y, golden[f"{case}.out"]) < 1e-6


def test_sliding_w1_is_identity(golden):
    q, k, v = golden["slide_w1.q"], golden["slide_w1.k"], golden["slide_w1.v"]
    np.testing.assert_allclose(O.sliding_window_attn(q, k, v, 1), v, rtol=0, atol=0)


def test_planted_error_is_caught(golden):
    """A mistake planted in the oracle's inputs must move rel-L2 far above the
    tolerances the parity tests use."""
    q, k, v = golden["c1.q"], golden["c1.k"], golden["c1.v"].copy()
    v[0, 1, 100, 3] += 1.0
    assert O.rel_l2(O.based_attn_reduced(q, k, v), golden["c1.out"]) > 1e-3


@pytest.mark.parametrize("case", ["ident", "ident_odd"])
def test_identity_numerator_matches_reference(golden, case):
    """oracle.identity_numerator / identity_chunked vs
    benchmarks/chunked_attention_benchmark.py:81 ref_identity_numerator, at
    several chunk sizes (the recurrence is exact algebra)."""
    q, k, v = golden[f"{case}.q"], golden[f"{case}.k"], golden[f"{case}.v"]
    want = golden[f"{case}.num"]
    assert O.rel_l2(O.identity_numerator(q, k, v), want) < 1e-6
    for chunk in (1, 13, 64, 1000):
        assert O.rel_l2(O.identity_chunked(q, k, v, chunk=chunk), want) < 1e-6


def test_identity_chunked_state_is_additive():
    """Seeding the second half with the first half's identity state gives the
    whole sequence (the sequence-split property the segmented kernels use)."""
    rng = np.random.default_rng(5)
    q, k = rng.standard_normal((2, 1, 2, 300, 16)) * 0.5
    v = rng.standard_normal((1, 2, 300, 24)) * 0.5
    whole = O.identity_chunked(q, k, v)
    a, s = O.identity_chunked(q[..., :128, :], k[..., :128, :], v[..., :128, :], return_state=True)
    b = O.identity_chunked(q[..., 128:, :], k[..., 128:, :], v[..., 128:, :], init_state=s)
    assert s.shape == (1, 2, 16, 25)
    assert O.rel_l2(np.concatenate([a, b], -2), whole) < 1e-12


def test_d64_refs_match_reference(golden):
    """d_qk = 64 (F = 2145), the reference chunked benchmark's default shape:
    the oracle's chunked recurrence and reduced form against its dense
    Taylor-feature references (benchmarks/chunked_attention_benchmark.py:55-76)."""
    q, k, v = (golden[f"dense64.{n}"].astype(np.float64) for n in "qkv")
    assert O.feature_dim(64) == 2145
    assert O.rel_l2(O.based_chunked(q, k, v), golden["dense64.out"]) < 1e-5
    assert O.rel_l2(O.based_chunked(q, k, v, normalize=False), golden["dense64.num"]) < 1e-5
    assert O.rel_l2(O.based_attn_reduced(q, k, v), golden["dense64.out"]) < 1e-5


@pytest.mark.parametrize("case", ["layer_w64", "layer_w129", "layer_d32_w7"])
def test_layer_matches_reference_composition(golden, case):
    """oracle.based_layer vs the reference's ref_based_attn +
    ref_sliding_window_attn on the same inputs (kernels/nki_attention_sliding.py:4-5)."""
    q, k, v = (golden[f"{case}.{n}"] for n in "qkv")
    y = O.based_layer(q, k, v, int(golden[f"{case}.window"]))
    assert O.rel_l2(y, golden[f"{case}.out"]) < 1e-6
