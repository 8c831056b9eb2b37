"""Host-side API behaviour on CPU: signatures mirror the reference, bad inputs
raise, CPU tensors are refused (no CPU fallback), and the plain-PyTorch
reference formulas the package re-exports agree with the oracle."""

import inspect

import numpy as np
import pytest
import torch

import oracle as O
import trainium_linear_attention_b200 as T
from trainium_linear_attention_b200 import ops
from trainium_linear_attention_b200.kernels import chunked_attention as CA
from trainium_linear_attention_b200.kernels import pytorch_attention as PA
from trainium_linear_attention_b200.kernels import sliding_attention as SA


def test_signatures_match_reference():
    # kernels/pytorch_attention.py:27,44,81
    for fn in (PA.ref_based_attn, PA.solution_nki, PA.solution):
        sig = inspect.signature(fn)
        assert list(sig.parameters) == ["q", "k", "v", "eps"]
        assert sig.parameters["eps"].default == 1e-6
    # benchmarks/chunked_attention_benchmark.py:96
    sig = inspect.signature(CA.chunked_nki_numerator)
    assert list(sig.parameters) == ["q", "k", "v", "chunk_size"]
    assert sig.parameters["chunk_size"].default == 64
    # benchmarks/sliding_attention_benchmark.py:59
    sig = inspect.signature(SA.nki_sliding_window_attn)
    assert list(sig.parameters) == ["q", "k", "v", "window_size", "block_size"]
    assert sig.parameters["window_size"].default == 64 and sig.parameters["block_size"].default == 64


def test_cpu_tensors_are_refused():
    q = torch.randn(1, 2, 8, 16)
    v = torch.randn(1, 2, 8, 64)
    for fn in (T.solution_nki, T.solution, T.chunked_nki_numerator, T.based_chunked):
        with pytest.raises(ValueError, match="CUDA"):
            fn(q, q, v)
    with pytest.raises(ValueError, match="CUDA"):
        T.nki_sliding_window_attn(q, q, q)


def test_bad_shapes_and_dtypes():
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(ValueError):
        ops._check_qkv(q, q, torch.randn(1, 2, 9, 64))
    with pytest.raises(ValueError):
        ops._check_qkv(q[0], q[0], q[0])
    with pytest.raises(TypeError):
        ops._dtype_code(q.half())
    with pytest.raises(TypeError):
        ops._check_qkv(q, q.double(), q)


def test_reference_formulas_agree_with_oracle(golden):
    q, k, v = (torch.from_numpy(golden[f"c1.{n}"]) for n in "qkv")
    y = PA.ref_based_attn(q, k, v)
    assert O.rel_l2(y.numpy(), golden["c1.out"]) < 1e-6
    q, k, v = (torch.from_numpy(golden[f"dense.{n}"]) for n in "qkv")
    assert O.rel_l2(CA.ref_based_attn(q, k, v).numpy(), golden["dense.out"]) < 1e-6
    assert O.rel_l2(CA.ref_based_numerator(q, k, v).numpy(), golden["dense.num"]) < 1e-6
    x = torch.from_numpy(golden["feat_d16.x"])
    np.testing.assert_allclose(CA.taylor_feature_map(x).numpy(), golden["feat_d16.phi"], rtol=1e-6)
    q, k, v = (torch.from_numpy(golden[f"slide_w16_odd.{n}"]) for n in "qkv")
    assert O.rel_l2(SA.ref_sliding_window_attn(q, k, v, 16).numpy(), golden["slide_w16_odd.out"]) < 1e-6


def test_native_check_is_false_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert PA._check_nki() is False


def test_based_modules_match_reference_wrappers():
    """benchmarks/based_attention_benchmark.py:24-69: same constructor
    arguments and parameter names; the reference-path module equals the
    projections around the oracle's BASED attention; the kernel module
    refuses CPU tensors (no CPU fallback)."""
    from trainium_linear_attention_b200.benchmarks import based_attention_benchmark as BM

    for cls in (BM.TrainiumBasedLinearAttention, BM.TrainiumBasedLinearAttentionNKI):
        sig = inspect.signature(cls.__init__)
        assert list(sig.parameters)[:4] == ["self", "dim", "heads", "eps"]
        assert sig.parameters["heads"].default == 8 and sig.parameters["eps"].default == 1e-6
    torch.manual_seed(3)
    ref = BM.TrainiumBasedLinearAttention(32, heads=2).double()
    assert sorted(ref.state_dict()) == ["k_proj.weight", "o_proj.weight", "q_proj.weight",
                                        "v_proj.weight"]
    x = torch.randn(2, 40, 32, dtype=torch.float64)
    with torch.no_grad():
        y = ref(x)
        heads = [p(x).view(2, 40, 2, 16).transpose(1, 2).numpy()
                 for p in (ref.q_proj, ref.k_proj, ref.v_proj)]
        att = torch.from_numpy(O.based_attn_reduced(*heads))
        want = ref.o_proj(att.transpose(1, 2).reshape(2, 40, 32))
    assert O.rel_l2(y.numpy(), want.numpy()) <= 1e-10
    mod = BM.TrainiumBasedLinearAttentionNKI(32, heads=2, window_size=8)
    mod.load_state_dict(ref.float().state_dict())
    with pytest.raises(ValueError, match="CUDA"):
        mod(x.float())
    with pytest.raises(ValueError):
        BM.TrainiumBasedLinearAttentionNKI(32, heads=2, attention="dense")
