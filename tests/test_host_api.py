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
