"""Generate the golden vectors that pin the CPU oracle to the reference.

Run once, in a container that has the reference checkout (its path is the
first argument, or $LA_REFERENCE_ROOT):

    python tests/golden/make_golden.py <reference-root>

It imports the reference's own PyTorch functions in place -- the reference
modules import ``torch_xla`` / ``neuronxcc`` at top level, which are replaced
by empty stub modules because only the pure-PyTorch reference functions are
called -- evaluates them on seeded inputs and writes ``golden.npz`` next to
this script.  The tests and the GPU box only ever read ``golden.npz``; they
never need the reference checkout.

Functions called (reference file:line):
  kernels/pytorch_attention.py:27                   ref_based_attn
  benchmarks/chunked_attention_benchmark.py:34      taylor_feature_map
  benchmarks/chunked_attention_benchmark.py:55      ref_based_attn (dense Taylor features)
  benchmarks/chunked_attention_benchmark.py:68      ref_based_numerator
  benchmarks/chunked_attention_benchmark.py:81      ref_identity_numerator
  benchmarks/sliding_attention_benchmark.py:32      ref_sliding_window_attn
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import numpy as np
import torch


def _install_stubs() -> None:
    for name in ("torch_xla", "torch_xla.core", "torch_xla.core.xla_model",
                 "neuronxcc", "neuronxcc.nki", "neuronxcc.nki.language"):
        sys.modules.setdefault(name, types.ModuleType(name))


def _randn(gen, shape, scale):
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * scale)


def main(ref_root: str) -> None:
    ref_root = str(Path(ref_root).resolve())
    _install_stubs()
    sys.path.insert(0, ref_root)
    from kernels.pytorch_attention import ref_based_attn as ref_reduced  # noqa: E402
    import benchmarks.chunked_attention_benchmark as cab  # noqa: E402
    import benchmarks.sliding_attention_benchmark as sab  # noqa: E402

    out = {}

    def based_case(name, shape_qk, dv, seed, eps=1e-6):
        gen = torch.Generator().manual_seed(seed)
        b, h, t, d = shape_qk
        q = _randn(gen, (b, h, t, d), 0.5)
        k = _randn(gen, (b, h, t, d), 0.5)
        v = _randn(gen, (b, h, t, dv), 0.5)
        out[f"{name}.q"], out[f"{name}.k"], out[f"{name}.v"] = q.numpy(), k.numpy(), v.numpy()
        out[f"{name}.out"] = ref_reduced(q, k, v, eps=eps).numpy()

    # benchmark configuration 1 exactly: B=1, H=4, N=256, d_qk=16, d_v=64, fp32, N(0,1)*0.5.
    based_case("c1", (1, 4, 256, 16), 64, seed=0)
    # ragged / odd lengths, d_v != d_qk, several heads
    based_case("par_odd", (2, 2, 65, 16), 32, seed=1)
    based_case("par_n1", (1, 2, 1, 16), 64, seed=2)
    based_case("par_d8", (1, 1, 130, 8), 24, seed=3)

    # feature maps
    gen = torch.Generator().manual_seed(10)
    for d in (16, 8, 4):
        x = _randn(gen, (5, d), 0.7)
        out[f"feat_d{d}.x"] = x.numpy()
        out[f"feat_d{d}.phi"] = cab.taylor_feature_map(x).numpy()

    # dense Taylor-feature references (normalised and numerator-only)
    gen = torch.Generator().manual_seed(20)
    q = _randn(gen, (1, 2, 192, 16), 0.5)
    k = _randn(gen, (1, 2, 192, 16), 0.5)
    v = _randn(gen, (1, 2, 192, 64), 0.5)
    out["dense.q"], out["dense.k"], out["dense.v"] = q.numpy(), k.numpy(), v.numpy()
    out["dense.out"] = cab.ref_based_attn(q, k, v, eps=1e-6).numpy()
    out["dense.num"] = cab.ref_based_numerator(q, k, v).numpy()

    # d_qk = 64: the reference chunked benchmark's default shape (B=1, H=2,
    # S=256, D=64, N(0,1) inputs; benchmarks/chunked_attention_benchmark.py:13-16)
    gen = torch.Generator().manual_seed(50)
    q = _randn(gen, (1, 2, 256, 64), 1.0)
    k = _randn(gen, (1, 2, 256, 64), 1.0)
    v = _randn(gen, (1, 2, 256, 64), 1.0)
    out["dense64.q"], out["dense64.k"], out["dense64.v"] = q.numpy(), k.numpy(), v.numpy()
    out["dense64.out"] = cab.ref_based_attn(q, k, v, eps=1e-6).numpy()
    out["dense64.num"] = cab.ref_based_numerator(q, k, v).numpy()

    # identity feature map, numerator only (fp32 inputs)
    def identity_case(name, shape_qk, dv, seed):
        gen = torch.Generator().manual_seed(seed)
        b, h, t, d = shape_qk
        q = _randn(gen, (b, h, t, d), 0.5)
        k = _randn(gen, (b, h, t, d), 0.5)
        v = _randn(gen, (b, h, t, dv), 0.5)
        out[f"{name}.q"], out[f"{name}.k"], out[f"{name}.v"] = q.numpy(), k.numpy(), v.numpy()
        out[f"{name}.num"] = cab.ref_identity_numerator(q, k, v).numpy()

    identity_case("ident", (1, 2, 192, 16), 64, seed=40)
    identity_case("ident_odd", (2, 2, 77, 16), 32, seed=41)

    # sliding window softmax
    def slide_case(name, shape, window, seed):
        gen = torch.Generator().manual_seed(seed)
        q = _randn(gen, shape, 1.0)
        k = _randn(gen, shape, 1.0)
        v = _randn(gen, shape, 1.0)
        out[f"{name}.q"], out[f"{name}.k"], out[f"{name}.v"] = q.numpy(), k.numpy(), v.numpy()
        out[f"{name}.window"] = np.array(window)
        out[f"{name}.out"] = sab.ref_sliding_window_attn(q, k, v, window_size=window).numpy()

    # the full BASED layer: the composition stated at
    # kernels/nki_attention_sliding.py:4-5 of the two reference functions
    def layer_case(name, shape_qk, dv, window, seed, scale):
        gen = torch.Generator().manual_seed(seed)
        b, h, t, d = shape_qk
        q = _randn(gen, (b, h, t, d), scale)
        k = _randn(gen, (b, h, t, d), scale)
        v = _randn(gen, (b, h, t, dv), scale)
        out[f"{name}.q"], out[f"{name}.k"], out[f"{name}.v"] = q.numpy(), k.numpy(), v.numpy()
        out[f"{name}.window"] = np.array(window)
        out[f"{name}.out"] = (ref_reduced(q, k, v, eps=1e-6)
                              + sab.ref_sliding_window_attn(q, k, v, window_size=window)).numpy()

    layer_case("layer_w64", (1, 2, 300, 16), 64, 64, seed=60, scale=0.5)
    layer_case("layer_w129", (1, 1, 400, 16), 32, 129, seed=61, scale=0.5)
    layer_case("layer_d32_w7", (2, 2, 77, 32), 32, 7, seed=62, scale=1.0)

    slide_case("slide_w64", (1, 1, 256, 64), 64, seed=30)
    slide_case("slide_w16_odd", (2, 2, 77, 32), 16, seed=31)
    slide_case("slide_w1", (1, 1, 10, 16), 1, seed=32)
    slide_case("slide_wbig", (1, 1, 100, 64), 300, seed=33)
    slide_case("slide_w100", (1, 1, 200, 64), 100, seed=34)

    dst = Path(__file__).with_name("golden.npz")
    np.savez_compressed(dst, **out)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LA_REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py <reference-root>")
    main(root)
