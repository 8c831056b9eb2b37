"""Run one kernel call on synthetic inputs, for profilers (ncu) and timing.

    python -m trainium_linear_attention_b200.profile_case --op chunked \\
        --batch 8 --heads 16 --seq-len 32768 [--calls 2] [--segments 0]

Inputs are generated on the device (iid N(0,1) * scale, seeded), one warm-up
call is made, then ``--calls`` calls; each call's device time is printed.
``--op`` is one of chunked, chunked_state, identity, layer, parallel, sliding.
"""

from __future__ import annotations

import argparse

import torch

from . import ops


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--op", choices=["chunked", "chunked_state", "identity", "layer", "parallel",
                                     "sliding"],
                    default="chunked")
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--seq-len", type=int, default=32768)
    ap.add_argument("--d-qk", type=int, default=16)
    ap.add_argument("--d-v", type=int, default=64)
    ap.add_argument("--window", type=int, default=64)
    ap.add_argument("--segments", type=int, default=0)
    ap.add_argument("--dtype", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--calls", type=int, default=2)
    args = ap.parse_args()

    dev = torch.device("cuda", 0)
    dtype = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    g = torch.Generator(device=dev).manual_seed(0)
    b, h, t = args.batch, args.heads, args.seq_len
    dqk = args.d_v if args.op == "sliding" else args.d_qk
    scale = 1.0 if args.op == "sliding" else 0.5
    q = (torch.randn(b, h, t, dqk, generator=g, device=dev) * scale).to(dtype)
    k = (torch.randn(b, h, t, dqk, generator=g, device=dev) * scale).to(dtype)
    v = (torch.randn(b, h, t, args.d_v, generator=g, device=dev) * scale).to(dtype)

    if args.op == "chunked":
        def call():
            return ops.based_chunked(q, k, v, segments=args.segments)
    elif args.op == "chunked_state":
        def call():
            return ops.based_chunked_state(k, v, segments=args.segments)
    elif args.op == "identity":
        def call():
            return ops.based_chunked(q, k, v, normalize=False, feature_map="identity",
                                     segments=args.segments)
    elif args.op == "layer":
        def call():
            return ops.based_layer(q, k, v, window_size=args.window, segments=args.segments)
    elif args.op == "parallel":
        def call():
            return ops.based_parallel(q, k, v)
    else:
        def call():
            return ops.sliding_window(q, k, v, window_size=args.window)

    call()
    torch.cuda.synchronize()
    for i in range(args.calls):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        call()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e)
        print(f"call {i}: {ms:.4f} ms  ({b * t / (ms / 1e3):.4e} tokens/s)")


if __name__ == "__main__":
    main()
