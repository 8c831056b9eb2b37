"""Measure the configurations other than the headline one, one JSON line each.

    python -m trainium_linear_attention_b200.sweep [--what c2,c3,c5] [--steps 20]

c2   chunked BASED, B=4, H=16, N=2048, d_qk=16, d_v=64 (configuration 2)
c3   sliding-window softmax attention, B=4, H=16, N=4096, d=64, W=64 (config 3)
c5   parallel and chunked BASED at B*N = 262144, H=16, N = 256 .. 65536 (by
     default; --c5-min-n / --c5-max-n): the crossover that ``solution()``
     dispatches on (config 5 is N = 512 .. 65536; N = 256 is the short side
     of the crossover)
ident   chunked identity-feature-map numerator, B=4, H=16, N=2048, d_qk=16, d_v=64
d64     chunked BASED at d_qk = d_v = 64 (F = 2145, the state split over a 16-CTA
        cluster), B=1, H=16, N=4096
share   configuration 4's per-rank work at 2, 4 and 8 GPUs (64, 32, 16 heads of
        N = 32768, heads sharded, no collective), timed on one GPU
layer   the full BASED layer (chunked BASED + sliding window W=64; the sliding
        kernel adds into the chunked kernel's output): B=4, H=16, N=2048,
        d_qk=16, d_v=64, and at d_qk = d_v = 64, B=1, H=16, N=4096

All inputs are bf16, iid N(0,1) * scale (0.5 for BASED, 1 for sliding),
generated on the device from a fixed seed.  Each point: warm-up calls, then
timed calls (at least --steps, or fewer when one call takes long), each
bracketed by CUDA events on the launching stream with a 256 MB L2 flush
before it (outside the events).  tokens/s counts B*N (heads not counted, the
reference's convention).  ``hbm_frac`` = algorithmic bytes/s over the
measured HBM peak (5120 B/token for BASED, 8192 for sliding at d=64);
``tc_frac`` = algorithmic flop/s over the measured bf16 peak, with the
parallel form's (N+1)/2 * H * (2 d_qk + 2 d_v + 4) flop per token.
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from . import ops

ROOT = Path(__file__).resolve().parent.parent
FLUSH_BYTES = 256 << 20


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]) * 1e9, float(d["bf16_tflops"]) * 1e12, "measured"
    return 6650e9, 1590e12, "fallback"


def time_calls(fn, steps: int, budget_s: float = 1.5):
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    times = []
    total = 0.0
    while len(times) < steps and (len(times) < 3 or total < budget_s):
        flush.fill_(len(times) & 0xFF)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ms = s.elapsed_time(e)
        times.append(ms)
        total += ms / 1e3
    return statistics.median(times), len(times)


def inputs(b, h, n, dqk, dv, scale, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(b, h, n, dqk, generator=g, device="cuda") * scale).bfloat16()
    k = (torch.randn(b, h, n, dqk, generator=g, device="cuda") * scale).bfloat16()
    v = (torch.randn(b, h, n, dv, generator=g, device="cuda") * scale).bfloat16()
    return q, k, v


def line(name, op, b, h, n, dqk, dv, ms, steps, bytes_per_token, flop_per_token, extra=None):
    hbm, tc, src = peaks()
    tok_s = b * n / (ms / 1e3)
    d = {"config": name, "op": op, "batch": b, "heads": h, "seq_len": n, "d_qk": dqk, "d_v": dv,
         "dtype": "bf16", "ms": round(ms, 4), "timed_calls": steps, "tokens_per_s": tok_s,
         "hbm_frac": tok_s * bytes_per_token / hbm,
         "tc_frac": tok_s * flop_per_token / tc if flop_per_token else None,
         "peak_source": src}
    if extra:
        d.update(extra)
    print(json.dumps(d), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--what", default="c2,c3,c5,share,ident,d64,layer")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--c5-min-n", type=int, default=256)
    ap.add_argument("--c5-max-n", type=int, default=65536)
    args = ap.parse_args()
    what = set(args.what.split(","))
    h, dqk, dv = 16, 16, 64
    based_bytes = h * ((2 * dqk + dv) * 2 + dv * 2)
    if "c2" in what:
        b, n = 4, 2048
        q, k, v = inputs(b, h, n, dqk, dv, 0.5)
        ms, st = time_calls(lambda: ops.based_chunked(q, k, v), args.steps)
        line("c2", "chunked", b, h, n, dqk, dv, ms, st, based_bytes, None)
    if "c3" in what:
        b, n, d, w = 4, 4096, 64, 64
        q, k, v = inputs(b, h, n, d, d, 1.0)
        ms, st = time_calls(lambda: ops.sliding_window(q, k, v, window_size=w), args.steps)
        line("c3", "sliding", b, h, n, d, d, ms, st, h * (3 * d * 2 + d * 2), h * w * 4 * d,
             {"window": w})
    if "share" in what:
        for ranks in (2, 4, 8):
            b_heads = 128 // ranks
            q, k, v = inputs(1, b_heads, 32768, dqk, dv, 0.5)
            ms, st = time_calls(lambda: ops.based_chunked(q, k, v), args.steps)
            g, _ = ops.chunked_plan(b_heads, 32768, dqk, dv, torch.bfloat16)
            # tokens/s and hbm_frac of this rank (b_heads / 16 of the B*N tokens);
            # job_tokens_per_s: all ranks at this time
            line("share", "chunked", b_heads / 16, 16, 32768, dqk, dv, ms, st, based_bytes, None,
                 {"ranks": ranks, "heads_per_rank": b_heads, "segments": g,
                  "job_tokens_per_s": 8 * 32768 / (ms / 1e3)})
            del q, k, v
    if "ident" in what:
        b, n = 4, 2048
        q, k, v = inputs(b, h, n, dqk, dv, 0.5)
        ms, st = time_calls(lambda: ops.based_chunked(q, k, v, normalize=False,
                                                      feature_map="identity"), args.steps)
        line("ident", "chunked_identity", b, h, n, dqk, dv, ms, st, based_bytes, None)
    if "d64" in what:
        b, n, d = 1, 4096, 64
        q, k, v = inputs(b, h, n, d, d, 0.5)
        ms, st = time_calls(lambda: ops.based_chunked(q, k, v), args.steps)
        f = 1 + d + d * (d + 1) // 2
        line("d64", "chunked_d64", b, h, n, d, d, ms, st, h * (4 * d * 2),
             h * (4 * f * (d + 1) + (64 + 1) / 2 * (2 * d + 2 * d + 4)))
    if "layer" in what:
        for b, n, d_qk, d_v in ((4, 2048, 16, 64), (1, 4096, 64, 64)):
            q, k, v = inputs(b, h, n, d_qk, d_v, 0.5)
            ms, st = time_calls(lambda: ops.based_layer(q, k, v, window_size=64), args.steps)
            line("layer", "based_plus_sliding", b, h, n, d_qk, d_v, ms, st,
                 h * ((2 * d_qk + d_v) * 2 + d_v * 2), None, {"window": 64})
            del q, k, v
    if "c5" in what:
        n = args.c5_min_n
        while n <= args.c5_max_n:
            b = 262144 // n
            q, k, v = inputs(b, h, n, dqk, dv, 0.5)
            for op in ("parallel", "chunked"):
                fn = (lambda: ops.based_parallel(q, k, v)) if op == "parallel" else \
                     (lambda: ops.based_chunked(q, k, v))
                ms, st = time_calls(fn, args.steps)
                flop = h * (n + 1) / 2 * (2 * dqk + 2 * dv + 4) if op == "parallel" else None
                line("c5", op, b, h, n, dqk, dv, ms, st, based_bytes, flop)
            del q, k, v
            n *= 2


if __name__ == "__main__":
    main()
