#!/usr/bin/env python
"""Benchmark of the chunked BASED hot path (benchmark configuration 4), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--mode heads|sp] [--seq-len N] [--segments G]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Default workload (benchmark configuration 4): chunked BASED, B=8, H=16, N=32768,
d_qk=16, d_v=64, bf16 inputs iid N(0,1)*0.5 (seeded per head), sharded by
batch x head over the ranks (no collective on the data path).  A step is one
pass of the chunked kernel over the rank's heads.  ``--mode sp`` runs the
sequence-parallel variant (B=1, H=16, N=262144 split over the ranks, one
NCCL all-gather of per-rank states per step).

Timing: W untimed warm-up steps, then exactly K steps, each bracketed by CUDA
events on the launching stream; the per-rank sum is max-reduced over ranks
after a barrier.  After the barrier and synchronize that open the timed
region, a ~0.1 ms spin kernel (outside the events) keeps the GPU busy while
the host enqueues the first step, so that the first step, like the others,
is timed from a queue the host has already filled (otherwise it alone would
include the host's ~30 us per-call launch cost and the idle GPU's wake-up;
``e2e`` keeps every host cost).  L2: a step streams 1.34 GB (config 4) through the 126 MB
L2, so no data of a step survives to the next; ``--l2 flush`` additionally
writes a 256 MB buffer before every timed step (outside the events; its dirty
lines are then written back during the step).  ``value`` = B*N tokens (heads not counted, the reference's
convention) / that time.  ``e2e`` repeats the measurement through the public
API with pinned host inputs copied in and the output copied back every step
(heads mode: ``based_chunked_host``, which copies one group of heads while
the kernels of the previous group run and the group before is copied back;
sequence-parallel mode: serial copies around the sequence-parallel forward).
``sp_phases_ms`` (sequence-parallel mode) splits a step into the state pass,
the NCCL all-gather with the prefix sum, and the seeded forward.
``--impl reference`` times the CPU port of the reference's chunked algorithm
(oracle/, numpy, one single-threaded worker process per usable core) on a
bounded sample of the same workload.
The other configurations (C2, C3 sliding window, the C5 parallel/chunked
crossover sweep) are measured by ``python -m trainium_linear_attention_b200.sweep``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WORKLOADS = {
    # name: (batch, heads, seq_len, d_qk, d_v, kind)
    "c4": (8, 16, 32768, 16, 64, "chunked"),
}
METRIC = "BASED chunked attn tokens/s @N=32K,H=16 on 1/2/4/8 B200; % of roofline"
L2_FLUSH_BYTES = 256 << 20
QUEUE_SPIN_CYCLES = 200_000  # ~0.1 ms at 1.9 GHz: longer than the host's enqueue of one step


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--mode", choices=["heads", "sp"], default="heads")
    ap.add_argument("--seq-len", type=int, default=None, help="override N (not a bench line)")
    ap.add_argument("--segments", type=int, default=0, help="0 = library's choice")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-groups", type=int, default=8,
                    help="head groups of the end-to-end leg (copies overlap the kernels)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--l2", choices=["none", "flush"], default="none",
                    help="none: the inputs (1.34 GB per step) exceed L2; flush: also write 256 MB "
                         "before every timed step")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    return args


# --------------------------------------------------------------------------- peaks

def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profile_traffic_per_token(kernel: str):
    """DRAM bytes per token from the committed ncu summary, if present.

    The summary line reads ``traffic_bytes_per_token: <float>`` and comes from
    one ``ncu`` capture of the named kernel (see the summary's own header)."""
    p = ROOT / "profiles" / f"{kernel}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_token:"):
            try:
                return float(line.split(":", 1)[1])
            except ValueError:
                return None
    return None


# --------------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML from start() to
    stop(), keeping only the samples taken while the window is open (the
    timed region): NVML is initialised and the thread started before the
    warm-up, so the GPU does not idle for them between warm-up and timing."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
        0x0000000000000002: "applications_clocks_setting",
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._window = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            if self._window.is_set():
                try:
                    self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                    mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    for bit, name in self.REASONS.items():
                        if mask & bit:
                            self.reasons.add(name)
                except Exception:
                    pass
            time.sleep(self.period)

    def start(self):
        if self.nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def open_window(self):
        self._window.set()

    def close_window(self):
        self._window.clear()

    def stop(self):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# --------------------------------------------------------------------------- inputs

def make_head_inputs(heads_range, seq_len, d_qk, d_v, scale, seed=1234):
    """Per-head seeded N(0,1)*scale inputs, generated on the host in fp32.

    Head ``i`` (flattened b*H + h) always gets generator seed ``seed + i``, so
    any rank's shard is reproducible on its own."""
    import torch
    qs, ks, vs = [], [], []
    for i in range(*heads_range):
        g = torch.Generator().manual_seed(seed + i)
        qs.append(torch.randn(seq_len, d_qk, generator=g) * scale)
        ks.append(torch.randn(seq_len, d_qk, generator=g) * scale)
        vs.append(torch.randn(seq_len, d_v, generator=g) * scale)
    return torch.stack(qs), torch.stack(ks), torch.stack(vs)


# --------------------------------------------------------------------------- reference arm

# The CPU arm: the oracle's numpy port of the reference chunked recurrence,
# the sampled heads split over single-threaded worker processes (one per
# usable core, at most one per head).  Its small per-chunk matmuls do not
# speed up with BLAS threads, so the heads are what runs in parallel.  The
# workers are started with "spawn" (safe after CUDA use in this process) and
# each generates its heads' inputs once, outside the timed passes.
def _cpu_worker_main(conn, heads, n, d_qk, d_v):
    import numpy as np
    from threadpoolctl import threadpool_limits
    import oracle as O
    limits = threadpool_limits(limits=1)  # noqa: F841  (held for the worker's life)
    inputs = []
    for head in heads:
        rng = np.random.default_rng(7 + head)
        inputs.append(tuple((rng.standard_normal((1, 1, n, d)) * 0.5).astype(np.float32)
                            for d in (d_qk, d_qk, d_v)))
    conn.send("ready")
    while conn.recv() == "go":
        for q, k, v in inputs:
            O.based_chunked(q, k, v, chunk=64, dtype=np.float32)
        conn.send("done")


def usable_cores():
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


class CpuPort:
    """Times `sample_heads` heads of `sample_tokens` tokens of the CPU port."""

    def __init__(self, d_qk, d_v, sample_heads, sample_tokens):
        import multiprocessing as mp
        ctx = mp.get_context("spawn")
        self.workers = max(1, min(usable_cores(), sample_heads))
        self.sample_heads, self.sample_tokens = sample_heads, sample_tokens
        self.conns, self.procs = [], []
        for w in range(self.workers):
            parent, child = ctx.Pipe()
            proc = ctx.Process(target=_cpu_worker_main, daemon=True,
                               args=(child, list(range(w, sample_heads, self.workers)),
                                     sample_tokens, d_qk, d_v))
            proc.start()
            self.conns.append(parent)
            self.procs.append(proc)
        for c in self.conns:
            if c.recv() != "ready":
                raise RuntimeError("CPU port worker failed to start")

    def sample(self, heads_in_metric):
        """(metric tokens/s, seconds) of one pass over the sampled heads: the
        metric counts B*N tokens for all `heads_in_metric` heads, so the sample
        stands for sample_tokens * sample_heads / heads_in_metric tokens."""
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("go")
        for c in self.conns:
            c.recv()
        dt = time.perf_counter() - t0
        return self.sample_tokens * self.sample_heads / heads_in_metric / dt, dt

    def describe(self):
        return (f"{self.sample_heads} heads x {self.sample_tokens} tokens per step, fp32 numpy "
                "port of the reference chunked recurrence (oracle/based_oracle.py based_chunked), "
                f"heads split over {self.workers} single-threaded worker processes")

    def close(self):
        for c in self.conns:
            try:
                c.send("stop")
            except (BrokenPipeError, OSError):
                pass
        for proc in self.procs:
            proc.join(timeout=30)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 alone runs the CPU arm
    b, h, n, dqk, dv, kind = WORKLOADS["c4"]
    n = args.seq_len or n
    sample_heads = 16 if args.mode == "heads" else 4
    port = CpuPort(dqk, dv, sample_heads, min(n, 32768))
    try:
        for _ in range(args.warmup):
            port.sample(h)
        secs = 0.0
        for _ in range(args.steps):
            secs += port.sample(h)[1]
    finally:
        port.close()
    value = args.steps * port.sample_tokens * port.sample_heads / h / secs
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, b, h, n, dqk, dv),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": port.workers,
                         "kind": "port", "sample": port.describe()},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def config_dict(args, b, h, n, dqk, dv):
    return {"workload": ("C4 chunked BASED, batch x head sharded" if args.mode == "heads"
                         else "C4-SP chunked BASED, sequence parallel"),
            "batch": b, "heads": h, "seq_len": n, "d_qk": dqk, "d_v": dv, "chunk_size": 64,
            "global_batch": b, "parallelism": (f"heads{args.gpus}" if args.mode == "heads"
                                               else f"sp{args.gpus}"),
            "inputs": "iid N(0,1)*0.5, seeded, bf16 (the reference arm: fp32 numpy sample)",
            "l2": ("flushed (256 MB write) before every timed step" if args.l2 == "flush" else
                   "not flushed: a rank's step reads and writes its share of config 4's "
                   "1.34 GB (>= 168 MB at 8 GPUs), more than the 126 MB L2")}


# --------------------------------------------------------------------------- our arm

def run_ours(args):
    import torch
    import torch.distributed as dist
    from trainium_linear_attention_b200 import distributed as D
    from trainium_linear_attention_b200 import ops

    rank, world, local = D.init_process_group_from_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    if args.mode == "heads":
        b, h, n, dqk, dv, _ = WORKLOADS["c4"]
        n = args.seq_len or n
        lo, hi = D.head_range(b * h, rank, world)
        tok_lo, tok_hi = 0, n
    else:
        b, h, n, dqk, dv = 1, 16, args.seq_len or 262144, 16, 64
        lo, hi = 0, b * h
        tok_lo, tok_hi = D.token_range(n, rank, world)
    local_heads = hi - lo
    t_local = tok_hi - tok_lo

    # inputs: host fp32 -> bf16 (pinned for the end-to-end leg) -> device
    if args.mode == "heads":
        qh, kh, vh = make_head_inputs((lo, hi), n, dqk, dv, 0.5)
    else:
        qf, kf, vf = make_head_inputs((0, h), n, dqk, dv, 0.5)
        qh, kh, vh = (x[:, tok_lo:tok_hi] for x in (qf, kf, vf))
    qh, kh, vh = (x.to(torch.bfloat16).reshape(1, local_heads, t_local, -1).contiguous().pin_memory()
                  for x in (qh, kh, vh))
    q, k, v = (x.to(dev) for x in (qh, kh, vh))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)

    seg = args.segments
    g, ws_bytes = ops.chunked_plan(local_heads, t_local, dqk, dv, torch.bfloat16, seg)
    workspace = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    if args.mode == "heads":
        def step():
            return ops.based_chunked(q, k, v, chunk_size=64, segments=seg, workspace=workspace)
    else:
        # phase events stay pending until after the timed steps (no host
        # wait inside a step)
        sp_timings = D.SPTimings()

        def step():
            return D.sequence_parallel_forward(q, k, v, chunk_size=64, timings=sp_timings)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident value: the launch count and the clock sampler
    # first, then the warm-up directly before the timed steps (no idle GPU
    # between them but the barrier)
    launches_per_step = count_library_launches(step)
    clk = ClockSampler(local).start()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for _ in range(args.warmup):
        step()
    if args.mode == "sp":
        sp_timings.reset()
    barrier()
    torch.cuda.synchronize()
    clk.open_window()
    torch.cuda._sleep(QUEUE_SPIN_CYCLES)  # busy GPU while the first step is enqueued
    for i in range(args.steps):
        if args.l2 == "flush":
            flush.zero_()
        starts[i].record(stream)
        step()
        ends[i].record(stream)
    torch.cuda.synchronize()
    clk.close_window()
    clk.stop()
    barrier()
    torch.cuda.synchronize()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(step_ms))
    tokens = b * n  # B*N, the reference's tokens convention (heads not counted)
    value = tokens * args.steps / (total_ms / 1e3)
    ms_per_step = total_ms / args.steps
    sp_split = None
    if args.mode == "sp":
        # per-step device time of each phase, max over ranks (state pass,
        # NCCL all-gather + prefix sum, seeded forward)
        sp_timings.resolve()
        n_sp = max(1, sp_timings.steps)
        sp_split = {key: max_over_ranks(getattr(sp_timings, key) / n_sp)
                    for key in ("state_ms", "exchange_ms", "forward_ms")}

    # ---- end to end through the public API (pinned host in, host out)
    e2e = None
    if not args.no_e2e:
        out_host = torch.empty((1, local_heads, t_local, dv), dtype=torch.bfloat16).pin_memory()
        from trainium_linear_attention_b200 import based_chunked_host as api_based_chunked_host

        if args.mode == "heads":
            def e2e_step():
                # copies of one group of heads overlap the kernels of the previous one
                api_based_chunked_host(qh, kh, vh, chunk_size=64, out=out_host,
                                       head_groups=args.e2e_groups)
        else:
            def e2e_step():
                qd = qh.to(dev, non_blocking=True)
                kd = kh.to(dev, non_blocking=True)
                vd = vh.to(dev, non_blocking=True)
                y = D.sequence_parallel_forward(qd, kd, vd, chunk_size=64)
                out_host.copy_(y, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        es = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        es[0].record(stream)
        for i in range(args.steps):
            e2e_step()
            es[i + 1].record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(es[0].elapsed_time(es[-1]))
        h2d = sum(x.numel() * x.element_size() for x in (qh, kh, vh))
        d2h = out_host.numel() * out_host.element_size()
        e2e = {"value": tokens * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "ms_per_step": e2e_ms / args.steps,
               "pipelining": (f"{args.e2e_groups} head groups, copies on two side streams"
                              if args.mode == "heads" else "serial copies")}

    # ---- roofline of the step on this rank (the chunked kernel dominates it)
    hbm_gbs, tflops, peak_kind = measured_peaks()
    local_tokens = local_heads * t_local  # token-heads this rank processes
    alg_bytes = local_tokens * (2 * dqk * 2 + dv * 2 + dv * 2)  # q,k,v read + out write, bf16
    rank_ms = sum(step_ms) / args.steps
    achieved = alg_bytes / (rank_ms / 1e3) / 1e9
    traffic_tok = profile_traffic_per_token("chunked_output_c4")
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_gbs, "unit": "GB/s",
                "frac": achieved / hbm_gbs, "peak_source": peak_kind,
                "traffic": (traffic_tok * local_tokens / 16 if traffic_tok else None),
                "alg_bytes_per_launch": alg_bytes,
                "flop_frac": (local_tokens / 16 * 1216592) / (rank_ms / 1e3) / (tflops * 1e12)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        port = CpuPort(dqk, dv, 16, min(n, 32768))
        try:
            port.sample(h)  # warm-up
            rates, secs = [], 0.0
            while secs < 12.0 and len(rates) < 12:
                r, dt = port.sample(h)
                rates.append(r)
                secs += dt
        finally:
            port.close()
        cpu = {"value": statistics.median(rates), "unit": "tokens/s", "cores": port.workers,
               "kind": "port", "sample": f"{port.describe()}, {len(rates)} runs (median)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": config_dict(args, b, h, n, dqk, dv),
            "plan": {"segments_per_head": g, "local_heads": local_heads,
                     "local_tokens": t_local},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clk.summary(), "gpu_launches": launches_per_step * args.steps,
        }
        if sp_split is not None:
            line["sp_phases_ms"] = sp_split
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def count_library_launches(step) -> int:
    """Kernels of this library one untimed step launches (its launch counter)."""
    import torch
    from trainium_linear_attention_b200 import _native as N
    before = N.lib().la_launch_count()
    step()
    torch.cuda.synchronize()
    return int(N.lib().la_launch_count() - before)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
