"""Multi-rank host logic on CPU ``gloo`` ranks: head partitioning, the
sequence-parallel prefix exchange, and failure handling -- no GPU involved.
The compute steps are the CPU oracle, injected into the product's exchange
code, so only the partitioning / collective logic is under test here."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from trainium_linear_attention_b200 import distributed as D


@pytest.mark.parametrize("bh,world", [(128, 8), (64, 3), (5, 8), (16, 16), (1, 2)])
def test_head_ranges_cover_exactly_once(bh, world):
    seen = []
    for r in range(world):
        a, b = D.head_range(bh, r, world)
        assert 0 <= a <= b <= bh
        seen.extend(range(a, b))
    assert seen == list(range(bh))
    sizes = [D.head_range(bh, r, world)[1] - D.head_range(bh, r, world)[0] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_shard_heads_views():
    x = torch.arange(2 * 3 * 4 * 5, dtype=torch.float32).reshape(2, 3, 4, 5)
    parts = [D.shard_heads(x, r, 4) for r in range(4)]
    assert torch.equal(torch.cat([p[0] for p in parts]), x.reshape(6, 4, 5))


def test_exclusive_prefix_order():
    states = torch.arange(4 * 3, dtype=torch.float64).reshape(4, 3)
    assert torch.equal(D.exclusive_prefix(states, 0), torch.zeros(3, dtype=torch.float64))
    assert torch.equal(D.exclusive_prefix(states, 3), states[:3].sum(0))


class _FakeEvent:
    """Stands in for a CUDA event: a timestamp in ms, and a count of waits."""

    def __init__(self, t):
        self.t, self.waits = t, 0

    def elapsed_time(self, other):
        return other.t - self.t

    def synchronize(self):
        self.waits += 1


def test_sp_timings_resolve_after_the_steps():
    """Phase events stay pending until resolve(), which adds each forward's
    three phases; reset() drops what the warm-up recorded."""
    t = D.SPTimings()
    t.pending.append([_FakeEvent(x) for x in (0.0, 1.0, 1.5, 4.0)])
    t.reset()
    assert (t.steps, t.state_ms, t.exchange_ms, t.forward_ms) == (0, 0.0, 0.0, 0.0)
    steps = [[_FakeEvent(x) for x in (0.0, 2.0, 2.5, 6.0)],
             [_FakeEvent(x) for x in (10.0, 11.0, 12.5, 13.0)]]
    t.pending.extend(steps)
    assert t.steps == 0 and t.state_ms == 0.0  # nothing read before resolve
    t.resolve()
    assert t.steps == 2 and not t.pending
    assert (t.state_ms, t.exchange_ms, t.forward_ms) == (3.0, 2.0, 4.0)
    assert all(ev[3].waits == 1 for ev in steps)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sp_worker(rank, world, port, data, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v = (torch.from_numpy(a) for a in data)
        ql, kl, vl = (D.shard_tokens(x, rank, world) for x in (q, k, v))

        def state_fn(k_, v_):
            s = O.chunked_state(k_.numpy(), v_.numpy())
            return torch.from_numpy(s.reshape((-1,) + s.shape[-2:]))

        def forward_fn(q_, k_, v_, prefix):
            b, h = q_.shape[:2]
            init = prefix.numpy().reshape((b, h) + tuple(prefix.shape[-2:]))
            return torch.from_numpy(O.based_chunked(q_.numpy(), k_.numpy(), v_.numpy(), init_state=init))

        out = D.sequence_parallel_forward(ql, kl, vl, state_fn=state_fn, forward_fn=forward_fn)
        result_q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_parallel_exchange_on_gloo(world):
    rng = np.random.default_rng(world)
    t = 333  # not divisible by the world size
    q = rng.standard_normal((1, 2, t, 16)) * 0.5
    k = rng.standard_normal((1, 2, t, 16)) * 0.5
    v = rng.standard_normal((1, 2, t, 64)) * 0.5
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sp_worker, args=(r, world, port, (q, k, v), result_q)) for r in range(world)]
    for p in procs:
        p.start()
    outs = dict(result_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    y = np.concatenate([outs[r] for r in range(world)], axis=2)
    want = O.based_attn_reduced(q, k, v)
    assert O.rel_l2(y, want) < 1e-10


def _timeout_worker(rank, world, port, result_q):
    """Rank 1 never reaches the liveness check before the exchange: rank 0's
    check must end with an error within its timeout instead of hanging."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    if rank == 1:
        result_q.put((rank, "skipped"))
        result_q.close()
        result_q.join_thread()
        import time
        time.sleep(8)  # alive but absent from the collective
        os._exit(0)
    try:
        D.check_peers(timeout_s=2.0)
        result_q.put((rank, "completed"))
    except RuntimeError as e:  # the expected path
        result_q.put((rank, f"error:{type(e).__name__}"))
    result_q.close()
    result_q.join_thread()
    os._exit(0)  # skip the teardown handshake with the absent peer


def test_missing_rank_surfaces_as_error():
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(result_q.get(timeout=60) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "skipped"
    assert res[0].startswith("error:")
