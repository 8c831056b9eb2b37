"""Multi-GPU execution: batch x head sharding and sequence parallelism.

The reference is single-device (it shards only over the SPMD grid of one
NeuronCore, kernels/nki_attention.py:67,113).  Two modes are added here, one
process per GPU, ``torch.distributed`` (NCCL) for the plumbing:

* **Head parallel.**  The flattened ``b*h`` heads are split into contiguous
  ranges, one per rank; each rank runs the chunked kernel on its range.  No
  collective is on the data path.
* **Sequence parallel.**  For one long sequence, rank ``r`` owns the token
  range ``[r*T/P, (r+1)*T/P)`` of every head.  (1) each rank computes the
  total state of its tokens (``la_based_chunked_state``), (2) the states are
  all-gathered (one NCCL all-gather of ``b*h*F*(d_v+1)`` fp32 per rank,
  1.1 MB at H=16, d_qk=16, d_v=64), (3) each rank sums the states of the ranks
  before it in rank order (deterministic) and (4) runs the chunked kernel
  seeded with that prefix.  The per-segment states of step (1) stay in the
  workspace and step (4) reuses them, so K and V are read twice, not three
  times.

The compute steps are injectable (``state_fn`` / ``forward_fn``) so the
exchange logic runs under CPU ``gloo`` ranks in the tests.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist


def head_range(batch_heads: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of flattened heads owned by ``rank``.

    The first ``batch_heads % world`` ranks own one extra head, so any
    ``batch_heads`` (also fewer heads than ranks) is covered exactly once.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, extra = divmod(batch_heads, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_heads(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The rank's heads of a global ``(b, h, t, d)`` tensor as ``(1, n_local, t, d)``."""
    b, h, t, d = x.shape
    start, stop = head_range(b * h, rank, world)
    return x.reshape(b * h, t, d)[start:stop].unsqueeze(0)


def token_range(seq_len: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of tokens owned by ``rank`` in sequence-parallel mode."""
    return head_range(seq_len, rank, world)


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The rank's token range of a global ``(b, h, t, d)`` tensor."""
    start, stop = token_range(x.shape[2], rank, world)
    return x[:, :, start:stop]


def exclusive_prefix(states: torch.Tensor, rank: int) -> torch.Tensor:
    """Sum of ``states[0:rank]`` (``states``: (P, ...)) in one reduction over
    the rank dimension (deterministic: same shapes, same order on every call;
    one kernel instead of one addition per earlier rank)."""
    if rank == 0:
        return torch.zeros_like(states[0])
    return states[:rank].sum(0)


@dataclass
class SPTimings:
    """Device-side milliseconds of sequence-parallel forwards (CUDA only).

    Each forward records four events on the stream (before the state pass,
    after it, after the exchange and prefix, after the seeded forward) and
    leaves them pending: nothing in the step waits for the device, so steps
    run back to back.  ``resolve()`` waits for the recorded events and adds
    each forward's phases to the totals; ``steps`` counts the forwards added.
    """
    state_ms: float = 0.0
    exchange_ms: float = 0.0
    forward_ms: float = 0.0
    steps: int = 0
    pending: list = field(default_factory=list)
    extra: dict = field(default_factory=dict)

    def resolve(self) -> "SPTimings":
        for ev in self.pending:
            ev[3].synchronize()
            self.state_ms += ev[0].elapsed_time(ev[1])
            self.exchange_ms += ev[1].elapsed_time(ev[2])
            self.forward_ms += ev[2].elapsed_time(ev[3])
            self.steps += 1
        self.pending.clear()
        return self

    def reset(self) -> None:
        self.resolve()
        self.state_ms = self.exchange_ms = self.forward_ms = 0.0
        self.steps = 0


def _default_state_fn(workspace_holder):
    from . import ops

    def state_fn(k, v):
        b, h, t, d = k.shape
        g, ws = ops.chunked_plan(b * h, t, d, v.shape[-1], k.dtype)
        workspace_holder["segments"] = g
        workspace_holder["ws"] = ops._workspace(ws, k.device)
        return ops.based_chunked_state(k, v, segments=g, workspace=workspace_holder["ws"])
    return state_fn


def _default_forward_fn(workspace_holder, chunk_size, eps):
    from . import ops

    def forward_fn(q, k, v, prefix):
        g = workspace_holder.get("segments", 0)
        return ops.based_chunked(q, k, v, chunk_size=chunk_size, eps=eps, init_state=prefix,
                                 segments=g, workspace=workspace_holder.get("ws"),
                                 reuse_segments=g > 1)
    return forward_fn


def sequence_parallel_forward(q, k, v, group=None, *, chunk_size: int = 64, eps: float = 1e-6,
                              state_fn=None, forward_fn=None, timings: SPTimings | None = None):
    """Normalised chunked BASED over a sequence split across the ranks of ``group``.

    ``q, k, v`` are this rank's token range ``(b, h, t_local, d)``; ranks hold
    consecutive ranges in rank order.  Returns this rank's output rows.  Every
    rank takes the same collective steps in the same order.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    holder: dict = {}
    state_fn = state_fn or _default_state_fn(holder)
    forward_fn = forward_fn or _default_forward_fn(holder, chunk_size, eps)
    cuda = q.device.type == "cuda"
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if (cuda and timings) else None

    if ev:
        ev[0].record()
    state = state_fn(k, v).contiguous()
    if ev:
        ev[1].record()
    flat = torch.empty((world * state.shape[0],) + tuple(state.shape[1:]), dtype=state.dtype,
                       device=state.device)
    dist.all_gather_into_tensor(flat, state, group=group)
    prefix = exclusive_prefix(flat.view((world,) + tuple(state.shape)), rank)
    if ev:
        ev[2].record()
    out = forward_fn(q, k, v, prefix)
    if ev:
        ev[3].record()
        timings.pending.append(ev)
    return out


def check_peers(group=None, timeout_s: float = 10.0) -> None:
    """Host-side liveness check before a collective step.

    Raises ``RuntimeError`` naming the missing ranks when a peer does not
    arrive within ``timeout_s`` (gloo ``monitored_barrier``).  With NCCL the
    process group's own timeout ends a collective that a peer never joins.
    """
    import datetime

    if dist.get_backend(group) == "gloo":
        dist.monitored_barrier(group=group, timeout=datetime.timedelta(seconds=timeout_s))
    else:
        dist.barrier(group=group)


def init_process_group_from_env(backend: str | None = None, timeout_s: float = 120.0):
    """Initialise the default group from torchrun's environment (127.0.0.1 rendezvous).

    Returns ``(rank, world, local_rank)``; a single process without torchrun
    variables gets ``(0, 1, 0)`` and no process group.
    """
    import datetime
    import os

    if "RANK" not in os.environ or int(os.environ.get("WORLD_SIZE", "1")) == 1:
        return 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if backend == "nccl":
        torch.cuda.set_device(local)
    kwargs = dict(backend=backend, rank=rank, world_size=world,
                  timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(**kwargs)
    return rank, world, local

