"""GPU parity: the CUDA kernels (through the C ABI) against the CPU oracle and
the reference's golden vectors.

Tolerances (rel-L2 over the whole output, the parity metric):
  * fp32 inputs:  <= 1e-4 against the fp32 reference;
  * bf16 inputs:  <= 2e-2 against the fp32/fp64 reference evaluated on the
    same bf16-rounded inputs.
"""

import numpy as np
import pytest
import torch

import oracle as O
import trainium_linear_attention_b200 as T
from trainium_linear_attention_b200 import ops

pytestmark = pytest.mark.gpu

TOL_FP32 = 1e-4
TOL_BF16 = 2e-2
DEV = "cuda"


def inputs(shape_qk, dv, seed, scale=0.5, dtype=torch.bfloat16):
    """Seeded N(0,1)*scale inputs generated on the host in fp32, cast to dtype."""
    g = torch.Generator().manual_seed(seed)
    b, h, t, d = shape_qk
    q = (torch.randn(b, h, t, d, generator=g) * scale).to(dtype)
    k = (torch.randn(b, h, t, d, generator=g) * scale).to(dtype)
    v = (torch.randn(b, h, t, dv, generator=g) * scale).to(dtype)
    return q, k, v


def np64(x):
    return x.float().cpu().numpy().astype(np.float64)


def cuda(*xs):
    return [x.to(DEV) for x in xs]


# ---------------------------------------------------------------- parallel ---

@pytest.mark.parametrize("case", ["c1", "par_odd", "par_n1", "par_d8"])
def test_parallel_fp32_golden(golden, case):
    q, k, v = (torch.from_numpy(golden[f"{case}.{n}"]).to(DEV) for n in "qkv")
    y = T.solution_nki(q, k, v)
    assert y.dtype == torch.float32 and y.shape == v.shape
    assert O.rel_l2(y.cpu().numpy(), golden[f"{case}.out"]) <= TOL_FP32


@pytest.mark.parametrize("shape,dv", [((2, 3, 1000, 16), 64), ((1, 2, 1, 16), 64),
                                      ((1, 2, 127, 16), 64), ((1, 1, 513, 16), 64),
                                      ((2, 2, 300, 32), 48)])
def test_parallel_bf16(shape, dv):
    q, k, v = inputs(shape, dv, seed=shape[2])
    y = T.solution_nki(*cuda(q, k, v))
    assert y.dtype == torch.bfloat16
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


@pytest.mark.parametrize("t", [1, 127, 128, 129, 256, 700])
def test_parallel_tensor_core_lengths(t):
    """The tcgen05 parallel kernel (bf16, d_qk 16, d_v 64) on ragged and
    tile-multiple lengths, against the oracle and against the chunked kernel."""
    q, k, v = inputs((2, 3, t, 16), 64, seed=100 + t)
    qc, kc, vc = cuda(q, k, v)
    y = ops.based_parallel(qc, kc, vc)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    assert O.rel_l2(np64(y), np64(ops.based_chunked(qc, kc, vc))) <= 1e-2


@pytest.mark.parametrize("b,h,t", [(2, 40, 384), (2, 40, 512), (2, 40, 513), (8, 80, 256),
                                   (8, 80, 300)])
def test_parallel_tensor_core_many_items(b, h, t):
    """The persistent kernel (N <= 512) runs several work items per CTA,
    both TMEM buffers and O accumulators in turn: single items at 80 heads,
    whole heads per CTA at 640; N = 513 takes the one-CTA-per-tile kernel.
    First, middle and last heads against the oracle."""
    q, k, v = inputs((b, h, t, 16), 64, seed=t + b)
    y = ops.based_parallel(*cuda(q, k, v))
    for bh in (0, 41, b * h - 1):
        bb, hh = divmod(bh, h)
        want = O.based_attn_reduced(np64(q[bb, hh]), np64(k[bb, hh]), np64(v[bb, hh]))
        assert O.rel_l2(np64(y[bb, hh]), want) <= TOL_BF16
    assert bool(torch.isfinite(y.float()).all())


def test_parallel_tensor_core_matches_cuda_core_path():
    """Aligned tensors take the tcgen05 kernel, unaligned copies of the same
    values the CUDA-core kernel; both agree."""
    q, k, v = cuda(*inputs((1, 4, 900, 16), 64, seed=41))

    def shifted(x):
        buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=DEV)
        y = buf[1:].view(x.shape)
        y.copy_(x)
        return y

    y_tc = ops.based_parallel(q, k, v)
    y_simt = ops.based_parallel(shifted(q), shifted(k), shifted(v))
    assert O.rel_l2(np64(y_tc), np64(y_simt)) <= 1e-2


# ----------------------------------------------------------------- chunked ---

def test_chunked_fp32_golden(golden):
    q, k, v = (torch.from_numpy(golden[f"dense.{n}"]).to(DEV) for n in "qkv")
    num = T.chunked_nki_numerator(q, k, v)
    assert O.rel_l2(num.cpu().numpy(), golden["dense.num"]) <= TOL_FP32
    y = T.based_chunked(q, k, v)
    assert O.rel_l2(y.cpu().numpy(), golden["dense.out"]) <= TOL_FP32


def test_chunked_config2():
    """Configuration 2: B=4, H=16, N=2048, d_qk=16, d_v=64, bf16, chunk 64."""
    q, k, v = inputs((4, 16, 2048, 16), 64, seed=2)
    y = T.based_chunked(*cuda(q, k, v), chunk_size=64)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    num = T.chunked_nki_numerator(*cuda(q, k, v), chunk_size=64)
    want_num = O.based_chunked(np64(q), np64(k), np64(v), normalize=False)
    assert O.rel_l2(np64(num), want_num) <= TOL_BF16


@pytest.mark.parametrize("t", [1, 63, 64, 65, 127, 128, 129, 1000])
def test_chunked_ragged_lengths(t):
    q, k, v = inputs((1, 3, t, 16), 64, seed=t)
    y = T.based_chunked(*cuda(q, k, v))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


@pytest.mark.parametrize("dqk,dv,dtype", [(16, 32, torch.float32), (8, 24, torch.float32),
                                          (16, 64, torch.float32), (32, 64, torch.bfloat16)])
def test_chunked_other_widths(dqk, dv, dtype):
    q, k, v = inputs((1, 2, 300, dqk), dv, seed=dqk + dv, dtype=dtype)
    y = T.based_chunked(*cuda(q, k, v))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    tol = TOL_FP32 if dtype == torch.float32 else TOL_BF16
    assert O.rel_l2(np64(y), want) <= tol


def test_chunked_d64_fp32_golden(golden):
    """d_qk = 64 (F = 2145: the state is split over a thread-block cluster)
    at the reference chunked benchmark's default shape, fp32, against the
    reference's own dense Taylor-feature outputs."""
    q, k, v = (torch.from_numpy(golden[f"dense64.{n}"]).to(DEV) for n in "qkv")
    y = T.based_chunked(q, k, v)
    assert O.rel_l2(y.cpu().numpy(), golden["dense64.out"]) <= TOL_FP32
    num = T.chunked_nki_numerator(q, k, v)
    assert O.rel_l2(num.cpu().numpy(), golden["dense64.num"]) <= TOL_FP32


@pytest.mark.parametrize("t,dv", [(1, 64), (63, 64), (64, 64), (65, 32), (300, 64), (1000, 64)])
def test_chunked_d64_bf16(t, dv):
    q, k, v = inputs((1, 3, t, 64), dv, seed=640 + t)
    y = T.based_chunked(*cuda(q, k, v))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


def test_chunked_d64_segments_and_state():
    """Segments (the state pass splits the features over independent CTAs),
    the final state against the oracle's, and a split sequence seeded with
    the first part's state."""
    q, k, v = cuda(*inputs((1, 2, 2000, 64), 64, seed=641, dtype=torch.float32))
    y1, s1 = ops.based_chunked(q, k, v, segments=1, return_state=True)
    y3, s3 = ops.based_chunked(q, k, v, segments=3, return_state=True)
    want, s_want = O.based_chunked(np64(q), np64(k), np64(v), return_state=True)
    assert O.rel_l2(np64(y1), want) <= TOL_FP32
    assert O.rel_l2(np64(y3), want) <= TOL_FP32
    assert O.rel_l2(s1.double().cpu().numpy(), s_want.reshape(2, 2145, 65)) <= TOL_FP32
    assert O.rel_l2(s3.double().cpu().numpy(), s_want.reshape(2, 2145, 65)) <= TOL_FP32
    st = ops.based_chunked_state(k, v, segments=3)
    assert O.rel_l2(st.double().cpu().numpy(), s_want.reshape(2, 2145, 65)) <= TOL_FP32
    a, sa = ops.based_chunked(q[:, :, :700], k[:, :, :700], v[:, :, :700], return_state=True)
    b = ops.based_chunked(q[:, :, 700:], k[:, :, 700:], v[:, :, 700:], init_state=sa)
    assert O.rel_l2(np64(torch.cat([a, b], 2)), want) <= TOL_FP32


@pytest.mark.parametrize("heads,t", [(2, 2000), (3, 4100)])
def test_chunked_d64_bf16_tensor_core_state(heads, t):
    """bf16 d_qk = 64 on the tensor-core kernel (16-CTA cluster, 160 feature
    slots per CTA): normalised and numerator outputs, one and three segments
    (the state pass), final states against the oracle's, the state entry
    point, and a split at a ragged token boundary seeded with the first
    part's state.  States carry bf16-rounded features: within 2e-3."""
    q, k, v = inputs((1, heads, t, 64), 64, seed=642 + t)
    qd, kd, vd = cuda(q, k, v)
    want, s_want = O.based_chunked(np64(q), np64(k), np64(v), return_state=True)
    s_want = s_want.reshape(heads, 2145, 65)
    for g in (1, 3):
        y, s = ops.based_chunked(qd, kd, vd, segments=g, return_state=True)
        assert O.rel_l2(np64(y), want) <= TOL_BF16
        assert O.rel_l2(s.double().cpu().numpy(), s_want) <= 2e-3
    num = ops.based_chunked(qd, kd, vd, normalize=False)
    num_want = O.based_chunked(np64(q), np64(k), np64(v), normalize=False)
    assert O.rel_l2(np64(num), num_want) <= TOL_BF16
    st = ops.based_chunked_state(kd, vd, segments=3)
    assert O.rel_l2(st.double().cpu().numpy(), s_want) <= 2e-3
    cut = 1000
    a, sa = ops.based_chunked(qd[:, :, :cut], kd[:, :, :cut], vd[:, :, :cut], return_state=True)
    b = ops.based_chunked(qd[:, :, cut:], kd[:, :, cut:], vd[:, :, cut:], init_state=sa)
    assert O.rel_l2(np64(torch.cat([a, b], 2)), want) <= TOL_BF16


def test_chunked_unaligned_pointers():
    """bf16 tensors whose data is not 16-byte aligned (TMA cannot address
    them) run on the CUDA-core kernels with the same result."""
    q, k, v = cuda(*inputs((1, 2, 500, 16), 64, seed=21))

    def shifted(x):
        buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=DEV)
        y = buf[1:].view(x.shape)
        y.copy_(x)
        return y

    qs, ks, vs = shifted(q), shifted(k), shifted(v)
    assert qs.data_ptr() % 16 != 0
    y = ops.based_chunked(qs, ks, vs)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    assert O.rel_l2(np64(y), np64(ops.based_chunked(q, k, v))) <= 1e-2


@pytest.mark.parametrize("segments", [2, 3, 8])
def test_chunked_segments_agree(segments):
    q, k, v = cuda(*inputs((1, 4, 3000, 16), 64, seed=7))
    y1 = ops.based_chunked(q, k, v, segments=1)
    yg = ops.based_chunked(q, k, v, segments=segments)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(yg), want) <= TOL_BF16
    assert O.rel_l2(np64(yg), np64(y1)) <= 1e-2


@pytest.mark.parametrize("t", [8000, 8192])
def test_chunked_lead_main_split(t):
    """96 heads on a 148-SM B200: segments=0 splits every head into a short
    lead and a long main piece.  Output, final state (from an initial state)
    and the oracle agree with the unsplit run."""
    b, h = 6, 16
    q, k, v = inputs((b, h, t, 16), 64, seed=t)
    qd, kd, vd = cuda(q, k, v)
    g, ws = ops.chunked_plan(b * h, t, 16, 64, torch.bfloat16)
    if torch.cuda.get_device_properties(0).multi_processor_count == 148:
        assert g == 2 and ws > 0  # the split is in use
    F = ops.feature_dim(16)
    s0 = torch.randn(b * h, F, 65, generator=torch.Generator().manual_seed(3)).abs().to(DEV)
    y, st = ops.based_chunked(qd, kd, vd, init_state=s0, return_state=True)
    y1, st1 = ops.based_chunked(qd, kd, vd, init_state=s0, return_state=True, segments=1)
    assert O.rel_l2(np64(y), np64(y1)) <= 1e-2
    assert O.rel_l2(st.double().cpu().numpy(), st1.double().cpu().numpy()) <= 1e-5
    yn = ops.based_chunked(qd, kd, vd)
    for bh in (0, b * h - 1):
        bb, hh = divmod(bh, h)
        want = O.based_chunked(np64(q[bb, hh]), np64(k[bb, hh]), np64(v[bb, hh]))
        assert O.rel_l2(np64(yn[bb, hh]), want) <= TOL_BF16


def test_launch_counter_counts_each_kernel():
    """la_launch_count: one output kernel unsegmented; state pass, running
    sums and output with three segments."""
    from trainium_linear_attention_b200 import _native as N
    q, k, v = cuda(*inputs((1, 2, 3000, 16), 64, seed=9))
    for segments, launches in ((1, 1), (3, 3)):
        before = N.lib().la_launch_count()
        ops.based_chunked(q, k, v, segments=segments)
        torch.cuda.synchronize()
        assert N.lib().la_launch_count() - before == launches


def test_chunked_state_roundtrip():
    """Seeding the second half with the first half's final state reproduces
    the whole sequence; the states match the oracle's."""
    q, k, v = cuda(*inputs((2, 2, 1500, 16), 64, seed=11))
    whole, s_whole = ops.based_chunked(q, k, v, return_state=True)
    cut = 700
    a, s_a = ops.based_chunked(q[:, :, :cut], k[:, :, :cut], v[:, :, :cut], return_state=True)
    b = ops.based_chunked(q[:, :, cut:], k[:, :, cut:], v[:, :, cut:], init_state=s_a)
    assert O.rel_l2(np64(torch.cat([a, b], 2)), np64(whole)) <= 1e-2
    want = O.chunked_state(np64(k), np64(v)).reshape(4, 153, 65)
    assert O.rel_l2(s_whole.cpu().numpy(), want) <= 1e-3
    st = ops.based_chunked_state(k, v)
    assert O.rel_l2(st.cpu().numpy(), want) <= 1e-3
    st3 = ops.based_chunked_state(k, v, segments=3)
    assert O.rel_l2(st3.cpu().numpy(), want) <= 1e-3


def test_chunked_reuse_segments():
    q, k, v = cuda(*inputs((1, 2, 2500, 16), 64, seed=12))
    g, ws_bytes = ops.chunked_plan(2, 2500, 16, 64, torch.bfloat16, segments=4)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    ops.based_chunked_state(k, v, segments=g, workspace=ws)
    y = ops.based_chunked(q, k, v, segments=g, workspace=ws, reuse_segments=True)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


@pytest.mark.parametrize("dqk,t,segments", [(16, 2500, 4), (64, 2100, 3)])
def test_chunked_reuse_segments_both_widths(dqk, t, segments):
    """The state entry point leaves the running sums a forward with
    reuse_segments seeds from, on the d_qk = 16 kernel and on the d_qk = 64
    cluster kernel (state pass without a cluster, then the 16-CTA forward)."""
    q, k, v = cuda(*inputs((1, 2, t, dqk), 64, seed=13 + dqk))
    g, ws_bytes = ops.chunked_plan(2, t, dqk, 64, torch.bfloat16, segments=segments)
    assert g == segments
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
    ops.based_chunked_state(k, v, segments=g, workspace=ws)
    y = ops.based_chunked(q, k, v, segments=g, workspace=ws, reuse_segments=True)
    assert torch.equal(y, ops.based_chunked(q, k, v, segments=g))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


def test_chunked_d64_unaligned_inputs():
    """bf16 d_qk = 64 tensors whose data is not 16-byte aligned (TMA cannot
    address them) run on the CUDA-core cluster kernel with the same result."""
    q, k, v = cuda(*inputs((1, 2, 300, 64), 64, seed=22))

    def shifted(x):
        buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=DEV)
        y = buf[1:].view(x.shape)
        y.copy_(x)
        return y

    y = ops.based_chunked(shifted(q), shifted(k), shifted(v))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    assert O.rel_l2(np64(y), np64(ops.based_chunked(q, k, v))) <= 1e-2


def test_chunked_sequence_parallel_emulated():
    """The sequence-parallel recipe (per-rank states, exclusive prefix, seeded
    forward) run for 4 emulated ranks on one GPU."""
    q, k, v = cuda(*inputs((1, 4, 4096, 16), 64, seed=13))
    world = 4
    parts = [(q[:, :, r * 1024:(r + 1) * 1024], k[:, :, r * 1024:(r + 1) * 1024],
              v[:, :, r * 1024:(r + 1) * 1024]) for r in range(world)]
    states = torch.stack([ops.based_chunked_state(pk, pv) for _, pk, pv in parts])
    outs = []
    for r, (pq, pk, pv) in enumerate(parts):
        prefix = states[:r].sum(0) if r else torch.zeros_like(states[0])
        outs.append(ops.based_chunked(pq, pk, pv, init_state=prefix))
    y = torch.cat(outs, 2)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


def test_chunked_full_size_properties():
    """Configuration 4 sizes (B=8, H=16, N=32768): eight heads spread over the
    batch (the last included) against the fp64 oracle, every head through
    size-independent properties -- the output is a convex combination of the
    values (weights 1+s+s^2/2 > 0), and the segmented and unsegmented runs
    agree."""
    q, k, v = inputs((8, 16, 32768, 16), 64, seed=4)
    qd, kd, vd = cuda(q, k, v)
    y = T.based_chunked(qd, kd, vd)
    for bh in (0, 17, 38, 55, 72, 93, 110, 127):
        b, h = divmod(bh, 16)
        want = O.based_chunked(np64(q[b, h]), np64(k[b, h]), np64(v[b, h]), chunk=1024)
        assert O.rel_l2(np64(y[b, h]), want) <= TOL_BF16
    vmax = vd.float().abs().amax(dim=2, keepdim=True)
    assert bool((y.float().abs() <= vmax * 1.01 + 1e-3).all())
    assert bool(torch.isfinite(y.float()).all())
    yg = ops.based_chunked(qd, kd, vd, segments=4)
    assert O.rel_l2(np64(yg), np64(y)) <= 1e-2


def test_sequence_parallel_full_length_emulated():
    """Configuration 4's sequence-parallel variant at full length (B=1, H=16,
    N=262144) with 8 ranks emulated on one GPU through the same calls a rank
    makes: its state pass with per-segment running sums left in its
    workspace, the exclusive prefix of the earlier ranks' states, and the
    seeded forward that reuses those segment sums.  Heads 0, 7 and 15 against
    the fp64 chunked oracle over all 262144 tokens; every head finite and a
    convex combination of the values."""
    world, n = 8, 262144
    q, k, v = inputs((1, 16, n, 16), 64, seed=262)
    qd, kd, vd = cuda(q, k, v)
    per = n // world
    states, outs = [], []
    holders = []
    for r in range(world):
        sl = slice(r * per, (r + 1) * per)
        kr, vr = kd[:, :, sl], vd[:, :, sl]
        g, ws_bytes = ops.chunked_plan(16, per, 16, 64, torch.bfloat16)
        ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=DEV)
        states.append(ops.based_chunked_state(kr, vr, segments=g, workspace=ws))
        holders.append((g, ws))
    for r in range(world):
        sl = slice(r * per, (r + 1) * per)
        prefix = torch.zeros_like(states[0])
        for j in range(r):
            prefix += states[j]
        g, ws = holders[r]
        outs.append(ops.based_chunked(qd[:, :, sl], kd[:, :, sl], vd[:, :, sl], init_state=prefix,
                                      segments=g, workspace=ws, reuse_segments=g > 1))
    y = torch.cat(outs, 2)
    for h in (0, 7, 15):
        want = O.based_chunked(np64(q[0, h]), np64(k[0, h]), np64(v[0, h]), chunk=1024)
        assert O.rel_l2(np64(y[0, h]), want) <= TOL_BF16
    assert bool(torch.isfinite(y.float()).all())
    vmax = vd.float().abs().amax(dim=2, keepdim=True)
    assert bool((y.float().abs() <= vmax * 1.01 + 1e-3).all())


@pytest.mark.parametrize("n", [2048, 8192, 65536])
def test_parallel_long_sequences_config5(n):
    """Configuration 5's parallel kernel at B*N = 262144, H = 16: at N = 65536
    each query tile walks up to 512 key tiles.  Two heads against the fp64
    chunked oracle, every head against the chunked kernel."""
    b = 262144 // n
    q, k, v = inputs((b, 16, n, 16), 64, seed=500 + n)
    qd, kd, vd = cuda(q, k, v)
    y = ops.based_parallel(qd, kd, vd)
    for bh in (0, b * 16 - 1):
        bb, hh = divmod(bh, 16)
        want = O.based_chunked(np64(q[bb, hh]), np64(k[bb, hh]), np64(v[bb, hh]), chunk=1024)
        assert O.rel_l2(np64(y[bb, hh]), want) <= TOL_BF16
    yc = ops.based_chunked(qd, kd, vd)
    err = (y.float() - yc.float()).reshape(b * 16, -1).norm(dim=1) / \
        yc.float().reshape(b * 16, -1).norm(dim=1)
    assert float(err.max()) <= 1e-2


def test_host_buffer_api_matches_device_call():
    """based_chunked_host (pinned host tensors, copies overlapped with the
    kernels per head group) gives the device call's result bit for bit, for
    head counts that do and do not divide into the groups."""
    for b, h, groups in ((2, 8, 8), (1, 5, 3), (1, 2, 8)):
        q, k, v = inputs((b, h, 1500, 16), 64, seed=40 + h)
        qp, kp, vp = (x.pin_memory() for x in (q, k, v))
        y = T.based_chunked_host(qp, kp, vp, head_groups=groups)
        torch.cuda.current_stream().synchronize()
        assert y.device.type == "cpu"
        # the same kernels on the same groups of heads (the segmentation, and
        # so the rounding, depends on a call's head count)
        qd, kd, vd = (x.reshape(1, b * h, 1500, -1) for x in cuda(q, k, v))
        step = -(-(b * h) // min(groups, b * h))
        want = torch.cat([ops.based_chunked(qd[:, lo:lo + step], kd[:, lo:lo + step],
                                            vd[:, lo:lo + step])
                          for lo in range(0, b * h, step)], 1).reshape(b, h, 1500, 64)
        assert torch.equal(y, want.cpu())
        oracle = O.based_attn_reduced(np64(q), np64(k), np64(v))
        assert O.rel_l2(np64(y), oracle) <= TOL_BF16


def test_deterministic():
    q, k, v = cuda(*inputs((2, 4, 2048, 16), 64, seed=5))
    a = ops.based_chunked(q, k, v, segments=3)
    b = ops.based_chunked(q, k, v, segments=3)
    assert torch.equal(a, b)
    assert torch.equal(T.solution_nki(q, k, v), T.solution_nki(q, k, v))


def test_deterministic_segment_states_lightly_loaded():
    """Few CTAs run far ahead of the memory system: the segment-state pass
    must still give bit-identical states on every run."""
    q, k, v = cuda(*inputs((1, 2, 4096, 16), 64, seed=6))
    g, ws_bytes = ops.chunked_plan(2, 4096, 16, 64, torch.bfloat16, segments=3)
    runs = []
    for _ in range(8):
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=DEV)
        ops.based_chunked_state(k, v, segments=g, workspace=ws)
        runs.append(ws)
    for ws in runs[1:]:
        assert torch.equal(ws, runs[0])
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    for _ in range(4):
        y = ops.based_chunked(q, k, v, segments=g)
        assert O.rel_l2(np64(y), want) <= 5e-3


# --------------------------------------------------------- full BASED layer ---

@pytest.mark.parametrize("case", ["layer_w64", "layer_w129", "layer_d32_w7"])
def test_layer_fp32_golden(golden, case):
    """based_layer (BASED + sliding window in one pass) against the reference's
    own two functions summed."""
    q, k, v = (torch.from_numpy(golden[f"{case}.{n}"]).to(DEV) for n in "qkv")
    y = T.based_layer(q, k, v, window_size=int(golden[f"{case}.window"]))
    assert O.rel_l2(y.cpu().numpy(), golden[f"{case}.out"]) <= TOL_FP32


@pytest.mark.parametrize("t,w,segments", [(1, 64, 0), (65, 64, 0), (1000, 64, 0), (2048, 64, 0),
                                          (3000, 129, 3), (700, 1, 0), (300, 129, 0),
                                          (129, 500, 0), (4100, 65, 0), (4100, 66, 2)])
def test_layer_bf16(t, w, segments):
    """bf16, d_qk = 16, d_v = 64: the chunked tensor-core kernel, then the
    sliding kernel adding the window term (spans of 192 keys for W <= 65, 256
    above)."""
    q, k, v = inputs((2, 4, t, 16), 64, seed=700 + t + w)
    if w > 129:
        with pytest.raises(RuntimeError):
            T.based_layer(*cuda(q, k, v), window_size=w)
        return
    y = ops.based_layer(*cuda(q, k, v), window_size=w, segments=segments)
    want = O.based_layer(np64(q), np64(k), np64(v), w)
    assert O.rel_l2(np64(y), want) <= TOL_BF16


@pytest.mark.parametrize("t,w,segments,dtype", [(256, 64, 0, torch.float32), (1000, 64, 0, torch.bfloat16),
                                                (1500, 129, 3, torch.bfloat16), (70, 7, 0, torch.float32)])
def test_layer_d64(t, w, segments, dtype):
    """The full BASED layer at d_qk = 64 (the reference module's head width,
    F = 2145): the state is split over a cluster, the window keys before a
    chunk come from memory."""
    q, k, v = inputs((1, 2, t, 64), 64, seed=750 + t, scale=0.5, dtype=dtype)
    y = ops.based_layer(*cuda(q, k, v), window_size=w, segments=segments)
    want = O.based_layer(np64(q), np64(k), np64(v), w)
    assert O.rel_l2(np64(y), want) <= (TOL_FP32 if dtype == torch.float32 else TOL_BF16)


def test_layer_segments_agree():
    """Segments seed the state from the earlier segments and read the window
    keys before their first token from memory: same result as one segment."""
    q, k, v = cuda(*inputs((1, 3, 2500, 16), 64, seed=710, dtype=torch.float32))
    y1 = ops.based_layer(q, k, v, window_size=100, segments=1)
    y4 = ops.based_layer(q, k, v, window_size=100, segments=4)
    assert O.rel_l2(np64(y4), np64(y1)) <= 1e-5
    want = O.based_layer(np64(q), np64(k), np64(v), 100)
    assert O.rel_l2(np64(y4), want) <= TOL_FP32


# ----------------------------------------------------------------- sliding ---

@pytest.mark.parametrize("case", ["slide_w64", "slide_w16_odd", "slide_w1", "slide_wbig",
                                  "slide_w100"])
def test_sliding_fp32_golden(golden, case):
    q, k, v = (torch.from_numpy(golden[f"{case}.{n}"]).to(DEV) for n in "qkv")
    y = T.nki_sliding_window_attn(q, k, v, window_size=int(golden[f"{case}.window"]))
    assert O.rel_l2(y.cpu().numpy(), golden[f"{case}.out"]) <= TOL_FP32


def test_sliding_config3():
    """Configuration 3: W=64, B=4, H=16, N=4096, d=64, bf16, N(0,1) inputs."""
    q, k, v = inputs((4, 16, 4096, 64), 64, seed=3, scale=1.0)
    y = T.nki_sliding_window_attn(*cuda(q, k, v), window_size=64)
    want = O.sliding_window_attn(np64(q), np64(k), np64(v), 64)
    assert O.rel_l2(np64(y), want) <= TOL_BF16


@pytest.mark.parametrize("t,w", [(1, 64), (65, 64), (200, 1), (300, 128), (129, 500), (1000, 65),
                                 (513, 129), (700, 130), (333, 66), (4097, 64), (130, 2)])
def test_sliding_edges_bf16(t, w):
    q, k, v = inputs((1, 2, t, 64), 64, seed=t + w, scale=1.0)
    y = T.nki_sliding_window_attn(*cuda(q, k, v), window_size=w)
    want = O.sliding_window_attn(np64(q), np64(k), np64(v), w)
    assert O.rel_l2(np64(y), want) <= TOL_BF16


def test_sliding_tensor_core_matches_cuda_core_path():
    """The tcgen05 kernel (aligned tensors) and the CUDA-core kernel
    (unaligned copies of the same values) agree."""
    q, k, v = cuda(*inputs((2, 3, 1500, 64), 64, seed=31, scale=1.0))

    def shifted(x):
        buf = torch.empty(x.numel() + 1, dtype=x.dtype, device=DEV)
        y = buf[1:].view(x.shape)
        y.copy_(x)
        return y

    for w in (64, 100):
        y_tc = T.nki_sliding_window_attn(q, k, v, window_size=w)
        y_simt = T.nki_sliding_window_attn(shifted(q), shifted(k), shifted(v), window_size=w)
        assert O.rel_l2(np64(y_tc), np64(y_simt)) <= 1e-2


# -------------------------------------------------------------- dispatch ---

def test_solution_dispatch_and_errors():
    q, k, v = cuda(*inputs((1, 2, 3000, 16), 64, seed=9))
    y = T.solution(q, k, v)
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    assert torch.equal(y, ops.based_chunked(q, k, v))  # long: the chunked kernel
    with pytest.raises(TypeError):
        T.solution(q.half(), k.half(), v.half())
    with pytest.raises(RuntimeError):  # d_qk beyond the kernels: raises, no fallback
        qq = torch.zeros(1, 1, 8, 256, device=DEV, dtype=torch.bfloat16)
        T.solution_nki(qq, qq, qq)
    with pytest.raises(RuntimeError):  # a state too wide even for a cluster
        qq = torch.zeros(1, 1, 8, 128, device=DEV, dtype=torch.bfloat16)
        T.based_chunked(qq, qq, qq)


@pytest.mark.parametrize("t", [256, 512])
def test_solution_short_sequence_takes_parallel_kernel(t):
    """N = 256 and 512 are at or below the measured crossover: solution() runs
    the parallel kernel (one launch, bit-identical to solution_nki, different
    from the chunked kernel's rounding) and matches the oracle."""
    from trainium_linear_attention_b200 import _native as N
    q, k, v = inputs((4, 16, t, 16), 64, seed=t)
    qd, kd, vd = cuda(q, k, v)
    torch.cuda.synchronize()
    before = N.lib().la_launch_count()
    y = T.solution(qd, kd, vd)
    torch.cuda.synchronize()
    assert N.lib().la_launch_count() - before == 1
    assert torch.equal(y, T.solution_nki(qd, kd, vd))
    assert not torch.equal(y, ops.based_chunked(qd, kd, vd))
    want = O.based_attn_reduced(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


# --------------------------------------------------------- identity map ---

@pytest.mark.parametrize("case", ["ident", "ident_odd"])
def test_identity_fp32_golden(golden, case):
    """chunked_identity_numerator (fp32) against the reference's own
    ref_identity_numerator outputs."""
    q, k, v = (torch.from_numpy(golden[f"{case}.{n}"]).to(DEV) for n in "qkv")
    y = T.chunked_identity_numerator(q, k, v)
    assert y.dtype == torch.float32
    assert O.rel_l2(y.cpu().numpy(), golden[f"{case}.num"]) <= TOL_FP32


@pytest.mark.parametrize("t,segments", [(1, 0), (65, 0), (1000, 0), (3000, 3), (4096, 0)])
def test_identity_bf16(t, segments):
    q, k, v = inputs((2, 4, t, 16), 64, seed=900 + t)
    qd, kd, vd = cuda(q, k, v)
    y = ops.based_chunked(qd, kd, vd, normalize=False, feature_map="identity", segments=segments)
    want = O.identity_numerator(np64(q), np64(k), np64(v))
    assert O.rel_l2(np64(y), want) <= TOL_BF16


def test_identity_state_roundtrip():
    q, k, v = cuda(*inputs((1, 2, 900, 16), 64, seed=77, dtype=torch.float32))
    y, s = ops.based_chunked(q, k, v, normalize=False, feature_map="identity", return_state=True)
    want, s_want = O.identity_chunked(np64(q), np64(k), np64(v), return_state=True)
    assert O.rel_l2(np64(y), want) <= TOL_FP32
    assert O.rel_l2(s.double().cpu().numpy(), s_want.reshape(2, 16, 65)) <= TOL_FP32
    a, sa = ops.based_chunked(q[:, :, :400], k[:, :, :400], v[:, :, :400], normalize=False,
                              feature_map="identity", return_state=True)
    b = ops.based_chunked(q[:, :, 400:], k[:, :, 400:], v[:, :, 400:], normalize=False,
                          feature_map="identity", init_state=sa)
    assert O.rel_l2(np64(torch.cat([a, b], 2)), want) <= TOL_FP32
    with pytest.raises(ValueError):
        ops.based_chunked(q, k, v, feature_map="identity")  # normalised identity: rejected


@pytest.mark.parametrize("heads,t", [(2, 900), (100, 8192)])
def test_identity_bf16_tensor_core_state(heads, t):
    """The identity map on the tensor-core kernel (bf16, d_qk = 16, d_v = 64):
    output and final state against the chunked restatement, and a split at a
    token boundary seeded with the first half's state.  100 heads of 8192
    tokens take the lead/main split (a state pass over each head's lead)."""
    q, k, v = inputs((1, heads, t, 16), 64, seed=78 + heads)
    qd, kd, vd = cuda(q, k, v)
    y, s = ops.based_chunked(qd, kd, vd, normalize=False, feature_map="identity",
                             return_state=True)
    want, s_want = O.identity_chunked(np64(q), np64(k), np64(v), return_state=True)
    assert O.rel_l2(np64(y), want) <= TOL_BF16
    assert O.rel_l2(s.double().cpu().numpy(), s_want.reshape(heads, 16, 65)) <= 1e-4
    h = t // 2
    a, sa = ops.based_chunked(qd[:, :, :h], kd[:, :, :h], vd[:, :, :h], normalize=False,
                              feature_map="identity", return_state=True)
    b = ops.based_chunked(qd[:, :, h:], kd[:, :, h:], vd[:, :, h:], normalize=False,
                          feature_map="identity", init_state=sa)
    assert O.rel_l2(np64(torch.cat([a, b], 2)), want) <= TOL_BF16


# ------------------------------------------------------------ traced dispatch ---

@pytest.mark.parametrize("t", [256, 3000])
def test_traced_solution_matches_eager(t):
    """trace_solution captures solution() for one shape in a CUDA graph (the
    parallel kernel at N = 256, the chunked kernel with its segment-state pass
    at N = 3000); replays on new inputs equal the eager call bit for bit."""
    from trainium_linear_attention_b200.kernels.pytorch_attention import (
        CROSSOVER_SEQ_LEN_BF16_TC, solution_kind)
    q, k, v = cuda(*inputs((1, 4, t, 16), 64, seed=t + 1))
    traced = T.trace_solution(q, k, v)
    want_kind = "parallel" if t <= CROSSOVER_SEQ_LEN_BF16_TC else "chunked"
    assert traced.kind == solution_kind(q, k, v) == want_kind
    for seed in (1, 2):
        q2, k2, v2 = cuda(*inputs((1, 4, t, 16), 64, seed=t + 10 * seed))
        y = traced(q2, k2, v2).clone()
        assert torch.equal(y, T.solution(q2, k2, v2))
    with pytest.raises(ValueError):
        traced(q[:, :, :10], k[:, :, :10], v[:, :, :10])


@pytest.mark.parametrize("dim,heads,t,dtype,attention,window", [
    (64, 4, 300, torch.float32, "parallel", None),   # head_dim 16, fp32: CUDA-core kernels
    (256, 4, 1100, torch.bfloat16, "auto", None),    # head_dim 64, bf16: chunked d_qk = 64 cluster kernel
    (64, 4, 500, torch.bfloat16, "parallel", 32),    # full BASED layer through the module
])
def test_based_module_matches_reference_module(dim, heads, t, dtype, attention, window):
    """The kernel module (benchmarks/based_attention_benchmark.py:47-69 names)
    with the reference module's weights gives the reference module's output
    (projections in fp64 around the oracle's attention, or the oracle's
    BASED + sliding-window sum)."""
    torch.manual_seed(11)
    ref = T.TrainiumBasedLinearAttention(dim, heads=heads).double()
    mod = T.TrainiumBasedLinearAttentionNKI(dim, heads=heads, window_size=window,
                                           attention=attention).to(DEV, dtype)
    mod.load_state_dict({k: w.to(dtype) for k, w in ref.state_dict().items()})
    x = (torch.randn(2, t, dim, dtype=torch.float64) * 0.5)
    with torch.no_grad():
        y = mod(x.to(DEV, dtype))
        # the oracle on the projections the kernel module computed
        hd = dim // heads
        qkv = [np64(p(x.to(DEV, dtype)).view(2, t, heads, hd).transpose(1, 2))
               for p in (mod.q_proj, mod.k_proj, mod.v_proj)]
        att = O.based_attn_reduced(*qkv)
        if window:
            att = att + O.sliding_window_attn(*qkv, window)
        att = torch.from_numpy(att).to(DEV, dtype).transpose(1, 2).reshape(2, t, dim)
        want = mod.o_proj(att)
    tol = TOL_FP32 if dtype == torch.float32 else TOL_BF16
    assert O.rel_l2(np64(y), np64(want)) <= tol
