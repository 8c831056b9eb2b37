"""Torch-facing calls into the native library (device memory + streams only).

Every function takes ``(b, h, t, d)`` CUDA tensors, enqueues the kernel on
``torch.cuda.current_stream()`` and returns a freshly allocated output in
``q.dtype``.  Inputs are never modified.  Failures raise; nothing falls back
to another implementation.
"""

from __future__ import annotations

import contextlib
import ctypes
import functools

import torch

from . import _native as N

_DTYPES = {torch.float32: N.LA_DTYPE_FLOAT32, torch.bfloat16: N.LA_DTYPE_BFLOAT16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16") from None


def _check_qkv(q, k, v, same_dv: bool = False):
    for name, t in (("q", q), ("k", k), ("v", v)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.dim() != 4:
            raise ValueError(f"{name} must be (batch, heads, seq_len, dim), got shape {tuple(t.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cuda":
            raise ValueError(f"{name} must be a CUDA tensor (got {t.device}); "
                             "this library has no CPU implementation")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v are on different devices")
    if q.shape != k.shape:
        raise ValueError(f"q and k shapes differ: {tuple(q.shape)} vs {tuple(k.shape)}")
    if v.shape[:3] != q.shape[:3]:
        raise ValueError(f"v shape {tuple(v.shape)} does not match q {tuple(q.shape)}")
    if same_dv and v.shape[-1] != q.shape[-1]:
        raise ValueError("v must have the same head dim as q for this op")
    return _dtype_code(q)


# Host cost matters: a call's launch latency is exposed whenever the GPU is
# idle, so the per-call Python work below avoids object churn (raw stream
# handle, plain ints for pointers, no device switch when already current,
# plan results cached per shape).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_ptr(device) -> int:
    """The raw cudaStream_t of the current stream of `device`."""
    index = torch.device(device).index
    if index is None:
        index = torch.cuda.current_device()
    if _raw_stream is not None:
        return _raw_stream(index)
    return torch.cuda.current_stream(index).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _on_device(device):
    """Make `device` current for the call (a no-op when it already is)."""
    index = torch.device(device).index
    if index is None or index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(index)


def based_parallel(q, k, v, eps: float = 1e-6) -> torch.Tensor:
    """Parallel (quadratic) BASED attention, normalised, causal."""
    code = _check_qkv(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    b, h, t, d = q.shape
    dv = v.shape[-1]
    out = torch.empty((b, h, t, dv), dtype=q.dtype, device=q.device)
    with _on_device(q.device):
        st = N.lib().la_based_parallel_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, t, d, dv,
                                           code, float(eps), _stream_ptr(q.device))
    N.check(st, "la_based_parallel_fwd")
    return out


def feature_dim(d_qk: int) -> int:
    return 1 + d_qk + d_qk * (d_qk + 1) // 2


def chunked_plan(batch_heads: int, seq_len: int, d_qk: int, d_v: int, dtype: torch.dtype,
                 segments: int = 0):
    """(segments, workspace_bytes) the library will use for this shape on the
    current device."""
    return _chunked_plan(int(batch_heads), int(seq_len), int(d_qk), int(d_v), _DTYPES[dtype],
                         int(segments), torch.cuda.current_device())


@functools.lru_cache(maxsize=1024)
def _chunked_plan(batch_heads, seq_len, d_qk, d_v, code, segments, device_index):
    g = ctypes.c_int(0)
    ws = ctypes.c_size_t(0)
    st = N.lib().la_based_chunked_plan(batch_heads, seq_len, d_qk, d_v, code, segments,
                                       ctypes.byref(g), ctypes.byref(ws))
    N.check(st, "la_based_chunked_plan")
    return g.value, ws.value


def _workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def based_chunked(q, k, v, chunk_size: int = 64, eps: float = 1e-6, normalize: bool = True,
                  init_state: torch.Tensor | None = None, return_state: bool = False,
                  segments: int = 0, workspace: torch.Tensor | None = None,
                  reuse_segments: bool = False, feature_map: str = "taylor"):
    """Chunked recurrent linear attention (BASED Taylor features by default).

    ``init_state`` / the returned final state are fp32 ``(b*h, F, d_v + 1)``
    in the key-side feature basis documented in ``include/la_attention.h``.
    ``feature_map="identity"`` uses phi(x) = x (F = d_qk, numerator only).
    """
    code = _check_qkv(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    b, h, t, d = q.shape
    dv = v.shape[-1]
    if chunk_size < 1:
        raise ValueError("chunk_size must be >= 1")
    if feature_map not in ("taylor", "identity"):
        raise ValueError(f"feature_map must be 'taylor' or 'identity', got {feature_map!r}")
    identity = feature_map == "identity"
    if identity and normalize:
        raise ValueError("the identity feature map is numerator-only (normalize=False)")
    F = d if identity else feature_dim(d)
    if init_state is not None:
        if (init_state.dtype != torch.float32 or init_state.device != q.device
                or tuple(init_state.shape) != (b * h, F, dv + 1)):
            raise ValueError(f"init_state must be float32 {(b * h, F, dv + 1)} on {q.device}")
        init_state = init_state.contiguous()
    out = torch.empty((b, h, t, dv), dtype=q.dtype, device=q.device)
    final = torch.empty((b * h, F, dv + 1), dtype=torch.float32, device=q.device) if return_state else None
    with _on_device(q.device):
        _, ws_bytes = chunked_plan(b * h, t, d, dv, q.dtype, segments)
        if workspace is None:
            workspace = _workspace(ws_bytes, q.device)
        elif workspace.numel() * workspace.element_size() < ws_bytes:
            raise ValueError(f"workspace too small: need {ws_bytes} bytes")
        flags = ((N.LA_CHUNKED_NORMALIZE if normalize else 0)
                 | (N.LA_CHUNKED_REUSE_SEGMENTS if reuse_segments else 0)
                 | (N.LA_CHUNKED_IDENTITY if identity else 0))
        st = N.lib().la_based_chunked_fwd(
            _ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, t, d, dv, code, int(chunk_size),
            float(eps), flags, _ptr(init_state), _ptr(final), _ptr(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            int(segments), _stream_ptr(q.device))
    N.check(st, "la_based_chunked_fwd")
    if return_state:
        return out, final
    return out


def based_chunked_state(k, v, segments: int = 0, workspace: torch.Tensor | None = None):
    """Total state sum_j phi_k(k_j) [v_j, 1]^T per head, fp32 ``(b*h, F, d_v+1)``."""
    code = _check_qkv(k, k, v)
    k, v = k.contiguous(), v.contiguous()
    b, h, t, d = k.shape
    dv = v.shape[-1]
    state = torch.empty((b * h, feature_dim(d), dv + 1), dtype=torch.float32, device=k.device)
    with _on_device(k.device):
        _, ws_bytes = chunked_plan(b * h, t, d, dv, k.dtype, segments)
        if workspace is None:
            workspace = _workspace(ws_bytes, k.device)
        st = N.lib().la_based_chunked_state(
            _ptr(k), _ptr(v), _ptr(state), b, h, t, d, dv, code, _ptr(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            int(segments), _stream_ptr(k.device))
    N.check(st, "la_based_chunked_state")
    return state


def sliding_window(q, k, v, window_size: int = 64) -> torch.Tensor:
    """Causal sliding-window softmax attention over [i - W + 1, i]."""
    code = _check_qkv(q, k, v, same_dv=True)
    if int(window_size) < 1:
        raise ValueError("window_size must be >= 1")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    b, h, t, d = q.shape
    out = torch.empty_like(q)
    with _on_device(q.device):
        st = N.lib().la_sliding_window_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, t, d, code,
                                           int(window_size), _stream_ptr(q.device))
    N.check(st, "la_sliding_window_fwd")
    return out


def based_layer(q, k, v, window_size: int = 64, eps: float = 1e-6, segments: int = 0,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The full BASED layer: chunked BASED attention plus sliding-window
    softmax attention over the same q, k, v (window <= 129): two tensor-core
    kernels for bf16, d_qk = 16, d_v = 64 (the second adds its term to the
    first's output), one pass on CUDA cores otherwise."""
    code = _check_qkv(q, k, v)
    if int(window_size) < 1:
        raise ValueError("window_size must be >= 1")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    b, h, t, d = q.shape
    dv = v.shape[-1]
    out = torch.empty((b, h, t, dv), dtype=q.dtype, device=q.device)
    with _on_device(q.device):
        g, ws_bytes = chunked_plan(b * h, t, d, dv, q.dtype, segments)
        if workspace is None:
            workspace = _workspace(ws_bytes, q.device)
        st = N.lib().la_based_layer_fwd(
            _ptr(q), _ptr(k), _ptr(v), _ptr(out), b, h, t, d, dv, code, int(window_size),
            float(eps), _ptr(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            int(segments), _stream_ptr(q.device))
    N.check(st, "la_based_layer_fwd")
    return out


_copy_streams: dict = {}


def _side_streams(device):
    """Two streams per device (host->device, device->host), created once."""
    key = torch.device(device).index
    if key not in _copy_streams:
        _copy_streams[key] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _copy_streams[key]


def based_chunked_host(q, k, v, chunk_size: int = 64, eps: float = 1e-6, normalize: bool = True,
                       head_groups: int = 8, device=None, out: torch.Tensor | None = None):
    """Chunked BASED attention on host-resident ``(b, h, t, d)`` tensors.

    The heads are processed in ``head_groups`` groups so that the host-to-
    device copy of one group, the kernels of the previous group and the
    device-to-host copy of the group before run at the same time (PCIe is
    full duplex): the copies run on two side streams of ``device`` and are
    joined back into its current stream before the call returns.  Inputs
    should be pinned (``pin_memory()``) for the copies to overlap.  The
    result is written into ``out`` (a pinned host tensor is allocated if it
    is None) and is complete once the current stream has reached this point
    (e.g. after ``torch.cuda.current_stream().synchronize()``).
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.device.type != "cpu":
            raise ValueError(f"{name} must be a host tensor for based_chunked_host")
    if q.shape != k.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError("q, k, v shapes do not match")
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    b, h, t, d = q.shape
    dv = v.shape[-1]
    bh = b * h
    if out is None:
        out = torch.empty((b, h, t, dv), dtype=q.dtype).pin_memory()
    elif out.shape != (b, h, t, dv) or out.dtype != q.dtype or out.device.type != "cpu":
        raise ValueError(f"out must be a host {q.dtype} tensor of shape {(b, h, t, dv)}")
    qf, kf, vf = (x.reshape(bh, t, x.shape[-1]) for x in (q, k, v))
    of = out.view(bh, t, dv)
    groups = max(1, min(int(head_groups), bh))
    step = -(-bh // groups)
    with _on_device(device):
        compute = torch.cuda.current_stream(device)
        h2d, d2h = _side_streams(device)
        qd = torch.empty((bh, t, d), dtype=q.dtype, device=device)
        kd = torch.empty_like(qd)
        vd = torch.empty((bh, t, dv), dtype=v.dtype, device=device)
        start = torch.cuda.Event()
        start.record(compute)  # the buffers are free once the compute stream is here
        h2d.wait_event(start)
        d2h.wait_event(start)
        for lo in range(0, bh, step):
            hi = min(bh, lo + step)
            with torch.cuda.stream(h2d):
                for dst, src in ((qd, qf), (kd, kf), (vd, vf)):
                    dst[lo:hi].copy_(src[lo:hi], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(h2d)
            compute.wait_event(ready)
            y = based_chunked(qd[lo:hi].unsqueeze(0), kd[lo:hi].unsqueeze(0),
                              vd[lo:hi].unsqueeze(0), chunk_size=chunk_size, eps=eps,
                              normalize=normalize)
            done = torch.cuda.Event()
            done.record(compute)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                of[lo:hi].copy_(y[0], non_blocking=True)
            y.record_stream(d2h)  # its memory is not reused before this copy ends
        finished = torch.cuda.Event()
        finished.record(d2h)
        compute.wait_event(finished)
        h2d_done = torch.cuda.Event()
        h2d_done.record(h2d)
        compute.wait_event(h2d_done)
    return out
