"""BASED causal attention: the reference's public API on B200 kernels.

Same names, signatures and defaults as kernels/pytorch_attention.py of the
reference:

* ``ref_based_attn(q, k, v, eps=1e-6)`` -- the reference formula in plain
  PyTorch (kernels/pytorch_attention.py:27-42), for comparisons only; no
  CUDA path calls it.
* ``solution_nki(q, k, v, eps=1e-6)`` -- the name of the reference's device
  path (kernels/pytorch_attention.py:44-78); here the sm_100a parallel fused
  kernel.  d_v may differ from d_qk (the reference assumes they are equal).
* ``solution(q, k, v, eps=1e-6)`` -- dispatch (kernels/pytorch_attention.py:
  81-92).  It picks the parallel or the chunked kernel by sequence length and
  RAISES on failure; unlike the reference it never falls back to PyTorch.
* ``_check_nki()`` -- whether the native kernels can run here
  (kernels/pytorch_attention.py:16-24).
* ``trace_solution(q, k, v, eps=1e-6)`` -- ``solution`` for one fixed shape
  captured in a CUDA graph, the counterpart of the traced dispatch the
  reference's crossover study measures against lazy dispatch
  (benchmarks/crossover_benchmark.py:98-165, ``torch_neuronx.trace``).
"""

from __future__ import annotations

import math

import torch

from .. import ops

_native_available = None

#: sequence length up to which ``solution`` uses the parallel kernel for bf16
#: inputs whose chunked form has no tensor-core kernel (both on CUDA cores);
#: longer sequences use the chunked kernel.
CROSSOVER_SEQ_LEN_BF16 = 1024
#: the same for fp32 inputs (both kernels on CUDA cores)
CROSSOVER_SEQ_LEN_FP32 = 2048
#: bf16 with d_qk = 16, d_v = 64 (both forms on tcgen05 kernels): measured at
#: B*N = 262144, H = 16 on B200, parallel 0.35 ms vs chunked 0.74 ms at
#: N = 256 and 0.53 vs 0.55 ms at N = 512 (the persistent parallel kernel,
#: up to 4 query tiles), but 0.96 vs 0.45 ms at N = 1024 (one CTA per query
#: tile) and 2.86 vs 0.40 at N = 4096
CROSSOVER_SEQ_LEN_BF16_TC = 512


def _check_nki() -> bool:
    """True when the native library loads and a CUDA device is visible."""
    global _native_available
    if _native_available is None:
        try:
            from .. import _native
            _native.lib()
            _native_available = torch.cuda.is_available()
        except Exception:
            _native_available = False
    return _native_available


def ref_based_attn(q, k, v, eps=1e-6):
    """Reference BASED causal attention in plain PyTorch (any device).

    q, k: (b, h, t, d_qk); v: (b, h, t, d_v).  Returns (b, h, t, d_v).
    Computed in the input dtype, as the reference does.
    """
    d = q.shape[-1]
    scale = 1.0 / math.sqrt(d)
    scores = torch.matmul(q * scale, k.transpose(-2, -1))
    poly = 1.0 + scores + 0.5 * scores * scores
    t = q.shape[-2]
    mask = torch.tril(torch.ones(t, t, device=q.device, dtype=q.dtype))
    masked = poly * mask
    den = masked.sum(dim=-1, keepdim=True) + eps
    return torch.matmul(masked, v) / den


def solution_nki(q, k, v, eps=1e-6):
    """BASED causal attention via the sm_100a parallel fused kernel.

    q, k: (b, h, t, d_qk); v: (b, h, t, d_v), CUDA, float32 or bfloat16.
    Returns (b, h, t, d_v) in q.dtype.
    """
    return ops.based_parallel(q, k, v, eps=eps)


def solution(q, k, v, eps=1e-6):
    """BASED causal attention on B200: parallel kernel for short sequences,
    chunked recurrent kernel for long ones.  Raises on any failure."""
    t = q.shape[-2]
    if q.dtype == torch.float32:
        limit = CROSSOVER_SEQ_LEN_FP32
    elif q.shape[-1] == 16 and v.shape[-1] == 64:
        limit = CROSSOVER_SEQ_LEN_BF16_TC
    else:
        limit = CROSSOVER_SEQ_LEN_BF16
    if t <= limit:
        return ops.based_parallel(q, k, v, eps=eps)
    return ops.based_chunked(q, k, v, eps=eps)


def solution_kind(q, k, v) -> str:
    """Which kernel ``solution`` runs for these inputs: "parallel" or "chunked"."""
    t = q.shape[-2]
    if q.dtype == torch.float32:
        limit = CROSSOVER_SEQ_LEN_FP32
    elif q.shape[-1] == 16 and v.shape[-1] == 64:
        limit = CROSSOVER_SEQ_LEN_BF16_TC
    else:
        limit = CROSSOVER_SEQ_LEN_BF16
    return "parallel" if t <= limit else "chunked"


class TracedSolution:
    """``solution`` for one shape, dtype and device, captured in a CUDA graph.

    The capture records the kernels ``solution`` launches for the example
    inputs (including the chunked path's segment-state pass) against static
    input and output buffers; a call copies new inputs into the static
    buffers (skipped for inputs that already are them) and replays the graph,
    removing the host-side dispatch of every later call.  The returned
    tensor is the static output buffer, overwritten by the next call: clone
    it to keep it.  Replays run on the current stream.
    """

    def __init__(self, q, k, v, eps=1e-6, warmup: int = 2):
        if q.device.type != "cuda":
            raise ValueError("trace_solution needs CUDA tensors")
        self.eps = float(eps)
        self.kind = solution_kind(q, k, v)
        self.q = q.detach().clone().contiguous()
        self.k = k.detach().clone().contiguous()
        self.v = v.detach().clone().contiguous()
        with torch.cuda.device(q.device):
            side = torch.cuda.Stream(q.device)
            side.wait_stream(torch.cuda.current_stream(q.device))
            with torch.cuda.stream(side):  # resolve symbols and kernel attributes first
                for _ in range(max(1, int(warmup))):
                    solution(self.q, self.k, self.v, eps=self.eps)
            torch.cuda.current_stream(q.device).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.out = solution(self.q, self.k, self.v, eps=self.eps)

    def replay(self):
        """Re-run the captured kernels on the static inputs; returns the static output."""
        self.graph.replay()
        return self.out

    def __call__(self, q, k, v):
        for dst, src in ((self.q, q), (self.k, k), (self.v, v)):
            if src.shape != dst.shape or src.dtype != dst.dtype or src.device != dst.device:
                raise ValueError(f"traced for {tuple(dst.shape)} {dst.dtype} on {dst.device}, "
                                 f"got {tuple(src.shape)} {src.dtype} on {src.device}")
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src)
        return self.replay()


def trace_solution(q, k, v, eps=1e-6) -> TracedSolution:
    """Capture ``solution`` for the shape of the example inputs (see TracedSolution)."""
    return TracedSolution(q, k, v, eps=eps)
