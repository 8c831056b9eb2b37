// la_based_chunked_fwd_noalloc: the chunked BASED forward for callers that
// cannot allocate device memory.
//
// A segmented chunked forward needs scratch for the per-segment states
// (la_based_chunked_workspace_size bytes).  Some callers cannot provide it:
// code loaded as a plugin by a host framework that owns all device memory
// and hands its plugins no allocation hook, or latency-critical paths that
// must not call cudaMalloc (which can synchronise the device).  This entry
// point takes its scratch from a fixed array compiled into the library
// instead, and otherwise behaves exactly like la_based_chunked_fwd, which it
// calls.  It calls no cudaMalloc, cudaFree or allocating library routine.
//
// Limits and sharing:
//   * the array holds kNoAllocScratchBytes (8 MiB) on every device that loads
//     the library, until the process exits: 210 (head, segment) states of the
//     d_qk = 16, d_v = 64 fast path (39,780 bytes each);
//   * a request whose scratch would exceed it fails with LA_ERR_WORKSPACE;
//   * every call on a device shares the one array and leaves its contents
//     behind; calls whose kernels overlap on the GPU (e.g. on two streams
//     without ordering) race on it.  The forward writes every scratch byte it
//     reads before reading it, so nothing needs clearing between calls.
//   * the array's address belongs to the CUDA context, not to the device: the
//     first call in each context resolves it (cudaGetSymbolAddress with that
//     context current) and caches it by the context's unique id; make that
//     first call before any stream capture.
#include "common.cuh"

namespace la {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, not a device address: the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

}  // namespace
}  // namespace la

extern "C" int la_based_chunked_fwd_noalloc(const void *q, const void *k, const void *v,
                                            void *out, int64_t batch, int64_t heads,
                                            int64_t seq_len, int64_t d_qk, int64_t d_v,
                                            int dtype, int64_t chunk_size, float eps,
                                            unsigned flags, const float *init_state,
                                            float *final_state, int segments, void *stream) {
  // The scratch never holds states this caller wrote with la_based_chunked_state.
  if (flags & LA_CHUNKED_REUSE_SEGMENTS) return LA_ERR_INVALID_ARGUMENT;
  if (batch < 0 || heads < 0 || seq_len < 0 || d_qk < 1 || d_v < 1 || segments < 0)
    return LA_ERR_INVALID_ARGUMENT;
  // the scratch this request needs, decided by the same planner as the
  // forward itself (pointer alignment included)
  if (batch * heads > 0 && seq_len > 0) {
    la::ChunkedFwdPlan plan;
    const int st = la::plan_chunked_fwd(q, k, v, out, batch * heads, seq_len, d_qk, d_v, dtype,
                                        segments, flags, &plan);
    if (st != LA_OK) return st;
    if (plan.scratch > la::kNoAllocScratchBytes) return LA_ERR_WORKSPACE;
  }
  void *scratch = la::context_symbol_address(&la::g_noalloc_scratch);
  if (!scratch) return LA_ERR_CUDA;
  return la_based_chunked_fwd(q, k, v, out, batch, heads, seq_len, d_qk, d_v, dtype, chunk_size,
                              eps, flags, init_state, final_state, scratch,
                              la::kNoAllocScratchBytes, segments, stream);
}
