// Shared helpers for the attention kernels (device side and launch side).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/la_attention.h"

namespace la {

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ---- element access ---------------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Index of the quadratic feature (a, b), a <= b, in the row-major upper
// triangle of a d x d matrix, offset by 1 + d (const + linear features).
__host__ __device__ __forceinline__ int quad_feature_index(int a, int b, int d) {
  // rows 0..a-1 contribute d, d-1, ..., d-a+1 entries
  return 1 + d + a * d - (a * (a - 1)) / 2 + (b - a);
}

__host__ __device__ __forceinline__ int64_t feature_dim(int64_t d) {
  return 1 + d + d * (d + 1) / 2;
}

// ---- launch helpers -------------------------------------------------------------
struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t smem_optin = 0;
};

// Properties of the current device (cached per device ordinal).
int current_device_info(DeviceInfo *info);

// Device address of the __device__ variable whose host-side name is `symbol`
// (a stand-in, not an address) in the CUDA context current on the calling
// thread; null if it cannot be resolved.  A module variable's address
// belongs to a context, not to a device (a host that makes its own driver
// contexts on a device gets its own copy of every such variable), so the
// address is resolved with cudaGetSymbolAddress once per context and cached
// by the context's unique id.
void *context_symbol_address(const void *symbol);

// Unique id (cuCtxGetId) of the context current on this thread; false if no
// context is current or the driver cannot tell.
bool current_context_id(unsigned long long *id);

// Raises `func`'s dynamic shared-memory limit to `bytes` in the current
// context, once: later calls make no CUDA API call, so a launch that follows
// can be captured into a CUDA graph.
int allow_dynamic_smem(const void *func, int bytes);

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? LA_OK : LA_ERR_CUDA; }

// Counts one kernel launch (la_launch_count).
void note_launch();

// Called after every kernel launch: counts it and returns LA_ERR_CUDA if it
// failed.
inline int check_launch() {
  note_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LA_OK : LA_ERR_CUDA;
}

// ---- SIMT kernel entry points (generic shapes, fp32 math) -----------------------
int launch_parallel_simt(const void *q, const void *k, const void *v, void *out, int64_t bh,
                         int64_t n, int dqk, int dv, int dtype, float eps, cudaStream_t s);

int launch_sliding_simt(const void *q, const void *k, const void *v, void *out, int64_t bh,
                        int64_t n, int d, int dtype, int64_t window, cudaStream_t s);

// Chunked: G segments of `seg_len` tokens each (multiple of the chunk tile).
// `identity` selects the identity feature map (phi(x) = x, F = d_qk) instead
// of the Taylor map (F = 1 + d + d(d+1)/2).
// state pass: per-(head, segment) state -> seg_states[bh][g][F][dv+1]
int launch_chunked_state_simt(const void *k, const void *v, float *seg_states, int64_t bh,
                              int64_t n, int dqk, int dv, int dtype, bool identity, int segments,
                              int64_t seg_len, cudaStream_t s);
// output pass: prefix = init_state + sum of earlier segments' states.
int launch_chunked_output_simt(const void *q, const void *k, const void *v, void *out,
                               const float *init_state, float *final_state,
                               const float *seg_states, int64_t bh, int64_t n, int dqk, int dv,
                               int dtype, bool identity, float eps, bool normalize, int segments,
                               int64_t seg_len, int64_t window, cudaStream_t s);

// Whether the SIMT chunked kernels hold a (features, d_v + 1) state on chip.
bool chunked_simt_supported(int64_t features, int64_t dqk, int64_t dv);
// ... and, for the full BASED layer (window > 0: sliding-window softmax added
// in the same pass), also the K/V of the two chunks before (W <= 129).
bool layer_simt_supported(int64_t dqk, int64_t dv, int64_t window);

// Chunked kernels whose Taylor state is split by feature rows over a
// thread-block cluster (cluster_chunked.cu), for widths whose state does not
// fit one CTA (d_qk = 64: F = 2145).
bool cluster_chunked_supported(int64_t dqk, int64_t dv);
int cluster_chunked_ctas_per_segment();
int launch_chunked_state_cluster(const void *k, const void *v, float *seg_states, int64_t bh,
                                 int64_t n, int dqk, int dv, int dtype, int segments,
                                 int n_launch, int64_t seg_len, cudaStream_t s);
int launch_chunked_output_cluster(const void *q, const void *k, const void *v, void *out,
                                  const float *init_state, float *final_state,
                                  const float *seg_states, int64_t bh, int64_t n, int dqk, int dv,
                                  int dtype, float eps, bool normalize, int segments,
                                  int64_t seg_len, int64_t window, cudaStream_t s);

// How la_based_chunked_fwd runs a request: the one place that decides the
// kernels, the segmentation and the scratch it needs.
struct ChunkedFwdPlan {
  bool identity = false;  // identity feature map (LA_CHUNKED_IDENTITY)
  int64_t features = 0;   // F: rows of a head's state
  bool tc = false;        // tcgen05 kernels (else the SIMT or cluster kernels)
  bool tc64 = false;      // d_qk = 64 tcgen05 kernels (state split over a 16-CTA cluster)
  bool cluster = false;   // the CUDA-core cluster kernels (state split over 8 CTAs)
  int64_t lead = 0;       // > 0: lead/main split with a lead of this many tokens
  int g = 1;              // equal segments per head
  int64_t seg_len = 0;    // tokens per segment
  int ratio = 1;          // state-pass pieces per segment
  size_t scratch = 0;     // workspace bytes the run needs
};
int plan_chunked_fwd(const void *q, const void *k, const void *v, const void *out, int64_t bh,
                     int64_t n, int64_t d_qk, int64_t d_v, int dtype, int segments,
                     unsigned flags, ChunkedFwdPlan *plan);

}  // namespace la
