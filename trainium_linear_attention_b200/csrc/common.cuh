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
// state pass: per-(head, segment) state -> seg_states[bh][g][F][dv+1]
int launch_chunked_state_simt(const void *k, const void *v, float *seg_states, int64_t bh,
                              int64_t n, int dqk, int dv, int dtype, int segments,
                              int64_t seg_len, cudaStream_t s);
// output pass: prefix = init_state + sum of earlier segments' states.
int launch_chunked_output_simt(const void *q, const void *k, const void *v, void *out,
                               const float *init_state, float *final_state,
                               const float *seg_states, int64_t bh, int64_t n, int dqk, int dv,
                               int dtype, float eps, bool normalize, int segments,
                               int64_t seg_len, cudaStream_t s);

// Largest (d_qk, d_v) the SIMT chunked kernels hold on chip.
bool chunked_simt_supported(int64_t dqk, int64_t dv);

// Workspace bytes la_based_chunked_fwd needs for these arguments (the exact
// need; la_based_chunked_plan may report more).
size_t chunked_fwd_scratch_bytes(int64_t bh, int64_t n, int64_t d_qk, int64_t d_v, int dtype,
                                 int segments, unsigned flags);

}  // namespace la
