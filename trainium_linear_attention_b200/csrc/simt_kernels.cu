// CUDA-core (SIMT) kernels: the fp32 path and the generic-shape path.
//
// These compute in fp32 on CUDA cores for any head widths up to 128 and any
// sequence length.  They are the permanent fp32 implementation (BASED config
// 1 asks for rel-L2 <= 1e-4 against the fp32 reference, beyond what bf16 /
// tf32 tensor-core operands give) and cover shapes the tensor-core kernels do
// not specialise.  Layout of every tensor: (batch*heads, seq_len, d) row-major.
#include "common.cuh"

#include <math.h>

namespace la {
namespace {

constexpr int kRows = 64;          // query rows per CTA
constexpr int kLanesPerRow = 4;    // threads cooperating on one query row
constexpr int kThreads = kRows * kLanesPerRow;
constexpr int kKeyTile = 64;       // keys staged in shared memory per step
constexpr int kMaxD = 128;
constexpr int kMaxCols = (kMaxD + 1 + kLanesPerRow - 1) / kLanesPerRow;  // 33

template <typename T>
__device__ __forceinline__ void load_tile(float *dst, int ld_dst, const T *src, int64_t row0,
                                          int64_t nrows_total, int rows, int cols, float mul) {
  for (int idx = threadIdx.x; idx < rows * cols; idx += blockDim.x) {
    int r = idx / cols, c = idx - r * cols;
    int64_t gr = row0 + r;
    float x = 0.f;
    if (gr >= 0 && gr < nrows_total) x = to_f32(src[gr * cols + c]) * mul;
    dst[r * ld_dst + c] = x;
  }
}

// Sum over the kLanesPerRow threads of one row (they are adjacent lanes).
__device__ __forceinline__ float row_allreduce(float x) {
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  return x;
}

// ---------------------------------------------------------------------------
// Parallel BASED (kernels/pytorch_attention.py:27-42 semantics).
// grid (ceil(n/64), bh); 256 threads = 64 query rows x 4 lanes.  Each lane
// owns output columns lane, lane+4, ...; the q.k dot product is split over the
// 4 lanes and all-reduced, so every lane sees the same poly weight.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads)
based_parallel_simt_kernel(const T *__restrict__ q, const T *__restrict__ k,
                           const T *__restrict__ v, T *__restrict__ out, int64_t n, int dqk,
                           int dv, float scale, float eps) {
  extern __shared__ float smem[];
  const int ldq = dqk + 1;
  float *qs = smem;                       // [64][dqk+1]
  float *ks = qs + kRows * ldq;           // [64][dqk+1]
  float *vs = ks + kKeyTile * ldq;        // [64][dv]

  const int64_t bh = blockIdx.y;
  const int64_t q0 = (int64_t)blockIdx.x * kRows;
  const int row = threadIdx.x / kLanesPerRow;
  const int lane = threadIdx.x % kLanesPerRow;
  const int64_t qi = q0 + row;
  const T *qh = q + bh * n * dqk;
  const T *kh = k + bh * n * dqk;
  const T *vh = v + bh * n * dv;

  load_tile(qs, ldq, qh, q0, n, kRows, dqk, scale);

  float acc[kMaxCols];
#pragma unroll
  for (int i = 0; i < kMaxCols; ++i) acc[i] = 0.f;
  float den = 0.f;

  const int64_t last_key = min64(n, q0 + kRows) - 1;
  for (int64_t k0 = 0; k0 <= last_key; k0 += kKeyTile) {
    __syncthreads();
    load_tile(ks, ldq, kh, k0, n, kKeyTile, dqk, 1.f);
    load_tile(vs, dv, vh, k0, n, kKeyTile, dv, 1.f);
    __syncthreads();
    const int jmax = (int)min64(kKeyTile, last_key - k0 + 1);
    for (int j = 0; j < jmax; ++j) {
      float s = 0.f;
      for (int a = lane; a < dqk; a += kLanesPerRow) s = fmaf(qs[row * ldq + a], ks[j * ldq + a], s);
      s = row_allreduce(s);
      float p = fmaf(s, fmaf(0.5f, s, 1.f), 1.f);  // 1 + s + s^2/2
      p = (k0 + j <= qi) ? p : 0.f;
      den += p;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        int c = lane + i * kLanesPerRow;
        if (c < dv) acc[i] = fmaf(p, vs[j * dv + c], acc[i]);
      }
    }
  }
  if (qi < n) {
    const float inv = 1.f / (den + eps);
    T *oh = out + (bh * n + qi) * dv;
#pragma unroll
    for (int i = 0; i < kMaxCols; ++i) {
      int c = lane + i * kLanesPerRow;
      if (c < dv) oh[c] = from_f32<T>(acc[i] * inv);
    }
  }
}

// ---------------------------------------------------------------------------
// Sliding-window softmax (benchmarks/sliding_attention_benchmark.py:32-56
// semantics), online softmax over the band [i-W+1, i] only.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads)
sliding_simt_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
                    T *__restrict__ out, int64_t n, int d, int64_t window, float scale) {
  extern __shared__ float smem[];
  const int ldq = d + 1;
  float *qs = smem;
  float *ks = qs + kRows * ldq;
  float *vs = ks + kKeyTile * ldq;

  const int64_t bh = blockIdx.y;
  const int64_t q0 = (int64_t)blockIdx.x * kRows;
  const int row = threadIdx.x / kLanesPerRow;
  const int lane = threadIdx.x % kLanesPerRow;
  const int64_t qi = q0 + row;
  const T *qh = q + bh * n * d;
  const T *kh = k + bh * n * d;
  const T *vh = v + bh * n * d;

  load_tile(qs, ldq, qh, q0, n, kRows, d, scale);

  float acc[kMaxCols];
#pragma unroll
  for (int i = 0; i < kMaxCols; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;

  const int64_t first_key = max64(0, q0 - window + 1);
  const int64_t last_key = min64(n, q0 + kRows) - 1;
  for (int64_t k0 = first_key; k0 <= last_key; k0 += kKeyTile) {
    __syncthreads();
    load_tile(ks, ldq, kh, k0, n, kKeyTile, d, 1.f);
    load_tile(vs, d, vh, k0, n, kKeyTile, d, 1.f);
    __syncthreads();
    const int jmax = (int)min64(kKeyTile, last_key - k0 + 1);
    for (int j = 0; j < jmax; ++j) {
      const int64_t key = k0 + j;
      float s = 0.f;
      for (int a = lane; a < d; a += kLanesPerRow) s = fmaf(qs[row * ldq + a], ks[j * ldq + a], s);
      s = row_allreduce(s);
      const bool valid = key <= qi && key >= qi - window + 1;
      if (!valid) continue;  // uniform across the 4 lanes of the row
      if (s > m) {
        const float corr = expf(m - s);  // exp(-inf) = 0 on the first valid key
        l *= corr;
#pragma unroll
        for (int i = 0; i < kMaxCols; ++i) acc[i] *= corr;
        m = s;
      }
      const float p = expf(s - m);
      l += p;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        int c = lane + i * kLanesPerRow;
        if (c < d) acc[i] = fmaf(p, vs[j * d + c], acc[i]);
      }
    }
  }
  if (qi < n) {
    const float inv = 1.f / l;
    T *oh = out + (bh * n + qi) * d;
#pragma unroll
    for (int i = 0; i < kMaxCols; ++i) {
      int c = lane + i * kLanesPerRow;
      if (c < d) oh[c] = from_f32<T>(acc[i] * inv);
    }
  }
}

// ---------------------------------------------------------------------------
// Chunked recurrent BASED (kernels/nki_attention_chunked.py:71-109 recurrence,
// plus the normaliser as state column d_v).  The state S[F][dv+1] (fp32) lives
// in shared memory for the whole segment.  Key-side basis phi_k = [1, k_a,
// k_a k_b (a<=b)], query side phi_q = [1, q_a/sqrt(d), q_a q_b w_ab].
// ---------------------------------------------------------------------------
constexpr int kChunk = 64;

// With a sliding window (the full BASED layer) the K/V chunks form a ring of
// kRing buffers: chunk cc (global index t0 / 64) sits in buffer cc % kRing,
// so the window's keys in the two chunks before stay on chip (W <= 129).
constexpr int kRing = 3;
constexpr int kMaxWindow = 2 * kChunk + 1;

struct ChunkSmem {
  float *S;      // [F][dv+1]
  float *qs;     // [64][dqk+1]   raw q
  float *ks;     // [64][dqk+1]   raw k of the current chunk
  float *vs;     // [64][dv+1]    v with a trailing 1 (normaliser column)
  float *kring;  // ring buffers (window > 0), stride kChunk * (dqk + 1)
  float *vring;  //                           stride kChunk * (dv + 1)
};

__device__ __forceinline__ ChunkSmem carve(float *smem, int F, int dqk, int dv, bool ring) {
  ChunkSmem c;
  c.S = smem;
  c.qs = c.S + F * (dv + 1);
  c.kring = c.ks = c.qs + kChunk * (dqk + 1);
  c.vring = c.vs = c.ks + (ring ? kRing : 1) * kChunk * (dqk + 1);
  return c;
}

// chunk cc's buffers (the ring slot cc % kRing; slot 0 without a ring)
__device__ __forceinline__ void select_chunk(ChunkSmem &c, int64_t cc, int dqk, int dv,
                                             bool ring) {
  const int slot = ring ? (int)(cc % kRing) : 0;
  c.ks = c.kring + slot * kChunk * (dqk + 1);
  c.vs = c.vring + slot * kChunk * (dv + 1);
}

template <typename T>
__device__ __forceinline__ void load_chunk_kv(float *ks, float *vs, const T *kh, const T *vh,
                                              int64_t t0, int64_t t_end, int dqk, int dv) {
  const int ldk = dqk + 1, ldv = dv + 1;
  for (int idx = threadIdx.x; idx < kChunk * dqk; idx += blockDim.x) {
    int r = idx / dqk, a = idx - r * dqk;
    int64_t t = t0 + r;
    ks[r * ldk + a] = t < t_end ? to_f32(kh[t * dqk + a]) : 0.f;
  }
  for (int idx = threadIdx.x; idx < kChunk * ldv; idx += blockDim.x) {
    int r = idx / ldv, e = idx - r * ldv;
    int64_t t = t0 + r;
    float x = 0.f;
    if (t < t_end) x = (e < dv) ? to_f32(vh[t * dv + e]) : 1.f;
    vs[r * ldv + e] = x;
  }
}

// S[f][e] += sum_{t in chunk} phi_k(k_t)[f] * vaug_t[e]; thread per feature row
// (rows strided by blockDim), columns in register blocks of 32.  The identity
// map has phi_k(k) = k (F = dqk); the Taylor map [1, k_a, k_a k_b (a <= b)].
__device__ void chunk_state_update(const ChunkSmem &c, int F, int dqk, int dv, int rows,
                                   bool identity) {
  const int ldk = dqk + 1, ldv = dv + 1;
  for (int f = threadIdx.x; f < F; f += blockDim.x) {
    // decode feature f -> (a, b) ; kind 0 const, 1 linear, 2 quadratic
    int kind, a = 0, b = 0;
    if (identity) {
      kind = 1;
      a = f;
    } else if (f == 0) {
      kind = 0;
    } else if (f <= dqk) {
      kind = 1;
      a = f - 1;
    } else {
      kind = 2;
      int r = f - 1 - dqk;
      a = 0;
      while (r >= dqk - a) {
        r -= dqk - a;
        ++a;
      }
      b = a + r;
    }
    for (int e0 = 0; e0 < ldv; e0 += 32) {
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0.f;
      for (int t = 0; t < rows; ++t) {
        float phi = 1.f;
        if (kind == 1) phi = c.ks[t * ldk + a];
        if (kind == 2) phi = c.ks[t * ldk + a] * c.ks[t * ldk + b];
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (e0 + i < ldv) acc[i] = fmaf(phi, c.vs[t * ldv + e0 + i], acc[i]);
      }
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (e0 + i < ldv) c.S[f * ldv + e0 + i] += acc[i];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
chunked_state_simt_kernel(const T *__restrict__ k, const T *__restrict__ v,
                          float *__restrict__ seg_states, int64_t n, int dqk, int dv,
                          int identity, int segments, int64_t seg_len) {
  extern __shared__ float smem[];
  const int F = identity ? dqk : (int)feature_dim(dqk);
  const int ldv = dv + 1;
  ChunkSmem c = carve(smem, F, dqk, dv, false);
  const int64_t bh = blockIdx.y;
  const int g = blockIdx.x;
  const int64_t t_begin = (int64_t)g * seg_len;
  const int64_t t_end = min64(n, t_begin + seg_len);
  const T *kh = k + bh * n * dqk;
  const T *vh = v + bh * n * dv;
  for (int i = threadIdx.x; i < F * ldv; i += blockDim.x) c.S[i] = 0.f;
  for (int64_t t0 = t_begin; t0 < t_end; t0 += kChunk) {
    __syncthreads();
    load_chunk_kv(c.ks, c.vs, kh, vh, t0, t_end, dqk, dv);
    __syncthreads();
    chunk_state_update(c, F, dqk, dv, (int)min64(kChunk, t_end - t0), identity != 0);
  }
  __syncthreads();
  float *dst = seg_states + (bh * segments + g) * (int64_t)F * ldv;
  for (int i = threadIdx.x; i < F * ldv; i += blockDim.x) dst[i] = c.S[i];
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
chunked_output_simt_kernel(const T *__restrict__ q, const T *__restrict__ k,
                           const T *__restrict__ v, T *__restrict__ out,
                           const float *__restrict__ init_state, float *__restrict__ final_state,
                           const float *__restrict__ seg_states, int64_t n, int dqk, int dv,
                           int identity, float eps, int normalize, int segments,
                           int64_t seg_len, int window) {
  extern __shared__ float smem[];
  const int F = identity ? dqk : (int)feature_dim(dqk);
  const int ldv = dv + 1, ldq = dqk + 1;
  const bool ring = window > 0;
  ChunkSmem c = carve(smem, F, dqk, dv, ring);
  const int64_t bh = blockIdx.y;
  const int g = blockIdx.x;
  const int64_t t_begin = (int64_t)g * seg_len;
  const int64_t t_end = min64(n, t_begin + seg_len);
  const T *qh = q + bh * n * dqk;
  const T *kh = k + bh * n * dqk;
  const T *vh = v + bh * n * dv;

  // prefix state: init + the sum of the earlier segments' states (slot g - 1
  // of seg_states after launch_prefix_segments)
  for (int i = threadIdx.x; i < F * ldv; i += blockDim.x) {
    float s = init_state ? init_state[bh * (int64_t)F * ldv + i] : 0.f;
    if (g > 0) s += seg_states[(bh * segments + g - 1) * (int64_t)F * ldv + i];
    c.S[i] = s;
  }

  const int row = threadIdx.x / kLanesPerRow;
  const int lane = threadIdx.x % kLanesPerRow;
  const float rsd = 1.f / sqrtf((float)dqk);
  const float w_diag = 1.f / (2.f * dqk), w_off = 1.f / (float)dqk;

  // the window of the segment's first rows reaches into the two chunks
  // before it: bring them into their ring slots
  if (ring) {
    for (int64_t cc = t_begin / kChunk - 2; cc < t_begin / kChunk; ++cc) {
      if (cc < 0) continue;
      select_chunk(c, cc, dqk, dv, true);
      load_chunk_kv(c.ks, c.vs, kh, vh, cc * kChunk, n, dqk, dv);
    }
  }
  for (int64_t t0 = t_begin; t0 < t_end; t0 += kChunk) {
    __syncthreads();
    select_chunk(c, t0 / kChunk, dqk, dv, ring);
    load_chunk_kv(c.ks, c.vs, kh, vh, t0, t_end, dqk, dv);
    for (int idx = threadIdx.x; idx < kChunk * dqk; idx += blockDim.x) {
      int r = idx / dqk, a = idx - r * dqk;
      int64_t t = t0 + r;
      c.qs[r * ldq + a] = t < t_end ? to_f32(qh[t * dqk + a]) : 0.f;
    }
    __syncthreads();
    const int rows = (int)min64(kChunk, t_end - t0);

    float acc[kMaxCols];
#pragma unroll
    for (int i = 0; i < kMaxCols; ++i) acc[i] = 0.f;
    const float *qr = c.qs + row * ldq;
    // inter-chunk: phi_q(q_t) . S (state before this chunk's update)
    if (identity) {
      // phi_q(q) = q / sqrt(d)
      for (int a = 0; a < dqk; ++a) {
        const float phi = qr[a] * rsd;
#pragma unroll
        for (int i = 0; i < kMaxCols; ++i) {
          int e = lane + i * kLanesPerRow;
          if (e < ldv) acc[i] = fmaf(phi, c.S[a * ldv + e], acc[i]);
        }
      }
    } else {
      int f = 0;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        int e = lane + i * kLanesPerRow;
        if (e < ldv) acc[i] = c.S[e];
      }
      f = 1;
      for (int a = 0; a < dqk; ++a, ++f) {
        const float phi = qr[a] * rsd;
#pragma unroll
        for (int i = 0; i < kMaxCols; ++i) {
          int e = lane + i * kLanesPerRow;
          if (e < ldv) acc[i] = fmaf(phi, c.S[f * ldv + e], acc[i]);
        }
      }
      for (int a = 0; a < dqk; ++a) {
        for (int b = a; b < dqk; ++b, ++f) {
          const float phi = qr[a] * qr[b] * (a == b ? w_diag : w_off);
#pragma unroll
          for (int i = 0; i < kMaxCols; ++i) {
            int e = lane + i * kLanesPerRow;
            if (e < ldv) acc[i] = fmaf(phi, c.S[f * ldv + e], acc[i]);
          }
        }
      }
    }
    // intra-chunk: causal 1 + s + s^2/2 (identity map: s) against this
    // chunk's keys.  The loop bound is uniform over the CTA (the all-reduce is
    // a full-warp shuffle); keys after the row are masked to weight 0.
    for (int j = 0; j < rows; ++j) {
      float s = 0.f;
      for (int a = lane; a < dqk; a += kLanesPerRow) s = fmaf(qr[a], c.ks[j * ldq + a], s);
      s = row_allreduce(s) * rsd;
      float p = identity ? s : fmaf(s, fmaf(0.5f, s, 1.f), 1.f);
      p = (j <= row) ? p : 0.f;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        int e = lane + i * kLanesPerRow;
        if (e < ldv) acc[i] = fmaf(p, c.vs[j * ldv + e], acc[i]);
      }
    }
    // the lane holding column dv broadcasts the denominator to its row
    float den_part = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxCols; ++i)
      if (lane + i * kLanesPerRow == dv) den_part = acc[i];
    const float den = row_allreduce(den_part);
    const float inv = normalize ? 1.f / (den + eps) : 1.f;
#pragma unroll
    for (int i = 0; i < kMaxCols; ++i) acc[i] *= inv;
    if (ring) {
      // the full BASED layer: + softmax over the window [t - W + 1, t] of
      // the same scores s = q.k / sqrt(d) (benchmarks/sliding_attention_
      // benchmark.py:32-56), online over the keys of this chunk and the two
      // before it; the key loop bounds are uniform over the CTA
      const int64_t t_row = t0 + row;
      float m = -INFINITY, l = 0.f;
      float sw[kMaxCols];
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) sw[i] = 0.f;
      for (int64_t kk = max64(0, t0 - window + 1); kk < t0 + rows; ++kk) {
        const int64_t kc = kk / kChunk;
        const int kr = (int)(kk - kc * kChunk);
        const int slot = (int)(kc % kRing);
        const float *krow = c.kring + (slot * kChunk + kr) * ldq;
        const float *vrow = c.vring + (slot * kChunk + kr) * ldv;
        float s = 0.f;
        for (int a = lane; a < dqk; a += kLanesPerRow) s = fmaf(qr[a], krow[a], s);
        s = row_allreduce(s) * rsd;
        if (kk <= t_row && kk > t_row - window && row < rows) {  // uniform per row
          if (s > m) {
            const float corr = expf(m - s);  // exp(-inf) = 0 on the first key
            l *= corr;
#pragma unroll
            for (int i = 0; i < kMaxCols; ++i) sw[i] *= corr;
            m = s;
          }
          const float pe = expf(s - m);
          l += pe;
#pragma unroll
          for (int i = 0; i < kMaxCols; ++i) {
            const int e = lane + i * kLanesPerRow;
            if (e < dv) sw[i] = fmaf(pe, vrow[e], sw[i]);
          }
        }
      }
      const float linv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) acc[i] = fmaf(sw[i], linv, acc[i]);
    }
    if (row < rows) {
      T *oh = out + (bh * n + t0 + row) * dv;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        int e = lane + i * kLanesPerRow;
        if (e < dv) oh[e] = from_f32<T>(acc[i]);
      }
    }
    __syncthreads();  // every row read S before the update
    chunk_state_update(c, F, dqk, dv, rows, identity != 0);
  }
  if (final_state && g == segments - 1) {
    __syncthreads();
    float *dst = final_state + bh * (int64_t)F * ldv;
    for (int i = threadIdx.x; i < F * ldv; i += blockDim.x) dst[i] = c.S[i];
  }
}

size_t chunked_simt_smem(int64_t F, int dqk, int dv, bool ring = false) {
  const int bufs = ring ? kRing : 1;
  return sizeof(float) *
         (size_t)(F * (dv + 1) + (1 + bufs) * kChunk * (dqk + 1) + bufs * kChunk * (dv + 1));
}

}  // namespace

bool chunked_simt_supported(int64_t features, int64_t dqk, int64_t dv) {
  if (dqk < 1 || dqk > kMaxD || dv < 1 || dv > kMaxD || features < 1) return false;
  return chunked_simt_smem(features, (int)dqk, (int)dv) <= 200 * 1024;
}

bool layer_simt_supported(int64_t dqk, int64_t dv, int64_t window) {
  if (dqk < 1 || dqk > kMaxD || dv < 1 || dv > kMaxD || window < 1 || window > kMaxWindow)
    return false;
  return chunked_simt_smem(feature_dim(dqk), (int)dqk, (int)dv, true) <= 200 * 1024;
}

#define LA_DISPATCH_DTYPE(dtype, T, ...)                    \
  do {                                                      \
    if ((dtype) == LA_DTYPE_FLOAT32) {                      \
      using T = float;                                      \
      __VA_ARGS__;                                          \
    } else if ((dtype) == LA_DTYPE_BFLOAT16) {              \
      using T = __nv_bfloat16;                              \
      __VA_ARGS__;                                          \
    } else {                                                \
      return LA_ERR_INVALID_ARGUMENT;                       \
    }                                                       \
  } while (0)

int launch_parallel_simt(const void *q, const void *k, const void *v, void *out, int64_t bh,
                         int64_t n, int dqk, int dv, int dtype, float eps, cudaStream_t s) {
  if (dqk > kMaxD || dv > kMaxD) return LA_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * (size_t)((kRows + kKeyTile) * (dqk + 1) + kKeyTile * dv);
  dim3 grid((unsigned)((n + kRows - 1) / kRows), (unsigned)bh);
  const float scale = 1.f / sqrtf((float)dqk);
  LA_DISPATCH_DTYPE(dtype, T, {
    if (smem > 48 * 1024) {
      if (allow_dynamic_smem((const void *)based_parallel_simt_kernel<T>, (int)smem) != LA_OK) return LA_ERR_CUDA;
    }
    based_parallel_simt_kernel<T><<<grid, kThreads, smem, s>>>(
        (const T *)q, (const T *)k, (const T *)v, (T *)out, n, dqk, dv, scale, eps);
  });
  return check_launch();
}

int launch_sliding_simt(const void *q, const void *k, const void *v, void *out, int64_t bh,
                        int64_t n, int d, int dtype, int64_t window, cudaStream_t s) {
  if (d > kMaxD) return LA_ERR_UNSUPPORTED;
  const size_t smem = sizeof(float) * (size_t)((kRows + kKeyTile) * (d + 1) + kKeyTile * d);
  dim3 grid((unsigned)((n + kRows - 1) / kRows), (unsigned)bh);
  const float scale = 1.f / sqrtf((float)d);
  LA_DISPATCH_DTYPE(dtype, T, {
    if (smem > 48 * 1024) {
      if (allow_dynamic_smem((const void *)sliding_simt_kernel<T>, (int)smem) != LA_OK) return LA_ERR_CUDA;
    }
    sliding_simt_kernel<T><<<grid, kThreads, smem, s>>>((const T *)q, (const T *)k, (const T *)v,
                                                        (T *)out, n, d, window, scale);
  });
  return check_launch();
}

int launch_chunked_state_simt(const void *k, const void *v, float *seg_states, int64_t bh,
                              int64_t n, int dqk, int dv, int dtype, bool identity, int segments,
                              int64_t seg_len, cudaStream_t s) {
  const int64_t F = identity ? dqk : feature_dim(dqk);
  if (!chunked_simt_supported(F, dqk, dv)) return LA_ERR_UNSUPPORTED;
  const size_t smem = chunked_simt_smem(F, dqk, dv);
  dim3 grid((unsigned)segments, (unsigned)bh);
  LA_DISPATCH_DTYPE(dtype, T, {
    if (allow_dynamic_smem((const void *)chunked_state_simt_kernel<T>, (int)smem) != LA_OK) return LA_ERR_CUDA;
    chunked_state_simt_kernel<T><<<grid, kThreads, smem, s>>>(
        (const T *)k, (const T *)v, seg_states, n, dqk, dv, identity ? 1 : 0, segments, seg_len);
  });
  return check_launch();
}

int launch_chunked_output_simt(const void *q, const void *k, const void *v, void *out,
                               const float *init_state, float *final_state,
                               const float *seg_states, int64_t bh, int64_t n, int dqk, int dv,
                               int dtype, bool identity, float eps, bool normalize, int segments,
                               int64_t seg_len, int64_t window, cudaStream_t s) {
  const int64_t F = identity ? dqk : feature_dim(dqk);
  if (window > 0 ? (identity || !layer_simt_supported(dqk, dv, window))
                 : !chunked_simt_supported(F, dqk, dv))
    return LA_ERR_UNSUPPORTED;
  const size_t smem = chunked_simt_smem(F, dqk, dv, window > 0);
  dim3 grid((unsigned)segments, (unsigned)bh);
  LA_DISPATCH_DTYPE(dtype, T, {
    if (allow_dynamic_smem((const void *)chunked_output_simt_kernel<T>, (int)smem) != LA_OK) return LA_ERR_CUDA;
    chunked_output_simt_kernel<T><<<grid, kThreads, smem, s>>>(
        (const T *)q, (const T *)k, (const T *)v, (T *)out, init_state, final_state, seg_states,
        n, dqk, dv, identity ? 1 : 0, eps, normalize ? 1 : 0, segments, seg_len, (int)window);
  });
  return check_launch();
}

}  // namespace la

namespace la {
namespace {
__global__ void prefix_segments_kernel(float *__restrict__ seg, float *__restrict__ total,
                                       int stride, int groups, int ratio, int64_t per_head) {
  constexpr int kMaxSlots = 16;
  // launched as the programmatic dependent of the state pass: wait for its
  // states, and let the output pass after this kernel be scheduled
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int64_t bh = blockIdx.y;
  const int slots = groups * ratio;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < per_head;
       i += (int64_t)gridDim.x * blockDim.x) {
    float *base = seg + bh * stride * per_head + i;
    float run = 0.f;
    if (slots <= kMaxSlots) {
      // every slot is read before any is written: the loads are all in flight
      float x[kMaxSlots];
#pragma unroll
      for (int j = 0; j < kMaxSlots; ++j) x[j] = j < slots ? base[(int64_t)j * per_head] : 0.f;
#pragma unroll
      for (int j = 0; j < kMaxSlots; ++j) {
        if (j < slots) {
          run += x[j];
          if (j % ratio == ratio - 1) base[(int64_t)(j / ratio) * per_head] = run;
        }
      }
    } else {
      for (int gr = 0; gr < groups; ++gr) {
        // read this group's slots [gr*ratio, (gr+1)*ratio) before writing slot gr <= gr*ratio
        for (int r = 0; r < ratio; ++r) run += base[(int64_t)(gr * ratio + r) * per_head];
        base[(int64_t)gr * per_head] = run;
      }
    }
    if (total) total[bh * per_head + i] = run;
  }
}
}  // namespace

int launch_prefix_segments(float *seg, float *total, int64_t bh, int stride, int groups,
                           int ratio, int64_t per_head, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((per_head + 255) / 256), (unsigned)bh);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, prefix_segments_kernel, seg, total, stride, groups, ratio,
                         per_head) != cudaSuccess) {
    note_launch();
    cudaGetLastError();
    return LA_ERR_CUDA;
  }
  return check_launch();
}
}  // namespace la
