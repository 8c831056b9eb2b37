// Chunked BASED attention for feature widths whose state does not fit one
// CTA: d_qk = 64 (F = 2145, a 2145 x 65 fp32 state of 557 KB per head) and
// other widths up to the limit of cluster_chunked_supported().
//
// One thread-block cluster of kCluster CTAs owns one (head, segment).  The
// state S[F][d_v + 1] (fp32, the key-side basis of include/la_attention.h,
// normaliser as the last column) is split by feature rows: CTA r keeps rows
// [r Fr, (r + 1) Fr) in its shared memory for the whole segment.  Per chunk
// of 64 tokens (the reference recurrence, kernels/nki_attention_chunked.py:
// 71-109, with the normaliser):
//
//   every CTA     part_r = phi_q(Q)[:, rows of r] S_r        (64 x (d_v+1) partial)
//   cluster barrier
//   CTA r         rows 8r .. 8r+7 of the chunk: sum of the kCluster partials
//                 (read from the other CTAs' shared memory), plus the
//                 intra-chunk term tril(1 + s + s^2/2) [V 1], normalised and
//                 stored;
//   every CTA     S_r += phi_k(K)[:, rows of r]^T [V 1]
//
// The partials are double-buffered by chunk parity, so one cluster barrier
// per chunk orders both their writes and their reads.  With a window W > 0
// (the full BASED layer) CTA r adds, for its rows, the softmax over the keys
// [t - W + 1, t] of the same scores (one warp per row; keys of this chunk from
// shared memory, earlier keys from global memory, where all CTAs of the
// cluster have just read them).  All arithmetic is
// fp32 on CUDA cores, in a fixed order (deterministic).  A segmented run
// seeds each segment from the running sums of the earlier segments' states
// (state pass below, which splits the features over independent CTAs).
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace la {
namespace {

constexpr int kCluster = 8;               // CTAs per (head, segment)
constexpr int kCT = 64;                   // tokens per chunk
constexpr int kThr = 256;
constexpr int kRowsPerRank = kCT / kCluster;  // output rows each CTA finishes
constexpr int kMaxD = 128;
constexpr int kMaxCols = (kMaxD + 1 + 3) / 4;  // value columns per thread (4 lanes per token)
constexpr size_t kSmemLimit = 200 * 1024;
constexpr int64_t kMaxWindow = 129;  // the full BASED layer's window (as the SIMT path)

// One feature of the Taylor basis: phi_k = ka * kb (a factor with index < 0
// is 1), phi_q = wq * qa * qb.
struct FeatDesc {
  short a, b;
  float wq;
};

__host__ __device__ inline FeatDesc feature_desc(int f, int d) {
  FeatDesc fd;
  if (f == 0) {
    fd.a = -1;
    fd.b = -1;
    fd.wq = 1.f;
  } else if (f <= d) {
    fd.a = (short)(f - 1);
    fd.b = -1;
    fd.wq = 1.f / sqrtf((float)d);
  } else {
    int r = f - 1 - d, a = 0;
    while (r >= d - a) {
      r -= d - a;
      ++a;
    }
    fd.a = (short)a;
    fd.b = (short)(a + r);
    fd.wq = fd.a == fd.b ? 1.f / (2.f * d) : 1.f / (float)d;
  }
  return fd;
}

// Shared-memory carve-up (floats unless noted), shared by host and device.
struct ClusterSmem {
  int fr, ldq, ldv;
  size_t off_s, off_q, off_k, off_v, off_part, off_pw, off_tmp, off_desc, bytes;
  __host__ __device__ ClusterSmem(int F, int dqk, int dv, bool output) {
    fr = (F + kCluster - 1) / kCluster;
    ldq = dqk + 1;
    ldv = dv + 1;
    size_t o = 0;
    off_s = o;    o += (size_t)fr * ldv;
    off_q = o;    o += output ? (size_t)kCT * ldq : 0;
    off_k = o;    o += (size_t)kCT * ldq;
    off_v = o;    o += (size_t)kCT * ldv;
    off_part = o; o += output ? (size_t)2 * kCT * ldv : 0;
    off_pw = o;   o += output ? (size_t)kRowsPerRank * kCT : 0;
    off_tmp = o;  o += output ? (size_t)kRowsPerRank * ldv : 0;
    off_desc = o; o += (size_t)fr * 2;  // FeatDesc = 8 bytes = 2 floats
    bytes = o * sizeof(float);
  }
};

template <typename T>
__device__ __forceinline__ void load_rows(float *dst, int ld, const T *src, int64_t t0,
                                          int64_t t_end, int cols, bool ones_col) {
  const int width = cols + (ones_col ? 1 : 0);
  for (int idx = threadIdx.x; idx < kCT * width; idx += kThr) {
    const int r = idx / width, c = idx - r * width;
    const int64_t t = t0 + r;
    float x = 0.f;
    if (t < t_end) x = c < cols ? to_f32(src[t * cols + c]) : 1.f;
    dst[r * ld + c] = x;
  }
}

// S[f][e] += sum_t phi_k(k_t)[f] vaug_t[e] over the CTA's features; work items
// are (feature, block of 17 columns) so every thread has a similar share.
__device__ __forceinline__ void state_update(float *S, const FeatDesc *desc, int nf,
                                             const float *ks, const float *vs, int ldq, int ldv,
                                             int rows) {
  constexpr int kBlk = 17;
  const int nblk = (ldv + kBlk - 1) / kBlk;
  for (int item = threadIdx.x; item < nf * nblk; item += kThr) {
    const int fl = item / nblk, e0 = (item - fl * nblk) * kBlk;
    const FeatDesc fd = desc[fl];
    float acc[kBlk];
#pragma unroll
    for (int i = 0; i < kBlk; ++i) acc[i] = 0.f;
    for (int t = 0; t < rows; ++t) {
      const float ka = fd.a >= 0 ? ks[t * ldq + fd.a] : 1.f;
      const float kb = fd.b >= 0 ? ks[t * ldq + fd.b] : 1.f;
      const float phi = ka * kb;
#pragma unroll
      for (int i = 0; i < kBlk; ++i)
        if (e0 + i < ldv) acc[i] = fmaf(phi, vs[t * ldv + e0 + i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < kBlk; ++i)
      if (e0 + i < ldv) S[fl * ldv + e0 + i] += acc[i];
  }
}

__device__ __forceinline__ void init_desc(FeatDesc *desc, int f0, int nf, int d) {
  for (int i = threadIdx.x; i < nf; i += kThr) desc[i] = feature_desc(f0 + i, d);
}

// ---------------------------------------------------------------------------
// Output pass: grid (kCluster * segments, bh), clusters of kCluster along x.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThr, 1)
cluster_chunked_output_kernel(const T *__restrict__ q, const T *__restrict__ k,
                              const T *__restrict__ v, T *__restrict__ out,
                              const float *__restrict__ init_state,
                              float *__restrict__ final_state,
                              const float *__restrict__ seg_states, int64_t n, int dqk, int dv,
                              float eps, int normalize, int segments, int64_t seg_len,
                              int window) {
  extern __shared__ float smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int F = (int)feature_dim(dqk);
  const ClusterSmem L(F, dqk, dv, true);
  const int ldq = L.ldq, ldv = L.ldv;
  float *S = smem + L.off_s;
  float *qs = smem + L.off_q;
  float *ks = smem + L.off_k;
  float *vs = smem + L.off_v;
  float *part = smem + L.off_part;
  float *pw = smem + L.off_pw;
  float *tmp = smem + L.off_tmp;
  FeatDesc *desc = (FeatDesc *)(smem + L.off_desc);

  const int64_t bh = blockIdx.y;
  const int g = blockIdx.x / kCluster;
  const int f0 = rank * L.fr;
  const int nf = max(0, min(F, f0 + L.fr) - f0);
  const int64_t t_begin = (int64_t)g * seg_len;
  const int64_t t_end = min64(n, t_begin + seg_len);
  const T *qh = q + bh * n * dqk;
  const T *kh = k + bh * n * dqk;
  const T *vh = v + bh * n * dv;
  const int64_t per_head = (int64_t)F * ldv;

  init_desc(desc, f0, nf, dqk);
  // the segment's seed: init_state + the running sum of the earlier segments
  for (int i = threadIdx.x; i < nf * ldv; i += kThr) {
    const int64_t gi = (int64_t)f0 * ldv + i;
    float s = init_state ? init_state[bh * per_head + gi] : 0.f;
    if (g > 0) s += seg_states[(bh * segments + g - 1) * per_head + gi];
    S[i] = s;
  }

  const int tok = threadIdx.x >> 2, lane4 = threadIdx.x & 3;
  const float rsd = 1.f / sqrtf((float)dqk);
  const int n_chunks = (int)((t_end - t_begin + kCT - 1) / kCT);
  for (int c = 0; c < n_chunks; ++c) {
    const int64_t t0 = t_begin + (int64_t)c * kCT;
    const int rows = (int)min64(kCT, t_end - t0);
    const int buf = c & 1;
    __syncthreads();  // the previous chunk's readers of qs / ks / vs are done
    load_rows(qs, ldq, qh, t0, t_end, dqk, false);
    load_rows(ks, ldq, kh, t0, t_end, dqk, false);
    load_rows(vs, ldv, vh, t0, t_end, dv, true);
    __syncthreads();
    // partial inter-chunk term of this CTA's features for all 64 rows
    {
      float acc[kMaxCols];
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) acc[i] = 0.f;
      const float *qr = qs + tok * ldq;
      for (int fl = 0; fl < nf; ++fl) {
        const FeatDesc fd = desc[fl];
        const float qa = fd.a >= 0 ? qr[fd.a] : 1.f;
        const float qb = fd.b >= 0 ? qr[fd.b] : 1.f;
        const float phi = fd.wq * qa * qb;
#pragma unroll
        for (int i = 0; i < kMaxCols; ++i) {
          const int e = lane4 + 4 * i;
          if (e < ldv) acc[i] = fmaf(phi, S[fl * ldv + e], acc[i]);
        }
      }
      float *pr = part + (size_t)(buf * kCT + tok) * ldv;
#pragma unroll
      for (int i = 0; i < kMaxCols; ++i) {
        const int e = lane4 + 4 * i;
        if (e < ldv) pr[e] = acc[i];
      }
    }
    // every CTA's partial for this chunk is complete and visible
    cluster.sync();
    // rows 8 rank .. 8 rank + 7: intra-chunk weights
    const int r0 = rank * kRowsPerRank;
    for (int idx = threadIdx.x; idx < kRowsPerRank * kCT; idx += kThr) {
      const int il = idx / kCT, j = idx - il * kCT, i = r0 + il;
      float s = 0.f;
      for (int a = 0; a < dqk; ++a) s = fmaf(qs[i * ldq + a], ks[j * ldq + a], s);
      s *= rsd;
      const float p = fmaf(s, fmaf(0.5f, s, 1.f), 1.f);
      pw[il * kCT + j] = (j <= i && j < rows) ? p : 0.f;
    }
    __syncthreads();
    // sum of the cluster's partials (fixed rank order) + P [V 1]
    for (int idx = threadIdx.x; idx < kRowsPerRank * ldv; idx += kThr) {
      const int il = idx / ldv, e = idx - il * ldv, i = r0 + il;
      float acc = 0.f;
      for (int src = 0; src < kCluster; ++src) {
        const float *rp = cluster.map_shared_rank(part, src);
        acc += rp[(size_t)(buf * kCT + i) * ldv + e];
      }
      for (int j = 0; j < kCT; ++j) acc = fmaf(pw[il * kCT + j], vs[j * ldv + e], acc);
      tmp[il * ldv + e] = acc;
    }
    __syncthreads();
    if (window > 0) {
      // warp il: row r0 + il; lanes split the q.k dot product and own value
      // columns e = lane + 32 m
      const int il = threadIdx.x >> 5, ln = threadIdx.x & 31, i = r0 + il;
      const int64_t t_row = t0 + i;
      float m = -INFINITY, l = 0.f, sw[kMaxD / 32];
#pragma unroll
      for (int u = 0; u < kMaxD / 32; ++u) sw[u] = 0.f;
      if (i < rows) {
        for (int64_t kk = max64(0, t_row - window + 1); kk <= t_row; ++kk) {
          const bool here = kk >= t0;
          float sp = 0.f;
          for (int a = ln; a < dqk; a += 32) {
            const float kv = here ? ks[(kk - t0) * ldq + a] : to_f32(kh[kk * dqk + a]);
            sp = fmaf(qs[i * ldq + a], kv, sp);
          }
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) sp += __shfl_xor_sync(0xffffffffu, sp, o);
          const float sc = sp * rsd;
          if (sc > m) {
            const float corr = expf(m - sc);  // exp(-inf) = 0 on the first key
            l *= corr;
#pragma unroll
            for (int u = 0; u < kMaxD / 32; ++u) sw[u] *= corr;
            m = sc;
          }
          const float pe = expf(sc - m);
          l += pe;
#pragma unroll
          for (int u = 0; u < kMaxD / 32; ++u) {
            const int e = ln + 32 * u;
            if (e < dv) sw[u] = fmaf(pe, here ? vs[(kk - t0) * ldv + e] : to_f32(vh[kk * dv + e]),
                                     sw[u]);
          }
        }
        const float den = tmp[il * ldv + dv] + eps;
#pragma unroll
        for (int u = 0; u < kMaxD / 32; ++u) {
          const int e = ln + 32 * u;
          if (e < dv)
            out[(bh * n + t0 + i) * dv + e] = from_f32<T>(tmp[il * ldv + e] / den + sw[u] / l);
        }
      }
    } else {
      for (int idx = threadIdx.x; idx < kRowsPerRank * dv; idx += kThr) {
        const int il = idx / dv, e = idx - il * dv, i = r0 + il;
        if (i < rows) {
          const float den = tmp[il * ldv + dv] + eps;
          const float y = normalize ? tmp[il * ldv + e] / den : tmp[il * ldv + e];
          out[(bh * n + t0 + i) * dv + e] = from_f32<T>(y);
        }
      }
    }
    // the state update of this CTA's features (reads ks / vs, writes S)
    state_update(S, desc, nf, ks, vs, ldq, ldv, rows);
  }
  // no CTA leaves while another may still read its partials
  cluster.sync();
  if (final_state && g == segments - 1) {
    __syncthreads();
    for (int i = threadIdx.x; i < nf * ldv; i += kThr)
      final_state[bh * per_head + (int64_t)f0 * ldv + i] = S[i];
  }
}

// ---------------------------------------------------------------------------
// State pass: grid (kCluster * n_launch, bh), no cluster: CTA (r, g) sums the
// features of block r over segment g into seg_states[bh][g] (stride
// `segments` states per head).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThr, 1)
cluster_chunked_state_kernel(const T *__restrict__ k, const T *__restrict__ v,
                             float *__restrict__ seg_states, int64_t n, int dqk, int dv,
                             int segments, int64_t seg_len) {
  extern __shared__ float smem[];
  const int F = (int)feature_dim(dqk);
  const ClusterSmem L(F, dqk, dv, false);
  const int ldq = L.ldq, ldv = L.ldv;
  float *S = smem + L.off_s;
  float *ks = smem + L.off_k;
  float *vs = smem + L.off_v;
  FeatDesc *desc = (FeatDesc *)(smem + L.off_desc);
  const int64_t bh = blockIdx.y;
  const int r = blockIdx.x % kCluster, g = blockIdx.x / kCluster;
  const int f0 = r * L.fr;
  const int nf = max(0, min(F, f0 + L.fr) - f0);
  const int64_t t_begin = (int64_t)g * seg_len;
  const int64_t t_end = min64(n, t_begin + seg_len);
  const T *kh = k + bh * n * dqk;
  const T *vh = v + bh * n * dv;
  init_desc(desc, f0, nf, dqk);
  for (int i = threadIdx.x; i < nf * ldv; i += kThr) S[i] = 0.f;
  for (int64_t t0 = t_begin; t0 < t_end; t0 += kCT) {
    __syncthreads();
    load_rows(ks, ldq, kh, t0, t_end, dqk, false);
    load_rows(vs, ldv, vh, t0, t_end, dv, true);
    __syncthreads();
    state_update(S, desc, nf, ks, vs, ldq, ldv, (int)min64(kCT, t_end - t0));
  }
  __syncthreads();
  float *dst = seg_states + (bh * segments + g) * (int64_t)F * ldv + (int64_t)f0 * ldv;
  for (int i = threadIdx.x; i < nf * ldv; i += kThr) dst[i] = S[i];
}

}  // namespace

bool cluster_chunked_supported(int64_t dqk, int64_t dv) {
  if (dqk < 1 || dqk > kMaxD || dv < 1 || dv > kMaxD) return false;
  return ClusterSmem((int)feature_dim(dqk), (int)dqk, (int)dv, true).bytes <= kSmemLimit;
}

int cluster_chunked_ctas_per_segment() { return kCluster; }

#define LA_CLUSTER_DISPATCH(dtype, T, ...)                  \
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

int launch_chunked_state_cluster(const void *k, const void *v, float *seg_states, int64_t bh,
                                 int64_t n, int dqk, int dv, int dtype, int segments,
                                 int n_launch, int64_t seg_len, cudaStream_t s) {
  if (!cluster_chunked_supported(dqk, dv)) return LA_ERR_UNSUPPORTED;
  const size_t smem = ClusterSmem((int)feature_dim(dqk), dqk, dv, false).bytes;
  const dim3 grid((unsigned)(kCluster * n_launch), (unsigned)bh);
  LA_CLUSTER_DISPATCH(dtype, T, {
    if (allow_dynamic_smem((const void *)cluster_chunked_state_kernel<T>, (int)smem) != LA_OK)
      return LA_ERR_CUDA;
    cluster_chunked_state_kernel<T><<<grid, kThr, smem, s>>>(
        (const T *)k, (const T *)v, seg_states, n, dqk, dv, segments, seg_len);
  });
  return check_launch();
}

int launch_chunked_output_cluster(const void *q, const void *k, const void *v, void *out,
                                  const float *init_state, float *final_state,
                                  const float *seg_states, int64_t bh, int64_t n, int dqk, int dv,
                                  int dtype, float eps, bool normalize, int segments,
                                  int64_t seg_len, int64_t window, cudaStream_t s) {
  if (!cluster_chunked_supported(dqk, dv)) return LA_ERR_UNSUPPORTED;
  if (window < 0 || window > kMaxWindow) return LA_ERR_UNSUPPORTED;
  const size_t smem = ClusterSmem((int)feature_dim(dqk), dqk, dv, true).bytes;
  const dim3 grid((unsigned)(kCluster * segments), (unsigned)bh);
  LA_CLUSTER_DISPATCH(dtype, T, {
    if (allow_dynamic_smem((const void *)cluster_chunked_output_kernel<T>, (int)smem) != LA_OK)
      return LA_ERR_CUDA;
    cluster_chunked_output_kernel<T><<<grid, kThr, smem, s>>>(
        (const T *)q, (const T *)k, (const T *)v, (T *)out, init_state, final_state, seg_states,
        n, dqk, dv, eps, normalize ? 1 : 0, segments, seg_len, (int)window);
  });
  return check_launch();
}

}  // namespace la
