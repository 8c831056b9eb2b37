// Chunked BASED attention at d_qk = 64 (F = 2145 Taylor features) on tcgen05
// tensor cores, the state split over a 16-CTA thread-block cluster.
//
// Fast path: bf16 q/k/v, d_qk = 64, d_v = 64.  One cluster owns one (head,
// segment) and walks its tokens in 128-token tiles.  CTA r of the cluster
// owns features [135 r, 135 r + 135) of the key-side basis of
// include/la_attention.h (160 feature slots, the padding zero) and keeps
// their part of the state, S_r^T (fp32, 128 TMEM lanes = value rows, row 64
// the normaliser), in TMEM for the whole segment.  Per tile c (Q, K, V the
// tile's rows):
//
//   every CTA   phi_r(K) -> smem, phi_r(Q) -> TMEM   (CUDA cores, its slots)
//               O_r    = phi_r(Q) S_r,c          M=128 N=80  K=160 (bf16 snapshot of S_r,c)
//               S_r^T += [V 1 0]^T phi_r(K)       M=128 N=160 K=128
//   CTA 0       scores = Q K^T                    M=128 N=128 K=64
//               P      = tril(1 + s/8 + s^2/128)   (CUDA cores, written over the scores)
//               O_0   += P [V 1]                  M=128 N=80  K=128
//   every CTA   O_r -> shared memory (fp32); cluster barrier
//   CTA r       rows 8r .. 8r+7: sum of the 16 partial rows (read from the other
//               CTAs' shared memory in rank order), / (O[:, 64] + eps); stored
//   cluster barrier (the partials may be overwritten)
//
// which is the reference recurrence of kernels/nki_attention_chunked.py:71-109
// with the normaliser, as in the d_qk = 16 kernel (tc_chunked.cu), whose
// operand layouts this kernel reuses: the sum over the cluster of phi_r(q) .
// phi_r(k) is the full Taylor kernel 1 + s + s^2/2 of s = q.k / 8.
//
// Features.  Slot s of CTA r is feature f = 135 r + s in the documented order
// [1, x_0 .. x_63, x_a x_b (a <= b) row-major]; it is the product of two
// entries of the token's row extended by x_64 = 1 and x_65 = 0 (constant,
// linear and padding slots use those), scaled on the query side by 1/8
// (linear), 1/64 (a < b) or 1/128 (a = b): exact powers of two, so each
// feature is the fp32 product of bf16 inputs rounded once to bf16, as in the
// d_qk = 16 kernel.  The token rows are first copied into a column-major
// bf16 table so that every thread reads its token's entries without bank
// conflicts.
//
// The phases of a tile run one after another (barriers between them); the
// next tile's Q, K, V load by TMA meanwhile.  The state-only variant
// (kStateOnly) runs the phi(K) / update path without a cluster (every CTA
// is independent) and writes its slots of the segment's state.
#include <cooperative_groups.h>

#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

namespace cg = cooperative_groups;

namespace la {
namespace {
using namespace tc;

constexpr int kCl = 16;        // CTAs per cluster
constexpr int kT = 128;        // tokens per tile
constexpr int kDqk = 64;
constexpr int kDv = 64;
constexpr int kF = 2145;       // 1 + 64 + 64 * 65 / 2
constexpr int kFr = 135;       // features per CTA (16 * 135 = 2160 >= 2145)
constexpr int kSlots = 160;    // slots per CTA: five 32-slot blocks
constexpr int kSV = kDv + 1;   // state columns in global memory
constexpr int kNO = 80;        // N of phi(Q) S and P [V 1]
constexpr int kThreads = 256;
constexpr int kRowsPerRank = kT / kCl;  // output rows each CTA finishes
static_assert(kCl * kFr >= kF && kFr <= kSlots && kSlots % 32 == 0, "feature split");

// TMEM columns (one CTA per SM owns all 512)
constexpr uint32_t kColS = 0;       // S^T    128 lanes x 160 fp32
constexpr uint32_t kColO = 160;     // O      128 lanes x 80 fp32
constexpr uint32_t kColPhiQ = 256;  // phi(Q) 128 lanes x 80 bf16 pairs
constexpr uint32_t kColSc = 384;    // scores 128 fp32 / P 64 bf16 pairs (CTA 0)
constexpr uint32_t kTmemCols = 512;

// Shared memory (offsets from a 1024-byte aligned base)
constexpr uint32_t kTileBytes = kT * 128;            // 128 rows x 128 B, 128B-swizzled
constexpr uint32_t kPhiBlock = kT * 64;              // 32 slots of 128 tokens, 64B-swizzled
constexpr uint32_t kPhiBytes = (kSlots / 32) * kPhiBlock;
constexpr uint32_t kSnapKBlock = kNO * 128;          // 64 slots of the 80 snapshot rows
constexpr uint32_t kSnapBytes = 3 * kSnapKBlock;
constexpr int kXRows = kDqk + 2;                     // x_0 .. x_63, 1, 0
constexpr int kStages = 2;

template <bool kStateOnly>
struct Layout64 {
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffK = kOffQ + (kStateOnly ? 0 : kStages * kTileBytes);
  static constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
  static constexpr uint32_t kOffOnes = kOffV + kStages * kTileBytes;  // 16 rows x 128 B
  static constexpr uint32_t kOffPhiK = kOffOnes + 2048;
  static constexpr uint32_t kOffSnap = kOffPhiK + kPhiBytes;
  static constexpr uint32_t kOffX = kOffSnap + (kStateOnly ? 0 : kSnapBytes);
  static constexpr uint32_t kOffPart = kOffX + kXRows * kT * 2;     // fp32 [128][65]
  static constexpr uint32_t kOffDesc = kOffPart + (kStateOnly ? 0 : kT * kSV * 4);
  static constexpr uint32_t kOffBar = kOffDesc + kSlots * 8;
  static constexpr uint32_t kSmemAlloc = kOffBar + 256 + 1024;  // + alignment slack
  static_assert(kOffV % 1024 == 0 && kOffOnes % 1024 == 0 && kOffPhiK % 1024 == 0 &&
                    kOffSnap % 1024 == 0,
                "swizzled regions need 1024-byte alignment");
  static_assert(kOffDesc % 8 == 0 && kOffBar % 8 == 0, "alignment");
  static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");
};

enum Bar64 { kFull = 0, kMma = kFull + kStages, kPv, kNumBars };

// Slot s of CTA `rank`: feature index (or -1), the two factors' rows of the
// extended token row (64 = the constant 1, 65 = zero) and the query-side
// weight.
struct SlotDesc {
  unsigned char a, b;
  short f;
  float wq;
};
__device__ __forceinline__ SlotDesc slot_desc(int rank, int s) {
  SlotDesc d;
  const int f = rank * kFr + s;
  if (s >= kFr || f >= kF) {
    d.a = d.b = kDqk + 1;
    d.f = -1;
    d.wq = 0.f;
  } else if (f == 0) {
    d.a = d.b = kDqk;
    d.f = 0;
    d.wq = 1.f;
  } else if (f <= kDqk) {
    d.a = (unsigned char)(f - 1);
    d.b = kDqk;
    d.f = (short)f;
    d.wq = 0.125f;  // 1 / sqrt(64)
  } else {
    int r = f - 1 - kDqk, a = 0;
    while (r >= kDqk - a) {
      r -= kDqk - a;
      ++a;
    }
    d.a = (unsigned char)a;
    d.b = (unsigned char)(a + r);
    d.f = (short)f;
    d.wq = a == a + r ? 1.f / 128.f : 1.f / 64.f;  // 1/(2d) on the diagonal, 1/d off it
  }
  return d;
}

struct Params64 {
  __nv_bfloat16 *out;
  const float *init_state;  // (bh, F, 65) or null
  float *final_state;       // (bh, F, 65) or null (written by the last segment)
  const float *seg_states;  // (bh, G, F, 65): prefix slots (output pass)
  float *seg_out;           // (bh, G, F, 65): this segment's state (state pass)
  int *err;
  int64_t n;
  int64_t seg_len;
  int segments;
  float eps;
  int normalize;
};

__device__ __forceinline__ bool wait_teardown(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  return true;
}

// Tile rows (128 tokens x 64 bf16, 128B-swizzled) -> the column-major table
// X[a][token] (bf16).  Thread t copies half a row.
__device__ __forceinline__ void stage_rows(uint32_t tile, __nv_bfloat16 *X) {
  const int token = threadIdx.x & (kT - 1), half = threadIdx.x >> 7;
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    uint32_t w[4];
    ld_shared_v4(tile + sw128_offset(token, 4 * half + ch), w[0], w[1], w[2], w[3]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int a = 32 * half + 8 * ch + 2 * i;
      X[a * kT + token] = __ushort_as_bfloat16((unsigned short)(w[i] & 0xFFFFu));
      X[(a + 1) * kT + token] = __ushort_as_bfloat16((unsigned short)(w[i] >> 16));
    }
  }
}

// Eight features (slots s0 .. s0+7) of `token`, each the fp32 product
// X[a] * X[b] * w rounded once to bf16, packed in four bf16x2 words.
__device__ __forceinline__ void features8(const SlotDesc *desc, const __nv_bfloat16 *X, int token,
                                          int s0, bool query, float scale, uint32_t *w) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float p[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const SlotDesc d = desc[s0 + 2 * i + h];
      const float xa = __bfloat162float(X[d.a * kT + token]);
      const float xb = __bfloat162float(X[d.b * kT + token]);
      p[h] = xa * xb * (query ? d.wq : 1.f) * scale;
    }
    w[i] = pack_bf16(p[0], p[1]);
  }
}

template <bool kStateOnly>
__global__ void __launch_bounds__(kThreads, 1)
chunked64_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params64 p) {
  using L = Layout64<kStateOnly>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + L::kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + L::kOffBar + 8 * kNumBars);
  volatile int *abort_flag = (volatile int *)(smem + L::kOffBar + 8 * kNumBars + 4);
  SlotDesc *desc = (SlotDesc *)(smem + L::kOffDesc);
  __nv_bfloat16 *X = (__nv_bfloat16 *)(smem + L::kOffX);
  float *part = (float *)(smem + L::kOffPart);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (kCl * segments, bh); clusters of kCl CTAs along x (output pass)
  const int rank = (int)(blockIdx.x % kCl);
  const int g = (int)(blockIdx.x / kCl);
  const int64_t bh = blockIdx.y;
  const int64_t t_begin = (int64_t)g * p.seg_len;
  const int64_t t_end = min64(p.n, t_begin + p.seg_len);
  const int n_tiles = (int)((t_end - t_begin + kT - 1) / kT);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
    grid_dependents_launch();
  }
  if (threadIdx.x < kSlots) desc[threadIdx.x] = slot_desc(rank, threadIdx.x);
  // the constant rows of the token table: x_64 = 1, x_65 = 0
  for (int i = threadIdx.x; i < 2 * kT; i += kThreads)
    X[kDqk * kT + i] = __float2bfloat16(i < kT ? 1.f : 0.f);
  // constant "ones" block: A-operand rows 64..127 of [V 1 0]^T for 16 tokens
  for (int i = threadIdx.x; i < 2048 / 4; i += kThreads) {
    const int row = (i * 4) / 128, byte = (i * 4) % 128;
    *(uint32_t *)(smem + L::kOffOnes + i * 4) = (byte == (row & 7) * 16) ? 0x3F80u : 0u;
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  cg::cluster_group cluster = cg::this_cluster();

  // inputs may be the previous kernel's output, and out may still be read by it
  grid_dependency_wait();
  const bool producer = threadIdx.x == 0;
  int issued = 0;  // tiles whose loads the producer has issued
  auto issue_loads = [&](int c) {
    ++issued;
    const int st = c % kStages;
    const int row = (int)(t_begin + (int64_t)c * kT);
    mbar_arrive_expect_tx(&bars[kFull + st], (kStateOnly ? 2 : 3) * kTileBytes);
    if (!kStateOnly)
      tma_load_3d(smem + L::kOffQ + st * kTileBytes, &tm_q, &bars[kFull + st], 0, row, (int)bh);
    tma_load_3d(smem + L::kOffK + st * kTileBytes, &tm_k, &bars[kFull + st], 0, row, (int)bh);
    tma_load_3d(smem + L::kOffV + st * kTileBytes, &tm_v, &bars[kFull + st], 0, row, (int)bh);
  };
  if (producer && n_tiles > 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    if (!kStateOnly) prefetch_tmap(&tm_q);
    issue_loads(0);
  }

  // ---- seed: S_0 = init_state + the prefix slot g - 1 (this CTA's slots),
  // into TMEM and (output pass) the bf16 snapshot; snapshot rows 65..79 zero
  const bool state_warp = warp >= 4 && warp < 7;  // lane quarters 0..2: S^T rows 0..95
  const int e = (warp & 3) * 32 + lane;          // S^T row of a state-warp thread
  if (state_warp) {
    const float *head_a =
        !kStateOnly && p.init_state ? p.init_state + (uint64_t)bh * kF * kSV : nullptr;
    const float *head_b =
        !kStateOnly && g > 0 ? p.seg_states + ((uint64_t)bh * p.segments + (g - 1)) * kF * kSV
                             : nullptr;
    for (int f0 = 0; f0 < kSlots; f0 += 16) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int f = desc[f0 + i].f;
        float x = 0.f;
        if (e < kSV && f >= 0) {
          if (head_a) x += head_a[(uint64_t)f * kSV + e];
          if (head_b) x += head_b[(uint64_t)f * kSV + e];
        }
        w[i] = __float_as_uint(x);
      }
      tmem_st16(taddr(tmem, (warp & 3) * 32, kColS + f0), w);
      if (!kStateOnly && e < kNO) {
        const uint32_t blk = sb + L::kOffSnap + (f0 >> 6) * kSnapKBlock;
        const int ch = (f0 & 63) >> 3;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          st_shared_v4(blk + sw128_offset(e, ch + h),
                       pack_bf16(__uint_as_float(w[8 * h + 0]), __uint_as_float(w[8 * h + 1])),
                       pack_bf16(__uint_as_float(w[8 * h + 2]), __uint_as_float(w[8 * h + 3])),
                       pack_bf16(__uint_as_float(w[8 * h + 4]), __uint_as_float(w[8 * h + 5])),
                       pack_bf16(__uint_as_float(w[8 * h + 6]), __uint_as_float(w[8 * h + 7])));
      }
    }
    tmem_wait_st();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  constexpr uint32_t id_qs = make_idesc_bf16(128, kNO, false, false);
  constexpr uint32_t id_pv = make_idesc_bf16(128, kNO, false, true);
  constexpr uint32_t id_up = make_idesc_bf16(128, kSlots, true, true);
  constexpr uint32_t id_sc = make_idesc_bf16(128, 128, false, false);
  // a K-step of 16 tokens of [V 1 0]^T / [V 1]: start +2048 B, LBO (distance to
  // the ones block) -2048 B
  constexpr uint64_t kStep = (uint64_t)(2048 >> 4) - ((uint64_t)(2048 >> 4) << 16);
  const uint32_t a_ones = sb + L::kOffOnes;
  const int token = threadIdx.x & (kT - 1), half = threadIdx.x >> 7;

  for (int c = 0; c < n_tiles; ++c) {
    const int st = c % kStages;
    const int64_t t0 = t_begin + (int64_t)c * kT;
    const int valid = (int)min64(kT, t_end - t0);
    // the next tile loads into the other stage (its last reader, tile c - 1,
    // is done: every phase of a tile ends at a barrier)
    if (producer && c + 1 < n_tiles) issue_loads(c + 1);
    mbar_wait(&bars[kFull + st], (c / kStages) & 1, abort_flag);

    // ---- phi(K) -> smem (64B-swizzled, MN-major B of the update)
    stage_rows(sb + L::kOffK + st * kTileBytes, X);
    __syncthreads();
    {
      const float kscale = token < valid ? 1.f : 0.f;  // padding tokens add nothing
      const uint32_t base = sb + L::kOffPhiK;
      for (int J = 10 * half; J < 10 * half + 10; ++J) {
        uint32_t w[4];
        features8(desc, X, token, 8 * J, false, kscale, w);
        st_shared_v4(base + (J >> 2) * kPhiBlock + sw64_offset(token, J & 3), w[0], w[1], w[2],
                     w[3]);
      }
    }
    __syncthreads();
    if (!kStateOnly) {
      // ---- phi(Q) -> TMEM (lane = token; warps w and w + 4 share a quarter)
      stage_rows(sb + L::kOffQ + st * kTileBytes, X);
      __syncthreads();
      const uint32_t qaddr = taddr(tmem, (warp & 3) * 32, kColPhiQ + 40 * half);
#pragma unroll 1
      for (int G = 0; G < 5; ++G) {  // 8 columns (16 slots) per store
        uint32_t w[8];
        features8(desc, X, token, 80 * half + 16 * G, true, 1.f, w);
        features8(desc, X, token, 80 * half + 16 * G + 8, true, 1.f, w + 4);
        tmem_st8(qaddr + 8 * G, w);
      }
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // ---- MMAs (warp 0): O_r = phi(Q) S_c; S^T += [V 1 0]^T phi(K); CTA 0: scores
    if (warp == 0) {
      const uint32_t v_base = sb + L::kOffV + st * kTileBytes;
      if (elect_one()) {
        if (!kStateOnly) {
          const uint64_t qs_b = make_sdesc(sb + L::kOffSnap, 16, 1024, kSwizzle128B);
#pragma unroll
          for (int j = 0; j < kSlots / 16; ++j) {
            const uint32_t boff = (j >> 2) * kSnapKBlock + (j & 3) * 32;
            umma_ts(tmem + kColO, tmem + kColPhiQ + 8 * j, qs_b + (boff >> 4), id_qs,
                    j > 0 ? 1u : 0u);
          }
        }
        const uint64_t db0 = make_sdesc(sb + L::kOffPhiK, kPhiBlock, 512, kSwizzle64B);
        const uint64_t da0 = make_sdesc(v_base, a_ones - v_base, 1024, kSwizzle128B);
#pragma unroll
        for (int j = 0; j < kT / 16; ++j)
          umma_ss(tmem + kColS, da0 + kStep * j, db0 + (uint64_t)((j * 1024) >> 4), id_up, 1u);
        if (!kStateOnly && rank == 0) {
          const uint64_t qd = make_sdesc(sb + L::kOffQ + st * kTileBytes, 16, 1024, kSwizzle128B);
          const uint64_t kd = make_sdesc(sb + L::kOffK + st * kTileBytes, 16, 1024, kSwizzle128B);
#pragma unroll
          for (int kk = 0; kk < kDqk / 16; ++kk)
            umma_ss(tmem + kColSc, qd + 2 * kk, kd + 2 * kk, id_sc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[kMma]);
      }
      __syncwarp();
    }
    mbar_wait(&bars[kMma], c & 1, abort_flag);
    tc_fence_after();

    if (!kStateOnly && rank == 0) {
      // ---- intra-tile term (CTA 0): P = tril(1 + s/8 + s^2/128) over the
      // tile's keys, then O_0 += P [V 1]
      if (warp < 4) {
        const int row = warp * 32 + lane;
        const uint32_t srow = taddr(tmem, warp * 32, kColSc);
        const int m = min(row, valid - 1);  // keys 0 .. m are visible to this row
        const uint64_t c128 = f2pack(1.f / 128.f, 1.f / 128.f), c8 = f2pack(0.125f, 0.125f);
        const uint64_t one2 = f2pack(1.f, 1.f);
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {  // keys 64 hh .. 64 hh + 63
          uint32_t r[64], w[32];
          tmem_ld16(srow + 64 * hh, r);
          tmem_ld16(srow + 64 * hh + 16, r + 16);
          tmem_ld16(srow + 64 * hh + 32, r + 32);
          tmem_ld16(srow + 64 * hh + 48, r + 48);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int j0 = 64 * hh + 2 * i;
            float p0, p1;
            const uint64_t s2 = f2pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            f2unpack(ffma2(s2, ffma2(s2, c128, c8), one2), p0, p1);
            w[i] = pack_bf16(j0 <= m ? p0 : 0.f, j0 + 1 <= m ? p1 : 0.f);
          }
          // P columns 32 hh .. 32 hh + 31 (keys 64 hh ..): score columns this
          // thread has already read
          tmem_st16(srow + 32 * hh, w);
          tmem_st16(srow + 32 * hh + 16, w + 16);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (warp == 0) {
        const uint32_t v_base = sb + L::kOffV + st * kTileBytes;
        const uint64_t db0 = make_sdesc(v_base, a_ones - v_base, 1024, kSwizzle128B);
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < kT / 16; ++j)
            umma_ts(tmem + kColO, tmem + kColSc + 8 * j, db0 + kStep * j, id_pv, 1u);
          umma_commit(&bars[kPv]);
        }
        __syncwarp();
      }
      mbar_wait(&bars[kPv], c & 1, abort_flag);
      tc_fence_after();
    }

    if (!kStateOnly) {
      // ---- O_r -> shared memory (warps 0..3, lane = row); S_{c+1} -> bf16
      // snapshot (warps 4..6, lane = S^T row)
      if (warp < 4) {
        const int row = warp * 32 + lane;
        const uint32_t obase = taddr(tmem, warp * 32, kColO);
        float *dst = part + row * kSV;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint32_t o[16];
          tmem_ld16(obase + 16 * q4, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[16 * q4 + i] = __uint_as_float(o[i]);
        }
        dst[kDv] = __uint_as_float(tmem_ld1(obase + kDv));
        tmem_wait_ld();
      } else if (state_warp && c + 1 < n_tiles) {
        const uint32_t base = taddr(tmem, (warp & 3) * 32, kColS);
        for (int f0 = 0; f0 < kSlots; f0 += 16) {
          uint32_t r[16];
          tmem_ld16(base + f0, r);
          tmem_wait_ld();
          if (e <= kDv) {
            const uint32_t blk = sb + L::kOffSnap + (f0 >> 6) * kSnapKBlock;
            const int ch = (f0 & 63) >> 3;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              st_shared_v4(blk + sw128_offset(e, ch + h),
                           pack_bf16(__uint_as_float(r[8 * h + 0]), __uint_as_float(r[8 * h + 1])),
                           pack_bf16(__uint_as_float(r[8 * h + 2]), __uint_as_float(r[8 * h + 3])),
                           pack_bf16(__uint_as_float(r[8 * h + 4]), __uint_as_float(r[8 * h + 5])),
                           pack_bf16(__uint_as_float(r[8 * h + 6]), __uint_as_float(r[8 * h + 7])));
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      // every CTA's partials of this tile are in its shared memory
      cluster.sync();
      tc_fence_after();
      // ---- rows 8 rank .. 8 rank + 7: warp w sums row 8 rank + w over the
      // cluster (rank order), lane l owns values l and l + 32
      {
        const int row = rank * kRowsPerRank + warp;
        float a0 = 0.f, a1 = 0.f, den = 0.f;
#pragma unroll 4
        for (int src = 0; src < kCl; ++src) {
          const float *rp = cluster.map_shared_rank(part, src) + row * kSV;
          a0 += rp[lane];
          a1 += rp[lane + 32];
          if (lane == 0) den += rp[kDv];
        }
        den = __shfl_sync(0xffffffffu, den, 0);
        const float inv = p.normalize ? 1.f / (den + p.eps) : 1.f;
        if (row < valid) {
          __nv_bfloat16 *o = p.out + ((uint64_t)bh * p.n + t0 + row) * kDv;
          o[lane] = __float2bfloat16_rn(a0 * inv);
          o[lane + 32] = __float2bfloat16_rn(a1 * inv);
        }
      }
      // no CTA overwrites its partials while another may still read them
      cluster.sync();
    }
  }

  // ---- the state after the segment: final state (output pass, last
  // segment) or this segment's state (state pass), this CTA's slots
  float *dst = nullptr;
  if (kStateOnly) dst = p.seg_out + ((uint64_t)bh * p.segments + g) * kF * kSV;
  else if (p.final_state != nullptr && g == p.segments - 1)
    dst = p.final_state + (uint64_t)bh * kF * kSV;
  if (dst && state_warp) {
    for (int f0 = 0; f0 < kSlots; f0 += 16) {
      uint32_t r[16];
      tmem_ld16(taddr(tmem, (warp & 3) * 32, kColS + f0), r);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int f = desc[f0 + i].f;
        if (e < kSV && f >= 0) dst[(uint64_t)f * kSV + e] = __uint_as_float(r[i]);
      }
    }
  }

  // ---- teardown: every issued copy has landed (each tile's loads were
  // waited for in its iteration, unless a wait gave up)
  if (producer) {
    for (int c = issued - kStages < 0 ? 0 : issued - kStages; c < issued; ++c)
      wait_teardown(&bars[kFull + c % kStages], (c / kStages) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
}

template <bool kStateOnly>
int launch64(const void *q, const void *k, const void *v, const Params64 &p, int64_t bh,
             int n_launch, cudaStream_t s) {
  if (bh > 65535 || p.n > INT32_MAX) return LA_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_3d(&mk, k, bh, p.n, kDqk, kT, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&mv, v, bh, p.n, kDv, kT, CU_TENSOR_MAP_SWIZZLE_128B))
    return LA_ERR_CUDA;
  if (kStateOnly) {
    mq = mk;
  } else if (!make_tmap_3d(&mq, q, bh, p.n, kDqk, kT, CU_TENSOR_MAP_SWIZZLE_128B)) {
    return LA_ERR_CUDA;
  }
  constexpr uint32_t kSmem = Layout64<kStateOnly>::kSmemAlloc;
  const void *fn = (const void *)chunked64_tc_kernel<kStateOnly>;
  if (allow_dynamic_smem(fn, (int)kSmem) != LA_OK) return LA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(kCl * n_launch), (unsigned)bh);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kStateOnly ? 1 : kCl;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cudaLaunchKernelEx(&cfg, chunked64_tc_kernel<kStateOnly>, mq, mk, mv, p) != cudaSuccess) {
    note_launch();
    cudaGetLastError();
    return LA_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace

bool chunked64_tc_available() {
  // 16-CTA clusters are a non-portable size: the attribute is set once per
  // context and the device must be able to hold at least one such cluster
  static thread_local int cached_device = -1;
  static thread_local bool cached = false;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (dev == cached_device) return cached;
  bool ok = false;
  const void *fn = (const void *)chunked64_tc_kernel<false>;
  constexpr uint32_t kSmem = Layout64<false>::kSmemAlloc;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
      allow_dynamic_smem(fn, (int)kSmem) == LA_OK) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCl, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    ok = cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) == cudaSuccess && clusters > 0;
  }
  cudaGetLastError();
  cached_device = dev;
  cached = ok;
  return ok;
}

int chunked64_tc_ctas_per_segment() { return kCl; }

int launch_chunked64_state_tc(const void *k, const void *v, float *seg_states, int64_t bh,
                              int64_t n, int segments, int n_launch, int64_t seg_len,
                              cudaStream_t s) {
  Params64 p{};
  p.seg_out = seg_states;
  p.err = device_error_word();
  p.n = n;
  p.seg_len = seg_len;
  p.segments = segments;
  if (!p.err) return LA_ERR_CUDA;
  return launch64<true>(nullptr, k, v, p, bh, n_launch, s);
}

int launch_chunked64_output_tc(const void *q, const void *k, const void *v, void *out,
                               const float *init_state, float *final_state,
                               const float *seg_states, int64_t bh, int64_t n, float eps,
                               bool normalize, int segments, int64_t seg_len, cudaStream_t s) {
  Params64 p{};
  p.out = (__nv_bfloat16 *)out;
  p.init_state = init_state;
  p.final_state = final_state;
  p.seg_states = seg_states;
  p.err = device_error_word();
  p.n = n;
  p.seg_len = seg_len;
  p.segments = segments;
  p.eps = eps;
  p.normalize = normalize ? 1 : 0;
  if (!p.err) return LA_ERR_CUDA;
  return launch64<false>(q, k, v, p, bh, segments, s);
}

}  // namespace la
