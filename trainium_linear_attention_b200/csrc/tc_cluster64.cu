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
//   CTA r < 8   the intra-tile term of keys 16r .. 16r+15:
//               scores = Q K_r^T                  M=128 N=16  K=64
//               P      = tril(1 + s/8 + s^2/128)   (CUDA cores, over the scores)
//               O_r   += P [V_r 1]                M=128 N=80  K=16
//   every CTA   O_r -> own shared memory; rows 8o .. 8o+7 -> CTA o (one bulk
//               copy per CTA, completing on CTA o's mbarrier)
//   CTA r       rows 8r .. 8r+7: sum of the 16 partial rows in rank order,
//               / (O[:, 64] + eps); stored
//
// which is the reference recurrence of kernels/nki_attention_chunked.py:71-109
// with the normaliser, as in the d_qk = 16 kernel (tc_chunked.cu), whose
// operand layouts this kernel reuses: summed over the cluster, phi_r(q) .
// phi_r(k) is the full Taylor kernel 1 + s + s^2/2 of s = q.k / 8, and the
// intra-tile partials sum to tril(P) [V 1].  An owner waits for its 16
// incoming blocks on its own mbarrier (bytes counted by the copies); a
// cluster barrier split into its two halves -- arrive after the owner sums,
// wait before the next tile's partials are staged -- keeps the staging and
// receiving buffers from being rewritten while a copy or an owner may still
// read them.
//
// Features.  Slot s of CTA r is feature f = 135 r + s in the documented order
// [1, x_0 .. x_63, x_a x_b (a <= b) row-major].  Four threads share a token;
// each holds the token's 64 (q_a, k_a) pairs in registers as bf16x2 words
// (plus u = (1, 1) for a token in the sequence, (1, 0) past its end) and
// computes a fixed quarter of the CTA's slots with code generated for that
// (CTA rank, quarter) from the compile-time slot list: one bf16x2 multiply
// x_a * x_b (or x_a * u, u * u) makes the query and the key feature, each the
// fp32 product of bf16 inputs rounded once to bf16; the query side is then
// scaled by 1/8 (linear), 1/64 (a < b) or 1/128 (a = b), exact powers of
// two, as in the d_qk = 16 kernel.
//
// The phases of a tile run one after another (barriers between them), with
// the owners' sums of tile c done during tile c + 1, while its MMAs run, so
// the partials' copies fly under the next tile's features; the next tile's
// Q, K, V load by TMA from the end of this tile's MMAs.  The
// state-only variant (kStateOnly) runs the phi(K) / update path without a
// cluster (every CTA is independent) and writes its slots of the segment's
// state.
#include <mutex>
#include <utility>

#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

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
constexpr int kThreads = 512;
constexpr int kRowsPerRank = kT / kCl;  // output rows each CTA finishes (8)
constexpr int kIntraRanks = 8;          // CTAs that take 16 keys of the intra-tile term
constexpr int kRecvLd = 68;             // floats per received partial row (65 + pad, 16 B)
static_assert(kCl * kFr >= kF && kFr <= kSlots && kSlots % 32 == 0, "feature split");
static_assert(kIntraRanks * 16 == kT && kIntraRanks <= kCl, "intra-tile split");

// TMEM columns (one CTA per SM owns all 512)
constexpr uint32_t kColS = 0;       // S^T    128 lanes x 160 fp32
constexpr uint32_t kColO = 160;     // O      128 lanes x 80 fp32
constexpr uint32_t kColPhiQ = 256;  // phi(Q) 128 lanes x 80 bf16 pairs
constexpr uint32_t kColSc = 384;    // scores 16 fp32 / P 8 bf16 pairs (CTAs r < 8)
constexpr uint32_t kTmemCols = 512;

// Shared memory (offsets from a 1024-byte aligned base)
constexpr uint32_t kTileBytes = kT * 128;            // 128 rows x 128 B, 128B-swizzled
constexpr uint32_t kPhiBlock = kT * 64;              // 32 slots of 128 tokens, 64B-swizzled
constexpr uint32_t kPhiBytes = (kSlots / 32) * kPhiBlock;
constexpr uint32_t kSnapKBlock = kNO * 128;          // 64 slots of the 80 snapshot rows
constexpr uint32_t kSnapBytes = 3 * kSnapKBlock;
constexpr uint32_t kRecvBytes = kCl * kRowsPerRank * kRecvLd * 4;  // one tile's partials
constexpr uint32_t kBlockBytes = kRowsPerRank * kRecvLd * 4;       // rows of one owner (2176 B)
static_assert(kBlockBytes % 16 == 0, "bulk copies move multiples of 16 bytes");

// The output pass holds one tile of Q, K and V (the next tile loads during
// the partial-sum exchange); the state pass keeps three tiles of K and V in
// flight (and so needs more than half the SM's shared memory: it runs alone
// on its SM, whose 512 TMEM columns it allocates).
template <bool kStateOnly>
struct Layout64 {
  static constexpr int kStages = kStateOnly ? 3 : 1;
  static constexpr uint32_t kStageBytes = (kStateOnly ? 2 : 3) * kTileBytes;
  static constexpr uint32_t kOffQ = 0;                               // stage: [Q] K V
  static constexpr uint32_t kOffK = kStateOnly ? 0 : kTileBytes;
  static constexpr uint32_t kOffV = kOffK + kTileBytes;
  static constexpr uint32_t kOffOnes = kStages * kStageBytes;         // 16 rows x 128 B
  static constexpr uint32_t kOffPhiK = kOffOnes + 2048;
  static constexpr uint32_t kOffSnap = kOffPhiK + kPhiBytes;
  static constexpr uint32_t kOffRecv = kOffSnap + (kStateOnly ? 0 : kSnapBytes);  // [src][8][68]
  static constexpr uint32_t kOffStage = kOffRecv + (kStateOnly ? 0 : kRecvBytes);  // [128][68]
  static constexpr uint32_t kOffDesc = kOffStage + (kStateOnly ? 0 : kRecvBytes);
  static constexpr uint32_t kOffBar = kOffDesc + kSlots * 8;
  static constexpr uint32_t kSmemAlloc = kOffBar + 64 + 1024;  // + alignment slack
  static_assert(kStageBytes % 1024 == 0 && kOffOnes % 1024 == 0 && kOffPhiK % 1024 == 0 &&
                    kOffSnap % 1024 == 0,
                "swizzled regions need 1024-byte alignment");
  static_assert(kOffRecv % 16 == 0 && kOffDesc % 8 == 0 && kOffBar % 8 == 0, "alignment");
  static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");
  static_assert(kSmemAlloc > 114 * 1024, "one CTA per SM");
};

constexpr int kMaxStages64 = 3;
enum Bar64 { kFull0 = 0, kMma = kFull0 + kMaxStages64, kPv, kRecv, kNumBars };

// Optional phase timeline (clock64 per tile) of thread 0 of every CTA of
// cluster (0, 0), compiled in with -DLA_TRACE only.
#ifdef LA_TRACE
constexpr int kTrTiles = 32, kTrEvents = 10;
__device__ long long la_trace64[kCl][kTrTiles][kTrEvents];
#define LA_TRACE64(tile, ev)                                                            \
  do {                                                                                 \
    if (blockIdx.y == 0 && blockIdx.x < kCl && threadIdx.x == 0 && (tile) < kTrTiles) \
      la_trace64[blockIdx.x][tile][ev] = clock64();                                    \
  } while (0)
#else
#define LA_TRACE64(tile, ev) \
  do {                       \
  } while (0)
#endif

// Slot s of CTA `rank`: its feature (or -1), the rows a, b of the token table
// whose product it is, and the bf16x2 weight (query-side scale, 1).
struct SlotDesc {
  unsigned char a, b;
  short f;
  uint32_t w;
};
__device__ __forceinline__ SlotDesc slot_desc(int rank, int s) {
  SlotDesc d;
  const int f = rank * kFr + s;
  uint32_t wq;  // bf16 bits of the query-side scale: exact powers of two
  if (s >= kFr || f >= kF) {
    d.a = d.b = kDqk + 1;
    d.f = -1;
    wq = 0u;
  } else if (f == 0) {
    d.a = d.b = kDqk;
    d.f = 0;
    wq = 0x3F80u;  // 1
  } else if (f <= kDqk) {
    d.a = (unsigned char)(f - 1);
    d.b = kDqk;
    d.f = (short)f;
    wq = 0x3E00u;  // 1/8 = 1/sqrt(64)
  } else {
    int r = f - 1 - kDqk, a = 0;
    while (r >= kDqk - a) {
      r -= kDqk - a;
      ++a;
    }
    d.a = (unsigned char)a;
    d.b = (unsigned char)(a + r);
    d.f = (short)f;
    wq = r == 0 ? 0x3C00u : 0x3C80u;  // 1/128 = 1/(2d) on the diagonal, 1/64 = 1/d off it
  }
  d.w = wq | (0x3F80u << 16);
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

// Shared-memory address of `saddr` in the CTA of the cluster with rank `rank`.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// The two halves of the cluster barrier (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Bulk copy of `bytes` from this CTA's shared memory to another CTA's (both
// addresses 16-byte aligned, `dst` and `mbar` shared::cluster addresses in
// the destination CTA); the destination's mbarrier counts the bytes.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, uint32_t src, uint32_t bytes,
                                                  uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst), "r"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

// Slot s of CTA `rank` at compile time: the rows a, b of the token's (q, k)
// pairs whose product it is (64 = u, a < 0: padding) and the bf16 bits of
// the query-side scale.
struct SlotAB {
  int a, b;
  uint32_t wq;
};
__host__ __device__ constexpr SlotAB slot_ab(int rank, int s) {
  const int f = rank * kFr + s;
  if (s >= kFr || f >= kF) return {-1, -1, 0u};
  if (f == 0) return {kDqk, kDqk, 0x3F80u};        // 1
  if (f <= kDqk) return {f - 1, kDqk, 0x3E00u};    // x_a / 8
  int r = f - 1 - kDqk, a = 0;
  while (r >= kDqk - a) {
    r -= kDqk - a;
    ++a;
  }
  return {a, a + r, r == 0 ? 0x3C00u : 0x3C80u};  // x_a^2 / 128, x_a x_b / 64
}
__host__ __device__ constexpr bool slot_ab_matches_desc() {
  // the compile-time list and the run-time table name the same features
  for (int r = 0; r < kCl; ++r)
    for (int s = 0; s < kSlots; ++s) {
      const SlotAB d = slot_ab(r, s);
      const int f = r * kFr + s;
      if ((d.a < 0) != (s >= kFr || f >= kF)) return false;
    }
  return true;
}
static_assert(slot_ab_matches_desc(), "slot lists");

// The quarter P of a CTA's slots one thread computes: [0, 32), [32, 80),
// [80, 128), [128, 160) (phi(Q) TMEM stores of 8 columns stay 8-aligned).
__host__ __device__ constexpr int part_lo(int P) { return P == 0 ? 0 : P == 1 ? 32 : P == 2 ? 80 : 128; }
__host__ __device__ constexpr int part_chunks(int P) { return P == 0 || P == 3 ? 2 : 3; }

template <int R, int S>
__device__ __forceinline__ uint32_t qk_feature(const uint32_t *x, uint32_t u) {
  constexpr SlotAB d = slot_ab(R, S);
  if constexpr (d.a < 0) {
    return 0u;
  } else {
    uint32_t xa, xb;
    if constexpr (d.a == kDqk) xa = u; else xa = x[d.a];
    if constexpr (d.b == kDqk) xb = u; else xb = x[d.b];
    const uint32_t p = hmul2_bf16(xa, xb);
    if constexpr (d.wq == 0x3F80u) return p;
    else return hmul2_bf16(p, d.wq | (0x3F80u << 16));
  }
}

// Slots S0 .. S0+15 of the thread's token: phi(K) -> smem (two 16-byte
// chunks of the 64B-swizzled MN-major layout), phi(Q) -> 8 TMEM columns.
template <bool kStateOnly, int R, int S0, int... I>
__device__ __forceinline__ void feature_chunk(const uint32_t *x, uint32_t u, uint32_t phik,
                                              uint32_t qaddr, int token,
                                              std::integer_sequence<int, I...>) {
  const uint32_t pq[16] = {qk_feature<R, S0 + I>(x, u)...};
  uint32_t qf[8], kf[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    qf[j] = bf16_pair<0, 0>(pq[2 * j], pq[2 * j + 1]);
    kf[j] = bf16_pair<1, 1>(pq[2 * j], pq[2 * j + 1]);
  }
  st_shared_v4(phik + (S0 >> 5) * kPhiBlock + sw64_offset(token, (S0 & 31) >> 3), kf[0], kf[1],
               kf[2], kf[3]);
  st_shared_v4(phik + ((S0 + 8) >> 5) * kPhiBlock + sw64_offset(token, ((S0 + 8) & 31) >> 3),
               kf[4], kf[5], kf[6], kf[7]);
  if (!kStateOnly) tmem_st8(qaddr + S0 / 2, qf);
}
template <bool kStateOnly, int R, int P, int... C>
__device__ __forceinline__ void part_features(const uint32_t *x, uint32_t u, uint32_t phik,
                                              uint32_t qaddr, int token,
                                              std::integer_sequence<int, C...>) {
  (feature_chunk<kStateOnly, R, part_lo(P) + 16 * C>(x, u, phik, qaddr, token,
                                                     std::make_integer_sequence<int, 16>{}),
   ...);
}
// The code for (rank, quarter) = (idx / 4, idx % 4).
template <bool kStateOnly, int... I>
__device__ __forceinline__ void features_for(int idx, const uint32_t *x, uint32_t u,
                                             uint32_t phik, uint32_t qaddr, int token,
                                             std::integer_sequence<int, I...>) {
  ((idx == I ? part_features<kStateOnly, I / 4, I % 4>(
                   x, u, phik, qaddr, token, std::make_integer_sequence<int, part_chunks(I % 4)>{})
             : void()),
   ...);
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
  const float *recv = (const float *)(smem + L::kOffRecv);

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

  // inputs may be the previous kernel's output, and out may still be read by it
  grid_dependency_wait();
  const bool producer = threadIdx.x == 0;
  int issued = 0;  // tiles whose loads the producer has issued
  auto issue_loads = [&](int c) {
    ++issued;
    const int st = c % L::kStages;
    uint8_t *base = smem + st * L::kStageBytes;
    const int row = (int)(t_begin + (int64_t)c * kT);
    mbar_arrive_expect_tx(&bars[kFull0 + st], L::kStageBytes);
    if (!kStateOnly) tma_load_3d(base + L::kOffQ, &tm_q, &bars[kFull0 + st], 0, row, (int)bh);
    tma_load_3d(base + L::kOffK, &tm_k, &bars[kFull0 + st], 0, row, (int)bh);
    tma_load_3d(base + L::kOffV, &tm_v, &bars[kFull0 + st], 0, row, (int)bh);
  };
  if (producer && n_tiles > 0) {
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    if (!kStateOnly) prefetch_tmap(&tm_q);
    for (int c = 0; c < L::kStages && c < n_tiles; ++c) issue_loads(c);
  }

  // State warps: lane quarters 0..2 (S^T rows 0..95), two column halves:
  // warps 4..6 columns 0..79, warps 8..10 columns 80..159.
  const bool state_warp = (warp >= 4 && warp < 7) || (warp >= 8 && warp < 11);
  const int e = (warp & 3) * 32 + lane;  // S^T row of a state-warp thread
  const int col0 = warp >= 8 ? 80 : 0;

  // ---- seed: S_0 = init_state + the prefix slot g - 1 (this CTA's slots),
  // into TMEM and (output pass) the bf16 snapshot; snapshot rows 65..79 zero
  if (state_warp) {
    const float *head_a =
        !kStateOnly && p.init_state ? p.init_state + (uint64_t)bh * kF * kSV : nullptr;
    const float *head_b =
        !kStateOnly && g > 0 ? p.seg_states + ((uint64_t)bh * p.segments + (g - 1)) * kF * kSV
                             : nullptr;
    for (int f0 = col0; f0 < col0 + 80; f0 += 16) {
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
  constexpr uint32_t id_sc = make_idesc_bf16(128, 16, false, false);
  // a K-step of 16 tokens of [V 1 0]^T / [V 1]: start +2048 B, LBO (distance to
  // the ones block) -2048 B
  constexpr uint64_t kStep = (uint64_t)(2048 >> 4) - ((uint64_t)(2048 >> 4) << 16);
  const uint32_t a_ones = sb + L::kOffOnes;
  const int token = threadIdx.x & (kT - 1), part = threadIdx.x >> 7;  // quarter of the slots
  const bool intra = !kStateOnly && rank < kIntraRanks;

  // Rows 8 rank .. 8 rank + 7 of tile cr, once its 16 blocks have landed:
  // warp w sums values 32 (w & 1) + lane of row 8 rank + w / 2 over the
  // partials in rank order, normalises and stores; then this CTA arrives on
  // the cluster barrier (its receiving buffer may be refilled).
  auto reduce_tile = [&](int cr) {
    mbar_wait(&bars[kRecv], cr & 1, abort_flag);
    const int64_t t0r = t_begin + (int64_t)cr * kT;
    const int r8 = warp >> 1, row = rank * kRowsPerRank + r8;
    const int ev = 32 * (warp & 1) + lane;
    const float *rb = recv + r8 * kRecvLd;
    float acc = 0.f, den = 0.f;
#pragma unroll
    for (int src = 0; src < kCl; ++src) {
      acc += rb[src * kRowsPerRank * kRecvLd + ev];
      den += rb[src * kRowsPerRank * kRecvLd + kDv];
    }
    const float inv = p.normalize ? 1.f / (den + p.eps) : 1.f;
    if (row < min64(kT, t_end - t0r))
      p.out[((uint64_t)bh * p.n + t0r + row) * kDv + ev] = __float2bfloat16_rn(acc * inv);
    cluster_arrive();
  };

  for (int c = 0; c < n_tiles; ++c) {
    const int st = c % L::kStages;
    const uint32_t stage = sb + st * L::kStageBytes;
    const int64_t t0 = t_begin + (int64_t)c * kT;
    const int valid = (int)min64(kT, t_end - t0);
    LA_TRACE64(c, 0);
    mbar_wait(&bars[kFull0 + st], (c / L::kStages) & 1, abort_flag);
    LA_TRACE64(c, 1);

    // ---- features: phi_r(K) -> smem (MN-major B of the update), phi_r(Q) -> TMEM
    {
      uint32_t x[kDqk];
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t qw[4] = {0u, 0u, 0u, 0u}, kw[4];
        if (!kStateOnly)
          ld_shared_v4(stage + L::kOffQ + sw128_offset(token, ch), qw[0], qw[1], qw[2], qw[3]);
        ld_shared_v4(stage + L::kOffK + sw128_offset(token, ch), kw[0], kw[1], kw[2], kw[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[8 * ch + 2 * i] = bf16_pair<0, 0>(qw[i], kw[i]);
          x[8 * ch + 2 * i + 1] = bf16_pair<1, 1>(qw[i], kw[i]);
        }
      }
      const uint32_t u = token < valid ? 0x3F803F80u : 0x00003F80u;
      LA_TRACE64(c, 2);
      features_for<kStateOnly>(rank * 4 + part, x, u, sb + L::kOffPhiK,
                               taddr(tmem, (warp & 3) * 32, kColPhiQ), token,
                               std::make_integer_sequence<int, 4 * kCl>{});
      if (!kStateOnly) tmem_wait_st();
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    LA_TRACE64(c, 3);

    // ---- MMAs (warp 0): O_r = phi(Q) S_c; S^T += [V 1 0]^T phi(K); CTAs r < 8:
    // scores of keys 16r .. 16r+15
    const uint32_t v_base = stage + L::kOffV;
    if (warp == 0) {
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
        if (intra) {
          // keys 16r .. 16r+15 are rows 16r.. of the K tile: 8-row groups 2r, 2r+1
          const uint64_t qd = make_sdesc(stage + L::kOffQ, 16, 1024, kSwizzle128B);
          const uint64_t kd = make_sdesc(stage + L::kOffK + rank * 2048, 16, 1024, kSwizzle128B);
#pragma unroll
          for (int kk = 0; kk < kDqk / 16; ++kk)
            umma_ss(tmem + kColSc, qd + 2 * kk, kd + 2 * kk, id_sc, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[kMma]);
      }
      __syncwarp();
    }
    // the previous tile's rows, while this tile's MMAs run (its partials
    // have been in flight since the end of the previous tile)
    if (!kStateOnly && c > 0) reduce_tile(c - 1);
    LA_TRACE64(c, 4);
    mbar_wait(&bars[kMma], c & 1, abort_flag);
    tc_fence_after();
    LA_TRACE64(c, 5);

    if (intra) {
      // ---- P = tril(1 + s/8 + s^2/128) for keys 16r .. 16r+15, then
      // O_r += P [V_r 1] (one K-step: V rows 16r ..)
      if (warp < 4) {
        const int row = warp * 32 + lane;
        const uint32_t srow = taddr(tmem, warp * 32, kColSc);
        const int m = min(row, valid - 1) - 16 * rank;  // keys 16r .. 16r+m are visible
        const uint64_t c128 = f2pack(1.f / 128.f, 1.f / 128.f), c8 = f2pack(0.125f, 0.125f);
        const uint64_t one2 = f2pack(1.f, 1.f);
        uint32_t r[16], w[8];
        tmem_ld16(srow, r);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float p0, p1;
          const uint64_t s2 = f2pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          f2unpack(ffma2(s2, ffma2(s2, c128, c8), one2), p0, p1);
          w[i] = pack_bf16(2 * i <= m ? p0 : 0.f, 2 * i + 1 <= m ? p1 : 0.f);
        }
        tmem_st8(srow, w);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (warp == 0) {
        const uint64_t db0 = make_sdesc(v_base, a_ones - v_base, 1024, kSwizzle128B);
        if (elect_one()) {
          umma_ts(tmem + kColO, tmem + kColSc, db0 + kStep * rank, id_pv, 1u);
          umma_commit(&bars[kPv]);
        }
        __syncwarp();
      }
      mbar_wait(&bars[kPv], c & 1, abort_flag);
      tc_fence_after();
    }
    LA_TRACE64(c, 6);
    // this tile's stage is free (the loads of the tile after the next, in the
    // state pass; of the next, in the output pass)
    if (producer && issued < n_tiles) issue_loads(issued);

    if (!kStateOnly) {
      // every owner has summed the previous tile: the staging and receiving
      // buffers are free
      if (c > 0) cluster_wait();
      // ---- O_r -> staging [row][68] (warps 0..3 values 0..31, warps 12..15
      // values 32..64; lane = row); S_{c+1} -> bf16 snapshot (state warps)
      if (warp < 4 || warp >= 12) {
        const int row = (warp & 3) * 32 + lane, h = warp >= 12 ? 1 : 0;
        const uint32_t obase = taddr(tmem, (warp & 3) * 32, kColO + 32 * h);
        const uint32_t dst = sb + L::kOffStage + (row * kRecvLd + 32 * h) * 4;
        uint32_t o[32];
        tmem_ld16(obase, o);
        tmem_ld16(obase + 16, o + 16);
        const uint32_t den = h ? tmem_ld1(obase + 32) : 0u;
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          st_shared_v4(dst + 16 * i, o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
        if (h) asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst + 32 * 4), "r"(den) : "memory");
      } else if (state_warp && c + 1 < n_tiles) {
        // 80 columns: the next group's TMEM load is in flight while this
        // group is packed and stored
        const uint32_t base = taddr(tmem, (warp & 3) * 32, kColS + col0);
        uint32_t r0[16], r1[16];
        tmem_ld16(base, r0);
#pragma unroll
        for (int grp = 0; grp < 5; ++grp) {
          uint32_t *cur = (grp & 1) ? r1 : r0;
          uint32_t *nxt = (grp & 1) ? r0 : r1;
          tmem_wait_ld();
          if (grp + 1 < 5) tmem_ld16(base + 16 * (grp + 1), nxt);
          const int f0 = col0 + 16 * grp;
          if (e <= kDv) {
            const uint32_t blk = sb + L::kOffSnap + (f0 >> 6) * kSnapKBlock;
            const int ch = (f0 & 63) >> 3;
#pragma unroll
            for (int h = 0; h < 2; ++h)
              st_shared_v4(blk + sw128_offset(e, ch + h),
                           pack_bf16(__uint_as_float(cur[8 * h + 0]), __uint_as_float(cur[8 * h + 1])),
                           pack_bf16(__uint_as_float(cur[8 * h + 2]), __uint_as_float(cur[8 * h + 3])),
                           pack_bf16(__uint_as_float(cur[8 * h + 4]), __uint_as_float(cur[8 * h + 5])),
                           pack_bf16(__uint_as_float(cur[8 * h + 6]), __uint_as_float(cur[8 * h + 7])));
          }
        }
      }
      // the copies start once the staging warps are done; the snapshot warps
      // finish meanwhile (the next tile's barrier orders their stores before
      // the MMAs that read them)
      fence_proxy_async_smem();
      tc_fence_before();
      if (warp < 4 || warp >= 12) named_barrier_sync(1, 256);
      LA_TRACE64(c, 7);
      if (warp == 0 && lane < kCl) {
        // lane o: rows 8o .. 8o+7 -> block [rank] of CTA o, counted on its
        // mbarrier; this CTA's own mbarrier expects the 16 blocks of its rows
        const uint32_t o = (uint32_t)lane;
        bulk_copy_to_peer(cluster_addr(sb + L::kOffRecv + rank * kBlockBytes, o),
                          sb + L::kOffStage + o * kBlockBytes, kBlockBytes,
                          cluster_addr(smem_u32(&bars[kRecv]), o));
        if (lane == 0) mbar_arrive_expect_tx(&bars[kRecv], kCl * kBlockBytes);
      }
    }
    LA_TRACE64(c, 8);
  }

  // ---- the state after the segment: final state (output pass, last
  // segment) or this segment's state (state pass), this CTA's slots
  float *dst = nullptr;
  if (kStateOnly) dst = p.seg_out + ((uint64_t)bh * p.segments + g) * kF * kSV;
  else if (p.final_state != nullptr && g == p.segments - 1)
    dst = p.final_state + (uint64_t)bh * kF * kSV;
  if (dst && state_warp) {
    for (int f0 = col0; f0 < col0 + 80; f0 += 16) {
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

  // the last tile's rows; then every owner has summed (so every bulk copy
  // of this CTA's partials, read from its staging buffer, has landed)
  // before any CTA of the cluster leaves
  if (!kStateOnly && n_tiles > 0) {
    reduce_tile(n_tiles - 1);
    cluster_wait();
  }

  // ---- teardown: every issued copy has landed (each tile's loads were
  // waited for in its iteration, unless a wait gave up)
  if (producer) {
    for (int c = issued - L::kStages < 0 ? 0 : issued - L::kStages; c < issued; ++c)
      wait_teardown(&bars[kFull0 + c % L::kStages], (c / L::kStages) & 1);
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

#ifdef LA_TRACE
extern "C" int la_debug_read_trace64(long long *dst, int count) {
  const int n = kCl * kTrTiles * kTrEvents;
  if (count < n) return -1;
  return cudaMemcpyFromSymbol(dst, la_trace64, sizeof(long long) * n) == cudaSuccess ? n : -1;
}
#endif

namespace {
// 16-CTA clusters the device of each context holds at once (0: none), found
// once per context: the non-portable cluster size is enabled for the kernel
// and the occupancy of one such cluster is queried.
int query_max_clusters() {
  const void *fn = (const void *)chunked64_tc_kernel<false>;
  constexpr uint32_t kSmem = Layout64<false>::kSmemAlloc;
  int clusters = 0;
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
    if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) clusters = 0;
  }
  cudaGetLastError();
  return clusters > 0 ? clusters : 0;
}

int max_clusters() {
  struct Entry {
    unsigned long long ctx;
    int clusters;
  };
  static std::mutex mu;
  static Entry cache[64];
  static int used = 0;
  unsigned long long ctx = 0;
  const bool known = current_context_id(&ctx);
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].ctx == ctx) return cache[i].clusters;
  }
  const int clusters = query_max_clusters();
  if (known) {
    std::lock_guard<std::mutex> lock(mu);
    if (used < 64) cache[used++] = Entry{ctx, clusters};
  }
  return clusters;
}
}  // namespace

bool chunked64_tc_available() { return max_clusters() > 0; }

int chunked64_tc_ctas_per_segment() { return kCl; }

// Segments per head: the g that minimises the estimated time of the output
// pass, in waves of the clusters the device holds at once (7 on a B200),
// plus the state pass over the first g - 1 segments (16 independent CTAs
// per segment) and the running-sum launch, at least 1024 tokens per segment.
// The state pass's cost per tile (0.7 of an output tile) and the launches'
// (3 tiles) are fitted to B=1, H=16, N=4096 on a B200: one segment (three
// waves of 7, 7 and 2 clusters) 0.546 ms, two segments 0.581 ms.
int chunked64_auto_segments(int64_t bh, int64_t n, int sm_count) {
  const int64_t w = max_clusters();
  if (bh <= 0 || n <= 0 || w <= 0) return 1;
  const int64_t tiles = (n + kT - 1) / kT;
  const int64_t max_g = (n + 1023) / 1024 < 16 ? (n + 1023) / 1024 : 16;
  int best = 1;
  double best_t = 0.0;
  for (int64_t g = 1; g <= max_g; ++g) {
    const double seg_tiles = (double)((tiles + g - 1) / g);
    const double out_waves = (double)((bh * g + w - 1) / w);
    const double st_waves = g > 1 ? (double)((kCl * bh * (g - 1) + sm_count - 1) / sm_count) : 0.0;
    const double t = out_waves * seg_tiles + 0.7 * st_waves * seg_tiles + (g > 1 ? 3.0 : 0.0);
    if (g == 1 || t < best_t) {
      best_t = t;
      best = (int)g;
    }
  }
  return best;
}

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
