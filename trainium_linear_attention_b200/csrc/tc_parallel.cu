// Parallel (quadratic) causal BASED attention on tcgen05 tensor cores (sm_100a).
//
// Fast path: bf16 q/k/v, d_qk = 16, d_v = 64.  A work item is one (head,
// 128-query tile qt); it walks the key tiles 0 .. qt:
//
//   S  = Q K_kt^T                   tcgen05 M=128 N=128 K=16  -> TMEM (fp32)
//   P  = 1 + s/4 + s^2/32           CUDA cores (s = q.k raw; d = 16), causal
//                                   mask on the diagonal tile, bf16 P over S
//   O += P [V_kt 1]                 tcgen05 M=128 N=80 K=128  (A = P in TMEM)
//   out = O[:, :64] / (O[:, 64] + eps)
//
// which is ref_based_attn / solution_nki (kernels/pytorch_attention.py:27-78)
// and the NKI kernel of kernels/nki_attention.py:25-115 (blocked causal
// polynomial attention with a numerator and a denominator): the denominator
// is the ones column of [V 1] (the row sum of P), from a 2 KB constant block
// addressed as the second 64-column block of the V operand.
//
// Two kernels.  Up to kPersistentMaxTiles query tiles per head (N <= 512),
// where per-CTA start-up and first loads would dominate, a persistent kernel:
// one CTA per SM walks the work items b, b + grid, ... (items ordered
// longest first: query tile N/128 - 1 of every head, then
// the next, so the round-robin split is balanced).  K/V tiles stream through
// an 8-stage TMA ring and Q through two slots; TMEM holds two S/P buffers,
// each with its own group of four polynomial warps (two key tiles in flight),
// and two O accumulators, so an item's output leaves TMEM while the next
// item accumulates.  Roles: warp 0 TMA, warp 1 MMA issuer (scores of key
// tile s issued before P V of tile s - 1), warps 2-9 polynomial, warps 10-13
// epilogue.  For longer sequences, one CTA (4 warps) per work item, two CTAs
// per SM (256 TMEM columns each), K/V through a 3-stage ring: measured faster
// there (N = 2048: 1.72 vs 1.95 ms; N = 256: 0.55 vs 0.41 ms).
#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

namespace la {
namespace {
using namespace tc;

constexpr int kT = 128;      // queries / keys per tile
constexpr int kDqk = 16;
constexpr int kDv = 64;
constexpr int kNO = 80;      // N of P [V 1]: 64 values, row sum, 15 zero columns
constexpr uint32_t kQBytes = kT * kDqk * 2;        // 4 KB, 32-byte rows
constexpr uint32_t kVBytes = kT * kDv * 2;         // 16 KB, 128-byte rows
constexpr int kPersistentMaxTiles = 4;

// ------------------------------------------------------------ one CTA per work item
namespace tile {
constexpr int kStages = 3;   // K/V ring

constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kQBytes;        // kStages x 4 KB
constexpr uint32_t kOffV = kOffK + kStages * kQBytes;     // 16384: kStages x 16 KB
constexpr uint32_t kOffOnes = kOffV + kStages * kVBytes;  // 65536: 16 rows x 128 B
constexpr uint32_t kOffBar = kOffOnes + 2048;
// padded so that two CTAs (256 TMEM columns each) share an SM, never three
// (a third CTA's tcgen05.alloc would wait for a neighbour to finish)
constexpr uint32_t kSmemAlloc = 80 * 1024;
static_assert(kOffV % 1024 == 0 && kOffOnes % 1024 == 0, "128B-swizzled tiles need 1024-byte alignment");
static_assert(kOffBar + 128 + 1024 <= kSmemAlloc, "shared memory layout");

constexpr uint32_t kColS = 0;      // S fp32 128 columns / P bf16 64 columns
constexpr uint32_t kColO = 128;    // O fp32 80 columns
constexpr uint32_t kTmemCols = 256;

struct ParallelParams {
  __nv_bfloat16 *out;
  int *err;
  int64_t n;
  float eps;
};

enum PBar { kFull0, kFull1, kFull2, kSReady, kPVDone, kNumPBars };

__global__ void __launch_bounds__(128)
parallel_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const ParallelParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + kOffBar + 8 * kNumPBars);
  volatile int *abort_flag = (volatile int *)(smem + kOffBar + 8 * kNumPBars + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int qt = blockIdx.x;
  const int q0 = qt * kT;
  const int nkt = qt + 1;  // key tiles 0 .. qt

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumPBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // ones block: rows 64..127 of the [V 1] operand's second 64-column block
  // (element 0 of each 128-byte row is 1, 128B-swizzled)
  for (int i = threadIdx.x; i < 2048 / 4; i += 128) {
    const int row = (i * 4) / 128, byte = (i * 4) % 128;
    *(uint32_t *)(smem + kOffOnes + i * 4) = (byte == (row & 7) * 16) ? 0x3F80u : 0u;
  }
  if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  constexpr uint32_t id_s = make_idesc_bf16(128, 128, false, false);
  constexpr uint32_t id_pv = make_idesc_bf16(128, kNO, false, true);
  // a K-step of 16 keys: start address +2048 B, LBO (distance to the ones block) -2048 B
  constexpr uint64_t kStep = (uint64_t)(2048 >> 4) - ((uint64_t)(2048 >> 4) << 16);
  auto load_kv = [&](int kt) {
    const int st = kt % kStages;
    mbar_arrive_expect_tx(&bars[kFull0 + st], (kt == 0 ? kQBytes : 0) + kQBytes + kVBytes);
    if (kt == 0) tma_load_3d(smem + kOffQ, &tm_q, &bars[kFull0 + st], 0, q0, (int)bh);
    tma_load_3d(smem + kOffK + st * kQBytes, &tm_k, &bars[kFull0 + st], 0, kt * kT, (int)bh);
    tma_load_3d(smem + kOffV + st * kVBytes, &tm_v, &bars[kFull0 + st], 0, kt * kT, (int)bh);
  };
  if (threadIdx.x == 0) {
    for (int kt = 0; kt < nkt && kt < kStages; ++kt) load_kv(kt);
  }

  const int row = warp * 32 + lane;  // query q0 + row, TMEM lane
  const uint32_t srow = taddr(tmem, warp * 32, kColS);
  const uint64_t c32 = f2pack(0.03125f, 0.03125f), c4 = f2pack(0.25f, 0.25f);
  const uint64_t one2 = f2pack(1.f, 1.f);
  for (int kt = 0; kt < nkt; ++kt) {
    const int st = kt % kStages;
    if (warp == 0) {
      // warp 0 waits converged and issues through one elected lane
      // S(kt) overwrites P(kt-1): P V of the previous tile has finished, which
      // also frees its K/V stage for tile kt+2
      if (kt > 0) mbar_wait_warp(&bars[kPVDone], (kt - 1) & 1, abort_flag);
      if (lane == 0 && kt > 0 && kt + kStages - 1 < nkt) load_kv(kt + kStages - 1);
      mbar_wait_warp(&bars[kFull0 + st], (kt / kStages) & 1, abort_flag);
      tc_fence_after();
      const uint64_t da = make_sdesc(sb + kOffQ, 16, 256, kSwizzle32B);
      const uint64_t db = make_sdesc(sb + kOffK + st * kQBytes, 16, 256, kSwizzle32B);
      if (elect_one()) {
        umma_ss(tmem + kColS, da, db, id_s, 0);
        umma_commit(&bars[kSReady]);
      }
      __syncwarp();
    }
    mbar_wait(&bars[kSReady], kt & 1, abort_flag);
    __syncwarp();
    tc_fence_after();
    // P = 1 + s/4 + s^2/32 in place: chunk c (S columns 32c .. 32c+31, keys
    // kt*128 + 32c ..) becomes P columns 16c .. 16c+15.  On the diagonal
    // tile key j is visible to query row r when j <= r; keys past n (read
    // as zero) are never visible.
    const bool diag = kt == qt;
    const int lim = (int)min64(diag ? row : kT - 1, p.n - 1 - (int64_t)kt * kT);
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t r[32], w[16];
      tmem_ld16(srow + 32 * cc, r);
      tmem_ld16(srow + 32 * cc + 16, r + 16);
      tmem_wait_ld();
      const int m = lim - 32 * cc;  // columns 0 .. m of this chunk are visible
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        const uint64_t s2 = f2pack(__uint_as_float(r[2 * t]), __uint_as_float(r[2 * t + 1]));
        float p0, p1;
        f2unpack(ffma2(s2, ffma2(s2, c32, c4), one2), p0, p1);
        p0 = 2 * t <= m ? p0 : 0.f;
        p1 = 2 * t + 1 <= m ? p1 : 0.f;
        w[t] = pack_bf16(p0, p1);
      }
      tmem_st16(srow + 16 * cc, w);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc_fence_after();
      const uint32_t v_base = sb + kOffV + st * kVBytes;
      const uint64_t db0 = make_sdesc(v_base, (sb + kOffOnes) - v_base, 1024, kSwizzle128B);
      if (elect_one()) {
#pragma unroll
        for (int j = 0; j < kT / 16; ++j)
          umma_ts(tmem + kColO, tmem + kColS + 8 * j, db0 + kStep * j, id_pv,
                  (kt > 0 || j > 0) ? 1u : 0u);
        umma_commit(&bars[kPVDone]);
      }
      __syncwarp();
    }
  }
  mbar_wait(&bars[kPVDone], (nkt - 1) & 1, abort_flag);
  __syncwarp();
  tc_fence_after();

  // ---------------------------------------------------------------- epilogue
  uint32_t w[32];
  const uint32_t obase = taddr(tmem, warp * 32, kColO);
  {
    uint32_t o[32];
    const uint32_t dbits = tmem_ld1(obase + kDv);
    tmem_ld16(obase, o);
    tmem_ld16(obase + 16, o + 16);
    tmem_wait_ld();
    // O[:, 64] = rowsum(P): the denominator before eps
    const float inv = 1.f / (__uint_as_float(dbits) + p.eps);
    const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
    for (int t = 0; t < 16; ++t)
      w[t] = pack_bf16x2(fmul2(f2pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1])), inv2));
    tmem_ld16(obase + 32, o);
    tmem_ld16(obase + 48, o + 16);
    tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < 16; ++t)
      w[16 + t] =
          pack_bf16x2(fmul2(f2pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1])), inv2));
  }
  // 4x4 transpose of 32-byte pieces inside each group of four lanes: each
  // store instruction then writes eight whole 128-byte rows
  const int gi = lane & 3;
#pragma unroll
  for (int mm = 2; mm >= 1; mm >>= 1) {
    const bool hi = (gi & mm) != 0;
#pragma unroll
    for (int kx = 0; kx < 2; ++kx) {
      const int s0 = mm == 2 ? kx : (kx << 1);
      const int s1 = s0 | mm;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const uint32_t send = hi ? w[8 * s0 + t] : w[8 * s1 + t];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, mm);
        if (hi) w[8 * s0 + t] = recv;
        else w[8 * s1 + t] = recv;
      }
    }
  }
  const int rbase = q0 + warp * 32 + (lane & ~3);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (rbase + j < p.n) {
      uint4 *dst = (uint4 *)(p.out + ((uint64_t)bh * p.n + rbase + j) * kDv) + 2 * gi;
      asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                   "r"(w[8 * j]), "r"(w[8 * j + 1]), "r"(w[8 * j + 2]), "r"(w[8 * j + 3]),
                   "r"(w[8 * j + 4]), "r"(w[8 * j + 5]), "r"(w[8 * j + 6]), "r"(w[8 * j + 7])
                   : "memory");
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // every issued copy has landed (all were waited on unless a wait gave up)
    for (int kt = nkt - kStages < 0 ? 0 : nkt - kStages; kt < nkt; ++kt) {
      const uint64_t t0 = globaltimer();
      while (!mbar_try_wait(&bars[kFull0 + kt % kStages], (kt / kStages) & 1))
        if (globaltimer() - t0 > kWaitTimeoutNs) break;
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
}

}  // namespace tile

// ------------------------------------------------------------ persistent
namespace persistent {
constexpr int kStages = 8;   // K/V ring
constexpr int kThreadsPar = 14 * 32;

constexpr uint32_t kOffV = 0;                                   // kStages x 16 KB
constexpr uint32_t kOffK = kOffV + kStages * kVBytes;           // kStages x 4 KB
constexpr uint32_t kOffQ = kOffK + kStages * kQBytes;           // 2 x 4 KB
constexpr uint32_t kOffOnes = kOffQ + 2 * kQBytes;              // 16 rows x 128 B
constexpr uint32_t kOffBar = kOffOnes + 2048;
constexpr uint32_t kSmemAlloc = kOffBar + 256 + 1024;           // + alignment slack
static_assert(kOffV % 1024 == 0 && kOffOnes % 1024 == 0, "128B-swizzled tiles need 1024-byte alignment");
static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");

constexpr uint32_t kColS = 0;      // S/P buffer b: fp32 S at 128 b .. / bf16 P in its first 64
constexpr uint32_t kColO = 256;    // O accumulator o: 80 fp32 columns at 256 + 128 o
constexpr uint32_t kTmemCols = 512;

struct ParallelParams {
  __nv_bfloat16 *out;
  int *err;
  int64_t n;
  int64_t items;  // bh * tiles
  int64_t bh;
  int tiles;      // query tiles per head
  int head_major; // a CTA takes whole heads (else single items, longest first)
  float eps;
};

// barriers: Q slots full / empty, K/V stages full / empty, per S/P buffer S
// ready / P ready / buffer free, per O accumulator ready / free, done
enum PBar {
  kQFull = 0,
  kQEmpty = kQFull + 2,
  kKVFull = kQEmpty + 2,
  kKVEmpty = kKVFull + kStages,
  kSReady = kKVEmpty + kStages,
  kPReady = kSReady + 2,
  kSPFree = kPReady + 2,
  kOReady = kSPFree + 2,
  kOFree = kOReady + 2,
  kDone = kOFree + 2,
  kNumPBars
};
static_assert(8 * kNumPBars + 8 <= 256, "barrier area");

// The work item of a CTA's j-th turn: query tile qt of head h.  Head-major
// (many heads per SM): the CTA takes heads b, b + grid, ..., each with its
// query tiles from the last down, so a head's K/V tiles are read again while
// they are still in L2.  Otherwise single items round-robin, longest first.
struct Item {
  int64_t h;
  int qt;
};
__device__ __forceinline__ Item item_of(const ParallelParams &p, int j) {
  if (p.head_major)
    return {blockIdx.x + (int64_t)(j / p.tiles) * gridDim.x, p.tiles - 1 - j % p.tiles};
  const int64_t idx = blockIdx.x + (int64_t)j * gridDim.x;
  return {idx % p.bh, p.tiles - 1 - (int)(idx / p.bh)};
}
__device__ __forceinline__ int item_count(const ParallelParams &p) {
  if (p.head_major)
    return (int64_t)blockIdx.x < p.bh ? (int)((p.bh - 1 - blockIdx.x) / gridDim.x + 1) * p.tiles : 0;
  return (int64_t)blockIdx.x < p.items ? (int)((p.items - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
}

__device__ __forceinline__ bool wait_teardown(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  return true;
}

__global__ void __launch_bounds__(kThreadsPar, 1)
parallel_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const ParallelParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + kOffBar + 8 * kNumPBars);
  volatile int *abort_flag = (volatile int *)(smem + kOffBar + 8 * kNumPBars + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = item_count(p);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumPBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // ones block: rows 64..127 of the [V 1] operand's second 64-column block
  // (element 0 of each 128-byte row is 1, 128B-swizzled)
  for (int i = threadIdx.x; i < 2048 / 4; i += kThreadsPar) {
    const int row = (i * 4) / 128, byte = (i * 4) % 128;
    *(uint32_t *)(smem + kOffOnes + i * 4) = (byte == (row & 7) * 16) ? 0x3F80u : 0u;
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      int s = 0;  // key-tile steps issued
      int jq = 0;
      bool ok = true;
      for (; ok && jq < count; ++jq) {
        const Item it = item_of(p, jq);
        const int qs = jq & 1;
        if (jq >= 2 && !mbar_wait(&bars[kQEmpty + qs], ((jq >> 1) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bars[kQFull + qs], kQBytes);
        tma_load_3d(smem + kOffQ + qs * kQBytes, &tm_q, &bars[kQFull + qs], 0, it.qt * kT, (int)it.h);
        for (int kt = 0; kt <= it.qt; ++kt, ++s) {
          const int st = s % kStages;
          if (s >= kStages && !mbar_wait(&bars[kKVEmpty + st], ((s / kStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars[kKVFull + st], kQBytes + kVBytes);
          tma_load_3d(smem + kOffK + st * kQBytes, &tm_k, &bars[kKVFull + st], 0, kt * kT, (int)it.h);
          tma_load_3d(smem + kOffV + st * kVBytes, &tm_v, &bars[kKVFull + st], 0, kt * kT, (int)it.h);
        }
      }
      // every issued copy must land before the CTA can exit
      for (int c = s - kStages < 0 ? 0 : s - kStages; c < s; ++c)
        wait_teardown(&bars[kKVFull + c % kStages], (c / kStages) & 1);
      for (int c = jq - 2 < 0 ? 0 : jq - 2; c < jq; ++c)
        wait_teardown(&bars[kQFull + (c & 1)], (c >> 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // the warp waits converged and issues through one elected lane
    {
      constexpr uint32_t id_s = make_idesc_bf16(128, 128, false, false);
      constexpr uint32_t id_pv = make_idesc_bf16(128, kNO, false, true);
      // a K-step of 16 keys: start address +2048 B, LBO (distance to the ones block) -2048 B
      constexpr uint64_t kStep = (uint64_t)(2048 >> 4) - ((uint64_t)(2048 >> 4) << 16);
      // scores of step s (key tile kt of the item of turn j)
      auto issue_s = [&](int s, int j, int kt, int qt) -> bool {
        const int st = s % kStages, b = s & 1, qs = j & 1;
        if (!mbar_wait_warp(&bars[kKVFull + st], (s / kStages) & 1, abort_flag)) return false;
        if (kt == 0 && !mbar_wait_warp(&bars[kQFull + qs], (j >> 1) & 1, abort_flag)) return false;
        if (s >= 2 && !mbar_wait_warp(&bars[kSPFree + b], ((s >> 1) - 1) & 1, abort_flag))
          return false;
        tc_fence_after();
        const uint64_t da = make_sdesc(sb + kOffQ + qs * kQBytes, 16, 256, kSwizzle32B);
        const uint64_t db = make_sdesc(sb + kOffK + st * kQBytes, 16, 256, kSwizzle32B);
        if (elect_one()) {
          umma_ss(tmem + kColS + 128 * b, da, db, id_s, 0);
          umma_commit(&bars[kSReady + b]);
          if (kt == qt) umma_commit(&bars[kQEmpty + qs]);  // the item's last read of Q
        }
        __syncwarp();
        return true;
      };
      // P V of step s into the O accumulator of turn j
      auto issue_pv = [&](int s, int j, int kt, int qt) -> bool {
        const int st = s % kStages, b = s & 1, o = j & 1;
        if (!mbar_wait_warp(&bars[kPReady + b], (s >> 1) & 1, abort_flag)) return false;
        if (kt == 0 && j >= 2 &&
            !mbar_wait_warp(&bars[kOFree + o], ((j >> 1) - 1) & 1, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t v_base = sb + kOffV + st * kVBytes;
        const uint64_t db0 = make_sdesc(v_base, (sb + kOffOnes) - v_base, 1024, kSwizzle128B);
        if (elect_one()) {
#pragma unroll
          for (int jj = 0; jj < kT / 16; ++jj)
            umma_ts(tmem + kColO + 128 * o, tmem + kColS + 128 * b + 8 * jj, db0 + kStep * jj,
                    id_pv, (kt > 0 || jj > 0) ? 1u : 0u);
          umma_commit(&bars[kSPFree + b]);
          umma_commit(&bars[kKVEmpty + st]);
          if (kt == qt) umma_commit(&bars[kOReady + o]);
        }
        __syncwarp();
        return true;
      };
      // in order: the scores of step s, then P V of step s - 1
      int s = 0;
      int pj = -1, pkt = 0, pqt = 0;  // the step whose P V is still to issue
      bool ok = true;
      for (int j = 0; ok && j < count; ++j) {
        const int qt = item_of(p, j).qt;
        for (int kt = 0; ok && kt <= qt; ++kt, ++s) {
          ok = issue_s(s, j, kt, qt);
          if (ok && pj >= 0) ok = issue_pv(s - 1, pj, pkt, pqt);
          pj = j, pkt = kt, pqt = qt;
        }
      }
      if (ok && pj >= 0) issue_pv(s - 1, pj, pkt, pqt);
      if (elect_one()) umma_commit(&bars[kDone]);
      __syncwarp();
      if (lane == 0) wait_teardown(&bars[kDone], 0);
      __syncwarp();
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ polynomial
    // Group g (warps 2+4g .. 5+4g) takes the steps s = g, g + 2, ... (S/P
    // buffer g).  Every wait returns at once after an abort, so the four warps
    // of a group run the same iterations and reach every named barrier.
    const int grp = (warp - 2) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;  // query row of the tile, TMEM lane
    const uint32_t srow = taddr(tmem, wq * 32, kColS + 128 * grp);
    const uint64_t c32 = f2pack(0.03125f, 0.03125f), c4 = f2pack(0.25f, 0.25f);
    const uint64_t one2 = f2pack(1.f, 1.f);
    int s = 0;
    for (int j = 0; j < count; ++j) {
      const int qt = item_of(p, j).qt;
      for (int kt = 0; kt <= qt; ++kt, ++s) {
        if ((s & 1) != grp) continue;
        mbar_wait(&bars[kSReady + grp], (s >> 1) & 1, abort_flag);
        __syncwarp();
        tc_fence_after();
        // P = 1 + s/4 + s^2/32 in place: chunk c (S columns 32c .. 32c+31,
        // keys kt*128 + 32c ..) becomes P columns 16c .. 16c+15.  On the
        // diagonal tile key j is visible to query row r when j <= r; keys
        // past n (read as zero) are never visible.
        const int lim = (int)min64(kt == qt ? row : kT - 1, p.n - 1 - (int64_t)kt * kT);
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t r[32], w[16];
          tmem_ld16(srow + 32 * cc, r);
          tmem_ld16(srow + 32 * cc + 16, r + 16);
          tmem_wait_ld();
          const int m = lim - 32 * cc;  // columns 0 .. m of this chunk are visible
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const uint64_t s2 = f2pack(__uint_as_float(r[2 * t]), __uint_as_float(r[2 * t + 1]));
            float p0, p1;
            f2unpack(ffma2(s2, ffma2(s2, c32, c4), one2), p0, p1);
            p0 = 2 * t <= m ? p0 : 0.f;
            p1 = 2 * t + 1 <= m ? p1 : 0.f;
            w[t] = pack_bf16(p0, p1);
          }
          tmem_st16(srow + 16 * cc, w);
        }
        tmem_wait_st();
        tc_fence_before();
        named_barrier_sync(1 + grp, 128);
        if (wq == 0 && lane == 0) mbar_arrive(&bars[kPReady + grp]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    const int gi = lane & 3;
    for (int j = 0; j < count; ++j) {
      const Item it = item_of(p, j);
      const int o = j & 1;
      mbar_wait(&bars[kOReady + o], (j >> 1) & 1, abort_flag);
      __syncwarp();
      tc_fence_after();
      uint32_t w[32];
      const uint32_t obase = taddr(tmem, wq * 32, kColO + 128 * o);
      {
        uint32_t ov[32];
        const uint32_t dbits = tmem_ld1(obase + kDv);
        tmem_ld16(obase, ov);
        tmem_ld16(obase + 16, ov + 16);
        tmem_wait_ld();
        // O[:, 64] = rowsum(P): the denominator before eps
        const float inv = 1.f / (__uint_as_float(dbits) + p.eps);
        const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
        for (int t = 0; t < 16; ++t)
          w[t] = pack_bf16x2(fmul2(f2pack(__uint_as_float(ov[2 * t]), __uint_as_float(ov[2 * t + 1])), inv2));
        tmem_ld16(obase + 32, ov);
        tmem_ld16(obase + 48, ov + 16);
        tmem_wait_ld();
        // O of this turn is in registers: the accumulator is free
        tc_fence_before();
        named_barrier_sync(3, 128);
        if (wq == 0 && lane == 0) mbar_arrive(&bars[kOFree + o]);
#pragma unroll
        for (int t = 0; t < 16; ++t)
          w[16 + t] =
              pack_bf16x2(fmul2(f2pack(__uint_as_float(ov[2 * t]), __uint_as_float(ov[2 * t + 1])), inv2));
      }
      // 4x4 transpose of 32-byte pieces inside each group of four lanes: each
      // store instruction then writes eight whole 128-byte rows
#pragma unroll
      for (int mm = 2; mm >= 1; mm >>= 1) {
        const bool hi = (gi & mm) != 0;
#pragma unroll
        for (int kx = 0; kx < 2; ++kx) {
          const int s0 = mm == 2 ? kx : (kx << 1);
          const int s1 = s0 | mm;
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const uint32_t send = hi ? w[8 * s0 + t] : w[8 * s1 + t];
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, mm);
            if (hi) w[8 * s0 + t] = recv;
            else w[8 * s1 + t] = recv;
          }
        }
      }
      const int rbase = it.qt * kT + wq * 32 + (lane & ~3);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (rbase + i < p.n) {
          uint4 *dst = (uint4 *)(p.out + ((uint64_t)it.h * p.n + rbase + i) * kDv) + 2 * gi;
          asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                       "r"(w[8 * i]), "r"(w[8 * i + 1]), "r"(w[8 * i + 2]), "r"(w[8 * i + 3]),
                       "r"(w[8 * i + 4]), "r"(w[8 * i + 5]), "r"(w[8 * i + 6]), "r"(w[8 * i + 7])
                       : "memory");
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  // The issuer has seen `done` (every MMA it issued has completed) and the
  // producer every copy it issued before either reaches this barrier.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
}

}  // namespace persistent

}  // namespace


int launch_parallel_tc(const void *q, const void *k, const void *v, void *out, int64_t bh,
                       int64_t n, float eps, const DeviceInfo &info, cudaStream_t s) {
  if (bh > 65535 || n > INT32_MAX - kT) return LA_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_3d(&mq, q, bh, n, kDqk, kT, CU_TENSOR_MAP_SWIZZLE_32B) ||
      !make_tmap_3d(&mk, k, bh, n, kDqk, kT, CU_TENSOR_MAP_SWIZZLE_32B) ||
      !make_tmap_3d(&mv, v, bh, n, kDv, kT, CU_TENSOR_MAP_SWIZZLE_128B))
    return LA_ERR_CUDA;
  const int tiles = (int)((n + kT - 1) / kT);
  if (tiles == 0 || bh == 0) return LA_OK;
  if (tiles > kPersistentMaxTiles) {
    tile::ParallelParams p{};
    p.out = (__nv_bfloat16 *)out;
    p.err = device_error_word();
    p.n = n;
    p.eps = eps;
    if (!p.err) return LA_ERR_CUDA;
    if (allow_dynamic_smem((const void *)tile::parallel_tc_kernel, (int)tile::kSmemAlloc) != LA_OK)
      return LA_ERR_CUDA;
    dim3 grid((unsigned)tiles, (unsigned)bh);
    tile::parallel_tc_kernel<<<grid, 128, tile::kSmemAlloc, s>>>(mq, mk, mv, p);
    return check_launch();
  }
  persistent::ParallelParams p{};
  p.out = (__nv_bfloat16 *)out;
  p.err = device_error_word();
  p.n = n;
  p.bh = bh;
  p.tiles = tiles;
  p.items = bh * tiles;
  p.eps = eps;
  if (!p.err) return LA_ERR_CUDA;
  if (allow_dynamic_smem((const void *)persistent::parallel_tc_kernel,
                         (int)persistent::kSmemAlloc) != LA_OK)
    return LA_ERR_CUDA;
  const int sms = info.sm_count > 0 ? info.sm_count : 1;
  // whole heads per CTA once every SM has at least four (at most one head
  // of imbalance in four)
  p.head_major = bh >= 4 * (int64_t)sms ? 1 : 0;
  const int64_t grid = p.items < sms ? p.items : sms;
  persistent::parallel_tc_kernel<<<(unsigned)grid, persistent::kThreadsPar, persistent::kSmemAlloc,
                                   s>>>(mq, mk, mv, p);
  return check_launch();
}

}  // namespace la
