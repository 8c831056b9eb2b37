// Sliding-window causal softmax attention on tcgen05 tensor cores (sm_100a).
//
// Fast path: bf16 q/k/v, d_qk 64 or 16, d_v 64, window W <= 129.  A tile is
// one (head, 128-query block).  Its queries [q0, q0+128) see keys
// [q0 - W + 1, q0 + 127], which fit in one span of kSpan keys starting at
// k0 = q0 + 128 - kSpan (192 keys for W <= 65, 256 for W <= 129):
//
//   S   = Q K^T          tcgen05 M=128 N=kSpan K=d_qk -> TMEM (fp32)
//   P   = exp(S/sqrt(d_qk) - m)  CUDA cores (as 2^x, ex2.approx), row max m over the
//                        row's window, masked to [max(0, i-W+1), i]; bf16 P
//                        written over S
//   O   = P V            tcgen05 M=128 N=64 K=kSpan   (A = P in TMEM)
//   out = O / sum(P)  [+ addend: the BASED layer adds the window term to the
//                      chunked kernel's output, read in the epilogue]
//
// which is ref_sliding_window_attn (benchmarks/sliding_attention_benchmark.py:
// 32-56) and the NKI kernel of kernels/nki_attention_sliding.py:30-132
// (banded softmax, fp32 statistics) without its additive mask tensor: the
// band is computed from indices.  The whole band of a row is in one S tile,
// so the softmax needs no running rescale.
//
// Persistent and pipelined: one CTA per SM walks the tiles b, b + grid, ...
// (neighbouring CTAs take neighbouring tiles of a head, so the key rows that
// two spans share are read from L2).  Q, K and V of a tile arrive by TMA in
// one transaction into a ring of stages (keys before 0 and past n read as
// zero and are masked), so the next tiles load while this one computes; with
// kSpan = 192 two TMEM buffers of S/P and O let the scores of the next tile
// and the P V of this one run under the softmax and the output stores.
// Roles: warp 0 TMA, warp 1 MMA issuer (and TMEM owner), warps 2-9 softmax
// (two groups, one per TMEM buffer), warps 10-13 epilogue (each group of four
// covers the four TMEM lane quarters).
#include <utility>

#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

namespace la {
namespace {
using namespace tc;

constexpr int kT = 128;  // queries per tile
constexpr int kD = 64;   // value head dim
constexpr int kMaxStages = 6;
constexpr int kThreadsSl = 14 * 32;
constexpr uint32_t kStageOverhead = 256 + 2 * kT * 4 + 1024;  // barriers, row sums, alignment

// kDqk: query/key head dim, 64 (128-byte, 128B-swizzled rows) or 16 (32-byte,
// 32B-swizzled rows)
template <int kSpan, int kDqk>
struct SlidingLayout {
  static constexpr uint32_t kQBytes = kT * kDqk * 2;
  static constexpr uint32_t kKBytes = kSpan * kDqk * 2;
  static constexpr uint32_t kVBytes = kSpan * kD * 2;  // kSpan rows x 128 B
  static constexpr uint32_t kOffK = kQBytes;
  static constexpr uint32_t kOffV = kQBytes + kKBytes;
  static constexpr uint32_t kStageBytes = kQBytes + kKBytes + kVBytes;
  // as many TMA stages as shared memory holds (at most kMaxStages); at
  // d_qk = 16 that is 6 or 5, which also keeps the CTA alone on its SM
  // (it allocates all 512 TMEM columns)
  static constexpr int fit_stages() {
    int n = kMaxStages;
    while (n > 2 && n * kStageBytes + kStageOverhead > 227 * 1024) --n;
    return n;
  }
  static constexpr int kStages = fit_stages();
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kOffRowSum = kOffBar + 256;  // fp32 row sums, per TMEM buffer
  static constexpr uint32_t kSmemAlloc = kOffRowSum + 2 * kT * 4 + 1024;  // + alignment slack
  static constexpr uint32_t kBufCols = kSpan + kD;       // S/P, then O
  static constexpr int kBufs = 2 * kBufCols <= 512 ? 2 : 1;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kLoadBytes = kStageBytes;
  static_assert(kOffV % 1024 == 0 && kStageBytes % 1024 == 0,
                "128B-swizzled tiles need 1024-byte alignment");
  static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");
  static_assert(kSmemAlloc > 114 * 1024, "one CTA per SM (all TMEM columns)");
  static_assert(kLoadBytes < (1u << 20), "one TMA transaction count");
};

struct SlidingParams {
  __nv_bfloat16 *out;
  const __nv_bfloat16 *addend;  // null, or (bh, n, 64) added to the output (may be out)
  int *err;
  int64_t n;
  int64_t tiles;       // bh * tiles_per_head
  int tiles_per_head;
  int window;
  float scale_log2;    // log2(e) / sqrt(d_qk)
};

// barriers: TMA stage full / empty, then per TMEM buffer: S ready, P ready,
// O ready, buffer free; `done` when every MMA has completed
enum SBar {
  kFull = 0,
  kEmpty = kFull + kMaxStages,
  kSReady = kEmpty + kMaxStages,
  kPReady = kSReady + 2,
  kOReady = kPReady + 2,
  kTFree = kOReady + 2,
  kDone = kTFree + 2,
  kNumSBars
};
static_assert(8 * kNumSBars + 8 <= 256, "barrier area");

// 2^x by the hardware approximation (ex2.approx.ftz.f32: relative error
// ~2^-22, results below 2^-126 flush to zero) -- P is rounded to bf16 and
// the row sum accumulates it in fp32, so neither sees the difference.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ bool wait_teardown(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  return true;
}

template <int kSpan, int kDqk>
__global__ void __launch_bounds__(kThreadsSl, 1)
sliding_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const SlidingParams p) {
  using L = SlidingLayout<kSpan, kDqk>;
  constexpr int kBufs = L::kBufs;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + L::kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + L::kOffBar + 8 * kNumSBars);
  volatile int *abort_flag = (volatile int *)(smem + L::kOffBar + 8 * kNumSBars + 4);
  float *row_sum = (float *)(smem + L::kOffRowSum);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's tiles: blockIdx.x + j * gridDim.x for j = 0 .. count-1
  const int count =
      (int64_t)blockIdx.x < p.tiles ? (int)((p.tiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumSBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::kTmemCols);
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
      int j = 0;
      for (; j < count; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&bars[kEmpty + s], ((j / kStages) - 1) & 1, abort_flag))
          break;
        const int64_t t = blockIdx.x + (int64_t)j * gridDim.x;
        const int bh = (int)(t / p.tiles_per_head);
        const int q0 = (int)(t % p.tiles_per_head) * kT;
        const int k0 = q0 + kT - kSpan;  // may be negative: rows before 0 read as zero
        uint8_t *st = smem + s * L::kStageBytes;
        mbar_arrive_expect_tx(&bars[kFull + s], L::kLoadBytes);
        tma_load_3d(st, &tm_q, &bars[kFull + s], 0, q0, bh);
        tma_load_3d(st + L::kOffK, &tm_k, &bars[kFull + s], 0, k0, bh);
        tma_load_3d(st + L::kOffV, &tm_v, &bars[kFull + s], 0, k0, bh);
      }
      // every issued copy must land before the CTA can exit
      for (int c = j - kStages < 0 ? 0 : j - kStages; c < j; ++c)
        wait_teardown(&bars[kFull + c % kStages], (c / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // With two TMEM buffers the scores of tile j are issued before P V of
    // tile j-1, so they are ready when the softmax warps finish tile j-1.
    // The warp waits converged and issues through one elected lane.
    {
      constexpr uint32_t id_s = make_idesc_bf16(128, kSpan, false, false);
      constexpr uint32_t id_o = make_idesc_bf16(128, kD, false, true);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages, b = j % kBufs;
        if (!mbar_wait_warp(&bars[kFull + s], (j / kStages) & 1, abort_flag)) return false;
        if (j >= kBufs && !mbar_wait_warp(&bars[kTFree + b], ((j / kBufs) - 1) & 1, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t st = sb + s * L::kStageBytes;
        // K-major Q and K: 128-byte rows (8-row groups 1024 B apart) at
        // d_qk = 64, 32-byte rows (groups 256 B apart) at d_qk = 16
        constexpr uint32_t kSbo = kDqk == 64 ? 1024 : 256;
        constexpr auto kSw = kDqk == 64 ? kSwizzle128B : kSwizzle32B;
        const uint64_t qd = make_sdesc(st, 16, kSbo, kSw);
        const uint64_t kd = make_sdesc(st + L::kOffK, 16, kSbo, kSw);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < kDqk / 16; ++kk)  // K steps of 16 (32 bytes) along the rows
            umma_ss(tmem + b * L::kBufCols, qd + 2 * kk, kd + 2 * kk, id_s, kk > 0 ? 1u : 0u);
          umma_commit(&bars[kSReady + b]);
        }
        __syncwarp();
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j % kStages, b = j % kBufs;
        if (!mbar_wait_warp(&bars[kPReady + b], (j / kBufs) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint64_t vd = make_sdesc(sb + s * L::kStageBytes + L::kOffV, 16, 1024, kSwizzle128B);
        const uint32_t sp = tmem + b * L::kBufCols;
        if (elect_one()) {
#pragma unroll
          for (int jj = 0; jj < kSpan / 16; ++jj)  // 16 keys (2048 bytes of V) per step
            umma_ts(sp + kSpan, sp + 8 * jj, vd + (uint64_t)((jj * 2048) >> 4), id_o,
                    jj > 0 ? 1u : 0u);
          umma_commit(&bars[kOReady + b]);
          umma_commit(&bars[kEmpty + s]);  // Q, K (read by S) and V are done with
        }
        __syncwarp();
        return true;
      };
      if (kBufs == 2) {
        bool ok = true;
        for (int j = 0; ok && j < count; ++j) {
          ok = issue_s(j);
          if (ok && j > 0) ok = issue_pv(j - 1);
        }
        if (ok && count > 0) issue_pv(count - 1);
      } else {
        for (int j = 0; j < count; ++j)
          if (!issue_s(j) || !issue_pv(j)) break;
      }
      if (elect_one()) umma_commit(&bars[kDone]);
      __syncwarp();
      if (lane == 0) wait_teardown(&bars[kDone], 0);
      __syncwarp();
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ softmax -> P
    // Two groups of four warps, one per TMEM buffer: group g takes the tiles
    // j = g, g + 2, ... (with one buffer, group 0 takes them all).  Every wait
    // returns at once after an abort, so the four warps of a group run the
    // same iterations and reach every named barrier.
    const int grp = (warp - 2) >> 2;
    const int wq = warp & 3;  // TMEM lane quarter: rows 32wq .. 32wq+31
    const int r = wq * 32 + lane;
    const int c_hi = r + kSpan - kT;
    // columns any row of this warp may use: [w_lo, w_hi], loaded 16 at a time
    const int w_lo = max(0, wq * 32 + kSpan - kT - p.window + 1) & ~15;
    const int w_hi = wq * 32 + 31 + kSpan - kT;
    const int nchunk = (w_hi - w_lo) / 16 + 1;
    for (int j = grp; grp < kBufs && j < count; j += kBufs) {
      const int b = j % kBufs;
      const int64_t t = blockIdx.x + (int64_t)j * gridDim.x;
      const int q0 = (int)(t % p.tiles_per_head) * kT;
      const int k0 = q0 + kT - kSpan;
      const bool row_ok = q0 + r < p.n;
      const int c_lo = max(-k0, c_hi - p.window + 1);  // row r sees S columns [c_lo, c_hi]
      mbar_wait(&bars[kSReady + b], (j / kBufs) & 1, abort_flag);
      __syncwarp();
      tc_fence_after();
      const uint32_t srow = taddr(tmem, wq * 32, b * L::kBufCols);
      // band of this row relative to the warp's first column; empty for rows
      // past n, so that no per-element test of the row is needed
      const int rel_lo = row_ok ? c_lo - w_lo : 1 << 20;
      const int rel_hi = row_ok ? c_hi - w_lo : -(1 << 20);
      float m = -INFINITY;
      for (int ch = 0; ch < nchunk; ++ch) {
        uint32_t x[16];
        tmem_ld16(srow + w_lo + 16 * ch, x);
        const int lo = rel_lo - 16 * ch, hi = rel_hi - 16 * ch;  // in-band: lo <= i <= hi
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          m = fmaxf(m, (i >= lo && i <= hi) ? __uint_as_float(x[i]) : -INFINITY);
      }
      const float mb = m * p.scale_log2;  // -inf for rows past n: every value masked below
      const uint64_t sc2 = f2pack(p.scale_log2, p.scale_log2), nmb2 = f2pack(-mb, -mb);
      float l = 0.f;
      for (int ch = 0; ch < nchunk; ++ch) {
        uint32_t x[16], pk[8];
        tmem_ld16(srow + w_lo + 16 * ch, x);
        const int lo = rel_lo - 16 * ch, hi = rel_hi - 16 * ch;
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a0, a1;
          f2unpack(ffma2(f2pack(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), sc2, nmb2),
                   a0, a1);
          const float e0 = (2 * i >= lo && 2 * i <= hi) ? ex2_approx(a0) : 0.f;
          const float e1 = (2 * i + 1 >= lo && 2 * i + 1 <= hi) ? ex2_approx(a1) : 0.f;
          l += e0 + e1;
          pk[i] = pack_bf16(e0, e1);
        }
        // P columns (w_lo + 16 ch) / 2 .. + 8: S columns this warp has already read
        tmem_st8(srow + (w_lo + 16 * ch) / 2, pk);
      }
      {
        // P columns outside [w_lo, w_lo + 16 nchunk) / 2 are zero for these rows
        uint32_t z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int pc = 0; pc < w_lo / 2; pc += 8) tmem_st8(srow + pc, z);
        for (int pc = (w_lo + 16 * nchunk) / 2; pc < kSpan / 2; pc += 8) tmem_st8(srow + pc, z);
      }
      row_sum[b * kT + r] = l;
      tmem_wait_st();
      tc_fence_before();
      named_barrier_sync(1 + 2 * grp, 128);
      if (wq == 0 && lane == 0) mbar_arrive(&bars[kPReady + b]);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const int gi = lane & 3;
    for (int j = 0; j < count; ++j) {
      const int b = j % kBufs;
      const int64_t t = blockIdx.x + (int64_t)j * gridDim.x;
      const int64_t bh = t / p.tiles_per_head;
      const int q0 = (int)(t % p.tiles_per_head) * kT;
      mbar_wait(&bars[kOReady + b], (j / kBufs) & 1, abort_flag);
      // the row sums: published by the softmax warps' P-ready arrival
      mbar_wait(&bars[kPReady + b], (j / kBufs) & 1, abort_flag);
      __syncwarp();
      tc_fence_after();
      const float l = row_sum[b * kT + r];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const uint64_t inv2 = f2pack(inv, inv);
      uint32_t w[32];
      const uint32_t orow = taddr(tmem, wq * 32, b * L::kBufCols + kSpan);
      // the addend's row q0 + r (this lane's row before the transpose below),
      // added in fp32 before the single rounding to bf16
      const bool add_row = p.addend != nullptr && q0 + r < p.n;
      const uint4 *arow = (const uint4 *)(p.addend + ((uint64_t)bh * p.n + (add_row ? q0 + r : 0)) * kD);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o[32];
        uint4 a[4] = {};
        if (add_row) {
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = arow[4 * h + i];
        }
        tmem_ld16(orow + 32 * h, o);
        tmem_ld16(orow + 32 * h + 16, o + 16);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t aw = i % 4 == 0 ? a[i / 4].x : i % 4 == 1 ? a[i / 4].y
                            : i % 4 == 2 ? a[i / 4].z : a[i / 4].w;
          const uint64_t add2 = f2pack(__uint_as_float(aw << 16), __uint_as_float(aw & 0xFFFF0000u));
          w[16 * h + i] = pack_bf16x2(ffma2(
              f2pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2, add2));
        }
      }
      // O and the row sums of buffer b are in registers: the buffer is free
      tc_fence_before();
      named_barrier_sync(2, 128);
      if (wq == 0 && lane == 0) mbar_arrive(&bars[kTFree + b]);
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
          for (int i = 0; i < 8; ++i) {
            const uint32_t send = hi ? w[8 * s0 + i] : w[8 * s1 + i];
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, mm);
            if (hi) w[8 * s0 + i] = recv;
            else w[8 * s1 + i] = recv;
          }
        }
      }
      const int rbase = q0 + wq * 32 + (lane & ~3);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (rbase + i < p.n) {
          uint4 *dst = (uint4 *)(p.out + ((uint64_t)bh * p.n + rbase + i) * kD) + 2 * gi;
          asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                       "r"(w[8 * i]), "r"(w[8 * i + 1]), "r"(w[8 * i + 2]), "r"(w[8 * i + 3]),
                       "r"(w[8 * i + 4]), "r"(w[8 * i + 5]), "r"(w[8 * i + 6]), "r"(w[8 * i + 7])
                       : "memory");
        }
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  // The issuer has seen `done` (every MMA it issued has completed) before it
  // reaches this barrier.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
}

template <int kSpan, int kDqk>
int launch(const void *q, const void *k, const void *v, const SlidingParams &p, int64_t bh,
           int sm_count, cudaStream_t s) {
  using L = SlidingLayout<kSpan, kDqk>;
  constexpr CUtensorMapSwizzle kQKSwizzle =
      kDqk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_3d(&mq, q, bh, p.n, kDqk, kT, kQKSwizzle) ||
      !make_tmap_3d(&mk, k, bh, p.n, kDqk, kSpan, kQKSwizzle) ||
      !make_tmap_3d(&mv, v, bh, p.n, kD, kSpan, CU_TENSOR_MAP_SWIZZLE_128B))
    return LA_ERR_CUDA;
  if (allow_dynamic_smem((const void *)sliding_tc_kernel<kSpan, kDqk>, (int)L::kSmemAlloc) !=
      LA_OK)
    return LA_ERR_CUDA;
  const int64_t grid = p.tiles < sm_count ? p.tiles : sm_count;
  sliding_tc_kernel<kSpan, kDqk><<<(unsigned)grid, kThreadsSl, L::kSmemAlloc, s>>>(mq, mk, mv, p);
  return check_launch();
}

}  // namespace

bool sliding_tc_supported(int64_t window) { return window >= 1 && window <= 2 * kT - kT + 1; }

int launch_sliding_tc(const void *q, const void *k, const void *v, void *out, int64_t bh,
                      int64_t n, int64_t d_qk, int64_t window, const void *addend,
                      const DeviceInfo &info, cudaStream_t s) {
  if (!sliding_tc_supported(window) || (d_qk != 16 && d_qk != 64)) return LA_ERR_UNSUPPORTED;
  if (bh > 65535 || n > INT32_MAX - 2 * kT) return LA_ERR_UNSUPPORTED;
  SlidingParams p{};
  p.out = (__nv_bfloat16 *)out;
  p.addend = (const __nv_bfloat16 *)addend;
  p.err = device_error_word();
  p.n = n;
  p.tiles_per_head = (int)((n + kT - 1) / kT);
  p.tiles = bh * p.tiles_per_head;
  p.window = (int)window;
  p.scale_log2 = 1.4426950408889634f / (d_qk == 64 ? 8.0f : 4.0f);  // log2(e) / sqrt(d_qk)
  if (!p.err) return LA_ERR_CUDA;
  if (p.tiles == 0) return LA_OK;
  const int sms = info.sm_count > 0 ? info.sm_count : 1;
  const bool narrow = window <= kT / 2 + 1;
  if (d_qk == 64)
    return narrow ? launch<192, 64>(q, k, v, p, bh, sms, s) : launch<256, 64>(q, k, v, p, bh, sms, s);
  return narrow ? launch<192, 16>(q, k, v, p, bh, sms, s) : launch<256, 16>(q, k, v, p, bh, sms, s);
}

}  // namespace la
