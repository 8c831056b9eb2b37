// Sliding-window causal softmax attention on tcgen05 tensor cores (sm_100a).
//
// Fast path: bf16 q/k/v, head_dim 64, window W <= 129.  One CTA (4 warps)
// owns one (head, 128-query tile).  Its queries [q0, q0+128) see keys
// [q0 - W + 1, q0 + 127], which fit in one span of kSpan keys starting at
// k0 = q0 + 128 - kSpan (192 keys for W <= 65, 256 for W <= 129):
//
//   S   = Q K^T          tcgen05 M=128 N=kSpan K=64   -> TMEM (fp32)
//   P   = exp(S/8 - m)   CUDA cores, row max m over the row's window, masked
//                        to [max(0, i-W+1), i]; bf16 P written over S
//   O   = P V            tcgen05 M=128 N=64 K=kSpan   (A = P in TMEM)
//   out = O / sum(P)
//
// which is ref_sliding_window_attn (benchmarks/sliding_attention_benchmark.py:
// 32-56) and the NKI kernel of kernels/nki_attention_sliding.py:30-132
// (banded softmax, fp32 statistics) without its additive mask tensor: the
// band is computed from indices.  The whole band of a row is in one S tile,
// so the softmax needs no running rescale.  Q, K and V arrive by TMA in one
// transaction (keys before 0 and past n read as zero and are masked).  With
// kSpan = 192 a CTA holds 256 TMEM columns and 65 KB of shared memory, so two
// CTAs share an SM and one's loads overlap the other's math.
#include <utility>

#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

namespace la {
namespace {
using namespace tc;

constexpr int kT = 128;  // queries per tile
constexpr int kD = 64;   // head dim

template <int kSpan>
struct SlidingLayout {
  static constexpr uint32_t kOffQ = 0;                  // 128 rows x 128 B
  static constexpr uint32_t kOffK = kT * 128;           // kSpan rows x 128 B
  static constexpr uint32_t kOffV = kOffK + kSpan * 128;
  static constexpr uint32_t kOffBar = kOffV + kSpan * 128;
  // barriers, alignment slack; padded so that only as many CTAs share an SM
  // as its TMEM holds (two with 256 columns each, one with 512): a third
  // CTA's tcgen05.alloc would otherwise wait for a neighbour to finish
  static constexpr uint32_t kSmemUsed = kOffBar + 64 + 1024;
  static constexpr uint32_t kSmemFloor = kSpan + kD <= 256 ? 80 * 1024 : 120 * 1024;
  static constexpr uint32_t kSmemAlloc = kSmemUsed > kSmemFloor ? kSmemUsed : kSmemFloor;
  static constexpr uint32_t kColS = 0;                  // S / P: kSpan fp32 columns
  static constexpr uint32_t kColO = kSpan;              // O: 64 fp32 columns
  static constexpr uint32_t kTmemCols = kSpan + kD <= 256 ? 256 : 512;
  static constexpr uint32_t kLoadBytes = (kT + 2 * kSpan) * 128;
  static_assert(kOffK % 1024 == 0 && kOffV % 1024 == 0, "128B-swizzled tiles need 1024-byte alignment");
  static_assert(kLoadBytes < (1u << 20), "one TMA transaction count");
};

struct SlidingParams {
  __nv_bfloat16 *out;
  int *err;
  int64_t n;
  int window;
  float scale_log2;  // log2(e) / sqrt(head_dim)
};

enum SBar { kBarLoad, kBarS, kBarO, kNumSBars };

// bf16 pair {lo, hi} of two fp32 values (round to nearest even)
__device__ __forceinline__ uint32_t pack2(float lo, float hi) { return pack_bf16(lo, hi); }

template <int kSpan>
__global__ void __launch_bounds__(128)
sliding_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const SlidingParams p) {
  using L = SlidingLayout<kSpan>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + L::kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + L::kOffBar + 8 * kNumSBars);
  volatile int *abort_flag = (volatile int *)(smem + L::kOffBar + 8 * kNumSBars + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int q0 = blockIdx.x * kT;
  const int k0 = q0 + kT - kSpan;  // first key of the span (may be negative)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumSBars; ++i) mbar_init(&bars[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, L::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---------------------------------------------------------------- loads, S = Q K^T
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[kBarLoad], L::kLoadBytes);
    tma_load_3d(smem + L::kOffQ, &tm_q, &bars[kBarLoad], 0, q0, (int)bh);
    tma_load_3d(smem + L::kOffK, &tm_k, &bars[kBarLoad], 0, k0, (int)bh);
    tma_load_3d(smem + L::kOffV, &tm_v, &bars[kBarLoad], 0, k0, (int)bh);
    if (mbar_wait(&bars[kBarLoad], 0, abort_flag)) {
      tc_fence_after();
      constexpr uint32_t id_s = make_idesc_bf16(128, kSpan, false, false);
      const uint64_t qd = make_sdesc(sb + L::kOffQ, 16, 1024, kSwizzle128B);
      const uint64_t kd = make_sdesc(sb + L::kOffK, 16, 1024, kSwizzle128B);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk)  // K steps of 16 along the 128-byte rows
        umma_ss(tmem + L::kColS, qd + 2 * kk, kd + 2 * kk, id_s, kk > 0 ? 1u : 0u);
    }
    umma_commit(&bars[kBarS]);
  }

  // ---------------------------------------------------------------- softmax -> P
  // row r of the tile (query i = q0 + r) sees S columns [c_lo, c_hi]
  const int r = warp * 32 + lane;
  const int i = q0 + r;
  const bool row_ok = i < p.n;
  const int c_hi = r + kSpan - kT;
  const int c_lo = max(-k0, c_hi - p.window + 1);
  // columns any row of this warp may use: [w_lo, w_hi], loaded 16 at a time
  const int w_lo = max(0, warp * 32 + kSpan - kT - p.window + 1) & ~15;
  const int w_hi = warp * 32 + 31 + kSpan - kT;
  const int nchunk = (w_hi - w_lo) / 16 + 1;
  mbar_wait(&bars[kBarS], 0, abort_flag);
  __syncwarp();
  tc_fence_after();
  const uint32_t srow = taddr(tmem, warp * 32, L::kColS);
  float m = -INFINITY;
  for (int ch = 0; ch < nchunk; ++ch) {
    uint32_t x[16];
    tmem_ld16(srow + w_lo + 16 * ch, x);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int col = w_lo + 16 * ch + j;
      if (col >= c_lo && col <= c_hi) m = fmaxf(m, __uint_as_float(x[j]));
    }
  }
  const float mb = row_ok ? m * p.scale_log2 : 0.f;
  float l = 0.f;
  for (int ch = 0; ch < nchunk; ++ch) {
    uint32_t x[16], pk[8];
    tmem_ld16(srow + w_lo + 16 * ch, x);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = w_lo + 16 * ch + 2 * j;
      float e0 = exp2f(fmaf(__uint_as_float(x[2 * j]), p.scale_log2, -mb));
      float e1 = exp2f(fmaf(__uint_as_float(x[2 * j + 1]), p.scale_log2, -mb));
      e0 = (row_ok && col >= c_lo && col <= c_hi) ? e0 : 0.f;
      e1 = (row_ok && col + 1 >= c_lo && col + 1 <= c_hi) ? e1 : 0.f;
      l += e0 + e1;
      pk[j] = pack2(e0, e1);
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
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();

  // ---------------------------------------------------------------- O = P V
  if (threadIdx.x == 0) {
    tc_fence_after();
    constexpr uint32_t id_o = make_idesc_bf16(128, kD, false, true);
    const uint64_t vd = make_sdesc(sb + L::kOffV, 16, 1024, kSwizzle128B);
#pragma unroll
    for (int j = 0; j < kSpan / 16; ++j)  // 16 keys (2048 bytes of V) per step
      umma_ts(tmem + L::kColO, tmem + L::kColS + 8 * j, vd + (uint64_t)((j * 2048) >> 4), id_o,
              j > 0 ? 1u : 0u);
    umma_commit(&bars[kBarO]);
  }
  mbar_wait(&bars[kBarO], 0, abort_flag);
  __syncwarp();
  tc_fence_after();

  // ---------------------------------------------------------------- epilogue
  const float inv = l > 0.f ? 1.f / l : 0.f;
  const uint64_t inv2 = f2pack(inv, inv);
  uint32_t w[32];
  const uint32_t orow = taddr(tmem, warp * 32, L::kColO);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint32_t o[32];
    tmem_ld16(orow + 32 * h, o);
    tmem_ld16(orow + 32 * h + 16, o + 16);
    tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < 16; ++t)
      w[16 * h + t] = pack_bf16x2(fmul2(f2pack(__uint_as_float(o[2 * t]), __uint_as_float(o[2 * t + 1])), inv2));
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
      uint4 *dst = (uint4 *)(p.out + ((uint64_t)bh * p.n + rbase + j) * kD) + 2 * gi;
      asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                   "r"(w[8 * j]), "r"(w[8 * j + 1]), "r"(w[8 * j + 2]), "r"(w[8 * j + 3]),
                   "r"(w[8 * j + 4]), "r"(w[8 * j + 5]), "r"(w[8 * j + 6]), "r"(w[8 * j + 7])
                   : "memory");
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
}

template <int kSpan>
int launch(const void *q, const void *k, const void *v, const SlidingParams &p, int64_t bh,
           cudaStream_t s) {
  using L = SlidingLayout<kSpan>;
  CUtensorMap mq, mk, mv;
  if (!make_tmap_3d(&mq, q, bh, p.n, kD, kT, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&mk, k, bh, p.n, kD, kSpan, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_tmap_3d(&mv, v, bh, p.n, kD, kSpan, CU_TENSOR_MAP_SWIZZLE_128B))
    return LA_ERR_CUDA;
  if (cudaFuncSetAttribute(sliding_tc_kernel<kSpan>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           L::kSmemAlloc) != cudaSuccess)
    return LA_ERR_CUDA;
  dim3 grid((unsigned)((p.n + kT - 1) / kT), (unsigned)bh);
  sliding_tc_kernel<kSpan><<<grid, 128, L::kSmemAlloc, s>>>(mq, mk, mv, p);
  return check_launch();
}

}  // namespace

bool sliding_tc_supported(int64_t window) { return window >= 1 && window <= 2 * kT - kT + 1; }

int launch_sliding_tc(const void *q, const void *k, const void *v, void *out, int64_t bh,
                      int64_t n, int64_t window, const DeviceInfo &info, cudaStream_t s) {
  (void)info;
  if (!sliding_tc_supported(window)) return LA_ERR_UNSUPPORTED;
  if (bh > 65535 || n > INT32_MAX - 2 * kT) return LA_ERR_UNSUPPORTED;
  SlidingParams p{};
  p.out = (__nv_bfloat16 *)out;
  p.err = device_error_word();
  p.n = n;
  p.window = (int)window;
  p.scale_log2 = 1.4426950408889634f / 8.0f;  // log2(e) / sqrt(64)
  if (!p.err) return LA_ERR_CUDA;
  return window <= kT / 2 + 1 ? launch<192>(q, k, v, p, bh, s) : launch<256>(q, k, v, p, bh, s);
}

}  // namespace la
