// Chunked recurrent BASED attention on tcgen05 tensor cores (sm_100a).
//
// Fast path: bf16 q/k/v, d_qk = 16, d_v = 64.  One CTA owns one (head,
// segment) and walks its tokens in 128-token tiles.  Per tile c (Q, K, V are
// the tile's rows, S_c the fp32 state of all earlier tokens, phi the Taylor
// feature map in the query/key-split basis of include/la_attention.h):
//
//   S^T   += [V 1 0]^T phi(K)       tcgen05 M=128 N=160 K=128  (fp32 state in TMEM)
//   O      = phi(Q) S_c             tcgen05 M=128 N=80  K=160  (A = phi(Q) in TMEM,
//                                                               B = bf16 snapshot of S_c)
//   scores = Q K^T                  tcgen05 M=128 N=128 K=16   -> TMEM
//   P      = tril(1 + s/4 + s^2/32) CUDA cores, bf16 P written over its scores
//   O     += P [V 1]                tcgen05 M=128 N=80  K=128  (A = P in TMEM)
//   out    = O[:, :64] / (O[:, 64] + eps)
//
// which is the reference recurrence of kernels/nki_attention_chunked.py:71-109
// (acc_o = Q_phi S; scores = Q_phi K_phi^T; S += K_phi^T V; acc_o +=
// tril(scores) V) with the intra-tile term evaluated in the equivalent
// polynomial form 1 + s + s^2/2 and the normaliser carried both as state row
// 64 (z = sum phi(k)) and as the ones column of [V 1] (the row sum of P).
// The 153 features never touch HBM: each token's phi(Q) is expanded in
// registers and stored to TMEM, its phi(K) to shared memory, by a thread that
// owns the token.
//
// A thread pays ~100 cycles to issue one M=128, K=16 tcgen05.mma (measured:
// one thread issues no faster than one per ~100-150 cycles, longer than an
// N <= 160 MMA runs), and ~90 per tcgen05.commit, so two threads issue: one
// the state updates UP(c), the other QS(c), PV(c) and the scores of tile
// c+1.  (Giving QS, PV and the scores a thread each, with P in its own TMEM
// columns, was measured 9% slower.)  The state snapshot and phi(K) of tile
// c+1 are produced while QS(c) and PV(c) run, phi(Q) of tile c+1 (by the
// epilogue warps, before they store the output of tile c) while PV(c) runs,
// and P of tile c+1 while UP(c+1) and QS(c+1) run.
//
// Warp roles (800 threads, one CTA per SM):
//   warp 19     TMA producer: Q/K tiles (2-stage ring) and V tiles (3-stage ring)
//   warp 23     TMEM allocator + update MMA issuer (S^T += ...)
//   warp 24     output MMA issuer (phi(Q) S, P [V 1], scores)
//   warps 0-3   features: phi(K) -> smem (2 buffers)
//   warps 4-11  polynomial: scores -> P (TMEM); two warps per TMEM lane quarter
//   warps 16-18, 20-22  state: S^T (TMEM, fp32) -> bf16 snapshot in smem (2
//               buffers); lane quarters 0-2 (S^T rows >= 96 are always zero),
//               two warps per quarter, 80 feature columns each
//   warps 12-15 epilogue: phi(Q) of tile c+1 -> TMEM, then O of tile c
//               (TMEM) -> normalised bf16 output rows
//
// The state-only variant (kStateOnly) runs just the phi(K) / update path and
// writes the segment's state; it seeds the later segments of a head.
#include <mutex>
#include <utility>

#include "tc_common.cuh"
#include "tc_kernels.cuh"
#include "tma_host.cuh"

namespace la {
namespace {
using namespace tc;

constexpr int kT = 128;       // tokens per tile
constexpr int kDqk = 16;
constexpr int kDv = 64;
constexpr int kF = 153;       // 1 + 16 + 136 features
constexpr int kFPad = 160;    // padded feature count (K of phi(Q) S, N of the update)
constexpr int kSV = kDv + 1;  // state columns in global memory: values + normaliser
constexpr int kNO = 80;       // N of phi(Q) S: 64 values, normaliser, 15 zero rows

// Warp roles.  A warp reaches the TMEM lanes of quarter warp % 4 only, so
// the TMEM roles come in sets that cover the quarters they need; the three
// single-thread roles fill the remaining slots.  (The register file is split
// between the four schedulers; 25 warps put 7 on one of them, which leaves 72
// registers per thread.)
constexpr int kWarpFeat = 0;     // 0..3    features
constexpr int kWarpPoly = 4;     // 4..11   polynomial (two warps per quarter)
constexpr int kWarpEpi = 12;     // 12..15  epilogue
constexpr int kWarpState0 = 16;  // 16..18  state, columns 0..79 (quarters 0..2)
constexpr int kWarpTma = 19;     //         TMA producer (Q/K and V rings)
constexpr int kWarpState1 = 20;  // 20..22  state, columns 80..159 (quarters 0..2)
constexpr int kWarpUpd = 23;     //         TMEM allocator + update MMA issuer
constexpr int kWarpOut = 24;     //         output MMA issuer
constexpr int kThreads = 25 * 32;
constexpr int kStateThreads = 6 * 32;

// TMEM columns (one CTA per SM owns all 512)
constexpr uint32_t kColS = 0;       // S^T    128 lanes x 160 fp32
constexpr uint32_t kColO = 160;     // O      128 lanes x 80 fp32
constexpr uint32_t kColPhiQ = 256;  // phi(Q) 128 lanes x 80 bf16 pairs
constexpr uint32_t kColSc = 384;    // scores 128 fp32 / P 64 bf16 pairs
constexpr uint32_t kTmemCols = 512;

// Shared memory (offsets from a 1024-byte aligned base)
constexpr uint32_t kQBytes = kT * kDqk * 2;         // 4 KB, 32B-swizzled rows
constexpr uint32_t kVBytes = kT * kDv * 2;          // 16 KB, 128B-swizzled rows
// phi(K): the MN-major B operand of the update, 64B-swizzled rows of 32
// features (5 blocks of 128 tokens x 64 B hold the 160 feature slots exactly;
// 128B rows would leave half of a third 64-feature block empty)
constexpr uint32_t kPhiBlock = kT * 64;             // 32 features of 128 tokens
constexpr uint32_t kPhiBytes = 5 * kPhiBlock;       // 160 features (5 blocks)
// Snapshots of S: the K-major B operand of phi(Q) S, 80 rows x 160 features
// in three 64-feature blocks of 80 x 128 B.  (Letting the two buffers share
// their half-used third block was measured 19% slower: the state warps then
// store into 128-byte rows the tensor core is reading.)
constexpr uint32_t kSnapKBlock = kNO * 128;         // 10 KB per 64-feature block
constexpr uint32_t kSnapBytes = 3 * kSnapKBlock;
constexpr int kMaxStages = 6;

// Shared-memory layout (offsets from a 1024-byte aligned base).  The full
// kernel: Q/K ring (2 stages), V ring (3), ones block, phi(K) x 2, snapshots
// x 2.  The state-only kernel needs no Q, phi(Q) or snapshots and spends the
// room on deeper K and V rings, since nothing else hides its load latency.
template <bool kStateOnly>
struct Layout {
  // (full kernel: a Q/K copy takes ~2,200 cycles to land under load and its
  // stage is released only by the scores MMA of its tile, late in the
  // tile, so both rings are several tiles deep)
  static constexpr int kQKStages = kStateOnly ? 6 : 4;
  static constexpr int kVStages = kStateOnly ? 6 : 3;
  static constexpr uint32_t kOffQ = 0;
  static constexpr uint32_t kOffK = kOffQ + (kStateOnly ? 0 : kQKStages * kQBytes);
  static constexpr uint32_t kOffV = kOffK + kQKStages * kQBytes;
  static constexpr uint32_t kOffOnes = kOffV + kVStages * kVBytes;  // 16 rows x 128 B
  static constexpr uint32_t kOffPhiK = kOffOnes + 2048;
  static constexpr uint32_t kOffSnap = kOffPhiK + 2 * kPhiBytes;
  static constexpr uint32_t kOffBar = kOffSnap + (kStateOnly ? 0 : 2 * kSnapBytes);
  static constexpr uint32_t kOffSlot = kOffBar + 512;            // slot map (kFPad shorts)
  static constexpr uint32_t kSmemAlloc = kOffSlot + 512 + 1024;  // + alignment slack
  static_assert(kQKStages <= kMaxStages && kVStages <= kMaxStages, "barrier slots");
  static_assert(kOffV % 1024 == 0 && kOffOnes % 1024 == 0 && kOffPhiK % 1024 == 0 &&
                    kPhiBytes % 1024 == 0 && kOffSnap % 1024 == 0 && kSnapKBlock % 1024 == 0,
                "128B-swizzled regions need 1024-byte alignment");
  static_assert(kSmemAlloc <= 227 * 1024, "shared memory budget");
};

// Barriers.  Ring stages have their own full/empty pairs; per-buffer pairs
// (..0/..1) complete once per two tiles (a producer that may run two tiles
// ahead of its consumer needs them).
enum Bar { kQKFull = 0, kQKEmpty = kQKFull + kMaxStages, kVFull = kQKEmpty + kMaxStages,
           kVEmpty = kVFull + kMaxStages, kPhiKReady0 = kVEmpty + kMaxStages, kPhiKReady1,
           kUpDone0, kUpDone1, kQSDone0, kQSDone1, kSnapReady0, kSnapReady1, kSRead, kPhiQReady, kScReady,
           kPReadyLo, kPReadyHi, kOReady, kOFree, kSReady, kDone, kNumBars };
static_assert(8 * kNumBars + 12 <= 512, "barrier area");

// Optional per-role timeline of CTA (0, 0), compiled in with -DLA_TRACE only.
#ifdef LA_TRACE
constexpr int kTraceChunks = 32, kTraceEvents = 8;
constexpr int kTraceMaxCtas = 128;
__device__ long long la_trace_buf[kTraceMaxCtas][6][kTraceChunks][kTraceEvents];
constexpr int kTraceCtas = 4096;
__device__ long long la_trace_cta[kTraceCtas][5];  // start ns, end ns, SM id, start clk, end clk
#define LA_TRACE_AT(role, chunk, ev)                                                   \
  do {                                                                                \
    if (blockIdx.x == 0 && blockIdx.y < kTraceMaxCtas && (chunk) < kTraceChunks && (threadIdx.x & 31) == 0) \
      la_trace_buf[blockIdx.y][role][chunk][ev] = clock64();                          \
  } while (0)
#else
#define LA_TRACE_AT(role, chunk, ev) \
  do {                               \
  } while (0)
#endif

// Feature slots.  S^T's columns, phi(K)'s smem columns and phi(Q)'s TMEM
// columns hold the 153 features of the query/key-split basis in the order
// below ("slots", two per bf16x2 pair), chosen so that almost every pair is a
// single bf16x2 product of an input word (x_b, x_b+1) and a broadcast x_a:
//   pairs 0..7    x_2i, x_2i+1                      (linear)
//   pair  8       1, 0                              (constant, padding)
//   pairs 9..44   x_a x_2j, x_a x_2j+1   a even, 2j >= a      (36 pairs)
//   pairs 45..72  x_a x_2j, x_a x_2j+1   a odd,  2j >  a      (28 pairs)
//   pairs 73..76  x_a^2, x_a'^2          a, a' = (1,3) (5,7) (9,11) (13,15)
//   pairs 77..79  0, 0                                        (padding)
// In HBM the state keeps the documented order [1, x_0..x_15, x_a x_b (a <= b)
// row-major]; slot_feature() maps a slot to it.
// Scales: key side unscaled; query side x_a / 4 (linear), x_a x_b / 16
// (a < b), x_a^2 / 32.  All are exact power-of-two rescalings of bf16 inputs,
// and a bf16 product of bf16 operands rounds the exact product once, so every
// feature equals the fp32 product rounded to bf16.
enum : int { kPairLin, kPairConst, kPairEven, kPairOdd, kPairDiag, kPairPad };
struct PairDesc {
  int type, a, b;  // kPairEven / kPairOdd: row a, word b; kPairDiag: rows a, b; kPairLin: word a
};
__host__ __device__ constexpr PairDesc pair_desc(int p) {
  if (p < 8) return {kPairLin, p, 0};
  if (p == 8) return {kPairConst, 0, 0};
  int q = p - 9;
  for (int a = 0; a < kDqk; a += 2) {  // even rows: words a/2 .. 7
    const int n = 8 - a / 2;
    if (q < n) return {kPairEven, a, a / 2 + q};
    q -= n;
  }
  for (int a = 1; a < kDqk; a += 2) {  // odd rows: words (a+1)/2 .. 7
    const int n = 8 - (a + 1) / 2;
    if (q < n) return {kPairOdd, a, (a + 1) / 2 + q};
    q -= n;
  }
  if (q < 4) return {kPairDiag, 4 * q + 1, 4 * q + 3};
  return {kPairPad, 0, 0};
}
// index of x_a x_b (a <= b) in the documented order
__host__ __device__ constexpr int quad_feature(int a, int b) {
  return 1 + kDqk + a * kDqk - a * (a - 1) / 2 + (b - a);
}
// documented feature index of slot s, or -1 for a padding slot
__host__ __device__ constexpr int slot_feature(int s) {
  const PairDesc d = pair_desc(s >> 1);
  const int h = s & 1;
  switch (d.type) {
    case kPairLin: return 1 + 2 * d.a + h;
    case kPairConst: return h ? -1 : 0;
    case kPairEven:
    case kPairOdd: return quad_feature(d.a, 2 * d.b + h);
    case kPairDiag: return h ? quad_feature(d.b, d.b) : quad_feature(d.a, d.a);
    default: return -1;
  }
}
struct alignas(16) SlotMap {
  short f[kFPad];
};
static_assert(sizeof(SlotMap) <= 512 && kFPad % 2 == 0, "slot map area");
__host__ __device__ constexpr SlotMap make_slot_map() {
  SlotMap m{};
  for (int s = 0; s < kFPad; ++s) m.f[s] = (short)slot_feature(s);
  return m;
}
__host__ __device__ constexpr bool slot_map_is_bijection() {
  int seen[kF] = {};
  for (int s = 0; s < kFPad; ++s) {
    const int f = slot_feature(s);
    if (f >= kF) return false;
    if (f >= 0) ++seen[f];
  }
  for (int f = 0; f < kF; ++f)
    if (seen[f] != 1) return false;
  return pair_desc(79).type == kPairPad && pair_desc(76).type == kPairDiag &&
         pair_desc(77).type == kPairPad;
}
static_assert(slot_map_is_bijection(), "every feature has exactly one slot");
// In global memory: each CTA copies it to shared memory at start (a uniform
// read of constant memory per slot costs a constant-cache miss per line and
// serialises; the copy is one coalesced load).
__device__ const SlotMap g_slot_map = make_slot_map();
// Identity feature map (phi(x) = x): slots 0..15 are x_0..x_15, the linear
// pairs 0..7 of the Taylor order, and every other slot is padding.  Its state
// keeps the d_qk features in input order.
__host__ __device__ constexpr SlotMap make_identity_slot_map() {
  SlotMap m{};
  for (int s = 0; s < kFPad; ++s) m.f[s] = (short)(s < kDqk ? s : -1);
  return m;
}
__device__ const SlotMap g_identity_slot_map = make_identity_slot_map();
// Feature slots the identity map uses: one 32-slot block of phi(K) (N of the
// update), two K-steps of phi(Q) S
constexpr int kIdSlots = 32;

// A token's inputs as bf16x2 words (x_2i lo, x_2i+1 hi): raw, and (query side)
// divided by 16 and by 32.  `one` is {1, 0}, or 0 for a padding key.
struct FeatIn {
  uint32_t w[8], s16[8], s32[8];
  uint32_t one;
};
template <bool kQ, int P>
__device__ __forceinline__ uint32_t pair_val(const FeatIn &s) {
  constexpr PairDesc d = pair_desc(P);
  if constexpr (d.type == kPairLin) {
    return kQ ? hmul2_bf16(s.w[d.a], 0x3E803E80u) : s.w[d.a];  // query side: x / 4
  } else if constexpr (d.type == kPairConst) {
    return s.one;
  } else if constexpr (d.type == kPairEven) {
    // row a even: x_a is the low half of word a/2; the diagonal pair of a
    // query row scales x_a^2 by 1/32 and x_a x_a+1 by 1/16
    uint32_t A;
    if constexpr (!kQ) A = bf16_pair<0, 0>(s.w[d.a >> 1], s.w[d.a >> 1]);
    else if constexpr (d.b == d.a / 2) A = bf16_pair<0, 0>(s.s32[d.a >> 1], s.s16[d.a >> 1]);
    else A = bf16_pair<0, 0>(s.s16[d.a >> 1], s.s16[d.a >> 1]);
    return hmul2_bf16(A, s.w[d.b]);
  } else if constexpr (d.type == kPairOdd) {
    const uint32_t x = kQ ? s.s16[d.a >> 1] : s.w[d.a >> 1];
    return hmul2_bf16(bf16_pair<1, 1>(x, x), s.w[d.b]);
  } else if constexpr (d.type == kPairDiag) {
    const uint32_t X = bf16_pair<1, 1>(s.w[d.a >> 1], s.w[d.b >> 1]);
    const uint32_t A = kQ ? bf16_pair<1, 1>(s.s32[d.a >> 1], s.s32[d.b >> 1]) : X;
    return hmul2_bf16(A, X);
  } else {
    return 0u;
  }
}

// A feature pair under either map: the identity map keeps the linear pairs
// (x_2i, x_2i+1; x / 4 on the query side, the 1/sqrt(d_qk) of its scores)
// and zeroes the rest.
template <bool kIdentity, bool kQ, int P>
__device__ __forceinline__ uint32_t feature_pair(const FeatIn &s) {
  if constexpr (kIdentity && pair_desc(P).type != kPairLin) return 0u;
  else return pair_val<kQ, P>(s);
}

// Slots 8J .. 8J+7 (pairs 4J .. 4J+3, one 16-byte chunk) of token `row` ->
// 64B-swizzled smem, 32 slots per 8 KB block: the MN-major B layout of
// phi(K) for the update MMA.
template <bool kIdentity, int J>
__device__ __forceinline__ void store_phik_chunk(const FeatIn &s, uint32_t base, int row) {
  st_shared_v4(base + (J >> 2) * kPhiBlock + sw64_offset(row, J & 3),
               feature_pair<kIdentity, false, 4 * J + 0>(s),
               feature_pair<kIdentity, false, 4 * J + 1>(s),
               feature_pair<kIdentity, false, 4 * J + 2>(s),
               feature_pair<kIdentity, false, 4 * J + 3>(s));
}
template <bool kIdentity, int... J>
__device__ __forceinline__ void store_phik(const FeatIn &s, uint32_t base, int row,
                                           std::integer_sequence<int, J...>) {
  (store_phik_chunk<kIdentity, J>(s, base, row), ...);
}

// phi(Q) TMEM columns [16G, 16G+16) = pairs 16G .. 16G+15 of TMEM lane `row`
template <bool kIdentity, int G, int... I>
__device__ __forceinline__ void store_phiq_group(const FeatIn &s, uint32_t addr,
                                                 std::integer_sequence<int, I...>) {
  const uint32_t w[16] = {feature_pair<kIdentity, true, 16 * G + I>(s)...};
  tmem_st16(addr, w);
}
template <bool kIdentity, int... G>
__device__ __forceinline__ void store_phiq(const FeatIn &s, uint32_t addr0,
                                           std::integer_sequence<int, G...>) {
  (store_phiq_group<kIdentity, G>(s, addr0 + 16 * G, std::make_integer_sequence<int, 16>{}),
   ...);
}

// Shared-memory address of the 16-byte chunk holding features f0 .. f0+7
// (f0 a multiple of 8) of snapshot row e in buffer `buf`.
__device__ __forceinline__ uint32_t snap_chunk_addr(uint32_t sb, int buf, int f0, int e) {
  return sb + Layout<false>::kOffSnap + buf * kSnapBytes + (f0 >> 6) * kSnapKBlock +
         sw128_offset(e, (f0 & 63) >> 3);
}

struct Params {
  __nv_bfloat16 *out;
  const float *init_state;  // (bh, F, 65) or null
  float *final_state;       // (bh, F, 65) or null (written by the last segment)
  const float *seg_states;  // (bh, G, F, 65): states of earlier segments (output pass)
  float *seg_out;           // (bh, G, F, 65): this segment's state (state pass)
  int *err;                 // device error word
  int64_t n;
  int64_t seg_len;
  int64_t lead_len;         // > 0: lead/main split (output pass: grid (bh, 2))
  int segments;             // segment count (the per-head stride of seg_states)
  float eps;
  int normalize;
};

__device__ __forceinline__ bool wait_teardown(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  return true;
}

// kIdentity: the identity feature map (numerator only): phi(K) and phi(Q)
// hold the 16 linear slots, the update runs at N = 32, phi(Q) S at K = 32 and
// P = tril(s / 4).
template <bool kStateOnly, bool kIdentity>
__global__ void __launch_bounds__(kThreads, 1)
chunked_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using L = Layout<kStateOnly>;
  constexpr int kQKStages = L::kQKStages, kVStages = L::kVStages;
  // features per head in global memory, feature slots the MMAs span
  constexpr int kFeat = kIdentity ? kDqk : kF;
  constexpr int kSlots = kIdentity ? kIdSlots : kFPad;
  constexpr uint32_t kOffQ = L::kOffQ, kOffK = L::kOffK, kOffV = L::kOffV, kOffOnes = L::kOffOnes,
                     kOffPhiK = L::kOffPhiK, kOffSnap = L::kOffSnap, kOffBar = L::kOffBar,
                     kOffSlot = L::kOffSlot;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  uint64_t *bars = (uint64_t *)(smem + kOffBar);
  uint32_t *tmem_slot = (uint32_t *)(smem + kOffBar + 8 * kNumBars);
  volatile int *abort_flag = (volatile int *)(smem + kOffBar + 8 * kNumBars + 4);
  volatile int *up_issued = (volatile int *)(smem + kOffBar + 8 * kNumBars + 8);
  const short *slot_map = (const short *)(smem + kOffSlot);  // slot -> feature (or -1)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Equal segments: grid (segments, bh), segment g covers [g seg_len, (g+1) seg_len).
  // Lead/main split: grid (bh, 2); y = 0 is the main piece [lead_len, n) (g = 1,
  // dispatched first), y = 1 the lead piece [0, lead_len) (g = 0).
  const bool split = p.lead_len > 0;
  const int g = split ? (blockIdx.y == 0 ? 1 : 0) : (int)blockIdx.x;
  const int64_t bh = split ? blockIdx.x : blockIdx.y;
  const int64_t t_begin = split ? (g ? p.lead_len : 0) : (int64_t)g * p.seg_len;
  const int64_t t_end = split ? (g ? p.n : p.lead_len) : min64(p.n, t_begin + p.seg_len);
  const int last_g = split ? 1 : p.segments - 1;
  const int n_chunks = (int)((t_end - t_begin + kT - 1) / kT);

#ifdef LA_TRACE
  if (threadIdx.x == 0 && !kStateOnly && blockIdx.y * gridDim.x + blockIdx.x < kTraceCtas) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    la_trace_cta[blockIdx.y * gridDim.x + blockIdx.x][0] = (long long)globaltimer();
    la_trace_cta[blockIdx.y * gridDim.x + blockIdx.x][2] = smid;
    la_trace_cta[blockIdx.y * gridDim.x + blockIdx.x][3] = clock64();
  }
#endif
  if (threadIdx.x == 0) {
    // every barrier: one arrival (a leader thread, a TMA expect-tx or a
    // tcgen05.commit), except: a Q/K stage is released by the phi(K) warps
    // and (full kernel) the phi(Q) warps and a polynomial warp once the
    // scores are done, a V stage by the update and (full kernel) P V,
    // `done` by both MMA issuers, each half of P by the four lane quarters'
    // polynomial warp pairs
    for (int i = 0; i < kNumBars; ++i) {
      uint32_t count = 1;
      if (i >= kQKEmpty && i < kQKEmpty + kMaxStages) count = kStateOnly ? 1 : 3;
      if (i >= kVEmpty && i < kVEmpty + kMaxStages) count = 2;
      if ((i == kUpDone0 || i == kUpDone1) && kStateOnly) count = 2;
      if (i == kDone) count = 2;
      if (i == kPReadyLo || i == kPReadyHi) count = 4;  // one polynomial warp pair per quarter
      mbar_init(&bars[i], count);
    }
    *abort_flag = 0;
    *up_issued = 0;
    fence_barrier_init();
    // the output pass that follows a state pass may take SMs as they free up
    if (kStateOnly) grid_dependents_launch();
  }
  if (threadIdx.x < kFPad / 2)
    ((uint32_t *)(smem + kOffSlot))[threadIdx.x] =
        ((const uint32_t *)(kIdentity ? g_identity_slot_map.f : g_slot_map.f))[threadIdx.x];
  // constant "ones" block: A-operand rows 64..127 of [V 1 0]^T for 16 tokens;
  // row 64 (element 0 of each token row, 128B-swizzled) is 1, the rest 0.
  for (int i = threadIdx.x; i < 2048 / 4; i += kThreads) {
    const int row = (i * 4) / 128, byte = (i * 4) % 128;
    const uint32_t one = (byte == (row & 7) * 16) ? 0x3F80u : 0u;
    *(uint32_t *)(smem + kOffOnes + i * 4) = one;
  }
  if (warp == kWarpUpd) tmem_alloc(tmem_slot, kTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kWarpTma) {
    // ------------------------------------------------------------ TMA producer
    // One thread feeds both rings, each released by its own consumers: it
    // issues whichever next copy has a free stage, so K can run ahead of V.
    if (lane == 0) {
      LA_TRACE_AT(5, 0, 2);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      if (!kStateOnly) prefetch_tmap(&tm_q);
      int cq = 0, cv = 0;  // next tiles to load
      uint64_t t_idle = globaltimer();
      while ((cq < n_chunks || cv < n_chunks) && !*abort_flag) {
        bool progress = false;
        if (cq < n_chunks) {
          const int st = cq % kQKStages, round = cq / kQKStages;
          if (round == 0 || mbar_try_wait(&bars[kQKEmpty + st], (round - 1) & 1)) {
            const int row = (int)(t_begin + (int64_t)cq * kT);
            LA_TRACE_AT(5, cq, 0);
            mbar_arrive_expect_tx(&bars[kQKFull + st], kStateOnly ? kQBytes : 2 * kQBytes);
            if (!kStateOnly)
              tma_load_3d(smem + kOffQ + st * kQBytes, &tm_q, &bars[kQKFull + st], 0, row, (int)bh);
            tma_load_3d(smem + kOffK + st * kQBytes, &tm_k, &bars[kQKFull + st], 0, row, (int)bh);
            ++cq;
            progress = true;
          }
        }
        if (cv < n_chunks) {
          const int st = cv % kVStages, round = cv / kVStages;
          if (round == 0 || mbar_try_wait(&bars[kVEmpty + st], (round - 1) & 1)) {
            const int row = (int)(t_begin + (int64_t)cv * kT);
            LA_TRACE_AT(5, cv, 1);
            mbar_arrive_expect_tx(&bars[kVFull + st], kVBytes);
            tma_load_3d(smem + kOffV + st * kVBytes, &tm_v, &bars[kVFull + st], 0, row, (int)bh);
            ++cv;
            progress = true;
          }
        }
        if (progress) {
          t_idle = globaltimer();
        } else {
          __nanosleep(64);
          if (globaltimer() - t_idle > kWaitTimeoutNs) *abort_flag = 1;
        }
      }
      // every issued copy must land before the CTA can exit
      for (int c = cq - kQKStages < 0 ? 0 : cq - kQKStages; c < cq; ++c)
        wait_teardown(&bars[kQKFull + c % kQKStages], (c / kQKStages) & 1);
      for (int c = cv - kVStages < 0 ? 0 : cv - kVStages; c < cv; ++c)
        wait_teardown(&bars[kVFull + c % kVStages], (c / kVStages) & 1);
    }
  } else if (warp == kWarpUpd || warp == kWarpOut) {
    // ------------------------------------------------------------ MMA issuers
    // Two warps issue into the same tensor pipe so each one's commits and
    // waits hide behind the other's MMAs:
    //   update issuer (warp 23): S^T += [V 1 0]^T phi(K) for every tile;
    //   output issuer (warp 24): per tile O = phi(Q) S_c, O += P [V 1], then
    //                            the scores of the next tile.
    // Each warp runs its loop converged (every lane waits, the warp agrees on
    // the outcome) and one elected lane issues the MMAs and their commits.
    constexpr uint32_t id_sc = make_idesc_bf16(128, 128, false, false);
    constexpr uint32_t id_qs = make_idesc_bf16(128, kNO, false, false);
    constexpr uint32_t id_pv = make_idesc_bf16(128, kNO, false, true);
    constexpr uint32_t id_up = make_idesc_bf16(128, kSlots, true, true);
    // a K-step of 16 tokens: start address +2048 B, LBO (distance to the ones block) -2048 B
    constexpr uint64_t kStep = (uint64_t)(2048 >> 4) - ((uint64_t)(2048 >> 4) << 16);
    const uint32_t a_ones = sb + kOffOnes;
    // The state-only kernel has no other MMAs, so its updates are split over
    // both issuing warps: tokens 0..63 of each tile into S^T, tokens 64..127
    // into a second accumulator (the full kernel's O columns) that starts at
    // zero; the two are summed when the state is written out.
    auto update_loop = [&](int j0, int j1, uint32_t dcol, bool second) {
      for (int c = 0; c < n_chunks; ++c) {
        const int b = c & 1;          // phi(K) buffer
        const int sv = c % kVStages;  // V stage
        if (!mbar_wait_warp(&bars[kVFull + sv], (c / kVStages) & 1, abort_flag)) break;
        LA_TRACE_AT(0, c, 7);
        if (!mbar_wait_warp(&bars[kPhiKReady0 + b], (c >> 1) & 1, abort_flag)) break;
        // S^T may change once the state warps have read S_c out of it
        if (!second && (c == 0 || !kStateOnly) &&
            !mbar_wait_warp(&bars[kSRead], c & 1, abort_flag))
          break;
        tc_fence_after();
        LA_TRACE_AT(0, c, 0);
        const uint32_t v_base = sb + kOffV + sv * kVBytes;
        // phi(K): 32-feature blocks kPhiBlock apart (LBO), 8-token groups 512 B
        // apart (SBO); a K-step of 16 tokens advances 1024 B
        const uint64_t db0 = make_sdesc(sb + kOffPhiK + b * kPhiBytes, kPhiBlock, 512, kSwizzle64B);
        const uint64_t da0 = make_sdesc(v_base, a_ones - v_base, 1024, kSwizzle128B);
        if (elect_one()) {
#pragma unroll
          for (int j = j0; j < j1; ++j)
            umma_ss(tmem + dcol, da0 + kStep * j, db0 + (uint64_t)((j * 1024) >> 4), id_up,
                    (second && c == 0 && j == j0) ? 0u : 1u);
          if (!kStateOnly) umma_commit(&bars[kSReady]);
          umma_commit(&bars[kUpDone0 + b]);
          umma_commit(&bars[kVEmpty + sv]);
          if (!second) *up_issued = c + 1;  // the state update of tile c is in the pipe
        }
        __syncwarp();
      }
      if (elect_one()) umma_commit(&bars[kDone]);
      __syncwarp();
    };
    if (warp == kWarpUpd) {
      update_loop(0, kStateOnly ? kT / 32 : kT / 16, kColS, false);
    } else if (kStateOnly) {
      update_loop(kT / 32, kT / 16, kColO, true);
    } else {
      const uint64_t qs_b_desc0 = make_sdesc(sb + kOffSnap, 16, 1024, kSwizzle128B);
      const uint64_t qs_b_desc1 = make_sdesc(sb + kOffSnap + kSnapBytes, 16, 1024, kSwizzle128B);
      auto issue_scores = [&](int c) {
        const int s = c % kQKStages;
        const uint64_t da = make_sdesc(sb + kOffQ + s * kQBytes, 16, 256, kSwizzle32B);
        const uint64_t db = make_sdesc(sb + kOffK + s * kQBytes, 16, 256, kSwizzle32B);
        // (the polynomial warps release the Q/K stage once they have seen
        // the scores complete: one commit fewer on this issuer's chain)
        if (elect_one()) {
          umma_ss(tmem + kColSc, da, db, id_sc, 0);
          umma_commit(&bars[kScReady]);
        }
        __syncwarp();
      };
      bool ok = mbar_wait_warp(&bars[kQKFull], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_scores(0);
      }
      for (int c = 0; ok && c < n_chunks; ++c) {
        const int b = c & 1;
        // O = phi(Q) S_c   (K = 160 features in 10 steps; S_c is snapshot b).
        // Its four conditions have usually all been met by the time this
        // warp gets here: test them together first, and wait on them one by
        // one only if one is still open.
        const bool ready = mbar_test_wait(&bars[kPhiQReady], c & 1) &&
                           mbar_test_wait(&bars[kSnapReady0 + b], (c >> 1) & 1) &&
                           (c == 0 || mbar_test_wait(&bars[kOFree], (c - 1) & 1)) &&
                           *up_issued >= c + 1;
        if (!__all_sync(0xffffffffu, ready)) {
          if (!mbar_wait_warp(&bars[kPhiQReady], c & 1, abort_flag)) break;
          LA_TRACE_AT(0, c, 4);
          if (!mbar_wait_warp(&bars[kSnapReady0 + b], (c >> 1) & 1, abort_flag)) break;
          LA_TRACE_AT(0, c, 5);
          if (c > 0 && !mbar_wait_warp(&bars[kOFree], (c - 1) & 1, abort_flag)) break;
          LA_TRACE_AT(0, c, 6);
          // let the update of tile c enter the pipe first: the next snapshot,
          // and so the next tile, waits on it
          if (!__all_sync(0xffffffffu, spin_until_at_least(up_issued, c + 1, abort_flag))) break;
        }
        tc_fence_after();
        LA_TRACE_AT(0, c, 1);
        const uint64_t qs_b_desc = b ? qs_b_desc1 : qs_b_desc0;
        if (elect_one()) {
#pragma unroll
          for (int j = 0; j < kSlots / 16; ++j) {
            const uint32_t boff = (j >> 2) * kSnapKBlock + (j & 3) * 32;
            umma_ts(tmem + kColO, tmem + kColPhiQ + 8 * j, qs_b_desc + (boff >> 4), id_qs,
                    j > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kQSDone0 + b]);
        }
        __syncwarp();
        // O += P [V 1]: B = V (64 columns) with the ones block as its second
        // 64-column block (LBO), so O[:, 64] also collects the row sum of P.
        // P arrives in two halves (keys 0..63, then 64..127): the first
        // half's MMAs run while the polynomial warps finish the second.
        const int sv = c % kVStages;
        if (!mbar_wait_warp(&bars[kVFull + sv], (c / kVStages) & 1, abort_flag)) break;
        const uint32_t v_base = sb + kOffV + sv * kVBytes;
        const uint64_t db0 = make_sdesc(v_base, a_ones - v_base, 1024, kSwizzle128B);
        bool pv_ok = true;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait_warp(&bars[h ? kPReadyHi : kPReadyLo], c & 1, abort_flag)) {
            pv_ok = false;
            break;
          }
          tc_fence_after();
          if (h == 0) LA_TRACE_AT(0, c, 2);
          if (elect_one()) {
#pragma unroll
            for (int j = 4 * h; j < 4 * h + 4; ++j)
              umma_ts(tmem + kColO, tmem + kColSc + 8 * j, db0 + kStep * j, id_pv, 1u);
            if (h == 1) umma_commit(&bars[kOReady]);
          }
          __syncwarp();
        }
        if (!pv_ok) break;
        // the scores of tile c+1 overwrite P(c): wait for P V to finish;
        // that also ends this issuer's use of TMA stage b
        if (!mbar_wait_warp(&bars[kOReady], c & 1, abort_flag)) break;
        if (lane == 0) mbar_arrive(&bars[kVEmpty + sv]);
        LA_TRACE_AT(0, c, 3);
        if (c + 1 < n_chunks) {
          const int c1 = c + 1;
          if (!mbar_wait_warp(&bars[kQKFull + c1 % kQKStages], (c1 / kQKStages) & 1, abort_flag))
            break;
          LA_TRACE_AT(1, c, 5);
          tc_fence_after();
          issue_scores(c + 1);
          LA_TRACE_AT(1, c, 6);
        }
      }
      if (elect_one()) umma_commit(&bars[kDone]);
      __syncwarp();
    }
  } else if (warp < kWarpPoly) {
    // ------------------------------------------------------------ features
    // phi(K) of every tile, into two shared-memory buffers (the state
    // chain: the update of tile c waits on it).  phi(Q) is the epilogue
    // warps' (it sits on the output chain, and they are idle between tiles).
    const int wq = warp & 3;
    const int row = wq * 32 + lane;  // token within the tile == TMEM lane
    const bool leader = (warp == kWarpFeat && lane == 0);
    auto do_phik = [&](int c) {
      const int s = c & 1;           // phi(K) buffer
      const int sq = c % kQKStages;  // Q/K stage
      mbar_wait(&bars[kQKFull + sq], (c / kQKStages) & 1, abort_flag);
      named_barrier_sync(1, 128);
      LA_TRACE_AT(1, c, 0);
      const int valid = (int)min64(kT, t_end - (t_begin + (int64_t)c * kT));
      const bool vrow = row < valid;
      uint32_t kw[8];
      const uint32_t kt = sb + kOffK + sq * kQBytes;
      ld_shared_v4(kt + sw32_offset(row, 0), kw[0], kw[1], kw[2], kw[3]);
      ld_shared_v4(kt + sw32_offset(row, 1), kw[4], kw[5], kw[6], kw[7]);
      // phi(K) into buffer c&1 once the update of tile c-2 has read it
      if (c >= 2) mbar_wait(&bars[kUpDone0 + s], ((c >> 1) - 1) & 1, abort_flag);
      named_barrier_sync(1, 128);
      LA_TRACE_AT(1, c, 3);
      {
        FeatIn fk;
#pragma unroll
        for (int i = 0; i < 8; ++i) fk.w[i] = vrow ? kw[i] : 0u;
        fk.one = vrow ? 0x3F80u : 0u;  // padding tokens add nothing to the state
        store_phik<kIdentity>(fk, sb + kOffPhiK + s * kPhiBytes, row,
                              std::make_integer_sequence<int, kSlots / 8>{});
      }
      LA_TRACE_AT(1, c, 4);
      fence_proxy_async_smem();
      named_barrier_sync(1, 128);
      if (leader) {
        mbar_arrive(&bars[kPhiKReady0 + s]);
        // K of tile c has been read (the full kernel's stage also waits for
        // the scores MMA and phi(Q))
        mbar_arrive(&bars[kQKEmpty + sq]);
      }
      LA_TRACE_AT(1, c, 1);
    };
    for (int c = 0; c < n_chunks; ++c) do_phik(c);
  } else if (warp < kWarpEpi) {
    // ------------------------------------------------------------ polynomial
    if (!kStateOnly) {
      const int wq = warp & 3;              // TMEM lane quarter: query rows 32wq ..
      const int half = (warp - kWarpPoly) >> 2;  // this warp's key groups: G = half, half + 2
      const int row = wq * 32 + lane;
      // Taylor: p = 1 + s/4 + s^2/32; identity: p = s/4 (= s * (0 s + 1/4) + 0, exact)
      const uint64_t c32 = kIdentity ? f2pack(0.f, 0.f) : f2pack(0.03125f, 0.03125f);
      const uint64_t c4 = f2pack(0.25f, 0.25f);
      const uint64_t one2 = kIdentity ? f2pack(0.f, 0.f) : f2pack(1.f, 1.f);
      for (int c = 0; c < n_chunks; ++c) {
        const int64_t t0 = t_begin + (int64_t)c * kT;
        const int valid = (int)min64(kT, t_end - t0);
        mbar_wait(&bars[kScReady], c & 1, abort_flag);
        named_barrier_sync(2, 256);
        // the scores MMA has read Q and K of tile c: its part of the stage is free
        if (warp == kWarpPoly && lane == 0) mbar_arrive(&bars[kQKEmpty + c % kQKStages]);
        tc_fence_after();
        LA_TRACE_AT(2, c, 0);
        // P = tril(1 + s/4 + s^2/32) for raw scores s = q.k (d = 16).  Key group
        // G (32 keys) lies below the diagonal for this warp's rows when G < wq,
        // holds the diagonal when G == wq and is all zero when G > wq.
#pragma unroll
        for (int G2 = 0; G2 < 2; ++G2) {
          const int G = 2 * G2 + half;
          uint32_t w[16];
          if (G <= wq) {
            uint32_t r[32];
            tmem_ld16(taddr(tmem, wq * 32, kColSc + 32 * G), r);
            tmem_ld16(taddr(tmem, wq * 32, kColSc + 32 * G + 16), r + 16);
            tmem_wait_ld();
            // keys 32G .. 32G + m of this group are visible to this row (one
            // masked body for every group keeps the hot loop's code small)
            const int m = min(row, valid - 1) - 32 * G;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint64_t s2 = f2pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
              float p0, p1;
              f2unpack(ffma2(s2, ffma2(s2, c32, c4), one2), p0, p1);
              p0 = 2 * i <= m ? p0 : 0.f;
              p1 = 2 * i + 1 <= m ? p1 : 0.f;
              w[i] = pack_bf16(p0, p1);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0u;
          }
          // P columns [16G, 16G + 16) hold keys [32G, 32G + 32).  They
          // overwrite score columns [16G, 16G + 16), i.e. keys of group G/2,
          // which the other warp of this quarter may still be reading: store
          // only after both warps have loaded their groups (barrier below).
          if (G2 == 0) {
            LA_TRACE_AT(2, c, 2);
            named_barrier_sync(5 + wq, 64);
            LA_TRACE_AT(2, c, 3);
          }
          tmem_st16(taddr(tmem, wq * 32, kColSc + 16 * G), w);
          // this quarter's half of P (keys 64 G2 .. 64 G2 + 63) is in TMEM
          tmem_wait_st();
          tc_fence_before();
          named_barrier_sync(5 + wq, 64);
          if (half == 0 && lane == 0) mbar_arrive(&bars[G2 ? kPReadyHi : kPReadyLo]);
        }
        LA_TRACE_AT(2, c, 1);
      }
    }
  } else if (warp >= kWarpState0) {
    // ------------------------------------------------------------ state
    const int wq = warp & 3;       // quarters 0..2: S^T rows 0..95
    const int half = warp >= kWarpState1 ? 1 : 0;
    const int e = wq * 32 + lane;  // row of S^T: value column e (< 64), normaliser (64)
    const int col0 = 80 * half;    // this warp's 80 feature columns
    const bool leader = (warp == kWarpState0 && lane == 0);
    const bool real = e < kSV;
    // S_0 = init_state + states of the earlier segments (fixed order).  Rows
    // 65..79 of both snapshot buffers are zero for good (S^T rows >= 65 never
    // change: their rows of [V 1 0]^T are zero).
    // The seed is init_state + the prefix slot g - 1; the 32 loads of a
    // group of 16 columns are independent and issued together.
    LA_TRACE_AT(3, 0, 3);
    const float *head_a =
        !kStateOnly && p.init_state ? p.init_state + (uint64_t)bh * kFeat * kSV : nullptr;
    const float *head_b =
        !kStateOnly && g > 0 ? p.seg_states + ((uint64_t)bh * p.segments + (g - 1)) * kFeat * kSV
                             : nullptr;
    // the seeds may come from the kernels launched just before this one on
    // the stream (state pass, running sums), which this grid may overlap
    if (!kStateOnly) grid_dependency_wait();
    if (leader) {  // the seeds, into L2 while the first group's loads are in flight
      if (head_a) prefetch_l2(head_a, sizeof(float) * kFeat * kSV);
      if (head_b) prefetch_l2(head_b, sizeof(float) * kFeat * kSV);
    }
    // Loads are unconditional (padding slots read feature 0 and are zeroed
    // after), so that all 32 of a group are in flight together.
    const bool seeded = real && (head_a || head_b);
    const float *seed_a = seeded ? (head_a ? head_a : head_b) + e : nullptr;
    const float *seed_b = seeded ? (head_b ? head_b : head_a) + e : nullptr;
    for (int grp = 0; grp < 5; ++grp) {
      const int f0 = col0 + 16 * grp;
      uint32_t w[16];
      if (seeded) {
        float xa[16], xb[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int f = slot_map[f0 + i];
          const int fi = f >= 0 ? f : 0;
          xa[i] = __ldg(seed_a + fi * kSV);
          xb[i] = __ldg(seed_b + fi * kSV);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int f = slot_map[f0 + i];
          const float x = (head_a ? xa[i] : 0.f) + (head_b ? xb[i] : 0.f);
          w[i] = __float_as_uint(f >= 0 ? x : 0.f);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0u;
      }
      tmem_st16(taddr(tmem, wq * 32, kColS + f0), w);
      if (!kStateOnly && e < kNO) {
#pragma unroll
        for (int buf = 0; buf < 2; ++buf) {
          if (buf == 1 && e <= kDv) continue;  // buffer 1: only the zero rows now
          st_shared_v4(snap_chunk_addr(sb, buf, f0, e),
                       pack_bf16(__uint_as_float(w[0]), __uint_as_float(w[1])),
                       pack_bf16(__uint_as_float(w[2]), __uint_as_float(w[3])),
                       pack_bf16(__uint_as_float(w[4]), __uint_as_float(w[5])),
                       pack_bf16(__uint_as_float(w[6]), __uint_as_float(w[7])));
          st_shared_v4(snap_chunk_addr(sb, buf, f0 + 8, e),
                       pack_bf16(__uint_as_float(w[8]), __uint_as_float(w[9])),
                       pack_bf16(__uint_as_float(w[10]), __uint_as_float(w[11])),
                       pack_bf16(__uint_as_float(w[12]), __uint_as_float(w[13])),
                       pack_bf16(__uint_as_float(w[14]), __uint_as_float(w[15])));
        }
      }
    }
    LA_TRACE_AT(3, 0, 4);
    tmem_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    named_barrier_sync(3, kStateThreads);
    LA_TRACE_AT(3, 0, 5);
    if (leader) {
      mbar_arrive(&bars[kSRead]);  // S_0 is in TMEM
      mbar_arrive(&bars[kSnapReady0]);
    }

    if (kStateOnly) {
      // the segment's state, once every update has completed
      mbar_wait(&bars[kDone], 0, abort_flag);
      named_barrier_sync(3, kStateThreads);
      {
        tc_fence_after();
        float *dst = p.seg_out + ((uint64_t)bh * p.segments + g) * kFeat * kSV;
        for (int grp = 0; grp < 5; ++grp) {
          uint32_t r[16], r2[16];
          tmem_ld16(taddr(tmem, wq * 32, kColS + col0 + 16 * grp), r);
          tmem_ld16(taddr(tmem, wq * 32, kColO + col0 + 16 * grp), r2);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int f = slot_map[col0 + 16 * grp + i];
            if (real && f >= 0)
              dst[(uint64_t)f * kSV + e] = __uint_as_float(r[i]) + __uint_as_float(r2[i]);
          }
        }
      }
    } else {
      const bool write_final = p.final_state != nullptr && g == last_g;
      // snapshot a group of 16 columns of row e (rows <= 64 carry data)
      auto put = [&](uint32_t snap, int f0, const uint32_t *r) {
        if (e <= kDv) {
          const uint32_t blk = snap + (f0 >> 6) * kSnapKBlock;
          const int ch = (f0 & 63) >> 3;
          st_shared_v4(blk + sw128_offset(e, ch),
                       pack_bf16(__uint_as_float(r[0]), __uint_as_float(r[1])),
                       pack_bf16(__uint_as_float(r[2]), __uint_as_float(r[3])),
                       pack_bf16(__uint_as_float(r[4]), __uint_as_float(r[5])),
                       pack_bf16(__uint_as_float(r[6]), __uint_as_float(r[7])));
          st_shared_v4(blk + sw128_offset(e, ch + 1),
                       pack_bf16(__uint_as_float(r[8]), __uint_as_float(r[9])),
                       pack_bf16(__uint_as_float(r[10]), __uint_as_float(r[11])),
                       pack_bf16(__uint_as_float(r[12]), __uint_as_float(r[13])),
                       pack_bf16(__uint_as_float(r[14]), __uint_as_float(r[15])));
        }
      };
      auto put_final = [&](int f0, const uint32_t *r) {
        float *dst = p.final_state + (uint64_t)bh * kFeat * kSV;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int f = slot_map[f0 + i];
          if (real && f >= 0) dst[(uint64_t)f * kSV + e] = __uint_as_float(r[i]);
        }
      };
      for (int c = 0; c < n_chunks; ++c) {
        // S^T holds S_{c+1} once the update of tile c is done; its snapshot
        // goes to buffer (c+1)&1, last read by phi(Q) S of tile c-1
        mbar_wait(&bars[kSReady], c & 1, abort_flag);
        LA_TRACE_AT(3, c, 2);
        if (c == n_chunks - 1) {
          // the state after the last tile: no tile reads its snapshot; the
          // last segment writes it out as the final state
          named_barrier_sync(3, kStateThreads);
          tc_fence_after();
          if (write_final) {
#pragma unroll 1
            for (int grp = 0; grp < 5; ++grp) {
              uint32_t r[16];
              tmem_ld16(taddr(tmem, wq * 32, kColS + col0 + 16 * grp), r);
              tmem_wait_ld();
              put_final(col0 + 16 * grp, r);
            }
          }
          break;
        }
        named_barrier_sync(3, kStateThreads);
        tc_fence_after();
        LA_TRACE_AT(3, c, 0);
        // S_{c+1} -> bf16 snapshot buffer (c+1)&1, last read by phi(Q) S of
        // tile c-1.  S^T is released to the next update as soon as the last
        // TMEM load has landed, before the last group is stored.
        if (c > 0) mbar_wait(&bars[kQSDone0 + ((c - 1) & 1)], ((c - 1) >> 1) & 1, abort_flag);
        {
          // groups of 16 columns that carry features: all 5 of each warp's 80
          // (Taylor); the first 2 of the column-0 warps (identity)
          constexpr int kGroups = kIdentity ? kIdSlots / 16 : 5;
          const bool active = !kIdentity || col0 == 0;
          const uint32_t snap = sb + kOffSnap + ((c + 1) & 1) * kSnapBytes;
          const uint32_t base = taddr(tmem, wq * 32, kColS + col0);
          uint32_t r0[16], r1[16];
          if (active) tmem_ld16(base, r0);
#pragma unroll
          for (int grp = 0; grp < kGroups; ++grp) {
            uint32_t *cur = (grp & 1) ? r1 : r0;
            uint32_t *nxt = (grp & 1) ? r0 : r1;
            if (active) tmem_wait_ld();
            if (grp + 1 < kGroups) {
              if (active) tmem_ld16(base + 16 * (grp + 1), nxt);
            } else {
              tc_fence_before();
              named_barrier_sync(3, kStateThreads);
              if (leader) mbar_arrive(&bars[kSRead]);
              LA_TRACE_AT(3, c, 6);
            }
            if (active) put(snap, col0 + 16 * grp, cur);
          }
        }
        LA_TRACE_AT(3, c, 7);
        fence_proxy_async_smem();
        tc_fence_before();
        named_barrier_sync(3, kStateThreads);
        if (leader) mbar_arrive(&bars[kSnapReady0 + ((c + 1) & 1)]);
        LA_TRACE_AT(3, c, 1);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    if (!kStateOnly) {
      const int wq = warp & 3;  // rows 32wq .. 32wq+31 of the tile, one per lane
      const bool leader = (warp == kWarpEpi && lane == 0);
      const int row = wq * 32 + lane;  // token within the tile == TMEM lane
      // phi(Q) of tile c -> TMEM (a single buffer, free once phi(Q) S of tile
      // c - 1 has read it).  Produced here, ahead of the output of tile
      // c - 1: phi(Q) S of tile c waits for it, while the output of tile
      // c - 1 only has to leave TMEM before phi(Q) S of tile c writes O.
      auto do_phiq = [&](int c) {
        const int sq = c % kQKStages;  // Q/K stage of tile c
        mbar_wait(&bars[kQKFull + sq], (c / kQKStages) & 1, abort_flag);
        uint32_t qw[8];
        const uint32_t qt = sb + kOffQ + sq * kQBytes;
        ld_shared_v4(qt + sw32_offset(row, 0), qw[0], qw[1], qw[2], qw[3]);
        ld_shared_v4(qt + sw32_offset(row, 1), qw[4], qw[5], qw[6], qw[7]);
        if (c > 0) mbar_wait(&bars[kQSDone0 + ((c - 1) & 1)], ((c - 1) >> 1) & 1, abort_flag);
        named_barrier_sync(4, 128);
        LA_TRACE_AT(4, c, 3);
        tc_fence_after();
        FeatIn fs;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          fs.w[i] = qw[i];
          fs.s16[i] = hmul2_bf16(qw[i], 0x3D803D80u);  // x / 16  (exact)
          fs.s32[i] = hmul2_bf16(qw[i], 0x3D003D00u);  // x / 32  (exact)
        }
        fs.one = 0x3F80u;
        store_phiq<kIdentity>(fs, taddr(tmem, wq * 32, kColPhiQ),
                              std::make_integer_sequence<int, kSlots / 32>{});
        tmem_wait_st();
        LA_TRACE_AT(4, c, 4);
        tc_fence_before();
        named_barrier_sync(4, 128);
        LA_TRACE_AT(4, c, 5);
        if (leader) {
          mbar_arrive(&bars[kPhiQReady]);
          mbar_arrive(&bars[kQKEmpty + sq]);  // Q of tile c has been read
        }
      };
      // this lane's store target after the transpose: piece (lane & 3) of row
      // (lane & ~3) of its quarter, advanced one tile per output; rows_left
      // counts the rows of the segment from that row on
      const int gi = lane & 3;
      uint4 *dst_row = (uint4 *)(p.out + ((uint64_t)bh * p.n + t_begin + wq * 32 + (lane & ~3)) * kDv) +
                       2 * gi;
      int64_t rows_left = t_end - (t_begin + wq * 32 + (lane & ~3));
      if (n_chunks > 0) do_phiq(0);
      for (int c = 0; c < n_chunks; ++c, dst_row += kT * kDv / 8, rows_left -= kT) {
        if (c + 1 < n_chunks) do_phiq(c + 1);
        mbar_wait(&bars[kOReady], c & 1, abort_flag);
        named_barrier_sync(4, 128);
        tc_fence_after();
        LA_TRACE_AT(4, c, 0);
        // O leaves TMEM in two round trips, (denominator, values 0..31) then
        // values 32..63, each normalised and packed to bf16 on arrival; TMEM
        // O is released before any global store is issued
        uint32_t w[32];
        const uint32_t obase = taddr(tmem, wq * 32, kColO);
        {
          uint32_t o[32];
          const uint32_t dbits = tmem_ld1(obase + kDv);
          tmem_ld16(obase, o);
          tmem_ld16(obase + 16, o + 16);
          tmem_wait_ld();
          // O[:, 64] = phi(q).z + rowsum(P): the full denominator before eps
          const float den = __uint_as_float(dbits) + p.eps;
          const float inv = p.normalize ? 1.f / den : 1.f;
          const uint64_t inv2 = f2pack(inv, inv);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(fmul2(f2pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2));
          tmem_ld16(obase + 32, o);
          tmem_ld16(obase + 48, o + 16);
          tmem_wait_ld();
          tc_fence_before();
          named_barrier_sync(4, 128);
          if (leader) mbar_arrive(&bars[kOFree]);  // O is in registers: TMEM O reusable
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[16 + i] =
                pack_bf16x2(fmul2(f2pack(__uint_as_float(o[2 * i]), __uint_as_float(o[2 * i + 1])), inv2));
        }
        LA_TRACE_AT(4, c, 1);
        // 4x4 transpose of 32-byte pieces inside each group of four lanes
        // (two butterfly stages): afterwards lane 4g+i holds piece i of rows
        // 4g..4g+3, and each store instruction writes eight whole rows
        {
#pragma unroll
          for (int m = 2; m >= 1; m >>= 1) {
            const bool hi = (gi & m) != 0;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              // the two slots this lane exchanges: bit m of the slot differs from bit m of gi
              const int s0 = m == 2 ? k : (k << 1);      // slot with bit m clear
              const int s1 = s0 | m;                     // slot with bit m set
#pragma unroll
              for (int r = 0; r < 8; ++r) {
                const uint32_t send = hi ? w[8 * s0 + r] : w[8 * s1 + r];
                const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m);
                if (hi) w[8 * s0 + r] = recv;
                else w[8 * s1 + r] = recv;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (j < rows_left) {
              uint4 *dst = dst_row + j * (kDv / 8);
              asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst),
                           "r"(w[8 * j]), "r"(w[8 * j + 1]), "r"(w[8 * j + 2]), "r"(w[8 * j + 3]),
                           "r"(w[8 * j + 4]), "r"(w[8 * j + 5]), "r"(w[8 * j + 6]), "r"(w[8 * j + 7])
                           : "memory");
            }
          }
        }
        LA_TRACE_AT(4, c, 2);
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpUpd) {
    if (lane == 0) wait_teardown(&bars[kDone], 0);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicExch(p.err, kErrTimeout);
#ifdef LA_TRACE
  if (threadIdx.x == 0 && !kStateOnly && blockIdx.y * gridDim.x + blockIdx.x < kTraceCtas)
  {
    la_trace_cta[blockIdx.y * gridDim.x + blockIdx.x][1] = (long long)globaltimer();
    la_trace_cta[blockIdx.y * gridDim.x + blockIdx.x][4] = clock64();
  }
#endif
}

// ---------------------------------------------------------------- host side
// 3-D map over (bh, n, d) bf16 with a (1, 128, d) box; rows past n read as zero.
bool make_map(CUtensorMap *map, const void *base, int64_t bh, int64_t n, int d,
              CUtensorMapSwizzle swz) {
  return make_tmap_3d(map, base, bh, n, d, kT, swz);
}

// pdl: launched as the programmatic dependent of the kernel before it on the
// stream (this library's state pass or running sums): its CTAs may start
// while that kernel drains and wait only where they read the seeds.
template <bool kStateOnly, bool kIdentity>
int launch(const void *q, const void *k, const void *v, const Params &p, int64_t bh, int n_launch,
           bool pdl, cudaStream_t s) {
  if (bh > 65535 || p.n > INT32_MAX) return LA_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv;
  if (!make_map(&mk, k, bh, p.n, kDqk, CU_TENSOR_MAP_SWIZZLE_32B) ||
      !make_map(&mv, v, bh, p.n, kDv, CU_TENSOR_MAP_SWIZZLE_128B))
    return LA_ERR_CUDA;
  if (kStateOnly) {
    mq = mk;
  } else if (!make_map(&mq, q, bh, p.n, kDqk, CU_TENSOR_MAP_SWIZZLE_32B)) {
    return LA_ERR_CUDA;
  }
  constexpr uint32_t kSmemAlloc = Layout<kStateOnly>::kSmemAlloc;
  if (allow_dynamic_smem((const void *)chunked_tc_kernel<kStateOnly, kIdentity>, (int)kSmemAlloc) !=
      LA_OK)
    return LA_ERR_CUDA;
  const dim3 grid = (!kStateOnly && p.lead_len > 0) ? dim3((unsigned)bh, 2u)
                                                   : dim3((unsigned)n_launch, (unsigned)bh);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemAlloc;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, chunked_tc_kernel<kStateOnly, kIdentity>, mq, mk, mv, p) !=
      cudaSuccess) {
    note_launch();
    cudaGetLastError();
    return LA_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace

#ifdef LA_TRACE
extern "C" int la_debug_read_trace(long long *dst, int count) {
  const int n = kTraceMaxCtas * 6 * kTraceChunks * kTraceEvents;
  if (count < n) return -1;
  return cudaMemcpyFromSymbol(dst, la_trace_buf, sizeof(long long) * n) == cudaSuccess ? n : -1;
}
extern "C" int la_debug_read_cta_trace(long long *dst, int count) {
  const int n = kTraceCtas * 5;
  if (count < n) return -1;
  return cudaMemcpyFromSymbol(dst, la_trace_cta, sizeof(long long) * n) == cudaSuccess ? n : -1;
}
#endif

int launch_chunked_state_tc(const void *k, const void *v, float *seg_states, int64_t bh,
                            int64_t n, int segments, int n_launch, int64_t seg_len, bool identity,
                            const DeviceInfo &info, cudaStream_t s) {
  (void)info;
  Params p{};
  p.seg_out = seg_states;
  p.err = device_error_word();
  p.n = n;
  p.seg_len = seg_len;
  p.segments = segments;
  if (!p.err) return LA_ERR_CUDA;
  return identity ? launch<true, true>(nullptr, k, v, p, bh, n_launch, false, s)
                  : launch<true, false>(nullptr, k, v, p, bh, n_launch, false, s);
}

int launch_chunked_output_tc(const void *q, const void *k, const void *v, void *out,
                             const float *init_state, float *final_state,
                             const float *seg_states, int64_t bh, int64_t n, float eps,
                             bool normalize, bool identity, int segments, int64_t seg_len,
                             int64_t lead_len, bool after_own_kernel, const DeviceInfo &info,
                             cudaStream_t s) {
  (void)info;
  Params p{};
  p.out = (__nv_bfloat16 *)out;
  p.init_state = init_state;
  p.final_state = final_state;
  p.seg_states = seg_states;
  p.err = device_error_word();
  p.n = n;
  p.seg_len = seg_len;
  p.lead_len = lead_len;
  p.segments = segments;
  p.eps = eps;
  p.normalize = normalize ? 1 : 0;
  if (!p.err) return LA_ERR_CUDA;
  if (identity && normalize) return LA_ERR_UNSUPPORTED;  // the identity map has no normaliser
  return identity ? launch<false, true>(q, k, v, p, bh, segments, after_own_kernel, s)
                  : launch<false, false>(q, k, v, p, bh, segments, after_own_kernel, s);
}

}  // namespace la
