// sm_100a building blocks written directly in inline PTX: mbarriers with
// bounded waits, TMA tensor loads, TMEM allocation / loads / stores, UMMA
// (tcgen05.mma) shared-memory and instruction descriptors.
//
// Descriptor bit layouts follow the PTX ISA "tcgen05 shared memory
// descriptor" and "instruction descriptor" tables (kind::f16, bf16 inputs,
// fp32 accumulate).  All TMA loads here are plain per-CTA loads.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace la {
namespace tc {

// A wait that has not completed after this many nanoseconds is a bug (a
// barrier that will never flip); the kernel records an error and unwinds.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

// Value written to the library's device error word when a wait timed out.
constexpr int kErrTimeout = 1;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier ---
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of whether the phase with the given parity has completed
// (acquire semantics, like a completed wait).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// As mbar_try_wait, but the thread may sleep in hardware until the phase
// completes or about `suspend_ns` nanoseconds pass, instead of returning at
// once: waiting warps then take no issue slots or shared-memory bandwidth.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity,
                                                    uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}
constexpr uint32_t kSuspendNs = 200000;  // one sleep; the abort flag and the clock are checked after each

// Waits for the phase with the given parity to complete.  Returns false if
// the CTA is aborting (flag set by any thread) or the wait timed out, in
// which case the CTA's abort flag is raised.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*abort_flag) return false;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, kSuspendNs)) {
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// Bounded spin until a shared counter written by another thread of the CTA
// reaches `target`.  Returns false on abort or timeout (flag raised).
__device__ __forceinline__ bool spin_until_at_least(volatile int *counter, int target,
                                                    volatile int *abort_flag) {
  if (*counter >= target) return true;
  const uint64_t t0 = globaltimer();
  uint32_t spins = 0;
  while (*counter < target) {
    __nanosleep(20);
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
  return true;
}

// Bounded wait by a whole converged warp: every lane waits on the barrier
// and the warp agrees on the outcome (false if any lane gave up), so the
// warp's control flow stays uniform.  (Polling with mbarrier.test_wait
// instead of sleeping in try_wait was measured 2% slower for the issuers.)
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity,
                                               volatile int *abort_flag) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
}

// True in exactly one lane of a converged warp (elect.sync): the lane that
// issues a single-thread tcgen05 instruction for the warp.  A warp that runs
// its MMA loop converged and issues through the elected lane issues
// tile-shaped tcgen05.mma sequences 18-38% faster than the same loop run by
// lane 0 alone (measured on B200: 8 ss N=160 MMAs 1096 -> 898 cycles, 10 ts
// N=80 MMAs 978 -> 606 cycles, each with its commit and wait).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// Programmatic dependent launch.  A kernel launched as the dependent of the
// kernel before it on the stream may start while that kernel still runs; it
// calls grid_dependency_wait() before reading anything that kernel wrote.
// grid_dependents_launch() lets this kernel's dependent be scheduled (its
// CTAs then take SMs as this kernel's CTAs leave).  Both are no-ops for a
// kernel launched without such a dependency.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------- fences ---
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// ---------------------------------------------------------------------- TMA ---
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Bring the 16-byte-aligned part of [p, p + bytes) into L2 (a hint: nothing
// is read into the SM; the edges that are not 16-byte aligned are skipped).
__device__ __forceinline__ void prefetch_l2(const void *p, size_t bytes) {
  const uintptr_t lo = ((uintptr_t)p + 15) & ~(uintptr_t)15;
  const uintptr_t hi = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
  if (hi > lo)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((uint32_t)(hi - lo))
                 : "memory");
}

// --------------------------------------------------------------------- TMEM ---
// Executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
}
// 32 lanes x 32 bits, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t *r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(addr));
}
// One 32-bit column per lane.
__device__ __forceinline__ uint32_t tmem_ld1(uint32_t addr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(addr));
  return r;
}
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t *r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(addr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
               "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32"
      " [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// -------------------------------------------------------------------- UMMA ---
enum : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

// Shared-memory matrix descriptor (sm_100 "version 1").
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor, kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn: operand is MN-major (else K-major).
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | ((a_mn ? 1u : 0u) << 15)     // A major
         | ((b_mn ? 1u : 0u) << 16)     // B major
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

// D[tmem] (+)= A[tmem] * B[smem]^T   (A is K-major in TMEM: lane = row)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z));
}

// Arrive on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ------------------------------------------------------- packed fp32 math ---
// sm_100 executes two fp32 lanes per instruction (f32x2); operands are 64-bit
// register pairs {lo, hi}.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// ---------------------------------------------------------------- packing ---
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(r) : "f"(lo), "f"(hi));
  return r;
}
// {lo, hi} fp32 pair -> bf16x2 (round to nearest even)
__device__ __forceinline__ uint32_t pack_bf16x2(uint64_t v) {
  float lo, hi;
  f2unpack(v, lo, hi);
  return pack_bf16(lo, hi);
}
// bf16x2 product, rounded once (== the fp32 product of the bf16 operands, RN)
__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// {half i of word a, half j of word b} as a bf16x2 word (i, j in {0 = lo, 1 = hi})
template <int I, int J>
__device__ __forceinline__ uint32_t bf16_pair(uint32_t a, uint32_t b) {
  constexpr uint32_t sel = (I ? 0x0032u : 0x0010u) | (J ? 0x7600u : 0x5400u);
  return __byte_perm(a, b, sel);
}
__device__ __forceinline__ float bf16lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16hi(uint32_t x) { return __uint_as_float(x & 0xFFFF0000u); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ void ld_shared_v4(uint32_t addr, uint32_t &a, uint32_t &b, uint32_t &c,
                                             uint32_t &d) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr)
               : "memory");
}

// Byte offset of the 16-byte chunk `chunk` of row `row` inside a 128B-swizzled
// region whose rows are 128 bytes and whose 8-row atoms are 1024 bytes apart.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + (((chunk ^ row) & 7u) << 4);
}
// Same for 64B swizzle with 64-byte rows (four 16-byte chunks per row; the
// pattern repeats every 8 rows = 512 bytes).
__device__ __forceinline__ uint32_t sw64_offset(uint32_t row, uint32_t chunk) {
  return row * 64u + (((chunk ^ (row >> 1)) & 3u) << 4);
}
// Same for 32B swizzle with 32-byte rows (two 16-byte chunks per row).
__device__ __forceinline__ uint32_t sw32_offset(uint32_t row, uint32_t chunk) {
  return row * 32u + (((chunk ^ (row >> 2)) & 1u) << 4);
}

}  // namespace tc
}  // namespace la
