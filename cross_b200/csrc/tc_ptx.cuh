// tcgen05 / mbarrier building blocks shared by the tensor-core kernels
// (sm_100a inline PTX): shared-memory addresses, bounded mbarrier waits,
// TMEM loads, and the exact 32-bit Barrett forms used by their epilogues.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace cross {
namespace tc {

constexpr uint64_t WAIT_NS = 2000000000ull;   // bound on any single wait

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `parity` to complete.  try_wait suspends the
// thread in hardware until the phase completes or a short system-defined
// interval passes, so a waiting role wakes as soon as its barrier flips.
// Returns false (and raises the CTA abort flag, recording `code`) when the
// bound expires or another role of the CTA has already aborted.  The first
// try is inline; the bounded loop is out of line.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int& abort, int* err, int code);
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int& abort, int* err, int code) {
  if (mbar_try(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort, err, code);
}
// The bounded loop with an explicit bound (bound_ns of global timer).
static __device__ __noinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int& abort, int* err,
                                                  int code, uint64_t bound_ns) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (abort) return false;
    if (globaltimer() - t0 > bound_ns) {
      atomicCAS(err, 0, code);
      abort = 1;
      return false;
    }
  }
}
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int& abort, int* err, int code) {
  return mbar_wait_for(bar, parity, abort, err, code, WAIT_NS);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive accumulator columns of this thread's TMEM lane (32x32b shape),
// loaded and waited for in one statement so that every use of v follows the
// wait (TMEM is not memory the compiler tracks, so no memory clobber).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// 16 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// The same 16-column load issued without waiting, and the wait for it.  The
// wait names the destination registers as read-write operands, so no use of
// them can be scheduled before it; nothing may read them in between.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15]));
}

// Barrett of finite_field.py:224-230 for w = 32 with the remainder taken in
// 32-bit arithmetic.  The reference forms r = z - t*q in uint64 and then keeps
// r >= q ? r - q : r truncated to uint32; t = floor(floor(z*m / 2^32) / 2^s_w)
// is computed exactly here (u = zhi*m + floor(zlo*m / 2^32) < 2^64, and only
// t mod 2^32 enters the 32-bit remainder), and whenever the true r lies in
// (-(2^32 - q), 2^32) the 32-bit remainder and comparison give the same uint32;
// min(r, r - q) is that comparison (r - q wraps above r exactly when r < q).
// Callers enable this path only when reduce_fast_ok (internal.hpp) holds for
// every modulus, which covers inputs z < 2^53 (contraction sums) and
// z < 2^31 * q + 2^32 (a word below 2^31 times a residue, plus a word).
__device__ __forceinline__ uint32_t reduce_fast2(uint32_t zlo, uint32_t zhi, uint32_t q, uint32_t m, uint32_t s_w) {
  const uint64_t u = (uint64_t)zhi * m + __umulhi(zlo, m);
  const uint32_t t = __funnelshift_r((uint32_t)u, (uint32_t)(u >> 32), s_w);
  const uint32_t r = zlo - t * q;
  return min(r, r - q);
}
__device__ __forceinline__ uint32_t reduce_fast(uint64_t z, uint32_t q, uint32_t m, uint32_t s_w) {
  return reduce_fast2((uint32_t)z, (uint32_t)(z >> 32), q, m, s_w);
}

// sum_p acc_p << 8p (ntt_mm.py:33-37); plain 64-bit shifts and adds compile
// to fewer instructions here than explicit wide multiply-adds.
__device__ __forceinline__ uint64_t combine4_mad(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3) {
  return (uint64_t)a0 + ((uint64_t)a1 << 8) + ((uint64_t)a2 << 16) + ((uint64_t)a3 << 24);
}

}  // namespace tc
}  // namespace cross
