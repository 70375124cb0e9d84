// mbarrier + bulk-copy (TMA engine) helpers for sm_100a kernels.
//
// Every wait is bounded: after kWaitNs of wall time (read from %globaltimer),
// or kWaitPolls polls if the timer does not advance, it returns false so the
// caller can record an error, drain its copies in flight and leave instead of
// spinning forever.  A kernel whose bulk copies have been issued must not
// exit before they land: see gemv.cu's producer drain.
#pragma once

#include <stdint.h>

namespace cb {

constexpr uint64_t kWaitNs = 1000000000ull;  // 1 s
constexpr uint32_t kWaitPolls = 1u << 28;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// The waiting thread is suspended (issuing nothing) until the phase
// completes or about kSuspendNs pass, so waiting warps leave the issue slots
// to the warps that share their scheduler.
constexpr uint32_t kSuspendNs = 10000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

// try_wait without a suspend-time hint: the thread wakes as soon as the phase
// completes.  For the short producer/consumer hand-offs of the tcgen05
// kernels, where a waiter suspended for a long hint would stall the chain.
__device__ __forceinline__ bool mbar_try_wait_short(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete; false on timeout.
// The clock is read every 256 polls, starting at the first such read (a
// %globaltimer read is slow; most waits end within their first polls).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitNs) {
  uint64_t start = 0;
  for (uint32_t i = 0; i < kWaitPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      const uint64_t now = global_ns();
      if (start == 0) start = now;
      else if (now - start > limit_ns) return false;
    }
  }
  return false;
}

// Grid-wide arrivals and tickets with release/acquire ordering instead of a
// full fence: the caller's block barrier orders its threads' earlier writes
// before the arriving thread, and a release at gpu scope is cumulative over
// them, so they are visible to whoever acquires the counter value.
__device__ __forceinline__ void arrive_release(unsigned* counter) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counter) : "memory");
}
__device__ __forceinline__ unsigned ticket_acq_rel(unsigned* counter) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

// Bulk copy global -> this CTA's shared memory, completing `bytes` of the
// barrier's transaction count.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

}  // namespace cb
