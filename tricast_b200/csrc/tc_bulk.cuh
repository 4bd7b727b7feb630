// mbarrier and 1-D bulk-copy (TMA, no multicast) helpers shared by the staged kernels. Every wait
// is bounded: mbar_wait gives up after about 2**22 polls and the caller reports the timeout.
//
// A kernel's pipeline waits take their poll limit from the launch (`polls`, negative = the default;
// tc_set_wait_limit sets it process-wide so that a test can make a wait run out). The waits that drain
// a kernel's own copies and MMAs before it exits always use the default limit.
#pragma once

#include <stdint.h>

namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after ~2**22 polls (each try_wait itself suspends for a while), or after
// `polls` polls when that is not negative (0: gives up at once).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int polls = -1) {
  const int limit = polls < 0 ? (1 << 22) : polls;
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bounded wait that lets the hardware suspend the thread between polls (up to ~64 us each), so
// waiting warps do not take issue slots from working ones; gives up after ~2**16 polls (seconds), or
// after `polls` polls when that is not negative.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, int polls = -1) {
  const int limit = polls < 0 ? (1 << 16) : polls;
  for (int i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(0x10000u)
        : "memory");
    if (ok) return true;
    __nanosleep(32);
  }
  return false;
}

// Global -> this CTA's shared memory, completing `bytes` on `bar`. Both addresses 16-byte aligned,
// bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// 16 bytes global -> shared without registers (both addresses 16-byte aligned). A thread's copies
// are complete after cp_async_wait_all; a following __syncthreads makes every thread's copies visible.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

}  // namespace tc
