// mbarrier / bulk-async-copy helpers shared by the sm_100a kernels.
//
// Every wait is bounded: after kWaitTimeoutNs of %globaltimer the waiter
// gives up, records ZIB_ERR_TIMEOUT in its translation unit's device error
// word and returns false so the kernel can drain and exit.
#pragma once

#include "zib_common.cuh"

// One device error word per translation unit (no relocatable device code);
// ZIB_DEFINE_ERROR_READER(name) emits the host reader for it.
static __device__ int g_zib_err_word = 0;

#define ZIB_DEFINE_ERROR_READER(fname)                                          \
  int fname() {                                                                 \
    int v = 0;                                                                  \
    if (cudaMemcpyFromSymbol(&v, g_zib_err_word, sizeof(int)) != cudaSuccess) { \
      cudaGetLastError();                                                       \
      return ZIB_ERR_LAUNCH;                                                    \
    }                                                                           \
    int zero = 0;                                                               \
    cudaMemcpyToSymbol(g_zib_err_word, &zero, sizeof(int));                     \
    return v;                                                                   \
  }

namespace zib {

constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that lets the thread sleep up to `hint_ns` (woken when the phase
// completes): a waiting warp re-polls rarely instead of spinning on issue slots
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
constexpr uint32_t kWaitSleepNs = 1000000u;  // 1 ms per poll; the bounded waits check their limit between polls

// Bounded wait; returns false after the timeout (error word set) or when
// *abort_flag is raised by another waiter.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) return true;
    if (abort_flag && *abort_flag) return false;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      if (abort_flag) *abort_flag = 1;
      atomicExch(&g_zib_err_word, (int)ZIB_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait that never raises anything (used while draining after an abort).
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) {
    if (globaltimer() - t0 > kWaitTimeoutNs) return;
  }
}

// 1-D bulk async copy global -> shared (no tensor map); 16-byte aligned
// addresses, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace zib
