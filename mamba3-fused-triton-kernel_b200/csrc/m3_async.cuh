// Asynchronous-copy primitives for sm_100a: mbarriers and 1-D bulk (TMA)
// copies global -> shared, written as inline PTX.
//
// Every wait is bounded: after kSpinLimit polls the waiting thread records
// M3_DEVERR_TIMEOUT in the library's device error word and gives up, so a
// lost transaction can never hang the GPU.  No copy here uses cluster
// multicast.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "mamba3_b200.h"

namespace m3 {

// Device-side error word of this translation unit (each kernel .cu file has
// its own copy; m3_device_error in the C ABI collects them all).
static __device__ int g_device_error = 0;

// Read (and optionally clear) this translation unit's error word.  Host
// side; synchronous.
static inline int device_error_of_this_unit(bool reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (reset && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

// Polls of mbarrier.try_wait before a wait is declared lost.  One poll
// returns after at most a hardware-defined suspend interval (well under a
// millisecond), so this bounds a wait to seconds.
constexpr long long kSpinLimit = 1ll << 22;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make the initialised barriers visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive once and add `bytes` to the transaction count of the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Add `bytes` to the transaction count of the current phase without
// arriving (for copies that join a phase another thread arrives on).
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (and records a timeout) if it did not complete within the bound.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit = kSpinLimit) {
  for (long long i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_device_error, M3_DEVERR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared through the TMA engine, completing
// `bytes` transactions on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

}  // namespace m3
