// async.cuh — mbarrier, TMA and bulk-copy helpers shared by the kernels that
// stage global data in shared memory with the asynchronous copy engine.
//
// Every wait is bounded: mbar_wait gives up after kAsyncWaitCycles (about one
// second at the boost clock) or once another warp of the CTA has set the
// abort flag, so a kernel whose copy never lands records a status and returns
// instead of hanging.  Loads carry no cluster multicast.
#pragma once

#include "kernels.cuh"

#include <cudaTypedefs.h>

namespace bitnet {

constexpr long long kAsyncWaitCycles = 2000000000LL;  // ~1 s at the boost clock

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `parity` to complete.  False when it has not
// completed within kAsyncWaitCycles, or (abort_flag given) once another warp of the
// CTA has given up.
static __device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (clock64() - t0 > kAsyncWaitCycles) return false;
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag);
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}
// One page of one kv head (K: kind 0, V: kind 1) of pool page z into dst.
__device__ __forceinline__ void tma_page(uint32_t dst, const CUtensorMap* map, int y, int z, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %2, %3, %4}], [%5], %6;\n" ::"r"(dst),
      "l"((uint64_t)map), "r"(0), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, bytes % 16 == 0).
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
          dst),
      "l"((uint64_t)src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// A failed wait: the first warp to give up records the status for the host.
__device__ __forceinline__ void give_up(volatile int* abort_flag, int32_t* status) {
  if (!*abort_flag) {
    *abort_flag = 1;
    atomicOr(status, kStatusWaitTimeout);
  }
}

}  // namespace bitnet
