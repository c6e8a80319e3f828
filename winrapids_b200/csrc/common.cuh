// common.cuh -- shared device helpers for the groupby kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "errbits.hpp"
#include "tambear_gb.h"

namespace tbgb {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier + 1-D bulk async copy (TMA engine, no multicast) -----------------
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

// try_wait with a suspend-time hint: the thread sleeps until the phase completes
// (or ~hint_ns passes) instead of spinning, leaving issue slots to working warps.
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

// Bounded wait: gives up after ~2 s of wall time and reports KERR_TIMEOUT
// instead of spinning forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && globaltimer_ns() - t0 > 2000000000ull) {
      atomicOr(err, KERR_TIMEOUT);
      return false;
    }
  }
}

// Global -> shared bulk copy completing on `bar`. dst, src and bytes must be
// multiples of 16 (callers check alignment on the host and in-kernel).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (no shared memory involved); src and
// bytes must be 16-byte aligned / multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- value helpers --------------------------------------------------------------
__device__ __forceinline__ bool is_nan(double v) { return v != v; }
__device__ __forceinline__ bool is_finite(double v) { return fabs(v) < __longlong_as_double(0x7FF0000000000000LL); }
__device__ __forceinline__ double pos_inf() { return __longlong_as_double(0x7FF0000000000000LL); }
__device__ __forceinline__ double neg_inf() { return __longlong_as_double(static_cast<long long>(0xFFF0000000000000ULL)); }
__device__ __forceinline__ double qnan() { return __longlong_as_double(0x7FF8000000000000LL); }

// Code for "this row holds a zero": rows are compared by index, sign in bit 0.
// The extrema of a group whose min (max) is zero take the sign of the group's
// first zero row -- what a sequential `if v < acc` scan produces.
__device__ __forceinline__ unsigned long long zero_code(long long row, double v) {
  return (static_cast<unsigned long long>(row) << 1) |
         (static_cast<unsigned long long>(__double_as_longlong(v)) >> 63);
}

}  // namespace tbgb
