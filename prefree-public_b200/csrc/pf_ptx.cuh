// Thin inline-PTX wrappers for sm_100a: mbarriers, bulk (non-tensor) TMA
// copies global -> shared, L2 cache policies, named barriers, the global timer.
// No cluster multicast anywhere: every copy lands in the issuing CTA's own
// shared memory.
#pragma once

#include <cstdint>

#include "pf_common.cuh"

namespace pf {
namespace ptx {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// make mbarrier initialisation visible to the async proxy (bulk copies)
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// true once the phase with the given parity has completed
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// waits at most about `hint_ns` (the hardware may return earlier), then
// reports whether the phase completed: a polling loop that sleeps instead of
// spinning
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// barrier over `nthreads` threads that also ANDs a predicate across them
__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same shared memory
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// asynchronous 8-byte copy global -> shared (zero-filled when !valid, no read)
__device__ __forceinline__ void cp_async8(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 8 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// non-blocking probe
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after `limit_ns` of wall time (returns false).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk copy global -> this CTA's shared memory, completion counted on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Read-only loads with an L2 eviction hint. Not volatile, so the compiler can
// batch several of them before their first use; callers make them
// unconditional (clamped addresses) so no load is ever speculated past a guard.
template <typename T>
__device__ __forceinline__ T ldg_hint(const T *p, uint64_t policy);

template <>
__device__ __forceinline__ double ldg_hint<double>(const double *p, uint64_t policy) {
  double v;
  asm("ld.global.nc.L2::cache_hint.f64 %0, [%1], %2;" : "=d"(v) : "l"(p), "l"(policy));
  return v;
}

template <>
__device__ __forceinline__ float ldg_hint<float>(const float *p, uint64_t policy) {
  float v;
  asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(policy));
  return v;
}

template <>
__device__ __forceinline__ int32_t ldg_hint<int32_t>(const int32_t *p, uint64_t policy) {
  int32_t v;
  asm("ld.global.nc.L2::cache_hint.s32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(policy));
  return v;
}

// x gathers: read-only loads that ask L2 for a 64-byte fill on a miss. A
// random 8-byte gather into a vector far larger than L2 then costs ~58 DRAM
// bytes instead of the ~107 of the default fill (measured on B200: 81.7 M vs
// 145.6 M sectors for 41.9 M gathers into 512 MB); hits are unchanged.
template <typename T>
__device__ __forceinline__ T ldg_x(const T *p);

template <>
__device__ __forceinline__ double ldg_x<double>(const double *p) {
  double v;
  asm("ld.global.nc.L2::64B.f64 %0, [%1];" : "=d"(v) : "l"(p));
  return v;
}

template <>
__device__ __forceinline__ float ldg_x<float>(const float *p) {
  float v;
  asm("ld.global.nc.L2::64B.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

template <typename H>
__device__ __forceinline__ H ldg_x_16(const H *p) {
  unsigned short v;
  asm("ld.global.nc.L2::64B.b16 %0, [%1];" : "=h"(v) : "l"(p));
  return half_from_bits<H>(v);
}

template <>
__device__ __forceinline__ __half ldg_x<__half>(const __half *p) {
  return ldg_x_16(p);
}

template <>
__device__ __forceinline__ __nv_bfloat16 ldg_x<__nv_bfloat16>(const __nv_bfloat16 *p) {
  return ldg_x_16(p);
}

// 16-byte pieces of a dense row gathered by column index (SpMM's X rows),
// with the same 64-byte fill
__device__ __forceinline__ double2 ldg_x_v2(const double2 *p) {
  double2 v;
  asm("ld.global.nc.L2::64B.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ float4 ldg_x_v4(const float4 *p) {
  float4 v;
  asm("ld.global.nc.L2::64B.v4.f32 {%0, %1, %2, %3}, [%4];"
      : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
      : "l"(p));
  return v;
}

// 16-bit values: a 16-bit load of the bit pattern
template <typename H>
__device__ __forceinline__ H ldg_hint_16(const H *p, uint64_t policy) {
  unsigned short v;
  asm("ld.global.nc.L2::cache_hint.b16 %0, [%1], %2;" : "=h"(v) : "l"(p), "l"(policy));
  return half_from_bits<H>(v);
}

template <>
__device__ __forceinline__ __half ldg_hint<__half>(const __half *p, uint64_t policy) {
  return ldg_hint_16(p, policy);
}

template <>
__device__ __forceinline__ __nv_bfloat16 ldg_hint<__nv_bfloat16>(const __nv_bfloat16 *p,
                                                                 uint64_t policy) {
  return ldg_hint_16(p, policy);
}

}  // namespace ptx
}  // namespace pf
