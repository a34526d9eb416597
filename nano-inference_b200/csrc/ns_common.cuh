// Device helpers shared by the sampler kernels (sm_100a).
//
// - mbarrier / bulk-copy (TMA, non-tensor) wrappers in inline PTX,
// - order-preserving float <-> uint32 keys for radix selection,
// - Philox4x32-10 (Salmon et al., SC'11) for the default uniform stream,
// - bounded waits: every spin gives up after kWaitTimeoutNs of wall time.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ns {

constexpr uint64_t kWaitTimeoutNs = 200ull * 1000ull * 1000ull;  // 200 ms

// ---------------------------------------------------------------------------
// keys
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t f2key(float f) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(f);
#else
  uint32_t u;
  __builtin_memcpy(&u, &f, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

// ---------------------------------------------------------------------------
// Philox4x32-10.  counter = (row_lo, row_hi, offset_lo, offset_hi),
// key = (seed_lo, seed_hi); u = (word0 >> 8) * 2^-24.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t offset, uint64_t row) {
  uint32_t c0 = (uint32_t)row, c1 = (uint32_t)(row >> 32);
  uint32_t c2 = (uint32_t)offset, c3 = (uint32_t)(offset >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
    const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    if (r < 9) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
  }
  return (float)(c0 >> 8) * (1.0f / 16777216.0f);
}

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`; false if it did not complete within
// kWaitTimeoutNs (the caller records an error and keeps control flow uniform).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

// System-scope flag protocol between GPUs (peer memory over NVLink): the
// writer fences its prior writes and releases the flag; a reader acquires it.
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Wait until *p >= target; false if that did not happen within kWaitTimeoutNs.
__device__ __forceinline__ bool flag_wait_bounded(const int64_t* p, int64_t target) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(p) >= target) return true;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16; this CTA only.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk copy) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// max that propagates NaN (PTX max.NaN, sm_80+): NaN if either input is NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// 2^a by the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22; results below 2^-126 flush to zero).
__device__ __forceinline__ float ex2_approx(float a) {
  float d;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(d) : "f"(a));
  return d;
}

// min that propagates NaN (PTX min.NaN, sm_80+).
__device__ __forceinline__ float fmin_nan(float a, float b) {
  float d;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace ns
