// tc_ptx.cuh — inline-PTX helpers for sm_100a: mbarriers with bounded waits,
// TMA bulk copies, and the library's device error word.
#pragma once

#include <stdint.h>

#include "paro_common.cuh"

namespace paro {

// Error bits a kernel sets (atomicOr) instead of hanging; read and cleared
// by paro_device_error_word().
constexpr uint32_t kErrMbarTimeout = 1u;
constexpr uint32_t kErrTmemAlloc = 2u;
constexpr uint32_t kErrGridWait = 4u;     // a wait for other CTAs of the same launch gave up

// One error word per translation unit (no relocatable device code needed);
// each .cu that uses these helpers exposes it through
// PARO_DEFINE_ERROR_ACCESSOR(name), and the C ABI ORs all of them.
static __device__ uint32_t g_device_error;

__device__ __forceinline__ void report_error(uint32_t bits) { atomicOr(&g_device_error, bits); }

#define PARO_DEFINE_ERROR_ACCESSOR(name)                                                   \
  uint32_t error_word_##name(int clear) {                                                  \
    uint32_t v = 0;                                                                        \
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return ~0u;  \
    if (clear && v) {                                                                      \
      const uint32_t z = 0;                                                                \
      if (cudaMemcpyToSymbol(g_device_error, &z, sizeof(z)) != cudaSuccess) return ~0u;   \
    }                                                                                      \
    return v;                                                                              \
  }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok;
}

// Wait for the phase with the given parity to complete.  Gives up after
// ~`limit_cycles` SM clocks (about half a second at the default), reports
// kErrMbarTimeout and returns false, so a broken pipeline ends the kernel
// instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          long long limit_cycles = 1000000000LL) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit_cycles) {
      report_error(kErrMbarTimeout);
      return false;
    }
  }
  return true;
}

// 1-D TMA bulk copy global -> shared, completing on `bar` (byte count must be
// a multiple of 16 and both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Partial sums shared between CTAs in 64-bit fixed point, 2^-28 units: range 2^35
// (a partial is at most G * 2^18 * |group scale|, so group scales up to
// ~900 in magnitude fit even for K = 18944; int4 weight scales are far
// smaller) and resolution 3.7e-9, below float32's spacing for any partial
// above 1e-3.  Integer addition makes a total independent of the order the
// partials arrive in, so the kernels that add them are deterministic.
__device__ __forceinline__ void red_add_fx(unsigned long long* p, float v) {
  const long long q = __float2ll_rn(v * 268435456.0f);
  asm volatile("red.global.add.u64 [%0], %1;" ::"l"(p), "l"((unsigned long long)q) : "memory");
}
__device__ __forceinline__ float ld_cg_fx(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return __ll2float_rn((long long)v) * 3.7252902984619141e-09f;   // 2^-28
}
__device__ __forceinline__ void st_cg_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.global.cg.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}


}  // namespace paro
