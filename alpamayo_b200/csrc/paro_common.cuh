// paro_common.cuh — shared definitions for the sm_100a ParoQuant W4A8 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/paro_b200.h"

namespace paro {

constexpr int kGroup = 128;          // int4 quantisation group (K channels)
constexpr int kRecRows = 16;         // output rows per tile record
constexpr int kRecCodeBytes = kRecRows * 64;              // 16 rows x 128 nibbles
constexpr int kRecScaleOff = kRecCodeBytes;               // 16 x fp16 scales
constexpr int kRecZeroOff = kRecCodeBytes + kRecRows * 2; // 16 x uint8 zero points
constexpr int kRecBytes = kRecZeroOff + kRecRows;         // 1072 (= 67 x 16)

static_assert(kRecBytes % 16 == 0, "records must stay 16-byte aligned");

// Byte offset of record (row block nb, group g) for a layer with G groups.
__host__ __device__ __forceinline__ size_t rec_offset(int nb, int g, int G) {
  return ((size_t)nb * G + g) * kRecBytes;
}

// Position of code k (0..127 within a group) inside a row's 64 bytes: with
// k = 64h + 32s + 16f + 4t + b it is byte t*16 + (2s + f)*4 + b, low nibble
// for h = 0 and high nibble for h = 1.
__host__ __device__ __forceinline__ int code_byte_pos(int k) {
  const int s = (k >> 5) & 1, f = (k >> 4) & 1, t = (k >> 2) & 3, b = k & 3;
  return t * 16 + (2 * s + f) * 4 + b;
}
__host__ __device__ __forceinline__ int code_nibble(int k) { return k >> 6; }

// ---------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

__device__ __forceinline__ float half_bits_to_f32(uint16_t b) {
  return __half2float(__ushort_as_half(b));
}

// Round a float32 to the nearest fp16 value (ties to even) and back.
__device__ __forceinline__ float round_fp16(float v) {
  return __half2float(__float2half_rn(v));
}

// Round half away from zero (libdevice round semantics used by the
// reference's Triton quantiser); calls the CUDA math library's roundf.
__device__ __forceinline__ float round_half_away(float v) { return roundf(v); }

// One Givens update of a channel: x' = x * p + partner * q, both products and
// the sum rounded separately (the reference evaluates c*a + s*b as two
// multiplies and an add), so the result does not depend on which operand
// comes first.
__device__ __forceinline__ float givens(float x, float partner, float p, float q) {
  return __fadd_rn(__fmul_rn(x, p), __fmul_rn(partner, q));
}

// The same on two rows at once (packed float32 pairs, sm_100).
__device__ __forceinline__ float2 givens2(float2 x, float2 partner, float p, float q) {
  uint64_t xv, wv, pv, qv, a, b, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(xv) : "f"(x.x), "f"(x.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(wv) : "f"(partner.x), "f"(partner.y));
  asm("mov.b64 %0, {%1, %1};" : "=l"(pv) : "f"(p));
  asm("mov.b64 %0, {%1, %1};" : "=l"(qv) : "f"(q));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(a) : "l"(xv), "l"(pv));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(b) : "l"(wv), "l"(qv));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}

// Loads of data that the previous kernel on the stream writes, in a kernel
// launched with programmatic dependent launch: it may start before that
// kernel ends, so these loads must stay after its griddepcontrol.wait.
// Plain loads through const __restrict__ pointers may be compiled as
// invariant (read-only path) loads, which the compiler is free to move above
// the wait; volatile asm with a memory clobber keeps them in place.
__device__ __forceinline__ uint32_t ld_dep_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_dep(const float* p) {
  float v;
  asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_dep(const __half* p) {
  unsigned short b;
  asm volatile("ld.global.u16 %0, [%1];" : "=h"(b) : "l"(p) : "memory");
  return __half2float(__ushort_as_half(b));
}
__device__ __forceinline__ float ld_dep(const __nv_bfloat16* p) {
  unsigned short b;
  asm volatile("ld.global.u16 %0, [%1];" : "=h"(b) : "l"(p) : "memory");
  return __uint_as_float((uint32_t)b << 16);  // bf16 is the high half of a float32
}

// L2 (.cg) accesses to data shared between CTAs or grids, as volatile asm
// with a memory clobber so that they keep their place relative to the
// fences, barriers and dependency waits that order them.
__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_cg_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}
// The same without the memory clobber, for loads issued in bulk whose order
// against other memory operations does not matter (they follow the
// dependency wait in program order: volatile asm keeps that order).
__device__ __forceinline__ uint4 ld_l2_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ int2 ld_l2_v2(const int* p) {
  int2 v;
  asm volatile("ld.global.cg.v2.s32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_cg_f32(float* p, float v) {
  asm volatile("st.global.cg.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// The decoder-layer step a decode-size linear can fuse into its rotation
// kernel's input load (rotq_decode.cu): none, residual add + RMSNorm, or
// SiLU(gate) * up.
constexpr int kProNone = 0;
constexpr int kProAddRmsnorm = 1;
constexpr int kProSiluMul = 2;

struct RotPro {
  const __nv_bfloat16* res_in;   // residual stream in [M, K] or null
  __nv_bfloat16* res_out;        // bf16(x + res_in) (x when null) [M, K]; must not overlap res_in or x
  const __nv_bfloat16* w;        // RMSNorm weight [K]
  float eps;
};

// Per-projection rotation tables of a group of linears that share their
// input (q / k / v, gate / up of a real checkpoint): the decode activation
// kernels take the table index from blockIdx.z and write one activation
// set per table.
constexpr int kMaxTables = 4;
struct RotTables {
  const uint32_t* rtab[kMaxTables];
  const uint16_t* cs[kMaxTables];
};

// Raise a kernel's dynamic shared-memory limit to `bytes` once per (kernel,
// device); later calls are a map lookup instead of a driver call.
cudaError_t ensure_smem_limit(const void* kernel, int bytes);

// ---------------------------------------------------------------------------
// small PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ int4 ldg_nc_v4(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

}  // namespace paro
