// gemm_decode.cu — int4 x int8 GEMM for decode shapes (small M), sm_100a.
//
// Memory-bound regime: the weight stream (N*K/2 bytes of codes plus group
// scales and zero points) dominates.  A CTA owns one 16-row block of the
// output features (one column of tile records) and walks the K groups with
// NW warps; each warp streams its groups' 1072-byte records with 16-byte
// non-allocating loads, expands the int4 codes to signed int8 (q - z) in
// registers, and feeds int8 mma.sync m16n8k32 (A = weights 16 rows x 32 K,
// B = 8 tokens).  Each group's int32 accumulators are exact; they are scaled
// by the group scale into float32 per group, summed across warps in shared
// memory, multiplied by the per-token scale and stored.
//
// The record layout puts, for lane (gid = lane/4, tig = lane%4), the A
// fragment words of rows gid and gid+8 for all four 32-K steps of a group in
// one 16-byte chunk each: low nibbles give a0/a1 (k = 4*tig..+3), high nibbles
// a2/a3 (k = 16 + 4*tig..+3).
#include "paro_common.cuh"

namespace paro {

constexpr int kDecWarps = 4;

__device__ __forceinline__ uint32_t expand_lo(uint32_t w, uint32_t zz) {
  // bytes 0x80 + q - z (no borrows since q, z <= 15), then flip the bias bit
  return (((w & 0x0F0F0F0Fu) | 0x80808080u) - zz) ^ 0x80808080u;
}
__device__ __forceinline__ uint32_t expand_hi(uint32_t w, uint32_t zz) {
  return ((((w >> 4) & 0x0F0F0F0Fu) | 0x80808080u) - zz) ^ 0x80808080u;
}

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ float load_as_f32(const void* p, size_t i) {
  return to_f32(static_cast<const T*>(p)[i]);
}

__device__ __forceinline__ float bias_at(const void* bias, int dtype, int n) {
  if (!bias) return 0.f;
  if (dtype == PARO_F16) return load_as_f32<__half>(bias, n);
  if (dtype == PARO_BF16) return load_as_f32<__nv_bfloat16>(bias, n);
  return load_as_f32<float>(bias, n);
}

__device__ __forceinline__ void store_out(void* out, int dtype, size_t idx, float v) {
  if (dtype == PARO_F16) static_cast<__half*>(out)[idx] = __float2half_rn(v);
  else if (dtype == PARO_BF16) static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else static_cast<float*>(out)[idx] = v;
}

// MT = number of 8-token tiles handled per CTA (tokens blockIdx.y*8*MT ...).
template <int MT>
__global__ void __launch_bounds__(kDecWarps * 32)
gemm_decode_kernel(const int8_t* __restrict__ xq, const float* __restrict__ xscale, int64_t M, int N, int K,
                   const uint8_t* __restrict__ packed, const void* __restrict__ bias, int bias_dtype,
                   void* __restrict__ out, int out_dtype) {
  __shared__ float red[kDecWarps][MT][4][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int nb = blockIdx.x;
  const int64_t tok0 = (int64_t)blockIdx.y * (8 * MT);
  const int G = K / kGroup;

  // token rows this lane feeds as the B operand (column gid of each tile)
  const int8_t* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int64_t t = tok0 + mt * 8 + gid;
    xvalid[mt] = t < M;
    xrow[mt] = xq + (xvalid[mt] ? t : 0) * (int64_t)K + 4 * tig;
  }

  float y[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;

  const uint8_t* rec0 = packed + rec_offset(nb, 0, G);
  int g = warp;
  int4 wa, wb;
  if (g < G) {
    const uint8_t* rec = rec0 + (size_t)g * kRecBytes;
    wa = ldg_nc_v4(rec + gid * 64 + tig * 16);
    wb = ldg_nc_v4(rec + (gid + 8) * 64 + tig * 16);
  }
  for (; g < G; g += kDecWarps) {
    const uint8_t* rec = rec0 + (size_t)g * kRecBytes;
    // scales / zero points of rows gid and gid+8
    const uint16_t* sp = reinterpret_cast<const uint16_t*>(rec + kRecScaleOff);
    const float s_lo = half_bits_to_f32(sp[gid]), s_hi = half_bits_to_f32(sp[gid + 8]);
    const uint32_t zz_lo = (uint32_t)rec[kRecZeroOff + gid] * 0x01010101u;
    const uint32_t zz_hi = (uint32_t)rec[kRecZeroOff + gid + 8] * 0x01010101u;
    const uint32_t wA[4] = {(uint32_t)wa.x, (uint32_t)wa.y, (uint32_t)wa.z, (uint32_t)wa.w};
    const uint32_t wB[4] = {(uint32_t)wb.x, (uint32_t)wb.y, (uint32_t)wb.z, (uint32_t)wb.w};
    // prefetch the next group's codes while this one computes
    const int gn = g + kDecWarps;
    if (gn < G) {
      const uint8_t* recn = rec0 + (size_t)gn * kRecBytes;
      wa = ldg_nc_v4(recn + gid * 64 + tig * 16);
      wb = ldg_nc_v4(recn + (gid + 8) * 64 + tig * 16);
    }
    int acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a0 = expand_lo(wA[j], zz_lo), a2 = expand_hi(wA[j], zz_lo);
      const uint32_t a1 = expand_lo(wB[j], zz_hi), a3 = expand_hi(wB[j], zz_hi);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int8_t* xp = xrow[mt] + (size_t)g * kGroup + 32 * j;
        const uint32_t b0 = xvalid[mt] ? ldg_nc_u32(xp) : 0u;
        const uint32_t b1 = xvalid[mt] ? ldg_nc_u32(xp + 16) : 0u;
        mma_s8(acc[mt], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      y[mt][0] = fmaf(s_lo, (float)acc[mt][0], y[mt][0]);
      y[mt][1] = fmaf(s_lo, (float)acc[mt][1], y[mt][1]);
      y[mt][2] = fmaf(s_hi, (float)acc[mt][2], y[mt][2]);
      y[mt][3] = fmaf(s_hi, (float)acc[mt][3], y[mt][3]);
    }
  }

#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) red[warp][mt][i][lane] = y[mt][i];
  __syncthreads();
  // every warp finishes a share of the (mt, i) slots
  for (int slot = warp; slot < MT * 4; slot += kDecWarps) {
    const int mt = slot >> 2, i = slot & 3;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) v += red[w][mt][i][lane];
    const int64_t t = tok0 + mt * 8 + 2 * tig + (i & 1);
    const int n = nb * kRecRows + gid + ((i >> 1) << 3);
    if (t < M) {
      v = v * xscale[t] + bias_at(bias, bias_dtype, n);
      store_out(out, out_dtype, (size_t)t * N + n, v);
    }
  }
}

cudaError_t launch_gemm_decode(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                               const void* bias, int bias_dtype, void* out, int out_dtype, cudaStream_t st) {
  const int nblk = N / kRecRows;
  const uint8_t* pk = static_cast<const uint8_t*>(packed);
#define PARO_DEC(MTV)                                                                                    \
  {                                                                                                      \
    dim3 grid(nblk, (unsigned)((M + 8 * MTV - 1) / (8 * MTV)));                                          \
    gemm_decode_kernel<MTV><<<grid, kDecWarps * 32, 0, st>>>(xq, xscale, M, N, K, pk, bias, bias_dtype, \
                                                            out, out_dtype);                             \
    return cudaGetLastError();                                                                           \
  }
  if (M <= 8) PARO_DEC(1)
  if (M <= 16) PARO_DEC(2)
  if (M <= 32) PARO_DEC(4)
  PARO_DEC(8)
#undef PARO_DEC
}

}  // namespace paro
