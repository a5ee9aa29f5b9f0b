// rotq.cu — the drop-in rotation kernel and the plain per-token quantiser
// (sm_100a).  The fused rotation + int8 kernel of the W4A8 path is in
// rotq_fused.cu.
//
//  * rotate_kernel : rotation::rotate (reference kernels/paroquant_kernels/src/
//                    rotation.cu:15-60): x * channel_scale, then KROT layers of
//                    disjoint Givens rotations per group, float32 math, stored in
//                    the input dtype.  Any KROT in {1,2,4,8,16}, group 64 or 128,
//                    and float32 / float16 / bfloat16 tensors and parameters.
//  * quant_kernel  : per_token_quant_int8 (vLLM int8_utils.py:106-128).
//
// rotate_kernel: a CTA owns 8 rows; warp w walks the groups w, w + 16, ...;
// per group it loads that group's pair indices and angles once (sin/cos via
// the __sincosf intrinsic, as the reference kernel), then rotates each row
// in a per-warp shared buffer (a layer's pairs are disjoint, so one
// __syncwarp per layer orders reads before writes).
#include "paro_common.cuh"

namespace paro {

constexpr int kRotWarps = 16;
constexpr int kRotThreads = kRotWarps * 32;
constexpr int kRotRows = 8;

__device__ __forceinline__ float load_param(const void* p, size_t idx, int dtype) {
  if (dtype == PARO_F16) return __half2float(static_cast<const __half*>(p)[idx]);
  if (dtype == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
  return static_cast<const float*>(p)[idx];
}

template <int KROT, int GS>
__global__ void __launch_bounds__(kRotThreads)
rotate_kernel_t(const void* __restrict__ xv, int x_dtype, int64_t M, int K, const void* __restrict__ scales,
                const void* __restrict__ theta, int param_dtype, const int16_t* __restrict__ pairs,
                void* __restrict__ outv) {
  static_assert(GS == 64 || GS == 128, "group size");
  constexpr int NP = GS / 64;   // pairs per lane
  constexpr int EPL = GS / 32;  // channels per lane
  __shared__ float wbuf_all[kRotWarps][GS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* wbuf = wbuf_all[warp];
  const int64_t row0 = (int64_t)blockIdx.x * kRotRows;
  const int nrows = (M - row0 < kRotRows) ? (int)(M - row0) : kRotRows;
  const int G = K / GS;

  for (int g = warp; g < G; g += kRotWarps) {
    int pi[KROT][NP], pj[KROT][NP];
    float cs[KROT][NP], sn[KROT][NP];
#pragma unroll
    for (int r = 0; r < KROT; ++r) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int pp = lane + 32 * p;
        const size_t off = (size_t)r * K + (size_t)g * GS + 2 * pp;
        // indices are masked into the group so a malformed table cannot reach
        // outside the warp's buffer (valid tables are permutations)
        pi[r][p] = pairs[off] & (GS - 1);
        pj[r][p] = pairs[off + 1] & (GS - 1);
        const float th = load_param(theta, (size_t)r * (K / 2) + (size_t)g * (GS / 2) + pp, param_dtype);
        __sincosf(th, &sn[r][p], &cs[r][p]);
      }
    }
    float sc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      sc[e] = scales ? load_param(scales, (size_t)g * GS + lane * EPL + e, param_dtype) : 1.f;

#pragma unroll 1
    for (int r = 0; r < nrows; ++r) {
      const size_t base = (size_t)(row0 + r) * K + (size_t)g * GS + lane * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e) wbuf[lane * EPL + e] = load_param(xv, base + e, x_dtype) * sc[e];
      __syncwarp();
#pragma unroll
      for (int l = 0; l < KROT; ++l) {
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const float c_ = cs[l][p], s_ = sn[l][p];
          const float xi = wbuf[pi[l][p]];
          const float xj = wbuf[pj[l][p]];
          wbuf[pi[l][p]] = xi * c_ + xj * s_;
          wbuf[pj[l][p]] = xi * (-s_) + xj * c_;
        }
        __syncwarp();
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const float v = wbuf[lane * EPL + e];
        if (x_dtype == PARO_F16) static_cast<__half*>(outv)[base + e] = __float2half_rn(v);
        else if (x_dtype == PARO_BF16) static_cast<__nv_bfloat16*>(outv)[base + e] = __float2bfloat16_rn(v);
        else static_cast<float*>(outv)[base + e] = v;
      }
      __syncwarp();
    }
  }
}

// Per-token int8 quantisation of an [M, K] tensor: one CTA per row.
template <typename InT>
__global__ void __launch_bounds__(256)
quant_kernel(const InT* __restrict__ x, int K, int8_t* __restrict__ out_q, float* __restrict__ out_scale) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const InT* xr = x + row * (int64_t)K;
  float a = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) a = fmaxf(a, fabsf(to_f32(xr[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  a = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) a = fmaxf(a, red[w]);
  a = fmaxf(a, 1e-10f);
  const float inv = __fdiv_rn(127.0f, a);
  if (threadIdx.x == 0) out_scale[row] = __fdiv_rn(a, 127.0f);
  int8_t* qr = out_q + row * (int64_t)K;
  for (int k = threadIdx.x; k < K; k += 256) qr[k] = (int8_t)(int)round_half_away(to_f32(xr[k]) * inv);
}

cudaError_t launch_rotate(int x_dtype, int krot, int group, const void* x, int64_t M, int K, const void* scales,
                          const void* theta, int pdt, const int16_t* pairs, void* out, cudaStream_t st) {
  dim3 grid((unsigned)((M + kRotRows - 1) / kRotRows));
#define PARO_ROT_CASE(KR, GSZ)                                                                         \
  if (krot == KR && group == GSZ) {                                                                    \
    rotate_kernel_t<KR, GSZ><<<grid, kRotThreads, 0, st>>>(x, x_dtype, M, K, scales, theta, pdt, pairs, out); \
    return cudaGetLastError();                                                                         \
  }
  PARO_ROT_CASE(1, 128) PARO_ROT_CASE(2, 128) PARO_ROT_CASE(4, 128) PARO_ROT_CASE(8, 128) PARO_ROT_CASE(16, 128)
  PARO_ROT_CASE(1, 64) PARO_ROT_CASE(2, 64) PARO_ROT_CASE(4, 64) PARO_ROT_CASE(8, 64) PARO_ROT_CASE(16, 64)
#undef PARO_ROT_CASE
  return cudaErrorInvalidValue;
}

cudaError_t launch_quant(int x_dtype, const void* x, int64_t M, int K, int8_t* q, float* s, cudaStream_t st) {
  dim3 grid((unsigned)M);
  switch (x_dtype) {
    case PARO_F32: quant_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(x), K, q, s); break;
    case PARO_F16: quant_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(x), K, q, s); break;
    case PARO_BF16:
      quant_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), K, q, s);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace paro
