// rotq.cu — activation-side kernels of the W4A8 rotated linear (sm_100a).
//
//  * rotate_kernel   : drop-in for rotation::rotate
//                      (reference kernels/paroquant_kernels/src/rotation.cu:15-60).
//  * rotq_kernel     : channel scale + Givens layers + per-token int8 quant in one
//                      pass (rotation.cu:15-60 followed by vLLM int8_utils.py:106-128).
//  * quant_kernel    : per-token int8 quant alone (int8_utils.py:106-128).
//
// Work decomposition (rotate / rotq): a CTA owns R consecutive rows and all K
// channels.  Warp w walks the groups g = w, w + NW, ...; for each group it
// loads that group's pair indices and angles once (sin/cos through the
// __sincosf intrinsic, exactly as the reference kernel), then rotates the
// group for each of its R rows in a per-warp shared buffer (the pairs of one
// layer are disjoint, so a layer needs only a __syncwarp between reads and
// writes).  rotq keeps every rotated row in shared memory until the row's
// absolute maximum is known, then writes int8 codes with 16-byte stores.
#include "paro_common.cuh"

namespace paro {

constexpr int kRotWarps = 16;
constexpr int kRotThreads = kRotWarps * 32;
constexpr int kMaxRowsPerCta = 16;

template <typename T> struct DT;
template <> struct DT<float> { static constexpr int id = PARO_F32; };
template <> struct DT<__half> { static constexpr int id = PARO_F16; };
template <> struct DT<__nv_bfloat16> { static constexpr int id = PARO_BF16; };

__device__ __forceinline__ float load_param(const void* p, size_t idx, int dtype) {
  if (dtype == PARO_F16) return __half2float(static_cast<const __half*>(p)[idx]);
  if (dtype == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
  return static_cast<const float*>(p)[idx];
}

// Pair indices of one lane for one layer: packed (i | j << 16).
template <typename PairT>
__device__ __forceinline__ uint32_t load_pair(const PairT* pairs, size_t off) {
  uint32_t i = (uint32_t)(uint16_t)pairs[off];
  uint32_t j = (uint32_t)(uint16_t)pairs[off + 1];
  return i | (j << 16);
}

// Per-warp rotation of one group row held in `buf` (GS floats).
template <int KROT, int GS>
__device__ __forceinline__ void givens_layers(float* buf, const uint32_t (&ij)[KROT][GS / 64 > 0 ? GS / 64 : 1],
                                              const float (&cs)[KROT][GS / 64 > 0 ? GS / 64 : 1],
                                              const float (&sn)[KROT][GS / 64 > 0 ? GS / 64 : 1]) {
  constexpr int NP = GS / 64;  // pairs per lane (group/2 pairs over 32 lanes)
#pragma unroll
  for (int r = 0; r < KROT; ++r) {
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      // indices are masked into the group so a malformed table cannot reach
      // outside the warp's buffer (valid tables are permutations of 0..GS-1)
      const int i = ij[r][p] & (GS - 1), j = (ij[r][p] >> 16) & (GS - 1);
      const float c_ = cs[r][p], s_ = sn[r][p];
      const float xi = buf[i];
      const float xj = buf[j];
      buf[i] = xi * c_ + xj * s_;
      buf[j] = xi * (-s_) + xj * c_;
    }
    __syncwarp();
  }
}

// MODE 0: rotate only, store rotated rows in OutT.  MODE 1: rotate + int8 quant.
template <typename InT, typename OutT, typename PairT, int KROT, int GS, int MODE>
__global__ void __launch_bounds__(kRotThreads)
rot_kernel(const InT* __restrict__ x, int64_t M, int K,
           const void* __restrict__ scales, const void* __restrict__ theta, int param_dtype,
           const PairT* __restrict__ pairs, int rows_per_cta, int fp16_round,
           OutT* __restrict__ out, int8_t* __restrict__ out_q, float* __restrict__ out_scale) {
  static_assert(GS == 64 || GS == 128, "group size");
  constexpr int NP = GS / 64;
  constexpr int EPL = GS / 32;  // channels per lane inside a group
  extern __shared__ __align__(16) float smem[];
  float* wbuf = smem + (threadIdx.x >> 5) * GS;          // per-warp group buffer
  float* stage = smem + kRotWarps * GS;                   // [rows][K] (MODE 1)
  __shared__ float red[kRotWarps][kMaxRowsPerCta];
  __shared__ float row_inv[kMaxRowsPerCta];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta;
  const int nrows = (M - row0 < rows_per_cta) ? (int)(M - row0) : rows_per_cta;
  const int G = K / GS;
  if (MODE == 1 && lane < kMaxRowsPerCta) red[warp][lane] = 0.f;
  __syncwarp();

  for (int g = warp; g < G; g += kRotWarps) {
    uint32_t ij[KROT][NP];
    float cs[KROT][NP], sn[KROT][NP];
#pragma unroll
    for (int r = 0; r < KROT; ++r) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int pp = lane + 32 * p;
        ij[r][p] = load_pair(pairs, (size_t)r * K + (size_t)g * GS + 2 * pp);
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
      const InT* xr = x + (row0 + r) * (int64_t)K + (size_t)g * GS + lane * EPL;
#pragma unroll
      for (int e = 0; e < EPL; ++e) wbuf[lane * EPL + e] = to_f32(xr[e]) * sc[e];
      __syncwarp();
      givens_layers<KROT, GS>(wbuf, ij, cs, sn);
      float v[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) v[e] = wbuf[lane * EPL + e];
      __syncwarp();
      if constexpr (MODE == 0) {
        OutT* orow = out + (row0 + r) * (int64_t)K + (size_t)g * GS + lane * EPL;
#pragma unroll
        for (int e = 0; e < EPL; ++e) orow[e] = from_f32<OutT>(v[e]);
      } else {
        float* srow = stage + (size_t)r * K + (size_t)g * GS + lane * EPL;
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float t = fp16_round ? round_fp16(v[e]) : v[e];
          srow[e] = t;
          a = fmaxf(a, fabsf(t));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) red[warp][r] = fmaxf(red[warp][r], a);
      }
    }
  }

  if constexpr (MODE == 1) {
    __syncthreads();
    if (threadIdx.x < nrows) {
      float a = 0.f;
#pragma unroll
      for (int w = 0; w < kRotWarps; ++w) a = fmaxf(a, red[w][threadIdx.x]);
      a = fmaxf(a, 1e-10f);
      row_inv[threadIdx.x] = __fdiv_rn(127.0f, a);
      out_scale[row0 + threadIdx.x] = __fdiv_rn(a, 127.0f);
    }
    __syncthreads();
    // quantise: 16 channels per thread-step, 16-byte stores
    const int chunks = K / 16;
    for (int idx = threadIdx.x; idx < nrows * chunks; idx += kRotThreads) {
      const int r = idx / chunks, c = idx - r * chunks;
      const float inv = row_inv[r];
      const float4* s4 = reinterpret_cast<const float4*>(stage + (size_t)r * K + c * 16);
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 f = s4[q];
        const int a0 = (int)round_half_away(f.x * inv), a1 = (int)round_half_away(f.y * inv);
        const int a2 = (int)round_half_away(f.z * inv), a3 = (int)round_half_away(f.w * inv);
        wv[q] = (uint32_t)(a0 & 0xFF) | ((uint32_t)(a1 & 0xFF) << 8) |
                ((uint32_t)(a2 & 0xFF) << 16) | ((uint32_t)(a3 & 0xFF) << 24);
      }
      *reinterpret_cast<int4*>(out_q + (row0 + r) * (int64_t)K + c * 16) =
          make_int4((int)wv[0], (int)wv[1], (int)wv[2], (int)wv[3]);
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

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
static int rows_for(int K, int elem_bytes_stage) {
  // keep the staged rows within ~160 KB of shared memory
  const size_t budget = 160 * 1024 - kRotWarps * kGroup * sizeof(float);
  int r = (int)(budget / ((size_t)K * elem_bytes_stage));
  if (r > kMaxRowsPerCta) r = kMaxRowsPerCta;
  return r;
}

template <typename InT, int KROT, int GS>
static cudaError_t launch_rotate_t(const void* x, int64_t M, int K, const void* scales, const void* theta,
                                   int pdt, const int16_t* pairs, void* out, cudaStream_t st) {
  const int rows = 8;
  const size_t smem = kRotWarps * GS * sizeof(float);
  dim3 grid((unsigned)((M + rows - 1) / rows));
  rot_kernel<InT, InT, int16_t, KROT, GS, 0><<<grid, kRotThreads, smem, st>>>(
      static_cast<const InT*>(x), M, K, scales, theta, pdt, pairs, rows, 0, static_cast<InT*>(out), nullptr,
      nullptr);
  return cudaGetLastError();
}

template <typename InT>
static cudaError_t launch_rotate_k(int krot, int group, const void* x, int64_t M, int K, const void* scales,
                                   const void* theta, int pdt, const int16_t* pairs, void* out,
                                   cudaStream_t st) {
#define PARO_ROT_CASE(KR, GSZ) \
  if (krot == KR && group == GSZ) return launch_rotate_t<InT, KR, GSZ>(x, M, K, scales, theta, pdt, pairs, out, st);
  PARO_ROT_CASE(1, 128) PARO_ROT_CASE(2, 128) PARO_ROT_CASE(4, 128) PARO_ROT_CASE(8, 128) PARO_ROT_CASE(16, 128)
  PARO_ROT_CASE(1, 64) PARO_ROT_CASE(2, 64) PARO_ROT_CASE(4, 64) PARO_ROT_CASE(8, 64) PARO_ROT_CASE(16, 64)
#undef PARO_ROT_CASE
  return cudaErrorInvalidValue;
}

cudaError_t launch_rotate(int x_dtype, int krot, int group, const void* x, int64_t M, int K, const void* scales,
                          const void* theta, int pdt, const int16_t* pairs, void* out, cudaStream_t st) {
  switch (x_dtype) {
    case PARO_F32: return launch_rotate_k<float>(krot, group, x, M, K, scales, theta, pdt, pairs, out, st);
    case PARO_F16: return launch_rotate_k<__half>(krot, group, x, M, K, scales, theta, pdt, pairs, out, st);
    case PARO_BF16: return launch_rotate_k<__nv_bfloat16>(krot, group, x, M, K, scales, theta, pdt, pairs, out, st);
  }
  return cudaErrorInvalidValue;
}

template <typename InT>
static cudaError_t launch_rotq_t(const void* x, int64_t M, int K, const uint16_t* scales, const uint16_t* theta,
                                 const uint8_t* pairs, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  const int rows = rows_for(K, sizeof(float));
  if (rows < 1) return cudaErrorInvalidValue;
  const size_t smem = kRotWarps * kGroup * sizeof(float) + (size_t)rows * K * sizeof(float);
  auto kern = rot_kernel<InT, InT, uint8_t, 8, 128, 1>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((M + rows - 1) / rows));
  kern<<<grid, kRotThreads, smem, st>>>(static_cast<const InT*>(x), M, K, scales, theta, PARO_F16, pairs, rows,
                                        fp16_round, nullptr, q, s);
  return cudaGetLastError();
}

cudaError_t launch_rotq(int x_dtype, const void* x, int64_t M, int K, const uint16_t* scales, const uint16_t* theta,
                        const uint8_t* pairs, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  switch (x_dtype) {
    case PARO_F32: return launch_rotq_t<float>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
    case PARO_F16: return launch_rotq_t<__half>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
    case PARO_BF16: return launch_rotq_t<__nv_bfloat16>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
  }
  return cudaErrorInvalidValue;
}

int rotq_max_k() { return (int)((160 * 1024 - kRotWarps * kGroup * sizeof(float)) / sizeof(float)); }

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
