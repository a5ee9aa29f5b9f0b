// elementwise.cu — the bf16 glue around the rotated linears of a decoder
// layer (decoder-stack benchmark): residual add + RMSNorm, and SiLU * up.
//
//  * add_rmsnorm_kernel: Qwen3VLTextRMSNorm (models/qwen3_vl/
//    modeling_qwen3_vl.py:340-357) with the residual add before it:
//    s = bf16(x + r); h = s * rsqrt(mean(s^2) + eps) in float32, rounded to
//    bf16, times the bf16 weight, rounded to bf16.  One CTA per row, 16-byte
//    vector accesses.
//  * silu_mul_kernel: act_fn(gate) * up on the fused gate_up output [M, 2I]:
//    bf16(bf16(g / (1 + exp(-g))) * u).
#include "paro_common.cuh"

namespace paro {

namespace {
__device__ __forceinline__ float bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}
}  // namespace

// K % 8 == 0, all rows 16-byte aligned.  residual may be null; if not, it is
// updated in place to x + residual (the next layer's residual stream).
__global__ void __launch_bounds__(256)
add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                   const __nv_bfloat16* __restrict__ weight, int K, float eps, __nv_bfloat16* __restrict__ out) {
  __shared__ float wsum[8];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * (int64_t)K);
  uint4* rr = residual ? reinterpret_cast<uint4*>(residual + row * (int64_t)K) : nullptr;
  const int n8 = K / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float a[8];
    unpack8(xr[i], a);
    if (rr) {
      float b[8];
      unpack8(rr[i], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] = bf(a[e] + b[e]);
      rr[i] = pack8(a);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(a[e], a[e], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) wsum[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += wsum[w];
  const float inv = rsqrtf(tot / (float)K + eps);
  const uint4* src = rr ? reinterpret_cast<const uint4*>(rr) : xr;
  const uint4* wr = reinterpret_cast<const uint4*>(weight);
  uint4* orow = reinterpret_cast<uint4*>(out + row * (int64_t)K);
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float a[8], w[8];
    unpack8(src[i], a);
    unpack8(wr[i], w);
#pragma unroll
    for (int e = 0; e < 8; ++e) a[e] = w[e] * bf(a[e] * inv);
    orow[i] = pack8(a);
  }
}

__global__ void __launch_bounds__(256)
silu_mul_kernel(const __nv_bfloat16* __restrict__ x, int64_t M, int I, __nv_bfloat16* __restrict__ out) {
  const int n8 = I / 8;
  const int64_t total = M * (int64_t)n8;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / n8;
    const int c8 = (int)(e - row * n8);
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * (int64_t)(2 * I));
    float g[8], u[8];
    unpack8(xr[c8], g);
    unpack8(xr[n8 + c8], u);
#pragma unroll
    for (int i = 0; i < 8; ++i) g[i] = bf(g[i] / (1.0f + expf(-g[i]))) * u[i];
    reinterpret_cast<uint4*>(out + row * (int64_t)I)[c8] = pack8(g);
  }
}

cudaError_t launch_add_rmsnorm(const void* x, void* residual, const void* weight, int64_t M, int K, float eps,
                               void* out, cudaStream_t st) {
  if (M > 0x7FFFFFFF) return cudaErrorInvalidValue;
  add_rmsnorm_kernel<<<(unsigned)M, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                    static_cast<__nv_bfloat16*>(residual),
                                                    static_cast<const __nv_bfloat16*>(weight), K, eps,
                                                    static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* x, int64_t M, int I, void* out, cudaStream_t st) {
  const int64_t total = M * (int64_t)(I / 8);
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  silu_mul_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), M, I,
                                                      static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace paro
