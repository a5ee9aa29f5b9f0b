// rotq_fused.cu — fused channel scale + Givens rotation + per-token int8
// quantisation (sm_100a): the activation half of one W4A8 rotated linear.
//
// Replaces the reference's rotation::rotate (kernels/paroquant_kernels/src/
// rotation.cu:15-60, RotateAccess<__half> in rotation.cuh:248-337) followed by
// vLLM's per_token_quant_int8 (int8_utils.py:106-128), in one pass over HBM.
//
// Owner-channel formulation: thread (group slot gs, channel ch) owns channel
// ch of a group for R rows and keeps those R values in registers through all
// layers.  A layer is a set of disjoint pairs; per layer each thread
//   1. publishes its R values to shared memory (consecutive threads write
//      consecutive slots, so the store is bank-conflict free),
//   2. one barrier,
//   3. reads its partner's R values and computes its own half of the
//      rotation:  i' = c*i + s*j  (role i),  j' = -s*i + c*j  (role j),
//      with both products and the sum rounded separately, as the
//      reference's c*a + s*b is evaluated.
// Shared buffers alternate between layers, so one barrier per layer is
// enough.  The per-channel table (partner, role, fp16 angle; built at load
// time by paro_prepare_rotation) is one 32-bit word per channel per layer;
// all layers' words are staged into shared memory with cp.async at start.
//
// The row's absolute maximum spans all K channels: a thread-block cluster of
// C <= 8 CTAs covers a row block's groups, each CTA reduces its rows' maxima,
// and the CTAs exchange them through distributed shared memory.  Rotated
// values never leave registers; the int8 codes are written once.
#include <cooperative_groups.h>

#include "paro_common.cuh"

namespace paro {

constexpr int kFusedMaxP = 8;

struct FusedGeom {
  int C, gpc, GB, P;
};

static FusedGeom fused_geom(int K) {
  const int G = K / kGroup;
  FusedGeom f;
  f.C = G < 8 ? G : 8;
  f.gpc = (G + f.C - 1) / f.C;
  f.GB = f.gpc < 4 ? f.gpc : 4;
  f.P = (f.gpc + f.GB - 1) / f.GB;
  return f;
}

template <int R>
__device__ __forceinline__ void st_vec(float* p, const float (&v)[R]) {
  if constexpr (R == 1) {
    p[0] = v[0];
  } else if constexpr (R == 2) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int q = 0; q < R / 4; ++q)
      reinterpret_cast<float4*>(p)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
}

template <int R>
__device__ __forceinline__ void ld_vec(const float* p, float (&v)[R]) {
  if constexpr (R == 1) {
    v[0] = p[0];
  } else if constexpr (R == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x;
    v[1] = a.y;
  } else {
#pragma unroll
    for (int q = 0; q < R / 4; ++q) {
      const float4 a = reinterpret_cast<const float4*>(p)[q];
      v[4 * q] = a.x;
      v[4 * q + 1] = a.y;
      v[4 * q + 2] = a.z;
      v[4 * q + 3] = a.w;
    }
  }
}

template <typename InT, int R, int PM>
__global__ void __launch_bounds__(512)
rotq_fused_kernel(const InT* x, int64_t M, int K, const uint16_t* __restrict__ scales,
                  const uint32_t* __restrict__ rtab, int fp16_round, int gpc, int GB, int P,
                  int8_t* __restrict__ out_q, float* __restrict__ out_scale) {
  namespace cg = cooperative_groups;
  // let the GEMM that consumes these codes start its weight stream now
  asm volatile("griddepcontrol.launch_dependents;");
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float smem_f[];
  uint32_t* tabs = reinterpret_cast<uint32_t*>(smem_f);      // [8][P][GB][128] rotation table slice
  float* xb = smem_f + (size_t)8 * P * GB * 128;             // [2][P][GB][128][R]
  __shared__ float wred[16][R];
  __shared__ float cta_max[R];
  __shared__ float row_inv[R];

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int ch = t & 127, gs = t >> 7;
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int G = K >> 7;
  const int64_t row0 = (int64_t)blockIdx.y * R;
  const int nrows = (M - row0 < R) ? (int)(M - row0) : R;
  const size_t plane = (size_t)P * GB * 128 * R;

  int goff[PM];   // channel offset of pass p's group, or -1
#pragma unroll
  for (int p = 0; p < PM; ++p) {
    const int gl = gs + p * GB;
    const int g = crank * gpc + gl;
    goff[p] = (p < P && gl < gpc && g < G) ? g * 128 + ch : -1;
  }

  // every layer's table entry of this thread's channels, copied to shared
  // memory asynchronously so all the loads are in flight at once; each
  // thread reads back only its own entries (no barrier needed)
  const size_t tslot = (size_t)gs * 128 + ch;
#pragma unroll
  for (int l = 0; l < 8; ++l)
#pragma unroll
    for (int p = 0; p < PM; ++p)
      if (goff[p] >= 0) {
        const uint32_t dst = smem_u32(tabs + ((size_t)l * P + p) * GB * 128 + tslot);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(rtab + (size_t)l * K + goff[p])
                     : "memory");
      }
  asm volatile("cp.async.commit_group;" ::: "memory");

  // x is the previous kernel's output: wait for that grid (a no-op when this
  // launch has no programmatic dependency)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float v[PM][R];
#pragma unroll
  for (int p = 0; p < PM; ++p) {
    const float sc = (goff[p] >= 0 && scales) ? half_bits_to_f32(scales[goff[p]]) : 1.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
      v[p][r] = (goff[p] >= 0 && r < nrows) ? ld_dep(x + (row0 + r) * (int64_t)K + goff[p]) * sc : 0.f;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");

#pragma unroll
  for (int l = 0; l < 8; ++l) {
    float* buf = xb + (l & 1) * plane;
#pragma unroll
    for (int p = 0; p < PM; ++p)
      if (p < P) st_vec<R>(buf + ((size_t)(p * GB + gs) * 128 + ch) * R, v[p]);
    __syncthreads();
#pragma unroll
    for (int p = 0; p < PM; ++p) {
      if (goff[p] >= 0) {
        const uint32_t tab = tabs[((size_t)l * P + p) * GB * 128 + tslot];
        const int partner = tab & 0x7F;
        const bool role_j = (tab >> 7) & 1;
        float s_, c_;
        __sincosf(half_bits_to_f32((uint16_t)(tab >> 16)), &s_, &c_);
        float w[R];
        ld_vec<R>(buf + ((size_t)(p * GB + gs) * 128 + partner) * R, w);
        // first element of the pair: c*i + s*j; second: -s*i + c*j
        const float cp = role_j ? -s_ : s_;
#pragma unroll
        for (int r = 0; r < R; ++r) v[p][r] = givens(v[p][r], w[r], c_, cp);
      }
    }
  }

  // fp16 store rounding of the reference's rotate kernel, row maxima
  float rmax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rmax[r] = 0.f;
#pragma unroll
  for (int p = 0; p < PM; ++p) {
    if (goff[p] >= 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (fp16_round) v[p][r] = round_fp16(v[p][r]);
        rmax[r] = fmaxf(rmax[r], fabsf(v[p][r]));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float a = rmax[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) wred[warp][r] = a;
  }
  __syncthreads();
  if (t < R) {
    float a = 0.f;
    const int nw = blockDim.x >> 5;
    for (int w = 0; w < nw; ++w) a = fmaxf(a, wred[w][t]);
    cta_max[t] = a;
  }
  cluster.sync();
  if (t < R) {
    float a = 0.f;
    for (int c = 0; c < csize; ++c) a = fmaxf(a, cluster.map_shared_rank(cta_max, c)[t]);
    a = fmaxf(a, 1e-10f);
    row_inv[t] = __fdiv_rn(127.0f, a);
    if (crank == 0 && t < nrows) out_scale[row0 + t] = __fdiv_rn(a, 127.0f);
  }
  // all remote reads are done before any CTA of the cluster exits, and
  // row_inv is visible to every thread of this CTA
  cluster.sync();
#pragma unroll
  for (int p = 0; p < PM; ++p) {
    if (goff[p] >= 0) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (r < nrows) out_q[(row0 + r) * (int64_t)K + goff[p]] = (int8_t)(int)round_half_away(v[p][r] * row_inv[r]);
    }
  }
}

template <typename InT, int R, int PM>
static cudaError_t launch_fused(const FusedGeom& f, const void* x, int64_t M, int K, const uint16_t* scales,
                                const uint32_t* rtab, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  const size_t smem = (8 + 2 * (size_t)R) * f.P * f.GB * 128 * sizeof(float);
  auto kern = rotq_fused_kernel<InT, R, PM>;
  cudaError_t e = ensure_smem_limit((const void*)kern, 200 * 1024);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)f.C, (unsigned)((M + R - 1) / R), 1);
  cfg.blockDim = dim3((unsigned)(128 * f.GB), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)f.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // overlap the table staging with the previous kernel's tail
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<const InT*>(x), M, K, scales, rtab, fp16_round, f.gpc, f.GB, f.P,
                            q, s);
}

// Rows per cluster: as many as the shared buffers allow, up to 8.
template <typename InT, int PM>
static cudaError_t launch_fused_r(const FusedGeom& f, const void* x, int64_t M, int K, const uint16_t* scales,
                                  const uint32_t* rtab, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  const size_t unit = (size_t)f.P * f.GB * 128 * sizeof(float);  // tables take 8 units, rows 2 units each
  const size_t budget = 200 * 1024;
  auto fits = [&](int r) { return (8 + 2 * (size_t)r) * unit <= budget; };
  if (M <= 1 || !fits(2)) return launch_fused<InT, 1, PM>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  if (M <= 2 || !fits(4)) return launch_fused<InT, 2, PM>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  if (M <= 4 || !fits(8)) return launch_fused<InT, 4, PM>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  return launch_fused<InT, 8, PM>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
}

template <typename InT>
static cudaError_t launch_fused_t(const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab,
                                  int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  const FusedGeom f = fused_geom(K);
  if (f.P <= 1) return launch_fused_r<InT, 1>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  if (f.P <= 2) return launch_fused_r<InT, 2>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  if (f.P <= 4) return launch_fused_r<InT, 4>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
  return launch_fused_r<InT, 8>(f, x, M, K, scales, rtab, fp16_round, q, s, st);
}

cudaError_t launch_rotq(int x_dtype, const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab,
                        int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  switch (x_dtype) {
    case PARO_F32: return launch_fused_t<float>(x, M, K, scales, rtab, fp16_round, q, s, st);
    case PARO_F16: return launch_fused_t<__half>(x, M, K, scales, rtab, fp16_round, q, s, st);
    case PARO_BF16: return launch_fused_t<__nv_bfloat16>(x, M, K, scales, rtab, fp16_round, q, s, st);
  }
  return cudaErrorInvalidValue;
}

// Largest K the fused kernel accepts: at most kFusedMaxP passes of 4 groups
// per CTA over an 8-CTA cluster.
int rotq_max_k() { return 8 * 4 * kFusedMaxP * kGroup; }

}  // namespace paro
