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
#include <cooperative_groups.h>

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

// ---------------------------------------------------------------------------
// Fused rotation + int8 quantisation, cluster version.
//
// A thread-block cluster of C CTAs owns R consecutive rows; CTA c of the
// cluster owns groups [c*gpc, (c+1)*gpc) and one warp per group, so all
// groups of a row block rotate in parallel.  Each warp loads its group's pair
// indices and angles once, then rotates all R rows together in a per-warp
// shared buffer laid out channel-major ([128][R], R floats per channel, so a
// Givens update moves R rows with vector loads).  The rotated values (fp16-
// rounded like the reference's rotate kernel output) stay in shared memory;
// each CTA's per-row absolute maxima are exchanged through distributed shared
// memory, and every warp then quantises its own group with the row scale.
// ---------------------------------------------------------------------------
template <int R>
struct RowVec;
template <> struct RowVec<1> { using T = float; };
template <> struct RowVec<2> { using T = float2; };
template <> struct RowVec<4> { using T = float4; };

template <int R>
__device__ __forceinline__ void ld_rows(const float* p, float (&v)[R]) {
  if constexpr (R == 1) {
    v[0] = p[0];
  } else if constexpr (R == 2) {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x; v[1] = a.y;
  } else {
#pragma unroll
    for (int q = 0; q < R / 4; ++q) {
      const float4 a = reinterpret_cast<const float4*>(p)[q];
      v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
    }
  }
}

template <int R>
__device__ __forceinline__ void st_rows(float* p, const float (&v)[R]) {
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

template <typename InT>
__device__ __forceinline__ void load4(const InT* p, float (&v)[4]) {
  if constexpr (sizeof(InT) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    const uint2 a = *reinterpret_cast<const uint2*>(p);
    const InT* h = reinterpret_cast<const InT*>(&a);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = to_f32(h[e]);
  }
}

template <typename InT, int R>
__global__ void __launch_bounds__(512)
rotq_cluster_kernel(const InT* __restrict__ x, int64_t M, int K, const uint16_t* __restrict__ scales,
                    const uint16_t* __restrict__ theta, const uint8_t* __restrict__ pairs, int fp16_round, int gpc,
                    int8_t* __restrict__ out_q, float* __restrict__ out_scale) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) float gbuf[];  // [gpc][128][R]
  __shared__ float wmax[32][R];
  __shared__ float cta_max[R];
  __shared__ float row_inv[R];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int G = K >> 7;
  const int64_t row0 = (int64_t)blockIdx.y * R;
  const int nrows = (M - row0 < R) ? (int)(M - row0) : R;
  float rmax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) rmax[r] = 0.f;

  for (int gl = warp; gl < gpc; gl += nwarps) {
    const int g = crank * gpc + gl;
    if (g >= G) break;
    float* gb = gbuf + (size_t)gl * 128 * R;
    // this lane's pairs p = lane, lane + 32 for every layer
    uint32_t pij[8][2];  // (i * R) | (j * R) << 16
    float cs[8][2], sn[8][2];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int pp = lane + 32 * h;
        const uint16_t pr = *reinterpret_cast<const uint16_t*>(pairs + (size_t)l * K + (size_t)g * 128 + 2 * pp);
        pij[l][h] = ((uint32_t)(pr & 0x7F) * R) | (((uint32_t)(pr >> 8) & 0x7F) * R << 16);
        __sincosf(half_bits_to_f32(theta[(size_t)l * (K / 2) + (size_t)g * 64 + pp]), &sn[l][h], &cs[l][h]);
      }
    }
    float sc[4];
    if (scales) {
      const uint2 s2 = *reinterpret_cast<const uint2*>(scales + (size_t)g * 128 + 4 * lane);
      const uint16_t* sh = reinterpret_cast<const uint16_t*>(&s2);
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] = half_bits_to_f32(sh[e]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) sc[e] = 1.f;
    }
    // load and scale R rows of this group: lane owns channels 4*lane..+3
    float xv[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nrows) {
        load4(x + (row0 + r) * (int64_t)K + (size_t)g * 128 + 4 * lane, xv[r]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) xv[r][e] = 0.f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float col[R];
#pragma unroll
      for (int r = 0; r < R; ++r) col[r] = xv[r][e] * sc[e];
      st_rows<R>(gb + (4 * lane + e) * R, col);
    }
    __syncwarp();
#pragma unroll
    for (int l = 0; l < 8; ++l) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float a[R], b[R];
        const int oi = pij[l][h] & 0xFFFF, oj = pij[l][h] >> 16;
        ld_rows<R>(gb + oi, a);
        ld_rows<R>(gb + oj, b);
        const float c_ = cs[l][h], s_ = sn[l][h];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float xi = a[r], xj = b[r];
          a[r] = xi * c_ + xj * s_;
          b[r] = xi * (-s_) + xj * c_;
        }
        st_rows<R>(gb + oi, a);
        st_rows<R>(gb + oj, b);
      }
      __syncwarp();
    }
    // fp16 store rounding of the reference and the per-row maxima
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float col[R];
      ld_rows<R>(gb + (4 * lane + e) * R, col);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (fp16_round) col[r] = round_fp16(col[r]);
        rmax[r] = fmaxf(rmax[r], fabsf(col[r]));
      }
      if (fp16_round) st_rows<R>(gb + (4 * lane + e) * R, col);
    }
  }

#pragma unroll
  for (int r = 0; r < R; ++r) {
    float a = rmax[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) wmax[warp][r] = a;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float a = 0.f;
    for (int w = 0; w < nwarps; ++w) a = fmaxf(a, wmax[w][threadIdx.x]);
    cta_max[threadIdx.x] = a;
  }
  cluster.sync();
  if (threadIdx.x < R) {
    float a = 0.f;
    for (int c = 0; c < csize; ++c) a = fmaxf(a, cluster.map_shared_rank(cta_max, c)[threadIdx.x]);
    a = fmaxf(a, 1e-10f);
    row_inv[threadIdx.x] = __fdiv_rn(127.0f, a);
    if (crank == 0 && threadIdx.x < nrows) out_scale[row0 + threadIdx.x] = __fdiv_rn(a, 127.0f);
  }
  // every remote read of cta_max is done before any CTA may exit, and
  // row_inv is visible to the whole CTA
  cluster.sync();

  for (int gl = warp; gl < gpc; gl += nwarps) {
    const int g = crank * gpc + gl;
    if (g >= G) break;
    const float* gb = gbuf + (size_t)gl * 128 * R;
    float col[4][R];
#pragma unroll
    for (int e = 0; e < 4; ++e) ld_rows<R>(gb + (4 * lane + e) * R, col[e]);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nrows) {
        const float inv = row_inv[r];
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) w |= ((uint32_t)(int)round_half_away(col[e][r] * inv) & 0xFFu) << (8 * e);
        *reinterpret_cast<uint32_t*>(out_q + (row0 + r) * (int64_t)K + (size_t)g * 128 + 4 * lane) = w;
      }
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

// Cluster geometry of the fused kernel: C CTAs (<= 8, portable) split the
// groups; each CTA runs one warp per group it owns.
struct RotqGeom {
  int csize, gpc, warps;
};

static RotqGeom rotq_geom(int K) {
  const int G = K / kGroup;
  RotqGeom g;
  g.csize = G < 8 ? G : 8;
  g.gpc = (G + g.csize - 1) / g.csize;
  g.warps = g.gpc < 16 ? g.gpc : 16;
  return g;
}

template <typename InT, int R>
static cudaError_t launch_rotq_r(const void* x, int64_t M, int K, const uint16_t* scales, const uint16_t* theta,
                                 const uint8_t* pairs, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  const RotqGeom geo = rotq_geom(K);
  const size_t smem = (size_t)geo.gpc * 128 * R * sizeof(float);
  auto kern = rotq_cluster_kernel<InT, R>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)geo.csize, (unsigned)((M + R - 1) / R), 1);
  cfg.blockDim = dim3((unsigned)(32 * geo.warps), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)geo.csize;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<const InT*>(x), M, K, scales, theta, pairs, fp16_round, geo.gpc,
                            q, s);
}

template <typename InT>
static cudaError_t launch_rotq_t(const void* x, int64_t M, int K, const uint16_t* scales, const uint16_t* theta,
                                 const uint8_t* pairs, int fp16_round, int8_t* q, float* s, cudaStream_t st) {
  if (M <= 1) return launch_rotq_r<InT, 1>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
  if (M <= 2) return launch_rotq_r<InT, 2>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
  if (M <= 4) return launch_rotq_r<InT, 4>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
  return launch_rotq_r<InT, 8>(x, M, K, scales, theta, pairs, fp16_round, q, s, st);
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

// Largest K the fused kernel accepts: the rows it keeps resident
// (gpc groups x 128 channels x 8 rows x 4 bytes per CTA) must fit in 200 KB.
int rotq_max_k() { return 8 * 48 * kGroup; }

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
