// rotq_decode.cu — the rotation half of a decode-size rotated linear
// (sm_100a): channel scale + 8 Givens layers per 128-channel group, rounded
// to fp16, plus each token row's |max|.  The int8 quantisation that needs
// the whole row's maximum happens after the kernel boundary
// (quant16_decode_kernel below), so no kernel here waits for another CTA.
//
// Geometry for a handful of tokens: one CTA per (group, token row) (the
// kernel is written for blocks of R rows; R = 1 is launched), 128 threads,
// thread ch owning channel ch of the group.  A 7B-class layer has 28
// (K = 3584) or 148 (K = 18944) groups per row, so the work spreads over
// many SMs instead of the 8-CTA cluster of the single-pass kernel, and a
// CTA's critical path is one table load, one activation load and 8
// exchange rounds.  Per layer each thread publishes
// its R values to shared memory, the CTA synchronises once, and each thread
// reads its partner's values and applies its own half of the pair with both
// products and the sum rounded separately (the arithmetic of the reference's
// rotate kernel, kernels/paroquant_kernels/src/rotation.cuh:248-337, and of
// rotq_fused.cu, operation for operation).  Row maxima: a warp reduction
// of the fp16 values' bit patterns (non-negative floats order like their
// bits), then one shared-memory atomic per warp and one global atomicMax per
// row and CTA.
//
// Output order (FRAG, for the streaming GEMM): within each group the 32
// quads of 4 channels are stored in the order its mma fragments read them
// (quad j*4 + t at position t*8 + j), so the quantiser writes its int8 codes
// straight into fragment order; without FRAG (for the tensor-core GEMM's
// tiled loads) the channels keep their order.  The scratch is private to the
// linear.
//
// Prologues (PRO, the decoder-layer step before the linear, fused into the
// load of the kernel's input; bf16 input only):
//  * kProAddRmsnorm: residual add + Qwen3VLTextRMSNorm.  Each CTA reads its
//    token's whole row to form the sum of squares of s = bf16(x + residual),
//    adding in exactly the order of add_rmsnorm_kernel (elementwise.cu: 256
//    threads, each over every 256th 8-element vector, a shuffle tree per
//    warp, then the 8 warp sums in order; here each of the 128 threads plays
//    two of those threads), so the normalised input bf16(w * bf16(s * inv))
//    is bit for bit the separate kernel's.  The CTAs of table 0 write s to
//    the residual output for their channels.
//  * kProSiluMul: x is the fused gate_up output [M, 2K]; the input is
//    bf16(bf16(silu(gate)) * up), as silu_mul_kernel computes it.
#include "tc_ptx.cuh"

namespace paro {

namespace {
__device__ __forceinline__ float bfr(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void unpack8_bf(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 ld_dep_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
               : "memory");
  return v;
}

// The sum of squares of vectors v0, v0 + 256, ... of a row (s = bf16(x + r)
// per element, r optional), one of add_rmsnorm_kernel's threads.
__device__ __forceinline__ float rms_part(const __nv_bfloat16* xr, const __nv_bfloat16* rr, int n8, int v0) {
  float ss = 0.f;
  for (int i = v0; i < n8; i += 256) {
    float a[8];
    unpack8_bf(ld_dep_v4(xr + 8 * i), a);
    if (rr) {
      float b[8];
      unpack8_bf(ld_dep_v4(rr + 8 * i), b);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] = bfr(a[e] + b[e]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(a[e], a[e], ss);
  }
  return ss;
}
}  // namespace

template <typename InT, int R, bool FRAG, int PRO>
__global__ void __launch_bounds__(128)
rot16_decode_kernel(const InT* x, int64_t M, int K, RotTables tabs, __half* __restrict__ y,
                    uint32_t* __restrict__ amax, RotPro pro) {
  static_assert(PRO != kProAddRmsnorm || R == 1, "the RMSNorm prologue runs one token row per CTA");
  // the GEMM that consumes these rows may launch now and start its weight
  // stream; it waits for this grid before reading y and amax
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float buf[2][R][128];
  __shared__ uint32_t cmax[R];
  const int ch = threadIdx.x, lane = ch & 31;
  const int c = blockIdx.x * 128 + ch;
  // where this channel's value goes: quad w = ch / 4 to position (w % 4) * 8 + w / 4
  const int cpos = FRAG ? blockIdx.x * 128 + ((((ch >> 2) & 3) << 3) + (ch >> 4)) * 4 + (ch & 3) : c;
  const int64_t r0 = (int64_t)blockIdx.y * R;
  const int nrows = M - r0 < R ? (int)(M - r0) : R;
  // table blockIdx.z: its rotation, its channel scales, its activation set
  // (picked by constant indices: a runtime index into the parameter's
  // arrays would copy them to local memory in every CTA)
  const int z = blockIdx.z;
  const uint32_t* __restrict__ rtab = z == 0 ? tabs.rtab[0] : z == 1 ? tabs.rtab[1] : z == 2 ? tabs.rtab[2] : tabs.rtab[3];
  const uint16_t* __restrict__ scales = z == 0 ? tabs.cs[0] : z == 1 ? tabs.cs[1] : z == 2 ? tabs.cs[2] : tabs.cs[3];
  static_assert(kMaxTables == 4, "table selection above");
  y += (size_t)blockIdx.z * M * K;
  amax += (size_t)blockIdx.z * M;

  int part[8];
  float cc[8], cp[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const uint32_t tab = __ldg(rtab + (size_t)l * K + c);
    part[l] = (int)(tab & 0x7F);
    float s_, c_;
    __sincosf(half_bits_to_f32((uint16_t)(tab >> 16)), &s_, &c_);
    cc[l] = c_;
    cp[l] = ((tab >> 7) & 1) ? -s_ : s_;
  }
  const float sc = scales ? half_bits_to_f32(scales[c]) : 1.f;
  if (ch < R) cmax[ch] = 0u;

  // x (and the zero state of amax) belong to the previous kernels on the
  // stream: wait for them before touching either
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float v[R];
  if constexpr (PRO == kProAddRmsnorm) {
    __shared__ float wsum[8];
    const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(x) + r0 * (int64_t)K;
    const __nv_bfloat16* rr = pro.res_in ? pro.res_in + r0 * (int64_t)K : nullptr;
    float s0 = rms_part(xr, rr, K / 8, ch), s1 = rms_part(xr, rr, K / 8, ch + 128);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (lane == 0) {
      wsum[ch >> 5] = s0;
      wsum[4 + (ch >> 5)] = s1;
    }
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += wsum[w];
    const float inv = rsqrtf(tot / (float)K + pro.eps);
    float sv = ld_dep(xr + c);
    if (rr) sv = bfr(sv + ld_dep(rr + c));
    if (blockIdx.z == 0) pro.res_out[r0 * (int64_t)K + c] = __float2bfloat16_rn(sv);
    v[0] = bfr(__bfloat162float(pro.w[c]) * bfr(sv * inv)) * sc;
  } else if constexpr (PRO == kProSiluMul) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      v[r] = 0.f;
      if (r < nrows) {
        const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(x) + (r0 + r) * (int64_t)(2 * K);
        const float g = ld_dep(xr + c), u = ld_dep(xr + K + c);
        v[r] = bfr(bfr(g / (1.0f + expf(-g))) * u) * sc;
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = r < nrows ? ld_dep(x + (r0 + r) * (int64_t)K + c) * sc : 0.f;
  }
#pragma unroll
  for (int l = 0; l < 8; ++l) {
#pragma unroll
    for (int r = 0; r < R; ++r) buf[l & 1][r][ch] = v[r];
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) v[r] = givens(v[r], buf[l & 1][r][part[l]], cc[l], cp[l]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const __half h = __float2half_rn(v[r]);
    uint32_t a = 0u;
    if (r < nrows) {
      y[(r0 + r) * (int64_t)K + cpos] = h;
      a = __float_as_uint(fabsf(__half2float(h)));
    }
    a = __reduce_max_sync(0xffffffffu, a);
    if (lane == 0 && a) atomicMax(&cmax[r], a);
  }
  __syncthreads();
  if (ch < nrows && cmax[ch]) atomicMax(amax + r0 + ch, cmax[ch]);
}

template <typename InT, int R, bool FRAG, int PRO>
static cudaError_t launch_r(const void* x, int64_t M, int K, const RotTables& tabs, int T, __half* y, uint32_t* amax,
                            const RotPro& pro, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(K / kGroup), (unsigned)((M + R - 1) / R), (unsigned)T);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rot16_decode_kernel<InT, R, FRAG, PRO>, static_cast<const InT*>(x), M, K, tabs, y,
                            amax, pro);
}

template <typename InT, bool FRAG, int PRO>
static cudaError_t launch_t(const void* x, int64_t M, int K, const RotTables& tabs, int T, __half* y, uint32_t* amax,
                            const RotPro& pro, cudaStream_t st) {
  // one row per CTA at decode sizes: a CTA with R rows runs its eight
  // exchange rounds R times longer, and there the kernel's latency is what
  // the linear waits for (measured on B200, 8 tokens: R = 8 cost 2.3 us more
  // per qkv / o linear than R = 1, 16 tokens on down 7 us more).  From 32
  // tokens the CTAs outnumber the SMs many times over and each one's table
  // loads and eight angle evaluations dominate: 2 or 4 rows share them (not
  // with the RMSNorm prologue, which reduces over whole rows).
  if constexpr (PRO != kProAddRmsnorm) {
    if (M >= 48) return launch_r<InT, 4, FRAG, PRO>(x, M, K, tabs, T, y, amax, pro, st);
    if (M >= 32) return launch_r<InT, 2, FRAG, PRO>(x, M, K, tabs, T, y, amax, pro, st);
  }
  return launch_r<InT, 1, FRAG, PRO>(x, M, K, tabs, T, y, amax, pro, st);
}

template <bool FRAG>
static cudaError_t launch_d(int x_dtype, const void* x, int64_t M, int K, const RotTables& tabs, int T, __half* y,
                            uint32_t* amax, int pro_kind, const RotPro& pro, cudaStream_t st) {
  if (pro_kind == kProAddRmsnorm) {
    if (x_dtype != PARO_BF16) return cudaErrorInvalidValue;
    return launch_t<__nv_bfloat16, FRAG, kProAddRmsnorm>(x, M, K, tabs, T, y, amax, pro, st);
  }
  if (pro_kind == kProSiluMul) {
    if (x_dtype != PARO_BF16) return cudaErrorInvalidValue;
    return launch_t<__nv_bfloat16, FRAG, kProSiluMul>(x, M, K, tabs, T, y, amax, pro, st);
  }
  switch (x_dtype) {
    case PARO_F32: return launch_t<float, FRAG, kProNone>(x, M, K, tabs, T, y, amax, pro, st);
    case PARO_F16: return launch_t<__half, FRAG, kProNone>(x, M, K, tabs, T, y, amax, pro, st);
    case PARO_BF16: return launch_t<__nv_bfloat16, FRAG, kProNone>(x, M, K, tabs, T, y, amax, pro, st);
  }
  return cudaErrorInvalidValue;
}

// amax must hold zeros for the M rows (the consuming kernels return it to
// zero); y receives M x K fp16 values, quads in fragment order when frag
// (for the streaming GEMM), in channel order otherwise (for the tensor-core
// GEMM's tiled loads).  pro_kind / pro: the fused prologue (kProNone,
// kProAddRmsnorm, kProSiluMul), bf16 input only for the latter two.
// T tables (1 .. kMaxTables): y and amax hold T consecutive sets of M x K
// values and M maxima.
cudaError_t launch_rot16_decode(int x_dtype, const void* x, int64_t M, int K, const RotTables& tabs, int T, __half* y,
                                uint32_t* amax, int frag, int pro_kind, const RotPro& pro, cudaStream_t st) {
  if (M <= 0 || M > 65535 || T < 1 || T > kMaxTables) return cudaErrorInvalidValue;
  return frag ? launch_d<true>(x_dtype, x, M, K, tabs, T, y, amax, pro_kind, pro, st)
              : launch_d<false>(x_dtype, x, M, K, tabs, T, y, amax, pro_kind, pro, st);
}

// Quantisation of the rotated rows: per (group, block of 8 rows) a CTA of 128
// threads, 16 per row, each turning 8 fp16 values into int8 with the row's
// scale (round half away from zero, vLLM's per_token_quant_int8,
// int8_utils.py:106-128).  The codes keep the scratch's fragment order; each
// (row, group) code sum goes to gsum[g][row] (rows padded to a multiple of
// 8) and the token scales to xscale.  The maxima stay as they are: the GEMM
// that reads these codes returns them to zero once this grid has finished.
__global__ void __launch_bounds__(128)
quant16_decode_kernel(const __half* y, uint32_t* amax, int64_t M, int K, int Mp, int8_t* __restrict__ xq,
                      float* __restrict__ xscale, int* __restrict__ gsum) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int t = threadIdx.x, part = t & 15;
  const int g = blockIdx.x;
  // activation set blockIdx.z (one per rotation table)
  y += (size_t)blockIdx.z * M * K;
  xq += (size_t)blockIdx.z * M * K;
  amax += (size_t)blockIdx.z * M;
  xscale += (size_t)blockIdx.z * M;
  gsum += (size_t)blockIdx.z * (K / kGroup) * Mp;
  const int64_t r = (int64_t)blockIdx.y * 8 + (t >> 4);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int sum = 0;
  if (r < M) {
    // both loads in flight before either value is used: one L2 round trip
    const size_t off = (size_t)r * K + (size_t)g * kGroup + part * 8;
    const uint4 u = ld_cg_v4(y + off);
    const float a = fmaxf(__uint_as_float(ld_cg_u32(amax + r)), 1e-10f);
    const float inv = __fdiv_rn(127.0f, a);
    if (g == 0 && part == 0) xscale[r] = __fdiv_rn(a, 127.0f);
    const __half* h = reinterpret_cast<const __half*>(&u);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      w0 |= ((uint32_t)(uint8_t)(int8_t)(int)round_half_away(__half2float(h[q]) * inv)) << (8 * q);
      w1 |= ((uint32_t)(uint8_t)(int8_t)(int)round_half_away(__half2float(h[q + 4]) * inv)) << (8 * q);
    }
    *reinterpret_cast<uint2*>(xq + off) = make_uint2(w0, w1);
    sum = __dp4a((int)w0, 0x01010101, __dp4a((int)w1, 0x01010101, 0));
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (part == 0 && r < Mp) gsum[(size_t)g * Mp + r] = sum;   // zero for padding rows
}

// Mp: rows of gsum per group (a multiple of 8, at least M; rows past M get
// zero sums).
cudaError_t launch_quant16_decode(const __half* y, uint32_t* amax, int64_t M, int K, int Mp, int8_t* xq,
                                  float* xscale, int* gsum, int T, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(K / kGroup), (unsigned)(Mp / 8), (unsigned)T);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, quant16_decode_kernel, y, amax, M, K, Mp, xq, xscale, gsum);
}

}  // namespace paro
