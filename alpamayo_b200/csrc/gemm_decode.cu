// gemm_decode.cu — int4 x int8 GEMM for decode shapes (small M), sm_100a.
//
// Memory-bound regime: the weight stream (N*K/2 bytes of codes plus group
// scales and zero points) dominates, so the kernel is built to keep every SM
// pulling weights at its share of HBM bandwidth:
//
//  * Persistent, load-balanced grid ("stream-K"): the layer's tile records —
//    one per (16-row block nb, 128-channel group g), stored nb-major so each
//    row block's K strip is contiguous — are split into one contiguous range
//    per CTA.  A CTA's range spans parts of a few row blocks (segments).
//  * TMA bulk copies: one producer thread streams the range through an
//    8-stage shared-memory ring (cp.async.bulk + mbarrier complete_tx).  A
//    chunk holds up to 8 records of one row block, one per consumer warp.
//  * 8 consumer warps expand each record's int4 codes to int8 (q - z) in
//    registers and run int8 mma.sync m16n8k32 against the token tile
//    (B fragments read from the L1-cached activations).  Each group's int32
//    accumulator is exact and is scaled into float32 per group.
//  * Segment end: the warps' partial sums are reduced in shared memory.  A
//    segment covering the whole row block is finished in place (token scale,
//    bias, store).  A boundary segment shared with a neighbouring CTA adds its
//    partial into a float32 workspace (red.global.add) and bumps the row
//    block's unit counter; the CTA that completes the count applies the
//    epilogue and returns the workspace slice and counter to zero, so the
//    workspace is zero again after every call.
//
// The record layout puts, for lane (gid = lane/4, tig = lane%4), the A
// fragment words of rows gid and gid+8 for all four 32-channel steps of a
// group in one 16-byte chunk each: low nibbles give a0/a1, high nibbles a2/a3.
#include "tc_ptx.cuh"

namespace paro {

constexpr int kDecConsumers = 8;
constexpr int kDecThreads = 32 * (kDecConsumers + 1);
constexpr int kDecStages = 8;
constexpr int kDecStageBytes = kDecConsumers * kRecBytes;
constexpr int kDecMaxTokens = 64;  // tokens per CTA slice (8 tiles of 8)

struct DecParams {
  const int8_t* xq;
  const float* xscale;
  int64_t M;
  int N, K;
  const uint8_t* packed;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  float* ws;        // [N][M] float32 partial sums, zero between calls
  uint32_t* cnt;    // [token slices][N/16] unit counters, zero between calls
  int64_t units;    // (N/16) * G
  int ctas;
};

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

__device__ __forceinline__ float bias_at(const void* bias, int dtype, int n) {
  if (!bias) return 0.f;
  if (dtype == PARO_F16) return __half2float(static_cast<const __half*>(bias)[n]);
  if (dtype == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
  return static_cast<const float*>(bias)[n];
}

__device__ __forceinline__ void store_out(void* out, int dtype, size_t idx, float v) {
  if (dtype == PARO_F16) static_cast<__half*>(out)[idx] = __float2half_rn(v);
  else if (dtype == PARO_BF16) static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else static_cast<float*>(out)[idx] = v;
}

// End of the chunk that starts at unit u: at most one record per consumer
// warp and never past the end of u's row block or of the CTA's range.
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

__device__ __forceinline__ int64_t chunk_end(int64_t u, int64_t u1, int G) {
  const int64_t seg_end = min64(u1, (u / G + 1) * (int64_t)G);
  return min64(u + kDecConsumers, seg_end);
}

template <int MT>
__global__ void __launch_bounds__(kDecThreads, 1) gemm_stream_kernel(DecParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
  uint64_t* empty = full + kDecStages;
  float* red = reinterpret_cast<float*>(empty + kDecStages);  // [consumers][MT*4][32]
  __shared__ int last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.K / kGroup;
  const int64_t u0 = (int64_t)blockIdx.x * p.units / p.ctas;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * p.units / p.ctas;
  const int64_t tok0 = (int64_t)blockIdx.y * kDecMaxTokens;
  uint32_t* cnt = p.cnt + (size_t)blockIdx.y * (p.N / kRecRows);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {  // producer
    if (lane == 0) {
      int64_t u = u0;
      for (int k = 0; u < u1; ++k) {
        const int64_t ce = chunk_end(u, u1, G);
        const int s = k % kDecStages;
        if (k >= kDecStages && !mbar_wait(&empty[s], ((k / kDecStages) - 1) & 1)) break;
        const uint32_t bytes = (uint32_t)(ce - u) * kRecBytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(smem + (size_t)s * kDecStageBytes, p.packed + u * kRecBytes, bytes, &full[s]);
        u = ce;
      }
    }
    return;
  }

  // consumers
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  const int gid = lane >> 2, tig = lane & 3;
  const int8_t* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int64_t t = tok0 + mt * 8 + gid;
    xvalid[mt] = t < p.M;
    xrow[mt] = p.xq + (xvalid[mt] ? t : 0) * (int64_t)p.K + 4 * tig;
  }
  float y[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;

  int64_t u = u0;
  for (int k = 0; u < u1; ++k) {
    const int64_t ce = chunk_end(u, u1, G);
    const int s = k % kDecStages;
    const int64_t my = u + cw;
    const bool have = my < ce;
    const int g = (int)(my % G);
    // activation fragments of this warp's group (independent of the stage)
    uint32_t bf[MT][4][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int8_t* xp = xrow[mt] + (size_t)g * kGroup + 32 * j;
        const bool v = have && xvalid[mt];
        bf[mt][j][0] = v ? ldg_nc_u32(xp) : 0u;
        bf[mt][j][1] = v ? ldg_nc_u32(xp + 16) : 0u;
      }
    if (!mbar_wait(&full[s], (k / kDecStages) & 1)) return;
    if (have) {
      const uint8_t* rec = smem + (size_t)s * kDecStageBytes + cw * kRecBytes;
      const uint4 wa = *reinterpret_cast<const uint4*>(rec + gid * 64 + tig * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(rec + (gid + 8) * 64 + tig * 16);
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(rec + kRecScaleOff);
      const float s_lo = half_bits_to_f32(sp[gid]), s_hi = half_bits_to_f32(sp[gid + 8]);
      const uint32_t zz_lo = (uint32_t)rec[kRecZeroOff + gid] * 0x01010101u;
      const uint32_t zz_hi = (uint32_t)rec[kRecZeroOff + gid + 8] * 0x01010101u;
      const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wB[4] = {wb.x, wb.y, wb.z, wb.w};
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
        for (int mt = 0; mt < MT; ++mt) mma_s8(acc[mt], a0, a1, a2, a3, bf[mt][j][0], bf[mt][j][1]);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        y[mt][0] = fmaf(s_lo, (float)acc[mt][0], y[mt][0]);
        y[mt][1] = fmaf(s_lo, (float)acc[mt][1], y[mt][1]);
        y[mt][2] = fmaf(s_hi, (float)acc[mt][2], y[mt][2]);
        y[mt][3] = fmaf(s_hi, (float)acc[mt][3], y[mt][3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool seg_done = (ce == u1) || (ce % G == 0);
    if (seg_done) {
      const int64_t nb = (ce - 1) / G;
      const int64_t seg_begin = max64(u0, nb * (int64_t)G);
      const int seg_units = (int)(ce - seg_begin);
      const bool whole = seg_units == G;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[(cw * MT * 4 + mt * 4 + i) * 32 + lane] = y[mt][i];
      named_barrier(1, kDecConsumers * 32);
      for (int slot = cw; slot < MT * 4; slot += kDecConsumers) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kDecConsumers; ++w) v += red[(w * MT * 4 + slot) * 32 + lane];
        const int mt = slot >> 2, i = slot & 3;
        const int64_t t = tok0 + mt * 8 + 2 * tig + (i & 1);
        const int n = (int)nb * kRecRows + gid + ((i >> 1) << 3);
        if (t < p.M) {
          if (whole) store_out(p.out, p.out_dtype, (size_t)t * p.N + n, v * p.xscale[t] + bias_at(p.bias, p.bias_dtype, n));
          else red_add_f32(p.ws + (size_t)n * p.M + t, v);
        }
      }
      if (!whole) {
        __threadfence();
        named_barrier(1, kDecConsumers * 32);
        if (ctid == 0) {
          const uint32_t old = atomicAdd(&cnt[nb], (uint32_t)seg_units);
          last_flag = (old + (uint32_t)seg_units == (uint32_t)G);
        }
        named_barrier(1, kDecConsumers * 32);
        if (last_flag) {
          __threadfence();
          const int ntok = (int)min64(kDecMaxTokens, p.M - tok0);
          for (int idx = ctid; idx < kRecRows * ntok; idx += kDecConsumers * 32) {
            const int r = idx / ntok, tt = idx - r * ntok;
            const int n = (int)nb * kRecRows + r;
            const int64_t t = tok0 + tt;
            float* wp = p.ws + (size_t)n * p.M + t;
            const float v = __ldcg(wp);
            __stcg(wp, 0.f);
            store_out(p.out, p.out_dtype, (size_t)t * p.N + n, v * p.xscale[t] + bias_at(p.bias, p.bias_dtype, n));
          }
          if (ctid == 0) cnt[nb] = 0u;
        }
      }
      named_barrier(1, kDecConsumers * 32);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;
    }
    u = ce;
  }
}

PARO_DEFINE_ERROR_ACCESSOR(decode)

static int g_num_sms = 0;

size_t gemm_decode_workspace(int64_t M, int N) {
  const int64_t slices = (M + kDecMaxTokens - 1) / kDecMaxTokens;
  size_t ws = (size_t)N * (size_t)M * sizeof(float);
  ws = (ws + 255) & ~(size_t)255;
  return ws + (size_t)slices * (N / kRecRows) * sizeof(uint32_t);
}

size_t gemm_decode_smem(int MT) {
  return (size_t)kDecStages * kDecStageBytes + 2 * kDecStages * sizeof(uint64_t) +
         (size_t)kDecConsumers * MT * 4 * 32 * sizeof(float);
}

template <int MT>
static cudaError_t launch_mt(DecParams p, cudaStream_t st) {
  const size_t smem = gemm_decode_smem(MT);
  cudaError_t e = cudaFuncSetAttribute(gemm_stream_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(p.ctas, (unsigned)((p.M + kDecMaxTokens - 1) / kDecMaxTokens));
  gemm_stream_kernel<MT><<<grid, kDecThreads, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm_decode(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                               const void* bias, int bias_dtype, void* out, int out_dtype, void* ws,
                               cudaStream_t st) {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  DecParams p;
  p.xq = xq;
  p.xscale = xscale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.packed = static_cast<const uint8_t*>(packed);
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.out_dtype = out_dtype;
  size_t wsf = ((size_t)N * (size_t)M * sizeof(float) + 255) & ~(size_t)255;
  p.ws = static_cast<float*>(ws);
  p.cnt = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + wsf);
  p.units = (int64_t)(N / kRecRows) * (K / kGroup);
  p.ctas = (int)min64(g_num_sms, p.units);
  if (M <= 8) return launch_mt<1>(p, st);
  if (M <= 16) return launch_mt<2>(p, st);
  if (M <= 32) return launch_mt<4>(p, st);
  return launch_mt<8>(p, st);
}

}  // namespace paro
