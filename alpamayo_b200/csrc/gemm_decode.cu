// gemm_decode.cu — int4 x int8 GEMM for decode shapes (small M), sm_100a.
//
// Memory-bound regime: the weight stream (N*K/2 bytes of codes plus group
// scales and zero points) dominates, so the kernel is built to keep every SM
// pulling weights at its share of HBM bandwidth:
//
//  * Persistent, load-balanced grid ("stream-K"): the layer's tile records —
//    one per (16-row block nb, 128-channel group g), stored nb-major so each
//    row block's K strip is contiguous — are split into one contiguous range
//    per CTA.  A CTA's range covers parts of a few row blocks (segments).
//  * TMA bulk copies: one producer thread streams the range through a shared
//    memory ring (cp.async.bulk + mbarrier complete_tx).  A chunk holds the
//    records of up to 16 consecutive groups of one row block, aligned to
//    16-group boundaries.
//  * 8 consumer warps; warp w owns the groups g = w (mod 8), so each chunk
//    gives every warp up to two independent records, and the activation
//    fragments a warp needs are the same for every row block.  The token
//    activations are staged once per CTA in shared memory in mma fragment
//    order (falls back to L1-cached global loads when they do not fit).
//  * Each record's int4 codes are expanded to int8 (q - z) in registers and
//    fed to int8 mma.sync m16n8k32 (A = 16 weight rows x 32 channels, B = 8
//    tokens); each group's int32 sum is exact and is scaled into float32.
//  * Segment end: partial sums of the 8 warps are reduced in shared memory.
//    A segment covering a whole row block is finished in place (token scale,
//    bias, store).  A boundary segment shared with a neighbouring CTA adds
//    its partial into a float32 workspace (red.global.add) and bumps the row
//    block's unit counter; the CTA that completes the count applies the
//    epilogue and returns the workspace slice and counter to zero, so the
//    workspace is zero again after every call.
//  * Programmatic dependent launch: the weight stream starts before the
//    activation kernel that produces this GEMM's input has finished; only
//    the reads of the activations wait (griddepcontrol.wait).
//
// Record layout: for lane (gid = lane/4, tig = lane%4), the A fragment words
// of rows gid and gid+8 for the four 32-channel steps of a group are one
// 16-byte chunk each: low nibbles give a0/a1, high nibbles a2/a3.
#include "tc_ptx.cuh"

namespace paro {

constexpr int kDecConsumers = 8;
constexpr int kDecThreads = 32 * (kDecConsumers + 1);
constexpr int kDecChunkGroups = 16;
constexpr int kDecStageBytes = kDecChunkGroups * kRecBytes;  // 17152
constexpr int kDecMaxStages = 8;
constexpr int kDecMaxTokens = 64;   // tokens per CTA slice (8 tiles of 8)
constexpr int kDecSmemBudget = 220 * 1024;

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
  int stages;
};

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// A = unsigned 8-bit codes (q, or 16*q from a high nibble), B = signed int8
// activations, int32 accumulate.
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Sum of the 32 int8 activations in a lane's 8 fragment words.
__device__ __forceinline__ int frag_sum(const uint32_t (&b)[8]) {
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = __dp4a((int)b[i], 0x01010101, s);
  return s;
}

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// End of the chunk starting at unit u: the next 16-group boundary of u's
// row block, the row block's end, or the CTA range end.
__device__ __forceinline__ int64_t chunk_end(int64_t u, int64_t u1, int G) {
  const int64_t nb = u / G;
  const int g = (int)(u - nb * G);
  const int gend = min(G, (g / kDecChunkGroups + 1) * kDecChunkGroups);
  return min64(u1, nb * G + gend);
}

// The 8 B-fragment words of (token tile, group g) for this lane: b0/b1 of
// the four 32-channel steps.
__device__ __forceinline__ void load_bfrag_global(const int8_t* xrow, bool valid, int g, uint32_t (&b)[8]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int8_t* xp = xrow + (size_t)g * kGroup + 32 * j;
    b[2 * j] = valid ? ldg_nc_u32(xp) : 0u;
    b[2 * j + 1] = valid ? ldg_nc_u32(xp + 16) : 0u;
  }
}

// One record: 16 rows x 128 channels against MT token tiles.
//   bf[mt][2s], bf[mt][2s+1] : B fragment of k-step s (channels 32s..32s+31)
//   sx[mt][0..1]             : group sums of this lane's two tokens
// The low nibbles of the lane's four words per row are, as unsigned bytes,
// the A fragments of k-steps 0-1; masked in place, the high nibbles are
// 16*q, the A fragments of k-steps 2-3 (a separate accumulator).  So
//   16 * sum_k (q - z) x = 16*lo + hi - 16*z*sum_k x,
// exact in int32 (and below 2^24, so the float conversion is exact), and
// scaled by s/16 it equals s * sum_k (q - z) x bit for bit.
template <int MT>
__device__ __forceinline__ void process_record(const uint8_t* rec, const uint32_t (&bf)[MT][8],
                                               const int (&sx)[MT][2], int gid, int tig, float (&y)[MT][4]) {
  const uint4 wa = *reinterpret_cast<const uint4*>(rec + gid * 64 + tig * 16);
  const uint4 wb = *reinterpret_cast<const uint4*>(rec + (gid + 8) * 64 + tig * 16);
  const uint16_t* sp = reinterpret_cast<const uint16_t*>(rec + kRecScaleOff);
  const float s16_lo = half_bits_to_f32(sp[gid]) * 0.0625f, s16_hi = half_bits_to_f32(sp[gid + 8]) * 0.0625f;
  const int nz_lo = -16 * (int)rec[kRecZeroOff + gid], nz_hi = -16 * (int)rec[kRecZeroOff + gid + 8];
  constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
  int lo[MT][4], hi[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) lo[mt][i] = hi[mt][i] = 0;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    mma_u8s8(lo[mt], wa.x & LO, wb.x & LO, wa.y & LO, wb.y & LO, bf[mt][0], bf[mt][1]);
    mma_u8s8(hi[mt], wa.x & HI, wb.x & HI, wa.y & HI, wb.y & HI, bf[mt][4], bf[mt][5]);
    mma_u8s8(lo[mt], wa.z & LO, wb.z & LO, wa.w & LO, wb.w & LO, bf[mt][2], bf[mt][3]);
    mma_u8s8(hi[mt], wa.z & HI, wb.z & HI, wa.w & HI, wb.w & HI, bf[mt][6], bf[mt][7]);
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int t0 = 16 * lo[mt][0] + hi[mt][0] + nz_lo * sx[mt][0];
    const int t1 = 16 * lo[mt][1] + hi[mt][1] + nz_lo * sx[mt][1];
    const int t2 = 16 * lo[mt][2] + hi[mt][2] + nz_hi * sx[mt][0];
    const int t3 = 16 * lo[mt][3] + hi[mt][3] + nz_hi * sx[mt][1];
    y[mt][0] = fmaf(s16_lo, (float)t0, y[mt][0]);
    y[mt][1] = fmaf(s16_lo, (float)t1, y[mt][1]);
    y[mt][2] = fmaf(s16_hi, (float)t2, y[mt][2]);
    y[mt][3] = fmaf(s16_hi, (float)t3, y[mt][3]);
  }
}

// XS: activations staged in shared memory (fragment order) instead of read
// from global memory per record.
template <int MT, bool XS>
__global__ void __launch_bounds__(kDecThreads, 1) gemm_stream_kernel(DecParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  const int G = p.K / kGroup;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kDecStageBytes);
  uint64_t* empty = full + kDecMaxStages;
  float* red = reinterpret_cast<float*>(empty + kDecMaxStages);                 // [8][MT*4][32]
  uint4* xs = reinterpret_cast<uint4*>(red + kDecConsumers * MT * 4 * 32);    // [G][MT][32][2]
  int* sxs = reinterpret_cast<int*>(xs + (XS ? 2 * G * MT * 32 : 0));         // [G][MT][8] group sums
  __shared__ int last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = (int64_t)blockIdx.x * p.units / p.ctas;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * p.units / p.ctas;
  const int64_t tok0 = (int64_t)blockIdx.y * kDecMaxTokens;
  uint32_t* cnt = p.cnt + (size_t)blockIdx.y * (p.N / kRecRows);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 0) {  // producer: weights do not depend on the previous kernel
    if (lane == 0) {
      int64_t u = u0;
      for (int k = 0; u < u1; ++k) {
        const int64_t ce = chunk_end(u, u1, G);
        const int s = k % S;
        if (k >= S && !mbar_wait(&empty[s], ((k / S) - 1) & 1)) break;
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
  grid_dependency_wait();  // the activations come from the previous kernel
  if constexpr (XS) {
    for (int e = ctid; e < G * MT * 32; e += kDecConsumers * 32) {
      const int l = e & 31, gm = e >> 5, mt = gm % MT, g = gm / MT;
      const int lgid = l >> 2, ltig = l & 3;
      const int64_t t = tok0 + mt * 8 + lgid;
      uint32_t b[8];
      load_bfrag_global(p.xq + (t < p.M ? t : 0) * (int64_t)p.K + 4 * ltig, t < p.M, g, b);
      xs[2 * e] = make_uint4(b[0], b[1], b[2], b[3]);
      xs[2 * e + 1] = make_uint4(b[4], b[5], b[6], b[7]);
      // the 4 lanes of one token row cover the group's 128 channels (the
      // trip count is uniform across a warp, so the shuffles are safe)
      int part = frag_sum(b);
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      if (ltig == 0) sxs[(g * MT + mt) * 8 + lgid] = part;
    }
    named_barrier(1, kDecConsumers * 32);
  }

  float y[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;

  int64_t u = u0;
  for (int k = 0; u < u1; ++k) {
    const int64_t ce = chunk_end(u, u1, G);
    const int s = k % S;
    const int64_t nb = u / G;
    const int gbase = (int)(u - nb * G) / kDecChunkGroups * kDecChunkGroups;
    if (!mbar_wait(&full[s], (k / S) & 1)) return;
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int g = gbase + slot * 8 + cw;
      const int64_t ur = nb * G + g;
      if (ur >= u && ur < ce) {
        uint32_t bf[MT][8];
        int sx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if constexpr (XS) {
            const uint4* xp = xs + 2 * ((g * MT + mt) * 32 + lane);
            const uint4 lo = xp[0], hi = xp[1];
            bf[mt][0] = lo.x; bf[mt][1] = lo.y; bf[mt][2] = lo.z; bf[mt][3] = lo.w;
            bf[mt][4] = hi.x; bf[mt][5] = hi.y; bf[mt][6] = hi.z; bf[mt][7] = hi.w;
            const int2 s2 = *reinterpret_cast<const int2*>(sxs + (g * MT + mt) * 8 + 2 * tig);
            sx[mt][0] = s2.x;
            sx[mt][1] = s2.y;
          } else {
            load_bfrag_global(xrow[mt], xvalid[mt], g, bf[mt]);
            // token row gid's sum, then the sums of this lane's C columns
            int part = frag_sum(bf[mt]);
            part += __shfl_xor_sync(0xffffffffu, part, 1);
            part += __shfl_xor_sync(0xffffffffu, part, 2);
            sx[mt][0] = __shfl_sync(0xffffffffu, part, 8 * tig);
            sx[mt][1] = __shfl_sync(0xffffffffu, part, 8 * tig + 4);
          }
        }
        process_record<MT>(smem + (size_t)s * kDecStageBytes + (size_t)(ur - u) * kRecBytes, bf, sx, gid, tig, y);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    const bool seg_done = (ce == u1) || (ce % G == 0);
    if (seg_done) {
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
          if (whole)
            store_out(p.out, p.out_dtype, (size_t)t * p.N + n, v * p.xscale[t] + bias_at(p.bias, p.bias_dtype, n));
          else
            red_add_f32(p.ws + (size_t)n * p.M + t, v);
        }
      }
      if (!whole) {
        // release: the CTA's partial adds (ordered before thread 0 by the
        // barrier) become visible before the counter moves; the CTA that
        // completes the count acquires them all
        named_barrier(1, kDecConsumers * 32);
        if (ctid == 0) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          const uint32_t old = atomicAdd(&cnt[nb], (uint32_t)seg_units);
          last_flag = (old + (uint32_t)seg_units == (uint32_t)G);
          if (last_flag) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
        named_barrier(1, kDecConsumers * 32);
        if (last_flag) {
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

static size_t fixed_smem(int MT) {
  return 2 * kDecMaxStages * sizeof(uint64_t) + (size_t)kDecConsumers * MT * 4 * 32 * sizeof(float);
}

template <int MT, bool XS>
static cudaError_t launch_mt(DecParams p, size_t xs_bytes, cudaStream_t st) {
  const size_t smem = (size_t)p.stages * kDecStageBytes + fixed_smem(MT) + (XS ? xs_bytes : 0);
  auto kern = gemm_stream_kernel<MT, XS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.ctas, (unsigned)((p.M + kDecMaxTokens - 1) / kDecMaxTokens), 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int MT>
static cudaError_t launch_pick(DecParams p, cudaStream_t st) {
  const int G = p.K / kGroup;
  const size_t xs_bytes = (size_t)G * MT * 32 * 32 + (size_t)G * MT * 8 * sizeof(int);
  const size_t base = fixed_smem(MT);
  const bool xs = base + xs_bytes + 3 * (size_t)kDecStageBytes <= (size_t)kDecSmemBudget;
  const size_t avail = kDecSmemBudget - base - (xs ? xs_bytes : 0);
  int stages = (int)(avail / kDecStageBytes);
  stages = stages > kDecMaxStages ? kDecMaxStages : stages;
  if (stages < 2) return cudaErrorInvalidValue;
  p.stages = stages;
  return xs ? launch_mt<MT, true>(p, xs_bytes, st) : launch_mt<MT, false>(p, xs_bytes, st);
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
  const size_t wsf = ((size_t)N * (size_t)M * sizeof(float) + 255) & ~(size_t)255;
  p.ws = static_cast<float*>(ws);
  p.cnt = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + wsf);
  p.units = (int64_t)(N / kRecRows) * (K / kGroup);
  p.ctas = (int)min64(g_num_sms, p.units);
  p.stages = 0;
  if (M <= 8) return launch_pick<1>(p, st);
  if (M <= 16) return launch_pick<2>(p, st);
  if (M <= 32) return launch_pick<4>(p, st);
  return launch_pick<8>(p, st);
}

}  // namespace paro
