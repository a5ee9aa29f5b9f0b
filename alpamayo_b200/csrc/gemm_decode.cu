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
constexpr int kDecThreads = 32 * (kDecConsumers + 2);  // producer + consumers + epilogue
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
  // fused activation (linear entry point): x -> rotation -> int8 in-kernel
  const void* x;            // [M, K] activations
  const uint16_t* cscale;   // [K] fp16 channel scales or null
  const uint32_t* rtab;     // [8, K] rotation table
  __half* rot16;            // [M, K] scratch: rotated rows, fp16
  uint32_t* amax;           // [M] row |max| bits, zero between calls
  uint32_t* gsync;          // [2] grid barrier and exit counters, zero between calls
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

template <int XIN>
__device__ __forceinline__ float load_x(const void* x, size_t i) {
  if constexpr (XIN == PARO_F16) return __half2float(static_cast<const __half*>(x)[i]);
  else if constexpr (XIN == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
  else return static_cast<const float*>(x)[i];
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Fused activation, phase A (the CTA's consumer threads, two halves of 128):
// half h rotates groups g = blockIdx.x + h * gridDim.x, ... for all M rows,
// 8 rows at a time, exactly as the activation kernels do (channel scale, 8
// Givens layers with separately rounded products, fp16 rounding); the rows go
// to the fp16 scratch and each row's |max| to amax (atomicMax on the bits).
template <int XIN>
__device__ __forceinline__ void fused_rotate(const DecParams& p, int ctid, float* xb) {
  const int half = ctid >> 7, ch = ctid & 127, lane = ctid & 31;
  const int G = p.K / kGroup;
  float* buf = xb + half * (2 * 8 * 128);
  for (int g = blockIdx.x + half * gridDim.x; g < G; g += 2 * gridDim.x) {
    const int c = g * kGroup + ch;
    int part[8];
    float cc[8], cp[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      const uint32_t tab = __ldg(p.rtab + (size_t)l * p.K + c);
      part[l] = (int)(tab & 0x7F);
      float s_, c_;
      __sincosf(half_bits_to_f32((uint16_t)(tab >> 16)), &s_, &c_);
      cc[l] = c_;
      cp[l] = ((tab >> 7) & 1) ? -s_ : s_;
    }
    const float sc = p.cscale ? half_bits_to_f32(p.cscale[c]) : 1.f;
    for (int64_t r0 = 0; r0 < p.M; r0 += 8) {
      float v[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) v[r] = (r0 + r < p.M) ? load_x<XIN>(p.x, (size_t)(r0 + r) * p.K + c) * sc : 0.f;
#pragma unroll
      for (int l = 0; l < 8; ++l) {
        float* b = buf + (l & 1) * (8 * 128);
#pragma unroll
        for (int r = 0; r < 8; ++r) b[r * 128 + ch] = v[r];
        named_barrier(2 + half, 128);
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = givens(v[r], b[r * 128 + part[l]], cc[l], cp[l]);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const __half h = __float2half_rn(v[r]);
        uint32_t a = 0u;
        if (r0 + r < p.M) {
          p.rot16[(size_t)(r0 + r) * p.K + c] = h;
          a = __float_as_uint(fabsf(__half2float(h)));
        }
        a = __reduce_max_sync(0xffffffffu, a);
        if (lane == 0 && a) atomicMax(p.amax + r0 + r, a);
      }
    }
  }
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

// Walks a CTA's unit range in chunks: a chunk is the records of up to 16
// consecutive groups of one row block, aligned to 16-group boundaries.
struct ChunkIter {
  int64_t u, u1;
  int nb, g, G;
  __device__ __forceinline__ ChunkIter(int64_t u0, int64_t u1_, int G_) : u(u0), u1(u1_), G(G_) {
    nb = (int)(u0 / G_);
    g = (int)(u0 - (int64_t)nb * G_);
  }
  __device__ __forceinline__ bool more() const { return u < u1; }
  __device__ __forceinline__ int count() const {
    const int gend = min(G, ((g >> 4) + 1) << 4);
    return (int)min64(gend - g, u1 - u);
  }
  // advance past a chunk of n records; true if that ended a segment
  __device__ __forceinline__ bool advance(int n) {
    u += n;
    g += n;
    if (g == G) {
      g = 0;
      ++nb;
      return true;
    }
    return u == u1;
  }
};

// XS: the token slice's int8 rows are bulk-copied into shared memory (rows
// padded by 16 bytes so the B-fragment reads of a warp hit 32 distinct
// banks) and the per-group sums computed there; otherwise fragments are read
// from global memory per record.
// XIN < 0: the int8 activations and token scales come from paro_rotq_int8;
// XIN = a paro dtype: the kernel computes them itself from x (fused linear,
// cooperative launch, M <= 64, XS only).
template <int MT, bool XS, int XIN>
__global__ void __launch_bounds__(kDecThreads, 1) gemm_stream_kernel(DecParams p) {
  constexpr bool FUSE = XIN >= 0;
  static_assert(!FUSE || XS, "the fused activation stages its int8 rows in shared memory");
  __shared__ float tok_scale_s[FUSE ? kDecMaxTokens : 1];
  __shared__ float tok_inv_s[FUSE ? kDecMaxTokens : 1];
  __shared__ int fuse_fail;
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  const int G = p.K / kGroup;
  constexpr int MP = 8 * MT;  // token rows of the slice
  const int xstride = p.K + 16;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kDecStageBytes);
  uint64_t* empty = full + kDecMaxStages;
  uint64_t* seg_full = empty + kDecMaxStages;   // [2]: all consumer slices written
  uint64_t* seg_free = seg_full + 2;             // [2]: epilogue has read them
  uint64_t* xbar = seg_free + 2;                 // activation rows landed
  float* red = reinterpret_cast<float*>(xbar + 2);                                    // [2][8][MT*4][32]
  uint8_t* xrows = reinterpret_cast<uint8_t*>(red + 2 * kDecConsumers * MT * 4 * 32);  // [MP][K + 16]
  int* sxs = reinterpret_cast<int*>(xrows + (XS ? (size_t)MP * xstride : 0));          // [G][MP] group sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t u0 = (int64_t)blockIdx.x * p.units / p.ctas;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * p.units / p.ctas;
  const int64_t tok0 = (int64_t)blockIdx.y * kDecMaxTokens;
  const int ntok_slice = (int)min64(MP, p.M - tok0);
  const int gid = lane >> 2, tig = lane & 3;
  constexpr int kSlice = MT * 4 * 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecConsumers);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&seg_full[b], kDecConsumers);
      mbar_init(&seg_free[b], 1);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the next kernel on the stream may launch as soon as SMs free up (it
  // waits for this grid's completion before reading its output)
  asm volatile("griddepcontrol.launch_dependents;");

  if (warp == 0) {  // producer: weights do not depend on the previous kernel
    if (lane == 0) {
      ChunkIter it(u0, u1, G);
      for (int k = 0; it.more(); ++k) {
        const int n = it.count();
        const int s = k % S;
        if (k >= S && !mbar_wait(&empty[s], ((k / S) - 1) & 1)) break;
        const uint32_t bytes = (uint32_t)n * kRecBytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        bulk_g2s(smem + (size_t)s * kDecStageBytes, p.packed + it.u * kRecBytes, bytes, &full[s]);
        it.advance(n);
        if (XS && !FUSE && (k == S - 1 || (!it.more() && k < S - 1))) {
          // the ring is full of weights: now fetch the activations, which
          // the previous kernel may still be writing
          grid_dependency_wait();
          mbar_arrive_expect_tx(xbar, (uint32_t)ntok_slice * p.K);
          for (int r = 0; r < ntok_slice; ++r)
            bulk_g2s(xrows + (size_t)r * xstride, p.xq + (tok0 + r) * (int64_t)p.K, (uint32_t)p.K, xbar);
        }
      }
      if (XS && !FUSE && u1 <= u0) {  // no weights to stream: still complete xbar
        grid_dependency_wait();
        mbar_arrive_expect_tx(xbar, (uint32_t)ntok_slice * p.K);
        for (int r = 0; r < ntok_slice; ++r)
          bulk_g2s(xrows + (size_t)r * xstride, p.xq + (tok0 + r) * (int64_t)p.K, (uint32_t)p.K, xbar);
      }
    }
    return;
  }

  if (warp == kDecConsumers + 1) {  // epilogue warp
    grid_dependency_wait();         // token scales come from the previous kernel
    uint32_t* cnt = p.cnt + (size_t)blockIdx.y * (p.N / kRecRows);
    const int nb0 = (int)(u0 / G);
    const int nseg = u1 > u0 ? (int)((u1 - 1) / G) - nb0 + 1 : 0;
    const int ntok = (int)min64(kDecMaxTokens, p.M - tok0);
    for (int q = 0; q < nseg; ++q) {
      const int par = q & 1, nb = nb0 + q;
      const int64_t seg_b = max64(u0, (int64_t)nb * G), seg_e = min64(u1, (int64_t)(nb + 1) * G);
      const int seg_units = (int)(seg_e - seg_b);
      if (!mbar_wait(&seg_full[par], (q >> 1) & 1)) return;
      float v[MT * 4];
#pragma unroll
      for (int sl = 0; sl < MT * 4; ++sl) {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kDecConsumers; ++w) a += red[(size_t)(par * kDecConsumers + w) * kSlice + sl * 32 + lane];
        v[sl] = a;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&seg_free[par]);
      const bool whole = seg_units == G;
#pragma unroll
      for (int sl = 0; sl < MT * 4; ++sl) {
        const int mt = sl >> 2, i = sl & 3;
        const int64_t t = tok0 + mt * 8 + 2 * tig + (i & 1);
        const int n = nb * kRecRows + gid + ((i >> 1) << 3);
        if (t < p.M) {
          if (whole)
            store_out(p.out, p.out_dtype, (size_t)t * p.N + n,
                      v[sl] * (FUSE ? tok_scale_s[t - tok0] : p.xscale[t]) + bias_at(p.bias, p.bias_dtype, n));
          else
            red_add_f32(p.ws + (size_t)n * p.M + t, v[sl]);
        }
      }
      if (!whole) {
        // release the warp's partial adds, count the units; the CTA that
        // completes the row block acquires every partial and finishes it
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          const uint32_t old = atomicAdd(&cnt[nb], (uint32_t)seg_units);
          last = (old + (uint32_t)seg_units == (uint32_t)G);
          if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          for (int idx = lane; idx < kRecRows * ntok; idx += 32) {
            const int r = idx / ntok, tt = idx - r * ntok;
            const int n = nb * kRecRows + r;
            const int64_t t = tok0 + tt;
            float* wp = p.ws + (size_t)n * p.M + t;
            const float a = __ldcg(wp);
            __stcg(wp, 0.f);
            store_out(p.out, p.out_dtype, (size_t)t * p.N + n,
                      a * (FUSE ? tok_scale_s[t - tok0] : p.xscale[t]) + bias_at(p.bias, p.bias_dtype, n));
          }
          __syncwarp();
          if (lane == 0) cnt[nb] = 0u;
        }
      }
    }
    return;
  }

  // consumers
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  const int8_t* xrow[MT];
  bool xvalid[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int64_t t = tok0 + mt * 8 + gid;
    xvalid[mt] = t < p.M;
    xrow[mt] = p.xq + (xvalid[mt] ? t : 0) * (int64_t)p.K + 4 * tig;
  }
  if constexpr (FUSE) {
    // phase A: rotate this CTA's groups (the shared activation area is the
    // exchange buffer until phase B fills it)
    fused_rotate<XIN>(p, ctid, reinterpret_cast<float*>(xrows));
    __threadfence();
    named_barrier(1, kDecConsumers * 32);
    // grid barrier: every CTA's rows and maxima are in place (cooperative
    // launch: all CTAs are resident; the wait is bounded)
    if (ctid == 0) {
      fuse_fail = 0;
      atomicAdd(p.gsync, 1u);
      const long long t0 = clock64();
      while (ld_acquire_gpu(p.gsync) < gridDim.x) {
        if (clock64() - t0 > 400000000LL) {
          report_error(kErrMbarTimeout);
          fuse_fail = 1;
          break;
        }
      }
    }
    named_barrier(1, kDecConsumers * 32);
    if (fuse_fail) return;
    // phase B: token scales, then the int8 rows into shared memory
    if (ctid < ntok_slice) {
      const float a = fmaxf(__uint_as_float(__ldcg(p.amax + tok0 + ctid)), 1e-10f);
      tok_inv_s[ctid] = __fdiv_rn(127.0f, a);
      tok_scale_s[ctid] = __fdiv_rn(a, 127.0f);
    }
    named_barrier(1, kDecConsumers * 32);
    const int k8n = p.K / 8;
    for (int e = ctid; e < ntok_slice * k8n; e += kDecConsumers * 32) {
      const int r = e / k8n, k8 = e - r * k8n;
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p.rot16 + (size_t)(tok0 + r) * p.K) + k8);
      const __half* h = reinterpret_cast<const __half*>(&u);
      const float inv = tok_inv_s[r];
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w0 |= ((uint32_t)(uint8_t)(int8_t)(int)round_half_away(__half2float(h[q]) * inv)) << (8 * q);
        w1 |= ((uint32_t)(uint8_t)(int8_t)(int)round_half_away(__half2float(h[q + 4]) * inv)) << (8 * q);
      }
      *reinterpret_cast<uint2*>(xrows + (size_t)r * xstride + (size_t)k8 * 8) = make_uint2(w0, w1);
    }
    named_barrier(1, kDecConsumers * 32);
    // the last CTA past this point returns the barrier state to zero
    if (ctid == 0) {
      __threadfence();
      const uint32_t old = atomicAdd(p.gsync + 1, 1u);
      if (old == gridDim.x - 1) {
        __threadfence();
        for (int64_t r = 0; r < p.M; ++r) p.amax[r] = 0u;
        p.gsync[0] = 0u;
        p.gsync[1] = 0u;
      }
    }
  }
  if constexpr (XS) {
    // rows beyond the slice's tokens hold stale bytes; they only feed output
    // columns that are never stored
    if (!FUSE && !mbar_wait(xbar, 0)) return;
    for (int e = ctid; e < G * MP; e += kDecConsumers * 32) {
      const int g = e / MP, r = e - g * MP;
      int sum = 0;
      if (r < ntok_slice) {
        const uint4* src = reinterpret_cast<const uint4*>(xrows + (size_t)r * xstride + (size_t)g * kGroup);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = src[c];
          sum = __dp4a((int)v.x, 0x01010101, sum);
          sum = __dp4a((int)v.y, 0x01010101, sum);
          sum = __dp4a((int)v.z, 0x01010101, sum);
          sum = __dp4a((int)v.w, 0x01010101, sum);
        }
      }
      sxs[e] = sum;
    }
    named_barrier(1, kDecConsumers * 32);
  } else {
    grid_dependency_wait();  // the activations come from the previous kernel
  }

  float y[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;

  ChunkIter it(u0, u1, G);
  int q = 0;
  for (int k = 0; it.more(); ++k) {
    const int n = it.count();
    const int s = k % S;
    const int gfirst = it.g, gbase = (it.g >> 4) << 4;
    if (!mbar_wait(&full[s], (k / S) & 1)) return;
#pragma unroll
    for (int slot = 0; slot < 2; ++slot) {
      const int g = gbase + slot * 8 + cw;
      if (g >= gfirst && g < gfirst + n) {
        uint32_t bf[MT][8];
        int sx[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          if constexpr (XS) {
            const uint8_t* xb = xrows + (size_t)(mt * 8 + gid) * xstride + (size_t)g * kGroup + 4 * tig;
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
              bf[mt][2 * s4] = *reinterpret_cast<const uint32_t*>(xb + 32 * s4);
              bf[mt][2 * s4 + 1] = *reinterpret_cast<const uint32_t*>(xb + 32 * s4 + 16);
            }
            const int2 s2 = *reinterpret_cast<const int2*>(sxs + (size_t)g * MP + mt * 8 + 2 * tig);
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
        process_record<MT>(smem + (size_t)s * kDecStageBytes + (size_t)(g - gfirst) * kRecBytes, bf, sx, gid, tig,
                           y);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);

    if (it.advance(n)) {  // segment end: hand this warp's partial to the epilogue warp
      const int par = q & 1;
      if (q >= 2 && !mbar_wait(&seg_free[par], ((q >> 1) - 1) & 1)) return;
      float* sl = red + (size_t)(par * kDecConsumers + cw) * kSlice;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sl[(mt * 4 + i) * 32 + lane] = y[mt][i];
          y[mt][i] = 0.f;
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&seg_full[par]);
      ++q;
    }
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
  // full/empty rings, seg_full/seg_free pairs, xbar (+1 slot keeps 16-byte
  // alignment), then the epilogue slices
  return (2 * kDecMaxStages + 6) * sizeof(uint64_t) + 2 * (size_t)kDecConsumers * MT * 4 * 32 * sizeof(float);
}

template <int MT, bool XS, int XIN = -1>
static cudaError_t launch_mt(DecParams p, size_t xs_bytes, cudaStream_t st) {
  const size_t smem = (size_t)p.stages * kDecStageBytes + fixed_smem(MT) + (XS ? xs_bytes : 0);
  auto kern = gemm_stream_kernel<MT, XS, XIN>;
  cudaError_t e = ensure_smem_limit((const void*)kern, kDecSmemBudget + 4096);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.ctas, (unsigned)((p.M + kDecMaxTokens - 1) / kDecMaxTokens), 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (XIN >= 0) {
    // the fused activation's grid barrier needs every CTA resident
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int MT>
static cudaError_t launch_pick(DecParams p, cudaStream_t st) {
  const int G = p.K / kGroup;
  const size_t xs_bytes = (size_t)8 * MT * (p.K + 16) + (size_t)G * 8 * MT * sizeof(int);
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
  DecParams p = {};
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

// ---------------------------------------------------------------------------
// fused linear for decode sizes: activation rotation + quantisation inside
// the GEMM kernel (see fused_rotate and the consumers' phase B)
// ---------------------------------------------------------------------------
size_t linear_decode_workspace(int64_t M, int N) {
  return gemm_decode_workspace(M, N) + (((size_t)M * sizeof(uint32_t) + 255) & ~(size_t)255) + 256;
}

template <int MT>
static cudaError_t launch_pick_fused(DecParams p, int x_dtype, cudaStream_t st) {
  const int G = p.K / kGroup;
  size_t xs_bytes = (size_t)8 * MT * (p.K + 16) + (size_t)G * 8 * MT * sizeof(int);
  const size_t xch = (size_t)2 * 2 * 8 * 128 * sizeof(float);  // phase A exchange buffers
  if (xs_bytes < xch) xs_bytes = xch;
  const size_t base = fixed_smem(MT);
  if (base + xs_bytes + 3 * (size_t)kDecStageBytes > (size_t)kDecSmemBudget) return cudaErrorNotSupported;
  int stages = (int)((kDecSmemBudget - base - xs_bytes) / kDecStageBytes);
  p.stages = stages > kDecMaxStages ? kDecMaxStages : stages;
  switch (x_dtype) {
    case PARO_F32: return launch_mt<MT, true, PARO_F32>(p, xs_bytes, st);
    case PARO_F16: return launch_mt<MT, true, PARO_F16>(p, xs_bytes, st);
    case PARO_BF16: return launch_mt<MT, true, PARO_BF16>(p, xs_bytes, st);
  }
  return cudaErrorInvalidValue;
}

// Returns cudaErrorNotSupported (nothing launched) for shapes whose int8
// rows do not fit in shared memory; callers then run the two kernels.
cudaError_t launch_linear_decode(const void* x, int x_dtype, const uint16_t* cscale, const uint32_t* rtab, int64_t M,
                                 int N, int K, const void* packed, const void* bias, int bias_dtype, void* out,
                                 int out_dtype, void* ws, void* scratch, cudaStream_t st) {
  if (M > kDecMaxTokens) return cudaErrorNotSupported;
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  DecParams p = {};
  p.xq = nullptr;
  p.xscale = nullptr;
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
  uint8_t* tail = static_cast<uint8_t*>(ws) + gemm_decode_workspace(M, N);
  p.amax = reinterpret_cast<uint32_t*>(tail);
  p.gsync = reinterpret_cast<uint32_t*>(tail + (((size_t)M * sizeof(uint32_t) + 255) & ~(size_t)255));
  p.x = x;
  p.cscale = cscale;
  p.rtab = rtab;
  p.rot16 = static_cast<__half*>(scratch);
  p.units = (int64_t)(N / kRecRows) * (K / kGroup);
  p.ctas = (int)min64(g_num_sms, p.units);
  p.stages = 0;
  if (M <= 8) return launch_pick_fused<1>(p, x_dtype, st);
  if (M <= 16) return launch_pick_fused<2>(p, x_dtype, st);
  if (M <= 32) return launch_pick_fused<4>(p, x_dtype, st);
  return launch_pick_fused<8>(p, x_dtype, st);
}

}  // namespace paro
