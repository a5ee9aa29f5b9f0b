// gemm_decode.cu — int4 x int8 GEMM for decode shapes (small M), sm_100a.
//
// Memory-bound regime: the weight stream (N*K/2 bytes of codes plus group
// scales and zero points) dominates, so the kernel is built to keep every SM
// pulling weights at its share of HBM bandwidth and to spend as few issue
// slots per weight byte as possible:
//
//  * Persistent, load-balanced grid ("stream-K"): the layer's tile records —
//    one per (16-row block nb, 128-channel group g), stored nb-major so each
//    row block's K strip is contiguous — are split into one contiguous range
//    per CTA.  A CTA's range covers parts of a few row blocks (segments).
//    The two end segments, which a CTA shares with its neighbours, are
//    visited first, so their fix-up through the workspace overlaps the rest
//    of the stream; the whole row blocks in between come last.
//  * TMA bulk copies: one producer thread streams the range through a shared
//    memory ring (cp.async.bulk + mbarrier complete_tx).  A chunk holds the
//    records of up to 32 consecutive groups of one row block, aligned to
//    32-group boundaries (a whole row block when K = 3584).
//  * Consumer warps (16 for up to 16 tokens, 8 beyond); warp w owns the
//    groups g = w (mod warps), so a chunk gives each warp up to two (16
//    warps) or four (8 warps) independent records.  The token slice's int8 rows are staged once per
//    CTA in shared memory and rearranged there into mma fragment order (a
//    lane's eight B words of a group are 32 contiguous bytes: two 16-byte
//    loads per record); rows that do not fit are read from global memory.
//  * Each record's int4 codes are expanded to int8 in registers and fed to
//    int8 mma.sync m16n8k32 (A = 16 weight rows x 32 channels, B = 8
//    tokens); each group's int32 sum is exact and is scaled into float32.
//  * Segment end: partial sums of the warps are reduced in shared memory by
//    an epilogue warp.  A segment covering a whole row block is finished in
//    place (token scale, bias, store).  A boundary segment shared with a
//    neighbouring CTA adds its partial into a 64-bit fixed-point workspace
//    (red_add_fx: the total does not depend on the order the CTAs arrive
//    in) and bumps the row block's unit counter; the CTA that
//    completes the count applies the epilogue and returns the workspace
//    slice and counter to zero, so the workspace is zero again after every
//    call.
//  * Programmatic dependent launch: the weight stream starts before the
//    activation kernel that produces this GEMM's input has finished; only
//    the reads of the activations wait (griddepcontrol.wait), and the
//    epilogue warp fetches them as soon as they are ready.
//
// Record layout: for lane (gid = lane/4, tig = lane%4), the A fragment words
// of rows gid and gid+8 for the four 32-channel steps of a group are one
// 16-byte chunk each: low nibbles give a0/a1, high nibbles a2/a3.
#include <cstdlib>
#include <cstring>

#include "stream_segs.cuh"
#include "tc_ptx.cuh"

namespace paro {

// consumer warps: 16 for up to 16 tokens (more warps hide the latency of
// each record's load -> mma -> scale chain), 8 for more tokens (more work
// per record, and the reduction slices would not fit)
__host__ __device__ constexpr int dec_consumers(int MT) { return MT <= 2 ? 16 : 8; }
// warps: producer, consumers, two epilogue warps (alternate segments, so two
// workspace fix-ups can be in flight at once)
__host__ __device__ constexpr int dec_threads(int MT) { return 32 * (dec_consumers(MT) + 3); }
constexpr int kDecChunkGroups = 32;
constexpr int kDecStageBytes = kDecChunkGroups * kRecBytes;  // 34304
constexpr int kDecMaxStages = 8;
constexpr int kDecMaxTokens = 64;   // tokens per CTA slice (8 tiles of 8)
constexpr int kDecSmemBudget = 220 * 1024;
constexpr int kXinPreQ = 17;        // gemm_stream_kernel's XIN for int8 rows in fragment order with code sums
constexpr int kXinPreQS = 18;       // ... the same rows and sums bulk-copied into shared memory
constexpr int kDecBulkXBytes = 32 * 1024;  // activation blocks above this are bulk-copied

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
  unsigned long long* ws;  // [N][M] fixed-point (red_add_fx) partial sums, zero between calls
  uint32_t* cnt;    // [token slices][N/16] unit counters, zero between calls
  // linear entry point (kXinPreQ, kXinPreQS): the row maxima the
  // rotation kernel accumulated and the quantiser read; this kernel
  // returns them to zero once the quantiser has finished
  uint32_t* amax;           // [M] row |max| bits, zero between calls
  int64_t units;    // (N/16) * G
  int ctas;
  int stages;
  int xrows_n;      // token rows staged in shared memory (XS)
  const int* gsum;  // kXinPreQ: per (group, token) code sums, [G][gsum_mp]
  int gsum_mp;
  // kXinPreQ with several rotation tables (a group of linears sharing their
  // input, weights concatenated along N): row blocks [tab_nb[t],
  // tab_nb[t + 1]) use activation set t; set t of xq / gsum / xscale / amax
  // starts t * set_xq bytes / t * set_gsum ints / t * M floats in
  int tables;
  int tab_nb[kMaxTables];
  int64_t set_xq, set_gsum;
};

// The activation set (rotation table) of row block nb.
__device__ __forceinline__ int table_of(const DecParams& p, int nb) {
  int t = 0;
#pragma unroll
  for (int i = 1; i < kMaxTables; ++i) t += (i < p.tables && nb >= p.tab_nb[i]) ? 1 : 0;
  return t;
}


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


// XS: the token slice's int8 rows are bulk-copied into shared memory (rows
// padded by 16 bytes so that the fragment reads of a warp hit 32 distinct
// banks), rearranged into fragment order, and their per-group sums computed
// there; otherwise fragments are read from global memory per record.
// XIN < 0: the int8 activations and token scales come from paro_rotq_int8;
// XIN = kXinPreQ: quant16_decode_kernel left the int8 rows in fragment order
// with their code sums, read per record from L2 (!XS); XIN = kXinPreQS: the
// same, bulk-copied into shared memory once (XS, no rearrangement).
template <int MT, bool XS, int XIN>
__global__ void __launch_bounds__(dec_threads(MT), 1) gemm_stream_kernel(DecParams p) {
  constexpr bool PREQ = XIN == kXinPreQ;
  constexpr bool PREQS = XIN == kXinPreQS;
  static_assert(!PREQ || !XS, "pre-quantised rows are read from global memory");
  static_assert(!PREQS || XS, "staged pre-quantised rows live in shared memory");
  constexpr int NC = dec_consumers(MT);
  constexpr int NCT = NC * 32;
  constexpr int SLOTS = kDecChunkGroups / NC;   // records per warp per chunk
  __shared__ float tok_scale_s[kMaxTables][kDecMaxTokens];
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages;
  const int G = p.K / kGroup;
  constexpr int MP = 8 * MT;  // token rows of the slice
  const int xstride = p.K + 16;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kDecStageBytes);
  uint64_t* empty = full + kDecMaxStages;
  uint64_t* seg_full = empty + kDecMaxStages;   // [2]: all consumer slices written
  uint64_t* seg_free = seg_full + 2;             // [2]: epilogue has read them
  uint64_t* xbar = seg_free + 2;                 // activation rows landed (bulk path)
  float* red = reinterpret_cast<float*>(xbar + 2);                           // [2][NC][MT*4][32]
  uint8_t* xrows = reinterpret_cast<uint8_t*>(red + 2 * NC * MT * 4 * 32);    // [xrows_n][K + 16]
  int* sxs = reinterpret_cast<int*>(xrows + (XS ? (size_t)p.xrows_n * xstride : 0));  // [G][MP] group sums

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
      mbar_init(&empty[s], NC);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&seg_full[b], NC);
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
      const Segs sg(u0, u1, G);
      int s = 0;
      uint32_t rnd = 0;   // passes over the ring so far
      bool ok = true;
      for (int i = 0; ok && i < sg.n; ++i) {
        int nb, g, ge;
        sg.get(i, nb, g, ge);
        const uint8_t* src = p.packed + ((int64_t)nb * G + g) * kRecBytes;
        while (g < ge) {
          const int n = min((g | (kDecChunkGroups - 1)) + 1, ge) - g;
          if (rnd > 0 && !mbar_wait(&empty[s], (rnd - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t bytes = (uint32_t)n * kRecBytes;
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(smem + (size_t)s * kDecStageBytes, src, bytes, &full[s]);
          src += bytes;
          g += n;
          if (++s == S) {
            s = 0;
            ++rnd;
          }
        }
      }
    }
    return;
  }

  if (warp > NC) {  // epilogue warps: warp NC + 1 + e takes the segments q = e (mod 2)
    const int ew = warp - (NC + 1);
    grid_dependency_wait();  // token scales (and rows) come from the previous kernel
    // both warps write the same token scales; each reads back its own
    for (int tb = 0; tb < p.tables; ++tb)
      for (int t = lane; t < ntok_slice; t += 32) tok_scale_s[tb][t] = p.xscale[tb * p.M + tok0 + t];
    __syncwarp();
    if constexpr (PREQ || PREQS) {
      // the quantiser that read the row maxima has finished: return them to
      // zero for the next call's rotation kernel
      if (blockIdx.x == 0 && blockIdx.y == 0 && ew == 0)
        for (int64_t t = lane; t < p.M * p.tables; t += 32) p.amax[t] = 0u;
    }
    uint32_t* cnt = p.cnt + (size_t)blockIdx.y * (p.N / kRecRows);
    if constexpr (PREQS) {
      // rows already in fragment order and their code sums ([G][MP], padding
      // tokens zero): bulk copies straight into place
      if (ew == 0 && lane == 0) {
        mbar_arrive_expect_tx(xbar, (uint32_t)ntok_slice * p.K + (uint32_t)(G * MP * 4));
        for (int r = 0; r < ntok_slice; ++r)
          bulk_g2s(xrows + (size_t)r * xstride, p.xq + (tok0 + r) * (int64_t)p.K, (uint32_t)p.K, xbar);
        bulk_g2s(sxs, p.gsum, (uint32_t)(G * MP * 4), xbar);
      }
    } else if constexpr (XS) {
      // large activation blocks: bulk copies of the rows (behind the weight
      // chunks already queued, but one copy per row)
      if (ew == 0 && lane == 0 && (int64_t)ntok_slice * p.K > kDecBulkXBytes) {
        mbar_arrive_expect_tx(xbar, (uint32_t)ntok_slice * p.K);
        for (int r = 0; r < ntok_slice; ++r)
          bulk_g2s(xrows + (size_t)r * xstride, p.xq + (tok0 + r) * (int64_t)p.K, (uint32_t)p.K, xbar);
      }
    }
    const int ntok = (int)min64(kDecMaxTokens, p.M - tok0);
    const Segs sg(u0, u1, G);
    for (int q = ew; q < sg.n; q += 2) {
      const int par = ew;
      int nb, gb, ge;
      sg.get(q, nb, gb, ge);
      const int seg_units = ge - gb;
      if (!mbar_wait(&seg_full[par], (q >> 1) & 1)) return;
      float v[MT * 4];
#pragma unroll
      for (int sl = 0; sl < MT * 4; ++sl) {
        float a = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < NC; ++w2) a += red[(size_t)(par * NC + w2) * kSlice + sl * 32 + lane];
        v[sl] = a;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&seg_free[par]);
      const bool whole = seg_units == G;
      const float* tsc = tok_scale_s[table_of(p, nb)];
#pragma unroll
      for (int sl = 0; sl < MT * 4; ++sl) {
        const int mt = sl >> 2, i = sl & 3;
        const int64_t t = tok0 + mt * 8 + 2 * tig + (i & 1);
        const int n = nb * kRecRows + gid + ((i >> 1) << 3);
        if (t < p.M) {
          if (whole)
            store_out(p.out, p.out_dtype, (size_t)t * p.N + n,
                      v[sl] * tsc[t - tok0] + bias_at(p.bias, p.bias_dtype, n));
          else
            red_add_fx(p.ws + (size_t)n * p.M + t, v[sl]);
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
          // up to 8 loads per lane in flight before the first store (each
          // load would otherwise wait out an L2 round trip on its own)
          const int nidx = kRecRows * ntok;
          for (int base = 0; base < nidx; base += 8 * 32) {
            float a[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int idx = base + j * 32 + lane;
              if (idx < nidx) {
                const int r = idx / ntok, tt = idx - r * ntok;
                a[j] = ld_cg_fx(p.ws + (size_t)(nb * kRecRows + r) * p.M + tok0 + tt);
              }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int idx = base + j * 32 + lane;
              if (idx < nidx) {
                const int r = idx / ntok, tt = idx - r * ntok;
                const int n = nb * kRecRows + r;
                const int64_t t = tok0 + tt;
                st_cg_u64(p.ws + (size_t)n * p.M + t, 0ull);
                store_out(p.out, p.out_dtype, (size_t)t * p.N + n,
                          a[j] * tsc[tt] + bias_at(p.bias, p.bias_dtype, n));
              }
            }
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
  const uint8_t* xrowf[MT];   // kXinPreQ: this lane's 32 bytes of group 0
  int xr[MT];   // staged row of this lane's token (clamped: rows past the tokens feed unused columns)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int64_t t = tok0 + mt * 8 + gid;
    xvalid[mt] = t < p.M;
    xrow[mt] = p.xq + (xvalid[mt] ? t : 0) * (int64_t)p.K + 4 * tig;
    xr[mt] = min(mt * 8 + gid, p.xrows_n - 1);
    xrowf[mt] = reinterpret_cast<const uint8_t*>(p.xq) + (xvalid[mt] ? t : 0) * (int64_t)p.K + 32 * tig;
  }
  if constexpr (PREQS) {
    grid_dependency_wait();
    if (!mbar_wait(xbar, 0)) return;   // rows and code sums landed (epilogue warp's copies)
  } else if constexpr (XS) {
    // Staged rows past the slice's tokens (when a later slice is short) hold
    // stale bytes, and lanes of tokens past the staged rows read the last
    // one; both only feed output columns that are never stored.  Each
    // (row, group) block's 32 words go to fragment order (word j*4 + t,
    // bytes 16j + 4t, to t*8 + j: lane tig's eight B words are then the 32
    // bytes at tig*32), and its code sum to sxs.
    grid_dependency_wait();
    for (int e = ctid; e < G * MP; e += NCT)
      if (e % MP >= ntok_slice) sxs[e] = 0;
    if ((int64_t)ntok_slice * p.K > kDecBulkXBytes) {
      // rows bulk-copied by the epilogue warp; a thread per block
      if (!mbar_wait(xbar, 0)) return;
      for (int e = ctid; e < ntok_slice * G; e += NCT) {
        const int r = e / G, g = e - r * G;
        uint4* blk = reinterpret_cast<uint4*>(xrows + (size_t)r * xstride + (size_t)g * kGroup);
        uint32_t o[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 v = blk[c];
          o[4 * c] = v.x;
          o[4 * c + 1] = v.y;
          o[4 * c + 2] = v.z;
          o[4 * c + 3] = v.w;
        }
        int sum = 0;
#pragma unroll
        for (int c = 0; c < 32; ++c) sum = __dp4a((int)o[c], 0x01010101, sum);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          blk[2 * t] = make_uint4(o[t], o[4 + t], o[8 + t], o[12 + t]);
          blk[2 * t + 1] = make_uint4(o[16 + t], o[20 + t], o[24 + t], o[28 + t]);
        }
        sxs[g * MP + r] = sum;
      }
    } else {
      // small blocks: loaded straight from global memory (L2: the previous
      // kernel just wrote them), a warp per block and a lane per word, so
      // they do not queue behind the weight stream's bulk copies
      // warp cw takes blocks cw, cw + NC, ... of the row-major (row, group)
      // order, walked with a running (row, group) pair
      constexpr int kBatch = 8;   // loads in flight per lane
      int r = 0, g = cw;
      while (g >= G) {
        g -= G;
        ++r;
      }
      while (r < ntok_slice) {
        uint32_t v[kBatch];
        int rr[kBatch], gg[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          rr[j] = r;
          gg[j] = g;
          if (r < ntok_slice)
            v[j] = ld_dep_u32(
                reinterpret_cast<const uint32_t*>(p.xq + (tok0 + r) * (int64_t)p.K + (size_t)g * kGroup) + lane);
          g += NC;
          while (g >= G) {
            g -= G;
            ++r;
          }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          if (rr[j] < ntok_slice) {   // uniform over the warp
            const int sum = __reduce_add_sync(0xffffffffu, __dp4a((int)v[j], 0x01010101, 0));
            reinterpret_cast<uint32_t*>(xrows + (size_t)rr[j] * xstride + (size_t)gg[j] * kGroup)
                [(lane & 3) * 8 + (lane >> 2)] = v[j];
            if (lane == 0) sxs[gg[j] * MP + rr[j]] = sum;
          }
        }
      }
    }
    named_barrier(1, NCT);
  } else {
    grid_dependency_wait();  // the activations come from the previous kernel
  }

  float y[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;

  const Segs sg(u0, u1, G);
  int s = 0;
  uint32_t rnd = 0;
  for (int q = 0; q < sg.n; ++q) {
    int nb, g, ge;
    sg.get(q, nb, g, ge);
    // this row block's activation set (several rotation tables: L2 route only)
    const int tset = PREQ ? table_of(p, nb) : 0;
    const int64_t xoff = tset * p.set_xq, goff = tset * p.set_gsum;
    while (g < ge) {
      const int n = min((g | (kDecChunkGroups - 1)) + 1, ge) - g;
      const int gbase = g & ~(kDecChunkGroups - 1);
      // pre-quantised rows from L2, one token tile: both slots' fragments and
      // code sums are requested before the wait for the weights, so their L2
      // latency overlaps it
      constexpr bool HOIST = PREQ && MT == 1;
      uint32_t hb[HOIST ? SLOTS : 1][8];
      int2 hs[HOIST ? SLOTS : 1];
      if constexpr (HOIST) {
#pragma unroll
        for (int slot = 0; slot < SLOTS; ++slot) {
          const int gg = min(gbase + slot * NC + cw, G - 1);
          if (xvalid[0]) {
            const uint4 b0 = ld_l2_v4(xrowf[0] + xoff + (size_t)gg * kGroup);
            const uint4 b1 = ld_l2_v4(xrowf[0] + xoff + (size_t)gg * kGroup + 16);
            hb[slot][0] = b0.x;
            hb[slot][1] = b0.y;
            hb[slot][2] = b0.z;
            hb[slot][3] = b0.w;
            hb[slot][4] = b1.x;
            hb[slot][5] = b1.y;
            hb[slot][6] = b1.z;
            hb[slot][7] = b1.w;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) hb[slot][i] = 0u;
          }
          hs[slot] = ld_l2_v2(p.gsum + goff + (size_t)gg * p.gsum_mp + tok0 + 2 * tig);
        }
      }
      if (!mbar_wait(&full[s], rnd & 1)) return;
#pragma unroll
      for (int slot = 0; slot < SLOTS; ++slot) {
        const int gg = gbase + slot * NC + cw;
        if (gg >= g && gg < g + n) {
          uint32_t bf[MT][8];
          int sx[MT][2];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            if constexpr (HOIST) {
#pragma unroll
              for (int i = 0; i < 8; ++i) bf[mt][i] = hb[slot][i];
              sx[mt][0] = hs[slot].x;
              sx[mt][1] = hs[slot].y;
            } else if constexpr (XS) {
              const uint4* xb = reinterpret_cast<const uint4*>(xrows + (size_t)xr[mt] * xstride +
                                                               (size_t)gg * kGroup + 32 * tig);
              const uint4 b0 = xb[0], b1 = xb[1];
              bf[mt][0] = b0.x;
              bf[mt][1] = b0.y;
              bf[mt][2] = b0.z;
              bf[mt][3] = b0.w;
              bf[mt][4] = b1.x;
              bf[mt][5] = b1.y;
              bf[mt][6] = b1.z;
              bf[mt][7] = b1.w;
              const int2 s2 = *reinterpret_cast<const int2*>(sxs + (size_t)gg * MP + mt * 8 + 2 * tig);
              sx[mt][0] = s2.x;
              sx[mt][1] = s2.y;
            } else if constexpr (PREQ) {
              // fragment-order rows and code sums in global memory (L2; .cg:
              // a previous call's lines in this SM's L1 could be stale)
              if (xvalid[mt]) {
                const uint4 b0 = ld_l2_v4(xrowf[mt] + xoff + (size_t)gg * kGroup);
                const uint4 b1 = ld_l2_v4(xrowf[mt] + xoff + (size_t)gg * kGroup + 16);
                bf[mt][0] = b0.x;
                bf[mt][1] = b0.y;
                bf[mt][2] = b0.z;
                bf[mt][3] = b0.w;
                bf[mt][4] = b1.x;
                bf[mt][5] = b1.y;
                bf[mt][6] = b1.z;
                bf[mt][7] = b1.w;
              } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) bf[mt][i] = 0u;
              }
              const int2 s2 = ld_l2_v2(p.gsum + goff + (size_t)gg * p.gsum_mp + tok0 + mt * 8 + 2 * tig);
              sx[mt][0] = s2.x;
              sx[mt][1] = s2.y;
            } else {
              load_bfrag_global(xrow[mt], xvalid[mt], gg, bf[mt]);
              // token row gid's sum, then the sums of this lane's C columns
              int part = frag_sum(bf[mt]);
              part += __shfl_xor_sync(0xffffffffu, part, 1);
              part += __shfl_xor_sync(0xffffffffu, part, 2);
              sx[mt][0] = __shfl_sync(0xffffffffu, part, 8 * tig);
              sx[mt][1] = __shfl_sync(0xffffffffu, part, 8 * tig + 4);
            }
          }
          process_record<MT>(smem + (size_t)s * kDecStageBytes + (size_t)(gg - g) * kRecBytes, bf, sx, gid, tig,
                             y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      g += n;
      if (++s == S) {
        s = 0;
        ++rnd;
      }
    }
    // segment end: hand this warp's partial to the epilogue warp
    const int par = q & 1;
    if (q >= 2 && !mbar_wait(&seg_free[par], ((q >> 1) - 1) & 1)) return;
    float* sl = red + (size_t)(par * NC + cw) * kSlice;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sl[(mt * 4 + i) * 32 + lane] = y[mt][i];
        y[mt][i] = 0.f;
      }
    __syncwarp();
    if (lane == 0) mbar_arrive(&seg_full[par]);
  }
}

PARO_DEFINE_ERROR_ACCESSOR(decode)

// Self-test of the bounded-wait error path: one thread waits, with the
// library's own mbar_wait, on a barrier that nothing arrives on.  No copy
// or other asynchronous operation is in flight, so the wait simply runs out
// after ~limit_cycles SM clocks, reports kErrMbarTimeout into this file's
// error word and the kernel returns normally.
__global__ void selftest_wait_kernel(long long limit_cycles) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, limit_cycles);
  }
}

cudaError_t launch_selftest_wait(long long limit_cycles, cudaStream_t st) {
  selftest_wait_kernel<<<1, 32, 0, st>>>(limit_cycles);
  return cudaGetLastError();
}

static size_t fixed_smem(int MT) {
  // full/empty rings, seg_full/seg_free pairs, xbar (+1 slot keeps 16-byte
  // alignment), then the reduction slices
  return (2 * kDecMaxStages + 6) * sizeof(uint64_t) +
         2 * (size_t)dec_consumers(MT) * MT * 4 * 32 * sizeof(float);
}

// Token rows staged per CTA: the slice's tokens (all of them below 64).
static int xrows_for(int MT, int64_t M) { return (int)(M < 8 * MT ? M : 8 * MT); }

// Shared memory of the staged int8 rows and their group sums for MT token
// tiles, or 0 if they do not fit beside three ring stages.
static size_t xs_bytes_for(int MT, int K, int64_t M) {
  const int G = K / kGroup;
  const size_t xs = (size_t)xrows_for(MT, M) * (K + 16) + (size_t)G * 8 * MT * sizeof(int);
  return fixed_smem(MT) + xs + 3 * (size_t)kDecStageBytes <= (size_t)kDecSmemBudget ? xs : 0;
}

template <int MT, bool XS, int XIN = -1>
static cudaError_t launch_mt(DecParams p, size_t xs_bytes, cudaStream_t st) {
  const size_t smem = (size_t)p.stages * kDecStageBytes + fixed_smem(MT) + (XS ? xs_bytes : 0);
  auto kern = gemm_stream_kernel<MT, XS, XIN>;
  cudaError_t e = ensure_smem_limit((const void*)kern, kDecSmemBudget + 4096);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.ctas, (unsigned)((p.M + kDecMaxTokens - 1) / kDecMaxTokens), 1);
  cfg.blockDim = dim3(dec_threads(MT), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

static void stages_for(DecParams& p, int MT, size_t xs_bytes) {
  const int stages = (int)((kDecSmemBudget - fixed_smem(MT) - xs_bytes) / kDecStageBytes);
  p.stages = stages > kDecMaxStages ? kDecMaxStages : stages;
}

template <int MT>
static cudaError_t launch_pick(DecParams p, cudaStream_t st) {
  const size_t xs_bytes = xs_bytes_for(MT, p.K, p.M);
  p.xrows_n = xrows_for(MT, p.M);
  stages_for(p, MT, xs_bytes);
  if (p.stages < 2) return cudaErrorInvalidValue;
  return xs_bytes ? launch_mt<MT, true>(p, xs_bytes, st) : launch_mt<MT, false>(p, 0, st);
}

static int g_num_sms = 0;

static void init_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
}

size_t gemm_decode_workspace(int64_t M, int N) {
  const int64_t slices = (M + kDecMaxTokens - 1) / kDecMaxTokens;
  size_t ws = (size_t)N * (size_t)M * sizeof(unsigned long long);
  ws = (ws + 255) & ~(size_t)255;
  return ws + (size_t)slices * (N / kRecRows) * sizeof(uint32_t);
}

// CTAs for nbk row blocks of G groups.  When the row blocks split evenly
// into at least 3/4 as many CTAs as SMs and a CTA's share is small (at most
// 64 records: the layer streams in a couple of microseconds), each CTA takes
// whole row blocks: no segment is shared, so no partial sums go through the
// workspace, whose fix-up latency would end the kernel; otherwise stream-K
// over all SMs keeps the per-CTA byte counts equal.
static int dec_ctas(int nbk, int G) {
  for (int k = 1; k <= 4; ++k) {
    if (nbk % k) continue;
    const int c = nbk / k;
    if (c <= g_num_sms && 4 * c >= 3 * g_num_sms && k * G <= 64) return c;
  }
  return (int)min64(g_num_sms, (int64_t)nbk * G);
}

static DecParams dec_params(int64_t M, int N, int K, const void* packed, const void* bias, int bias_dtype, void* out,
                            int out_dtype, void* ws) {
  init_sms();
  DecParams p = {};
  p.M = M;
  p.N = N;
  p.K = K;
  p.packed = static_cast<const uint8_t*>(packed);
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.out_dtype = out_dtype;
  const size_t wsf = ((size_t)N * (size_t)M * sizeof(unsigned long long) + 255) & ~(size_t)255;
  p.ws = static_cast<unsigned long long*>(ws);
  p.cnt = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + wsf);
  p.units = (int64_t)(N / kRecRows) * (K / kGroup);
  p.ctas = dec_ctas(N / kRecRows, K / kGroup);
  p.stages = 0;
  p.tables = 1;
  return p;
}

cudaError_t launch_gemm_rows(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                             const void* bias, int bias_dtype, void* out, int out_dtype, void* ws, uint32_t* amax,
                             const int* gsum, int gsum_mp, cudaStream_t st, int any_shape);

// Which decode GEMM runs: gemm_stream_kernel, unless the environment sets
// PARO_DECODE_GEMM=rows (read once per process), which sends the shapes
// where gemm_rows_kernel (gemm_rows.cu) measured at least as fast per launch
// (gate_up-wide layers, up to 8 tokens) to it.  Off by default: in the
// decode sweep of all four projections the streaming kernel alone was 2 %
// faster (2,249 against 2,205 GB/s of weights on B200).
static bool rows_kernel_enabled() {
  static const int on = [] {
    const char* v = getenv("PARO_DECODE_GEMM");
    return (v && strcmp(v, "rows") == 0) ? 1 : 0;
  }();
  return on != 0;
}

cudaError_t launch_gemm_decode(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                               const void* bias, int bias_dtype, void* out, int out_dtype, void* ws,
                               cudaStream_t st) {
  if (rows_kernel_enabled()) {
    const cudaError_t e = launch_gemm_rows(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, ws, nullptr,
                                           nullptr, 0, st, 0);
    if (e != cudaErrorNotSupported) return e;
  }
  DecParams p = dec_params(M, N, K, packed, bias, bias_dtype, out, out_dtype, ws);
  p.xq = xq;
  p.xscale = xscale;
  if (M <= 8) return launch_pick<1>(p, st);
  if (M <= 16) return launch_pick<2>(p, st);
  if (M <= 32) return launch_pick<4>(p, st);
  return launch_pick<8>(p, st);
}

// ---------------------------------------------------------------------------
// decode linear: rot16_decode_kernel rotates the activations into an fp16
// scratch and records each row's |max|, quant16_decode_kernel writes the
// int8 codes in fragment order with their group sums, and the GEMM, whose
// weight stream started during both, consumes them
// ---------------------------------------------------------------------------
cudaError_t launch_rot16_decode(int x_dtype, const void* x, int64_t M, int K, const RotTables& tabs, int T, __half* y,
                                uint32_t* amax, int frag, int pro_kind, const RotPro& pro, cudaStream_t st);
int gemm_tc_supported(int64_t M, int N, int K);
size_t gemm_tc_workspace(int64_t M, int N, int K);
cudaError_t launch_gemm_tc(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                           const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                           size_t workspace_bytes, cudaStream_t st);
cudaError_t launch_gemm_tc_sets(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, cudaStream_t st);
cudaError_t launch_gemm_tc_tile(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, int bt, cudaStream_t st,
                                uint32_t* zero_after, int zero_n, int out_mc);
int gemm_tc_sets_ok(int T, const int* tab_nb);

// Linears of up to 64 tokens whose GEMM is faster on the tensor cores
// (64-token tiles, split-K over the CTA pairs): from 13 tokens on long rows
// (down), 17 on gate_up-wide layers, 24 on the rest (gemm_tc_supported's
// measured crossovers).  Their rows still take this file's rotation +
// quantiser chain, in channel order.
int linear_decode_tc(int64_t M, int N, int K) {
  if (M > kDecMaxTokens || N % kRecRows || K % kGroup) return 0;
  return gemm_tc_supported(M, N, K);
}

// Workspace of the decode linear for T rotation tables (the GEMM's, then
// the row maxima of the T activation sets).
size_t linear_decode_workspace(int64_t M, int N, int K, int T) {
  const size_t tc = linear_decode_tc(M, N, K) ? gemm_tc_workspace(M, N, K) : 0;
  const size_t dec = gemm_decode_workspace(M, N);
  return (tc > dec ? tc : dec) + (((size_t)T * M * sizeof(uint32_t) + 255) & ~(size_t)255);
}

static int token_tiles(int64_t M) { return M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8; }

cudaError_t launch_quant16_decode(const __half* y, uint32_t* amax, int64_t M, int K, int Mp, int8_t* xq, float* xscale,
                                  int* gsum, int T, cudaStream_t st);

// Whether the GEMM stages the quantised rows in shared memory (kXinPreQS)
// or reads each record's fragments from L2 (kXinPreQ), measured on B200:
// staged for large layers (gate_up at 1 / 8 / 16 tokens: 19.3 / 20.8 / 26.2
// us against 24.7 / 27.5 / 35.4 us from L2), from L2 when each CTA streams
// few records (qkv, o: the copies' latency is most of their time, 0.2-0.3 us
// more per linear staged) or the rows do not fit.  Both beat quantising
// in the GEMM's own prologue, which this kernel did before (its exit
// counter and row reads delayed every CTA's first records).
static bool stage_rows(const DecParams& p) { return p.units > 64 * (int64_t)p.ctas; }

static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

// Scratch of the decode linear for T rotation tables: T activation sets of
// fp16 rotated rows, int8 codes, token scales and per-group code sums.
size_t linear_decode_scratch(int64_t M, int K, int T) {
  const size_t Mp = (size_t)8 * token_tiles(M);
  return al256((size_t)T * M * K * 2) + al256((size_t)T * M * K) + al256((size_t)T * M * 4) +
         al256((size_t)T * (K / kGroup) * Mp * 4);
}

template <int MT>
static cudaError_t launch_pick_preq(DecParams p, cudaStream_t st) {
  // the staged copy lands the code sums as one block: their row pitch must
  // be the kernel's (8 per token tile)
  const size_t xs_bytes = stage_rows(p) && p.gsum_mp == 8 * MT ? xs_bytes_for(MT, p.K, p.M) : 0;
  if (xs_bytes) {
    p.xrows_n = xrows_for(MT, p.M);
    stages_for(p, MT, xs_bytes);
    return launch_mt<MT, true, kXinPreQS>(p, xs_bytes, st);
  }
  p.xrows_n = 0;
  stages_for(p, MT, 0);
  return launch_mt<MT, false, kXinPreQ>(p, 0, st);
}

// Returns cudaErrorNotSupported (nothing launched) above kDecMaxTokens
// tokens; callers then run the two-kernel path.  T rotation tables (a group
// of linears sharing x, weights concatenated along N): tabs.rtab / cs[t]
// apply to row blocks [tab_nb[t], tab_nb[t + 1]) (tab_nb[0] = 0); with
// T > 1 the GEMM is the tensor-core kernel where the combined shape takes
// it and every table starts on a 256-row tile (each tile loads its table's
// activation set), otherwise the streaming kernel reading each set's
// fragments from L2.
cudaError_t launch_linear_decode_tables(const void* x, int x_dtype, const RotTables& tabs, int T, const int* tab_nb,
                                        int64_t M, int N, int K, const void* packed, const void* bias, int bias_dtype,
                                        void* out, int out_dtype, void* ws, void* scratch, int pro_kind,
                                        const RotPro& pro, cudaStream_t st) {
  if (M > kDecMaxTokens || M <= 0) return cudaErrorNotSupported;
  if (T < 1 || T > kMaxTables) return cudaErrorInvalidValue;
  DecParams p = dec_params(M, N, K, packed, bias, bias_dtype, out, out_dtype, ws);
  // (the tensor-core GEMM's row stores want a 16-byte aligned output; with
  // several tables, each table must start on one of its 256-row tiles)
  const bool tc = linear_decode_tc(M, N, K) && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                  gemm_tc_sets_ok(T, tab_nb);
  const size_t tcb = tc ? gemm_tc_workspace(M, N, K) : 0;
  const size_t decb = gemm_decode_workspace(M, N);
  uint8_t* tail = static_cast<uint8_t*>(ws) + (tcb > decb ? tcb : decb);
  p.amax = reinterpret_cast<uint32_t*>(tail);
  // rotation into the fp16 scratch, quantisation (fragment order + code
  // sums, or channel order for the tensor-core GEMM), then the GEMM
  __half* rot16 = static_cast<__half*>(scratch);
  cudaError_t e = launch_rot16_decode(x_dtype, x, M, K, tabs, T, rot16, p.amax, tc ? 0 : 1, pro_kind, pro, st);
  if (e != cudaSuccess) return e;
  uint8_t* sp = static_cast<uint8_t*>(scratch) + al256((size_t)T * M * K * 2);
  int8_t* xq = reinterpret_cast<int8_t*>(sp);
  float* xs = reinterpret_cast<float*>(sp + al256((size_t)T * M * K));
  int* gsum = reinterpret_cast<int*>(sp + al256((size_t)T * M * K) + al256((size_t)T * M * 4));
  const int Mp = 8 * token_tiles(M);
  e = launch_quant16_decode(rot16, p.amax, M, K, Mp, xq, xs, gsum, T, st);
  if (e != cudaSuccess) return e;
  if (tc) {
    // the tensor-core GEMM (launched behind the quantiser with programmatic
    // dependent launch) returns the row maxima to zero once the quantiser has
    // completed
    return launch_gemm_tc_tile(xq, xs, M, N, K, packed, bias, bias_dtype, out, out_dtype, tcb ? ws : nullptr, tcb, T,
                               tab_nb, 0, st, p.amax, (int)(T * M), 0);
  }
  if (T == 1 && rows_kernel_enabled()) {
    e = launch_gemm_rows(xq, xs, M, N, K, packed, bias, bias_dtype, out, out_dtype, ws, p.amax, gsum, Mp, st, 0);
    if (e != cudaErrorNotSupported) return e;
  }
  p.xq = xq;
  p.xscale = xs;
  p.gsum = gsum;
  p.gsum_mp = Mp;
  if (T > 1) {
    p.tables = T;
    for (int t = 0; t < T; ++t) p.tab_nb[t] = tab_nb[t];
    p.set_xq = M * (int64_t)K;
    p.set_gsum = (int64_t)(K / kGroup) * Mp;
    p.xrows_n = 0;
    switch (token_tiles(M)) {
      case 1: stages_for(p, 1, 0); return launch_mt<1, false, kXinPreQ>(p, 0, st);
      case 2: stages_for(p, 2, 0); return launch_mt<2, false, kXinPreQ>(p, 0, st);
      case 4: stages_for(p, 4, 0); return launch_mt<4, false, kXinPreQ>(p, 0, st);
    }
    stages_for(p, 8, 0);
    return launch_mt<8, false, kXinPreQ>(p, 0, st);
  }
  switch (token_tiles(M)) {
    case 1: return launch_pick_preq<1>(p, st);
    case 2: return launch_pick_preq<2>(p, st);
    case 4: return launch_pick_preq<4>(p, st);
  }
  return launch_pick_preq<8>(p, st);
}

cudaError_t launch_linear_decode(const void* x, int x_dtype, const uint16_t* cscale, const uint32_t* rtab, int64_t M,
                                 int N, int K, const void* packed, const void* bias, int bias_dtype, void* out,
                                 int out_dtype, void* ws, void* scratch, int pro_kind, const RotPro& pro,
                                 cudaStream_t st) {
  RotTables tabs = {};
  tabs.rtab[0] = rtab;
  tabs.cs[0] = cscale;
  const int nb0 = 0;
  return launch_linear_decode_tables(x, x_dtype, tabs, 1, &nb0, M, N, K, packed, bias, bias_dtype, out, out_dtype, ws,
                                     scratch, pro_kind, pro, st);
}

}  // namespace paro
