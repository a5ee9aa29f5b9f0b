// gemm_rows.cu — int4 x int8 GEMM for decode shapes (up to 16 tokens),
// sm_100a, with one row block per consumer warp.
//
// Same contract, record layout and workspace as gemm_stream_kernel
// (gemm_decode.cu); what changes is who adds what:
//
//  * The CTA's contiguous range of tile records (stream-K over all SMs, or
//    whole row blocks for small layers) is cut into segments, one per
//    16-row block, as before.  Segments are dealt out in rounds of 16
//    "items", one per consumer warp: with 16 or more segments a warp owns a
//    whole segment; with fewer, each segment is cut along its groups into
//    pieces so that all 16 warps stay busy.  A warp keeps its item's 16 x 8
//    (or 16 x 16) output sums in registers across all of the item's groups,
//    so no partial sum crosses warps except where a segment was cut.
//  * Ring stages hold one slot per warp (C records of that warp's row
//    block); the producer thread fills a stage with one bulk copy per warp
//    (cp.async.bulk + mbarrier complete_tx), so each warp's next records
//    are contiguous in its slot.
//  * A warp whose item is a whole row block that it owns alone applies the
//    token scales and bias and stores its outputs itself.  Cut or boundary
//    segments go through shared memory to an epilogue warp, which adds the
//    pieces in a fixed order and either stores (row block inside the CTA)
//    or adds into the 64-bit fixed-point workspace with a unit counter
//    (shared with a neighbouring CTA; the CTA that completes the count
//    finishes it and returns the workspace to zero), as gemm_stream_kernel
//    does.
//  * Per record a warp does two 16-byte loads of codes, its B fragments and
//    code sums (loaded before it waits for the stage), 16 mask operations,
//    4 mma.sync m16n8k32 u8.s8 per 8-token tile, and per output an integer
//    zero-point fold and one float FMA with the raw group scale; the 1/16
//    of the high-nibble trick is applied once, at the end (a power of two:
//    the result is the same as scaling every term).
//
// Activations come as in gemm_stream_kernel: int8 rows in channel order
// (paro_rotq_int8) bulk-copied and rearranged in shared memory into
// fragment order with their group sums, or (linear route) rows already in
// fragment order with their sums from quant16_decode_kernel, bulk-copied
// into place.
#include "stream_segs.cuh"
#include "tc_ptx.cuh"

namespace paro {

constexpr int kRwWarps = 16;                      // consumer warps
constexpr int kRwThreads = 32 * (kRwWarps + 3);   // producer, consumers, two epilogue warps
constexpr int kRwMaxStages = 8;
constexpr int kRwSmemBudget = 220 * 1024;
constexpr int kRwMaxTokens = 16;
constexpr int kRwBulkXBytes = 32 * 1024;          // channel-order blocks above this are bulk-copied
constexpr int kXinRowsChan = 0;                   // int8 rows in channel order (paro_rotq_int8)
constexpr int kXinRowsFrag = 1;                   // rows in fragment order + code sums (quant16_decode_kernel)

struct RwItem {
  int nb;          // row block
  short gb, ge;    // this warp's groups [gb, ge)
  short w0, k;     // the segment's pieces are warps w0 .. w0 + k - 1 (k = 0: no work)
  short sgb, sge;  // the segment's groups (its unit count toward the row block)
};

struct RwParams {
  const int8_t* xq;
  const float* xscale;
  int M, N, K;
  const uint8_t* packed;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  unsigned long long* ws;  // [N][M] fixed-point partial sums, zero between calls
  uint32_t* cnt;           // [N/16] unit counters, zero between calls
  uint32_t* amax;          // fragment-order route: row maxima to return to zero (or null)
  const int* gsum;         // fragment-order route: per (group, token) code sums [G][gsum_mp]
  int gsum_mp;
  int64_t units;
  int ctas;
  int stages;
  int xrows_n;
};

__device__ __forceinline__ void rw_mma(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void grid_dependency_wait_rw() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float rw_bias(const void* bias, int dtype, int n) {
  if (!bias) return 0.f;
  if (dtype == PARO_F16) return __half2float(static_cast<const __half*>(bias)[n]);
  if (dtype == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
  return static_cast<const float*>(bias)[n];
}

__device__ __forceinline__ void rw_store(void* out, int dtype, size_t idx, float v) {
  if (dtype == PARO_F16) static_cast<__half*>(out)[idx] = __float2half_rn(v);
  else if (dtype == PARO_BF16) static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else static_cast<float*>(out)[idx] = v;
}

// One record (16 rows x 128 channels) against MT token tiles, accumulated
// into y with the raw group scale: y += s * (16 * sum_k (q - z) x), exact in
// int32 up to the float FMA.  The low nibbles of a lane's four words per row
// are the A fragments of k-steps 0-1 (channels 0-63), the high nibbles
// masked in place are 16 * q for k-steps 2-3 (channels 64-127), so
//   16 * sum_k (q - z) x = 16 * (lo - z * sum_k x) + hi.
template <int MT>
__device__ __forceinline__ void rw_record(const uint8_t* rec, const uint32_t (&bf)[MT][8], const int (&sx)[MT][2],
                                          int gid, int tig, float (&y)[MT][4]) {
  const uint4 wa = *reinterpret_cast<const uint4*>(rec + gid * 64 + tig * 16);
  const uint4 wb = *reinterpret_cast<const uint4*>(rec + (gid + 8) * 64 + tig * 16);
  const uint16_t* sp = reinterpret_cast<const uint16_t*>(rec + kRecScaleOff);
  const float s_lo = half_bits_to_f32(sp[gid]), s_hi = half_bits_to_f32(sp[gid + 8]);
  const int z_lo = rec[kRecZeroOff + gid], z_hi = rec[kRecZeroOff + gid + 8];
  constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
  int lo[MT][4], hi[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) lo[mt][i] = hi[mt][i] = 0;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    rw_mma(lo[mt], wa.x & LO, wb.x & LO, wa.y & LO, wb.y & LO, bf[mt][0], bf[mt][1]);
    rw_mma(hi[mt], wa.x & HI, wb.x & HI, wa.y & HI, wb.y & HI, bf[mt][4], bf[mt][5]);
    rw_mma(lo[mt], wa.z & LO, wb.z & LO, wa.w & LO, wb.w & LO, bf[mt][2], bf[mt][3]);
    rw_mma(hi[mt], wa.z & HI, wb.z & HI, wa.w & HI, wb.w & HI, bf[mt][6], bf[mt][7]);
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int t0 = 16 * (lo[mt][0] - z_lo * sx[mt][0]) + hi[mt][0];
    const int t1 = 16 * (lo[mt][1] - z_lo * sx[mt][1]) + hi[mt][1];
    const int t2 = 16 * (lo[mt][2] - z_hi * sx[mt][0]) + hi[mt][2];
    const int t3 = 16 * (lo[mt][3] - z_hi * sx[mt][1]) + hi[mt][3];
    y[mt][0] = fmaf(s_lo, (float)t0, y[mt][0]);
    y[mt][1] = fmaf(s_lo, (float)t1, y[mt][1]);
    y[mt][2] = fmaf(s_hi, (float)t2, y[mt][2]);
    y[mt][3] = fmaf(s_hi, (float)t3, y[mt][3]);
  }
}

// The segments of a CTA's unit range in the visit order of Segs (the head
// of its last row block and the tail of its first, the two it shares with
// neighbouring CTAs, then the whole row blocks between), in 32-bit
// arithmetic (the host only launches this kernel when units * CTAs < 2^31).
struct RwSegs {
  int nb0, g0, nbL, gL1, G, n;
  __device__ __forceinline__ RwSegs(int u0, int u1, int G_) : G(G_) {
    if (u1 <= u0) {
      n = nb0 = g0 = nbL = gL1 = 0;
      return;
    }
    nb0 = u0 / G;
    g0 = u0 - nb0 * G;
    nbL = (u1 - 1) / G;
    gL1 = u1 - nbL * G;
    n = nbL == nb0 ? 1 : nbL - nb0 + 1;
  }
  __device__ __forceinline__ void get(int i, int& nb, int& gb, int& ge) const {
    if (nbL == nb0) {
      nb = nb0;
      gb = g0;
      ge = gL1;
    } else if (i == 0) {
      nb = nbL;
      gb = 0;
      ge = gL1;
    } else if (i == 1) {
      nb = nb0;
      gb = g0;
      ge = G;
    } else {
      nb = nb0 + i - 1;
      gb = 0;
      ge = G;
    }
  }
};

constexpr unsigned kFull = 0xffffffffu;

// Round r of a CTA's schedule, computed by one whole warp (every warp that
// needs it computes the same thing; no shared memory, no barrier).  The
// segments are dealt out in rounds of up to kRwWarps; lane j < m holds
// segment j of the round.  With fewer segments than warps, segment j is cut
// into k_j = ceil(L_j / P) pieces of ceil(L_j / k_j) groups, P the smallest
// length from ceil(T / kRwWarps) up for which all pieces fit the warps (T =
// the round's records), so no piece is empty.  Returns the item of warp slot
// `lane` (slots >= the number of pieces get an empty item), the round's
// ring stages (its longest piece / C) and whether any of its segments needs
// the epilogue warps (cut into pieces, or shared with another CTA).
// Rounds of a CTA: when its range has whole row blocks between two end
// segments and at least one end is shared with a neighbouring CTA, the two
// ends form round 0 (their fix-up through the workspace then overlaps the
// stream of the rest), and the whole row blocks follow in rounds of up to
// kRwWarps; otherwise all segments are dealt out evenly.
__device__ __forceinline__ int rw_head(const RwSegs& sg) {
  return (sg.n > 2 && (sg.gL1 < sg.G || sg.g0 > 0)) ? 2 : 0;
}
__device__ __forceinline__ int rw_rounds(const RwSegs& sg) {
  const int head = rw_head(sg);
  return (head ? 1 : 0) + (sg.n - head + kRwWarps - 1) / kRwWarps;
}

__device__ __forceinline__ RwItem rw_round(const RwSegs& sg, int rounds, int r, int G, int C, int lane, int& nst,
                                           int& epi) {
  const int head = rw_head(sg);
  int s0, m;
  if (head && r == 0) {
    s0 = 0;
    m = head;
  } else {
    const int rb = r - (head ? 1 : 0), nbr = rounds - (head ? 1 : 0), body = sg.n - head;
    s0 = head + (body * rb) / nbr;
    m = head + (body * (rb + 1)) / nbr - s0;
  }
  int nb = 0, gb = 0, ge = 0;
  if (lane < m) sg.get(s0 + lane, nb, gb, ge);
  const int L = lane < m ? ge - gb : 0;
  int k = lane < m ? 1 : 0;
  if (m < kRwWarps) {
    const int T = __reduce_add_sync(kFull, L);
    int P = max(1, (T + kRwWarps - 1) / kRwWarps);
    for (int tries = 0; tries < 64; ++tries, ++P) {
      const int kk = lane < m ? (L + P - 1) / P : 0;
      if (__reduce_add_sync(kFull, kk) <= kRwWarps) {
        k = kk;
        break;
      }
    }
  }
  const int pl = k > 0 ? (L + k - 1) / k : 0;
  int incl = k;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  const int w0 = incl - k;
  const int total = __shfl_sync(kFull, incl, 31);
  nst = (__reduce_max_sync(kFull, (unsigned)pl) + C - 1) / C;
  epi = __any_sync(kFull, k > 0 && !(k == 1 && gb == 0 && ge == G)) ? 1 : 0;
  // slot `lane` belongs to the segment whose pieces start at or before it
  const unsigned starts = __reduce_or_sync(kFull, k > 0 ? (1u << w0) : 0u);
  const int j = max(0, __popc(starts & ((2u << lane) - 1u)) - 1);
  const int snb = __shfl_sync(kFull, nb, j), sgb = __shfl_sync(kFull, gb, j), sge = __shfl_sync(kFull, ge, j);
  const int spl = __shfl_sync(kFull, pl, j), sw0 = __shfl_sync(kFull, w0, j), sk = __shfl_sync(kFull, k, j);
  RwItem it;
  if (lane < total) {
    const int b = sgb + (lane - sw0) * spl;
    it.nb = snb;
    it.gb = (short)b;
    it.ge = (short)min(sge, b + spl);
    it.w0 = (short)sw0;
    it.k = (short)sk;
    it.sgb = (short)sgb;
    it.sge = (short)sge;
  } else {
    it.nb = 0;
    it.gb = it.ge = 0;
    it.w0 = (short)lane;
    it.k = 0;
    it.sgb = it.sge = 0;
  }
  return it;
}

__device__ __forceinline__ RwItem rw_item_from(const RwItem& it, int src) {
  RwItem o;
  o.nb = __shfl_sync(kFull, it.nb, src);
  o.gb = (short)__shfl_sync(kFull, (int)it.gb, src);
  o.ge = (short)__shfl_sync(kFull, (int)it.ge, src);
  o.w0 = (short)__shfl_sync(kFull, (int)it.w0, src);
  o.k = (short)__shfl_sync(kFull, (int)it.k, src);
  o.sgb = (short)__shfl_sync(kFull, (int)it.sgb, src);
  o.sge = (short)__shfl_sync(kFull, (int)it.sge, src);
  return o;
}

template <int MT, int C, int XIN>
__global__ void __launch_bounds__(kRwThreads, 1) gemm_rows_kernel(RwParams p) {
  constexpr int NC = kRwWarps;
  constexpr int NCT = NC * 32;
  constexpr int MP = 8 * MT;
  constexpr int kSlice = MT * 4 * 32;
  constexpr int kSlotBytes = C * kRecBytes;
  constexpr int kStageBytes = NC * kSlotBytes;
  constexpr bool FRAGIN = XIN == kXinRowsFrag;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float tok_scale_s[kRwMaxTokens];

  const int S = p.stages;
  const int G = p.K / kGroup;
  const int xstride = p.K + 16;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kStageBytes);
  uint64_t* empty = full + kRwMaxStages;
  uint64_t* seg_full = empty + kRwMaxStages;   // [2]: every consumer warp handed its round over
  uint64_t* seg_free = seg_full + 2;            // [2]: the epilogue warp has read the slots
  uint64_t* xbar = seg_free + 2;                // activation rows landed
  float* red = reinterpret_cast<float*>(xbar + 2);                         // [2][NC][kSlice]
  uint8_t* xrows = reinterpret_cast<uint8_t*>(red + 2 * NC * kSlice);     // [xrows_n][K + 16]
  int* sxs = reinterpret_cast<int*>(xrows + (size_t)p.xrows_n * xstride);  // [G][MP]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const unsigned units = (unsigned)p.units, ctas = (unsigned)p.ctas;
  const RwSegs sg((int)(blockIdx.x * units / ctas), (int)((blockIdx.x + 1) * units / ctas), G);
  const int rounds = rw_rounds(sg);

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

  if (warp == 0) {
    // producer warp (weights do not depend on the previous kernel): lane w
    // streams warp slot w's records; lane 0 accounts for the stage's bytes
    int s = 0;
    uint32_t pass = 0;
    for (int r = 0; r < rounds; ++r) {
      int nst, epi;
      const RwItem it = rw_round(sg, rounds, r, G, C, lane, nst, epi);
      const uint8_t* src = p.packed + rec_offset(it.nb, it.gb, G);
      for (int st = 0; st < nst; ++st) {
        int ok = 1;
        if (lane == 0 && pass > 0) ok = mbar_wait(&empty[s], (pass - 1) & 1) ? 1 : 0;
        if (!__shfl_sync(kFull, ok, 0)) return;
        const int n = max(0, min(C, it.ge - (it.gb + st * C)));
        const uint32_t bytes = __reduce_add_sync(kFull, (uint32_t)n * kRecBytes);
        if (lane == 0) mbar_arrive_expect_tx(&full[s], bytes);
        __syncwarp();
        if (n > 0) bulk_g2s(smem + (size_t)s * kStageBytes + lane * kSlotBytes, src, (uint32_t)n * kRecBytes, &full[s]);
        src += C * kRecBytes;
        if (++s == S) {
          s = 0;
          ++pass;
        }
      }
    }
    return;
  }

  if (warp > NC) {  // epilogue warps: warp NC + 1 + e takes the epilogue rounds e (mod 2)
    const int ew = warp - (NC + 1);
    grid_dependency_wait_rw();  // token scales (and rows) come from the previous kernel
    if (ew == 0 && (FRAGIN || p.M * p.K > kRwBulkXBytes)) {
      // rows (and, in fragment order, their code sums) by bulk copies, one
      // per lane, issued before anything else: the consumers wait for them
      if (lane == 0)
        mbar_arrive_expect_tx(xbar, (uint32_t)p.M * p.K + (FRAGIN ? (uint32_t)(G * MP * 4) : 0u));
      __syncwarp();
      if (lane < p.M) bulk_g2s(xrows + (size_t)lane * xstride, p.xq + (int64_t)lane * p.K, (uint32_t)p.K, xbar);
      if (FRAGIN && lane == 31) bulk_g2s(sxs, p.gsum, (uint32_t)(G * MP * 4), xbar);
    }
    for (int t = lane; t < p.M; t += 32) tok_scale_s[t] = ld_dep(p.xscale + t);
    __syncwarp();
    if (FRAGIN && p.amax && blockIdx.x == 0 && ew == 0)
      for (int t = lane; t < p.M; t += 32) p.amax[t] = 0u;   // the quantiser that read them has finished
    int e = 0;
    for (int r = 0; r < rounds; ++r) {
      int nst, epi;
      const RwItem mine = rw_round(sg, rounds, r, G, C, lane, nst, epi);
      if (!epi) continue;
      const int par = e & 1;
      if (par == ew) {
        if (!mbar_wait(&seg_full[par], (e >> 1) & 1)) return;
        // segments for this warp: first pieces whose segment is cut or shared
        unsigned todo = __ballot_sync(kFull, lane < NC && mine.k > 0 && mine.w0 == lane &&
                                                 !(mine.k == 1 && mine.sgb == 0 && mine.sge == G));
        while (todo) {
          const int w = __ffs(todo) - 1;
          todo &= todo - 1;
          const RwItem s = rw_item_from(mine, w);
          const bool whole = s.sgb == 0 && s.sge == G;
          float v[MT * 4];
#pragma unroll
          for (int sl = 0; sl < MT * 4; ++sl) {
            float a = 0.f;
            for (int q = 0; q < s.k; ++q) a += red[(size_t)(par * NC + w + q) * kSlice + sl * 32 + lane];
            v[sl] = a * 0.0625f;
          }
#pragma unroll
          for (int sl = 0; sl < MT * 4; ++sl) {
            const int mt = sl >> 2, i = sl & 3;
            const int t = mt * 8 + 2 * tig + (i & 1);
            const int n = s.nb * kRecRows + gid + ((i >> 1) << 3);
            if (t < p.M) {
              if (whole)
                rw_store(p.out, p.out_dtype, (size_t)t * p.N + n,
                         v[sl] * tok_scale_s[t] + rw_bias(p.bias, p.bias_dtype, n));
              else
                red_add_fx(p.ws + (size_t)n * p.M + t, v[sl]);
            }
          }
          if (!whole) {
            // release the partial adds, count the units; the CTA that
            // completes the row block acquires every partial and finishes it
            __syncwarp();
            int last = 0;
            const int seg_units = s.sge - s.sgb;
            if (lane == 0) {
              asm volatile("fence.acq_rel.gpu;" ::: "memory");
              const uint32_t old = atomicAdd(&p.cnt[s.nb], (uint32_t)seg_units);
              last = (old + (uint32_t)seg_units == (uint32_t)G);
              if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
            }
            last = __shfl_sync(kFull, last, 0);
            if (last) {
              const int nidx = kRecRows * p.M;
              for (int base = 0; base < nidx; base += 8 * 32) {
                float a[8];
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const int idx = base + jj * 32 + lane;
                  if (idx < nidx) {
                    const int rr = idx / p.M, tt = idx - rr * p.M;
                    a[jj] = ld_cg_fx(p.ws + (size_t)(s.nb * kRecRows + rr) * p.M + tt);
                  }
                }
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                  const int idx = base + jj * 32 + lane;
                  if (idx < nidx) {
                    const int rr = idx / p.M, tt = idx - rr * p.M;
                    const int n = s.nb * kRecRows + rr;
                    st_cg_u64(p.ws + (size_t)n * p.M + tt, 0ull);
                    rw_store(p.out, p.out_dtype, (size_t)tt * p.N + n,
                             a[jj] * tok_scale_s[tt] + rw_bias(p.bias, p.bias_dtype, n));
                  }
                }
              }
              __syncwarp();
              if (lane == 0) p.cnt[s.nb] = 0u;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&seg_free[par]);
      }
      ++e;
    }
    return;
  }

  // ---- consumers ----------------------------------------------------------
  const int cw = warp - 1;
  const int ctid = threadIdx.x - 32;
  grid_dependency_wait_rw();   // the activations come from the previous kernel
  if constexpr (FRAGIN) {
    if (!mbar_wait(xbar, 0)) return;   // rows and code sums landed (epilogue warp's copies)
  } else {
    // token rows past M feed output columns that are never stored: zero
    // their sums; rows in channel order go to fragment order (word j*4 + t
    // to t*8 + j) with their per-group sums
    for (int e = ctid; e < G * MP; e += NCT)
      if (e % MP >= p.M) sxs[e] = 0;
    if (p.M * p.K > kRwBulkXBytes) {
      if (!mbar_wait(xbar, 0)) return;
      for (int e = ctid; e < p.M * G; e += NCT) {
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
      // small blocks straight from L2, a warp per (row, group) block and a
      // lane per word, several loads in flight per lane
      constexpr int kBatch = 8;
      int r = 0, g = cw;
      while (g >= G) {
        g -= G;
        ++r;
      }
      while (r < p.M) {
        uint32_t v[kBatch];
        int rr[kBatch], gg[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          rr[j] = r;
          gg[j] = g;
          if (r < p.M)
            v[j] = ld_dep_u32(reinterpret_cast<const uint32_t*>(p.xq + (int64_t)r * p.K + (size_t)g * kGroup) + lane);
          g += NC;
          while (g >= G) {
            g -= G;
            ++r;
          }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          if (rr[j] < p.M) {   // uniform over the warp
            const int sum = __reduce_add_sync(0xffffffffu, __dp4a((int)v[j], 0x01010101, 0));
            reinterpret_cast<uint32_t*>(xrows + (size_t)rr[j] * xstride + (size_t)gg[j] * kGroup)
                [(lane & 3) * 8 + (lane >> 2)] = v[j];
            if (lane == 0) sxs[gg[j] * MP + rr[j]] = sum;
          }
        }
      }
    }
    named_barrier(1, NCT);
  }

  // this lane's token rows (rows past the staged ones read the last staged
  // row; they only feed output columns that are never stored) and the token
  // scales of its output columns
  int xr[MT];
  float tsc[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    xr[mt] = min(mt * 8 + gid, p.xrows_n - 1);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = mt * 8 + 2 * tig + j;
      tsc[mt][j] = t < p.M ? ld_dep(p.xscale + t) : 0.f;
    }
  }

  int s = 0;
  uint32_t pass = 0;
  int e = 0;
  for (int r = 0; r < rounds; ++r) {
    int nst, epi;
    const RwItem it = rw_item_from(rw_round(sg, rounds, r, G, C, lane, nst, epi), cw);
    float y[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) y[mt][i] = 0.f;
    int g = it.gb;
    for (int st = 0; st < nst; ++st) {
      // B fragments and code sums of this stage's records, loaded before
      // waiting for the weights
      uint32_t bf[C][MT][8];
      int sx[C][MT][2];
#pragma unroll
      for (int j = 0; j < C; ++j) {
        const int gg = min(g + j, G - 1);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint4* xb =
              reinterpret_cast<const uint4*>(xrows + (size_t)xr[mt] * xstride + (size_t)gg * kGroup + 32 * tig);
          const uint4 b0 = xb[0], b1 = xb[1];
          bf[j][mt][0] = b0.x;
          bf[j][mt][1] = b0.y;
          bf[j][mt][2] = b0.z;
          bf[j][mt][3] = b0.w;
          bf[j][mt][4] = b1.x;
          bf[j][mt][5] = b1.y;
          bf[j][mt][6] = b1.z;
          bf[j][mt][7] = b1.w;
          const int2 s2 = *reinterpret_cast<const int2*>(sxs + (size_t)gg * MP + mt * 8 + 2 * tig);
          sx[j][mt][0] = s2.x;
          sx[j][mt][1] = s2.y;
        }
      }
      if (!mbar_wait(&full[s], pass & 1)) return;
      const uint8_t* slot = smem + (size_t)s * kStageBytes + cw * kSlotBytes;
#pragma unroll
      for (int j = 0; j < C; ++j)
        if (g + j < it.ge) rw_record<MT>(slot + j * kRecBytes, bf[j], sx[j], gid, tig, y);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      g += C;
      if (++s == S) {
        s = 0;
        ++pass;
      }
    }
    const bool own = it.k == 1 && it.sgb == 0 && it.sge == G;
    if (own) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = mt * 8 + 2 * tig + (i & 1);
          const int n = it.nb * kRecRows + gid + ((i >> 1) << 3);
          if (t < p.M)
            rw_store(p.out, p.out_dtype, (size_t)t * p.N + n,
                     y[mt][i] * 0.0625f * tsc[mt][i & 1] + rw_bias(p.bias, p.bias_dtype, n));
        }
    }
    if (epi) {
      const int par = e & 1;
      if (e >= 2 && !mbar_wait(&seg_free[par], ((e >> 1) - 1) & 1)) return;
      if (!own && it.k > 0) {
        float* sl = red + (size_t)(par * NC + cw) * kSlice;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) sl[(mt * 4 + i) * 32 + lane] = y[mt][i];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&seg_full[par]);
      ++e;
    }
  }
}

PARO_DEFINE_ERROR_ACCESSOR(rows)

static size_t rw_fixed_smem(int MT) {
  // full/empty rings, seg_full/seg_free pairs, xbar (+1 slot keeps 16-byte
  // alignment), then the reduction slots
  return (2 * kRwMaxStages + 6) * sizeof(uint64_t) + 2 * (size_t)kRwWarps * MT * 4 * 32 * sizeof(float);
}

static size_t rw_xs_bytes(int MT, int K, int M) {
  return (size_t)M * (K + 16) + (size_t)(K / kGroup) * 8 * MT * sizeof(int);
}

static int g_rw_sms = 0;

static int rw_sms() {
  if (g_rw_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_rw_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_rw_sms <= 0) g_rw_sms = 148;
  }
  return g_rw_sms;
}

// CTAs as gemm_stream_kernel chooses them: whole row blocks per CTA when
// they split evenly into at least 3/4 as many CTAs as SMs and a CTA's share
// is small, stream-K over all SMs otherwise.
static int rw_ctas(int nbk, int G) {
  const int sms = rw_sms();
  for (int k = 1; k <= 4; ++k) {
    if (nbk % k) continue;
    const int c = nbk / k;
    if (c <= sms && 4 * c >= 3 * sms && k * G <= 64) return c;
  }
  return (int)min64(sms, (int64_t)nbk * G);
}

// Launch plan: records per warp per stage (C) and stages, or false when
// this kernel does not take the shape (more than 16 tokens, rows that do
// not fit beside three stages, or more rounds than the schedule holds).
struct RwPlan {
  int MT, C, stages, ctas;
  size_t smem;
};

// any_shape: every shape the kernel handles (the explicit route), otherwise
// only where it measured at least as fast as the streaming kernel.
static bool rw_plan(int64_t M, int N, int K, RwPlan& pl, bool any_shape = false) {
  if (M < 1 || M > kRwMaxTokens || N % kRecRows || K % kGroup) return false;
  const int G = K / kGroup, nbk = N / kRecRows;
  pl.MT = M <= 8 ? 1 : 2;
  pl.ctas = rw_ctas(nbk, G);
  // Where this kernel measured at least as fast as gemm_stream_kernel on
  // B200 (per-launch times in a CUDA graph, weights > L2): up to 8 tokens on
  // layers whose CTAs own 16 or more whole row blocks each (gate_up at 1 /
  // 4 / 8 tokens: 16.6 / 16.8 / 17.0 us against 16.5 / 17.0 / 18.3).  Where
  // its row blocks are cut into pieces (qkv, o, down) the streaming kernel
  // was 2-5 us faster per launch.
  if (!any_shape && (M > 8 || (int64_t)nbk < 16 * (int64_t)pl.ctas)) return false;
  // the kernel walks its unit range in 32-bit arithmetic
  const int64_t units = (int64_t)nbk * G;
  if (units * (pl.ctas + 1) >= (int64_t)1 << 31 || (int64_t)M * K >= (int64_t)1 << 31) return false;
  const size_t base = rw_fixed_smem(pl.MT) + rw_xs_bytes(pl.MT, K, (int)M);
  if (base >= (size_t)kRwSmemBudget) return false;
  const size_t room = (size_t)kRwSmemBudget - base;
  // two records (2 KB bulk copies) per warp per stage, at least 4 stages
  // (1 KB copies streamed at about half the rate on B200)
  pl.C = 2;
  const size_t stage = (size_t)kRwWarps * 2 * kRecBytes;
  const int st = (int)(room / stage);
  if (st < 4) return false;
  pl.stages = st > kRwMaxStages ? kRwMaxStages : st;
  pl.smem = base + (size_t)pl.stages * stage;
  return true;
}

int gemm_rows_supported(int64_t M, int N, int K) {
  RwPlan pl;
  return rw_plan(M, N, K, pl) ? 1 : 0;
}

template <int MT, int C, int XIN>
static cudaError_t rw_launch(const RwParams& p, size_t smem, cudaStream_t st) {
  auto kern = gemm_rows_kernel<MT, C, XIN>;
  cudaError_t e = ensure_smem_limit((const void*)kern, kRwSmemBudget);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.ctas, 1, 1);
  cfg.blockDim = dim3(kRwThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int XIN>
static cudaError_t rw_dispatch(const RwParams& p, const RwPlan& pl, cudaStream_t st) {
  if (pl.MT == 1) return pl.C == 2 ? rw_launch<1, 2, XIN>(p, pl.smem, st) : rw_launch<1, 1, XIN>(p, pl.smem, st);
  return pl.C == 2 ? rw_launch<2, 2, XIN>(p, pl.smem, st) : rw_launch<2, 1, XIN>(p, pl.smem, st);
}

// ws: gemm_decode_workspace(M, N) bytes (the same layout: [N][M] fixed-point
// sums, then the row-block counters), zero-filled and left so.
// amax / gsum / gsum_mp: the fragment-order route (quant16_decode_kernel's
// output; gsum_mp must be 8 * token tiles); amax == nullptr and gsum ==
// nullptr for int8 rows in channel order.  Returns cudaErrorNotSupported
// (nothing launched) for shapes rw_plan does not take.
cudaError_t launch_gemm_rows(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                             const void* bias, int bias_dtype, void* out, int out_dtype, void* ws, uint32_t* amax,
                             const int* gsum, int gsum_mp, cudaStream_t st, int any_shape) {
  RwPlan pl;
  if (!rw_plan(M, N, K, pl, any_shape != 0)) return cudaErrorNotSupported;
  if (gsum && gsum_mp != 8 * pl.MT) return cudaErrorNotSupported;
  RwParams p = {};
  p.xq = xq;
  p.xscale = xscale;
  p.M = (int)M;
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
  p.amax = amax;
  p.gsum = gsum;
  p.gsum_mp = gsum_mp;
  p.units = (int64_t)(N / kRecRows) * (K / kGroup);
  p.ctas = pl.ctas;
  p.stages = pl.stages;
  p.xrows_n = (int)M;
  return gsum ? rw_dispatch<kXinRowsFrag>(p, pl, st) : rw_dispatch<kXinRowsChan>(p, pl, st);
}

}  // namespace paro
