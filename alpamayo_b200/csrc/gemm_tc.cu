// gemm_tc.cu — int4 x int8 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::i8, int32 accumulators in tensor memory) for prefill shapes, sm_100a.
//
// y[m, n] = xscale[m] * sum_g s[g, n] * sum_{k in g} (q[n, k] - z[g, n]) x[m, k] (+ bias[n])
//
// Persistent grid of CTA pairs (clusters of two): pair P walks the tiles
// P, P + pairs, ... of the (N / 256) x (M / BT) tile grid, so one tile's
// final stores overlap the next tile's loads and MMAs.  A pair computes a
// 256 (output rows n) x BT (tokens m) tile of y^T with cta_group::2 MMAs
// (M = 256, N = BT, K = 32); BT is 256 for prefill and 64 for 17-128 tokens
// (TcTile).  Each CTA holds 128 weight rows (half of the MMA's A operand)
// and BT / 2 tokens (half of its B operand) in shared memory, and its tensor
// memory holds the int32 sums of its own 128 rows for all BT tokens.
// The weights are the MMA's M operand and the tokens its N operand, so a TMEM
// lane is one output row and each epilogue thread owns one row (its group
// scale is one scalar per group).  K is walked one 128-channel group per
// pipeline stage (6 stages for BT = 256, 8 for BT = 64):
//
//  * warp 0 (producer, each CTA): per group, one tensor TMA of the CTA's
//    activation half (BT / 2 tokens x 128 int8 channels, 128-byte swizzle =
//    the UMMA K-major canonical layout) and one 3-D tensor TMA of its 8
//    weight records (16 rows x 128 channels each; the packed buffer viewed
//    as [N/16][G][1072 bytes]), which land in the stage's weight area.
//  * warpgroup 1 (expansion, each CTA): thread t reads row t's int4 codes
//    and zero point into registers, the warpgroup synchronises (records and
//    expanded rows share the area), thread t writes row t as signed int8
//    (q - z) in the swizzled K-major layout, and each warp then arrives on
//    the leader CTA's "stage ready" barrier.
//  * warp 1 of the leader CTA (MMA): once both CTAs' stage is ready and the
//    accumulator buffer has been drained by both epilogues, issues 4 MMAs
//    into one of 2 (BT = 256) or 4 (BT = 64) BT-column TMEM buffers (the
//    first overwriting it) and
//    commits completion to the stage-free and accumulator-full barriers of
//    both CTAs (tcgen05.commit multicast).
//  * warpgroups 2-3 (epilogue, each CTA): fold each finished group into
//    float32 registers while the tensor core works on the next group: each
//    int32 group sum (|acc| < 2^18, so the conversion is exact) is converted
//    to float32 and one packed FMA per two elements applies the row's group
//    scale; then each warp arrives on the leader's "buffer drained" barrier.
//    After the last group: token scale, bias, convert, store.
//
// Launched with programmatic dependent launch: set-up (barriers, tensor
// memory) and the first stages' weight boxes overlap the previous kernel on
// the stream; the activation boxes, the token scales and every store wait
// for it (griddepcontrol.wait).
//
// Per SM and group this moves 8.5 KB of records + BT / 2 x 128 bytes of
// activations from L2 for 128 x BT x 128 MACs.  No load uses cluster multicast.  All
// mbarrier waits are bounded (report kErrMbarTimeout and drop out), and the
// tensor memory is freed on every path out of the kernel, after both CTAs
// have stopped using it.
#include "umma.cuh"

namespace paro {

PARO_DEFINE_ERROR_ACCESSOR(tc)

constexpr int kTcRows = 128;                              // output rows per CTA (half the MMA's M)
constexpr int kTcThreads = 512;
constexpr int kTcRecs = kTcRows / kRecRows;               // 8 records per group
constexpr int kTcWBytes = kTcRows * kGroup;               // 16 KB expanded weights
static_assert(kTcRecs * kRecBytes <= kTcWBytes, "records land in the expanded-weight area");

// Tile shapes: BT tokens per tile (the MMA's N), 256 for prefill and 64 for
// 17-128 tokens, where a 256-token tile would spend most of every MMA and
// of the epilogue's per-group fold on padding.
template <int BT>
struct TcTile {
  static_assert(BT == 256 || BT == 64, "tile tokens");
  static constexpr int kTok = BT;                        // tokens per tile (MMA N)
  static constexpr int kTokHalf = BT / 2;                // tokens staged per CTA
  static constexpr int kStages = BT == 256 ? 6 : 8;
  static constexpr int kBufs = BT == 256 ? 2 : 4;        // TMEM accumulators in flight
  static constexpr int kTmemCols = kBufs * BT;           // 512 or 256 (a power of two)
  static constexpr int kXBytes = kTokHalf * kGroup;      // 16 KB or 4 KB activations per stage
  static constexpr int kCols = kTokHalf;                 // token columns per epilogue thread
  static constexpr int kPairs = kCols / 2;               // packed f32x2 accumulators per thread
  // shared memory plan (offsets from a 1024-byte aligned base; identical in
  // both CTAs, which the pair MMA's descriptors rely on)
  static constexpr int kOffW = 0;
  static constexpr int kOffX = kOffW + kStages * kTcWBytes;
  static constexpr int kOffXs = kOffX + kStages * kXBytes;   // [8 warps][kTokHalf] float token scales
  static constexpr int kOffBar = kOffXs + 8 * kTokHalf * 4;
  static constexpr int kSmem = kOffBar + 512 + 1024;         // barriers + alignment slack
  // instruction descriptor: s32 accumulate, A s8, B s8, both K-major,
  // N = BT, M = 256 (the CTA pair)
  static constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BT >> 3) << 17) |
                                     ((uint32_t)((2 * kTcRows) >> 4) << 24);
  static_assert((3 * kStages + 2 * kBufs + 1) * 8 + 4 <= 512, "barrier area");
  static_assert(kXBytes % 1024 == 0, "128-byte swizzle atoms stay 1024-byte aligned");
};

struct TcParams {
  const float* xscale;
  int64_t M;
  int N, K;
  int tiles_n, tiles;   // tiles along N (256 rows each) and in total
  int splits, gper;     // K splits per tile and groups per split (split-K when tiles are few)
  int items;            // tiles * splits
  const uint8_t* packed;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  unsigned long long* ws;  // splits > 1: [M][N] int64 fixed-point (2^-28) partial sums, zero between calls
  uint32_t* cnt;        // splits > 1: [tiles][2 CTAs][8 epilogue warps] counters, zero between calls
  // activation sets (one per rotation table of a projection group, weights
  // concatenated along N): the activations are [tables][M][K], the token
  // scales [tables][M]; rows from 16 * tab_nb[t] on use set t, and every
  // table starts on a 256-row tile
  int tables;
  int tab_nb[kMaxTables];
  // words the previous kernel on the stream read last (the decode chain's
  // row maxima): zeroed once that kernel has completed, or null
  uint32_t* zero_after;
  int zero_n;
  // out is an NVLink multicast address: bf16 stores as multimem.st (the
  // other ranks' copies of the buffer receive them too)
  int out_mc;
};

// The activation set of the 256-row tile starting at output row n.
__device__ __forceinline__ int tc_set(const TcParams& p, int n) {
  int t = 0;
#pragma unroll
  for (int i = 1; i < kMaxTables; ++i) t += (i < p.tables && n >= p.tab_nb[i] * kRecRows) ? 1 : 0;
  return t;
}


__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the barrier at this offset in both CTAs of the pair once every
// MMA the calling thread issued before has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(both)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Arrive on the barrier at the same offset in CTA `rank` of this cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n .reg .b32 ra;\n mapa.shared::cluster.u32 ra, %0, %1;\n"
      " mbarrier.arrive.shared::cluster.b64 _, [ra];\n}\n" ::"r"(smem_u32(bar)),
      "r"(rank)
      : "memory");
}

// Bounded wait on a barrier the peer CTA also arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, long long limit_cycles = 1000000000LL) {
  auto try_once = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (try_once()) return true;
  const long long t0 = clock64();
  while (!try_once()) {
    if (clock64() - t0 > limit_cycles) {
      report_error(kErrMbarTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}






__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// packed float32 pair arithmetic (sm_100)
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

__device__ __forceinline__ uint32_t ldg_nc_u16(const uint16_t* p) {
  uint16_t r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}


__device__ __forceinline__ float tc_bias(const void* bias, int dtype, int n) {
  if (!bias) return 0.f;
  if (dtype == PARO_F16) return __half2float(static_cast<const __half*>(bias)[n]);
  if (dtype == PARO_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
  return static_cast<const float*>(bias)[n];
}

// Stores one output row's `valid` (<= 2 NP) tokens: out[j * N] = y_j * xs[j] + bias,
// with the token scales xs staged in shared memory.
template <typename T, int NP>
__device__ __forceinline__ void store_row(const uint64_t (&y)[NP], T* __restrict__ out, int N,
                                          const float* __restrict__ xs, float bias, int valid) {
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    if (2 * j < valid) {
      const float2 f = unpack2(y[j]);
      const float2 a = *reinterpret_cast<const float2*>(xs + 2 * j);
      out[(size_t)(2 * j) * N] = from_f32<T>(f.x * a.x + bias);
      if (2 * j + 1 < valid) out[(size_t)(2 * j + 1) * N] = from_f32<T>(f.y * a.y + bias);
    }
  }
}

// The same stores as store_row for bf16 output written through an NVLink
// multicast address (every GPU bound to the multicast object receives them;
// multimem stores are at least 32 bits wide): lanes 2i and 2i + 1 hold
// output columns n and n + 1; per token pair the even lane stores token 2j's
// two columns and the odd lane token 2j + 1's, after one exchange.  All lanes
// of the warp call it (ok: this lane's row is inside the layer).
template <int NP>
__device__ __forceinline__ void store_row_mc(const uint64_t (&y)[NP], __nv_bfloat16* out, int N,
                                             const float* __restrict__ xs, float bias, int valid, bool ok,
                                             int lane) {
  const bool odd = lane & 1;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float2 f = unpack2(y[j]);
    const float2 a = *reinterpret_cast<const float2*>(xs + 2 * j);
    const float v0 = f.x * a.x + bias, v1 = f.y * a.y + bias;   // tokens 2j, 2j + 1 of this column
    const float recv = __shfl_xor_sync(0xffffffffu, odd ? v0 : v1, 1);
    const int tok = 2 * j + (odd ? 1 : 0);
    const __nv_bfloat16 lo = __float2bfloat16_rn(odd ? recv : v0), hi = __float2bfloat16_rn(odd ? v1 : recv);
    const uint32_t w = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
    __nv_bfloat16* dst = out + (size_t)tok * N - (odd ? 1 : 0);
    if (ok && tok < valid)
      asm volatile("multimem.st.global.bf16x2 [%0], %1;" ::"l"(dst), "r"(w) : "memory");
  }
}

template <int BT>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                const __grid_constant__ CUtensorMap wmap, TcParams p) {
  using C = TcTile<BT>;
  constexpr int kStages = C::kStages, kBufs = C::kBufs, kTokHalf = C::kTokHalf;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);     // [stages] this CTA's loads landed
  uint64_t* ready = full + kStages;                                     // [stages] leader: both CTAs' stage expanded
  uint64_t* freed = ready + kStages;                                    // [stages] MMAs done with the stage
  uint64_t* acc_full = freed + kStages;                                 // [bufs] group's MMAs complete
  uint64_t* acc_empty = acc_full + kBufs;                               // [bufs] leader: both epilogues drained
  uint64_t* mma_done = acc_empty + kBufs;                               // [1] leader: every MMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the tensor maps' descriptors, fetched while the set-up runs
  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
  }
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int G = p.K / kGroup;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  // tile t: output rows (t % tiles_n) * 256 + rank * 128 .. (this CTA's
  // half), tokens (t / tiles_n) * 256 ..
  auto tile_n0 = [&](int t) { return (t % p.tiles_n) * (2 * kTcRows) + (int)rank * kTcRows; };
  auto tile_m0 = [&](int t) { return (int64_t)(t / p.tiles_n) * BT; };
  auto tile_nrec = [&](int n0) { return max(0, min(kTcRecs, (p.N - n0) / kRecRows)); };
  // work item w: tile w / splits, groups [gb, ge) of its K split
  auto item_groups = [&](int w, int& gb, int& ge) {
    gb = (w - (w / p.splits) * p.splits) * p.gper;
    ge = min(G, gb + p.gper);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 8);      // 4 expansion warps x 2 CTAs
      mbar_init(&freed[s], 1);
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 16); // 8 epilogue warps x 2 CTAs
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "n"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers initialised and tensor memory allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the next kernel on the stream may launch as SMs free up (it waits for
  // this grid's completion before reading what it writes)
  asm volatile("griddepcontrol.launch_dependents;");
  bool failed = false;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    if (warp == 0 && lane == 0) {
      // producer.  The weights do not depend on the previous kernel on the
      // stream (the launch may overlap it): the first stages' weight boxes
      // go out before griddepcontrol.wait, every activation box after it.
      uint32_t npre = 0;
      for (int w = pair; w < p.items && npre < (uint32_t)kStages; w += pairs) {
        int gb, ge;
        item_groups(w, gb, ge);
        const int n0 = tile_n0(w / p.splits);
        for (int g = gb; g < ge && npre < (uint32_t)kStages; ++g, ++npre) {
          // a box always delivers all its bytes (rows past the layer's end
          // read as zeros)
          mbar_arrive_expect_tx(&full[npre], (uint32_t)(C::kXBytes + kTcRecs * kRecBytes));
          tma_load_3d(smem + C::kOffW + npre * kTcWBytes, &wmap, 0, g, n0 / kRecRows, &full[npre]);
        }
      }
      grid_dep_wait();
      uint32_t it = 0;  // groups issued by this CTA so far
      for (int w = pair; w < p.items && !failed; w += pairs) {
        const int t = w / p.splits;
        int gb, ge;
        item_groups(w, gb, ge);
        const int n0 = tile_n0(t);
        const int ty = (int)(tile_m0(t) + rank * kTokHalf);
        const int xset = tc_set(p, (t % p.tiles_n) * (2 * kTcRows));
        for (int g = gb; g < ge; ++g, ++it) {
          const uint32_t s = it % kStages;
          if (it >= (uint32_t)kStages) {
            if (!mbar_wait(&freed[s], ((it / kStages) - 1) & 1)) {
              failed = true;
              break;
            }
            mbar_arrive_expect_tx(&full[s], (uint32_t)(C::kXBytes + kTcRecs * kRecBytes));
            tma_load_3d(smem + C::kOffW + s * kTcWBytes, &wmap, 0, g, n0 / kRecRows, &full[s]);
          }
          tma_load_3d(smem + C::kOffX + s * C::kXBytes, &xmap, g * kGroup, ty, xset, &full[s]);
        }
      }
    } else if (warp == 1 && lane == 0 && leader) {
      // MMA issuer (leader CTA only)
      const uint32_t w_base = smem_u32(smem + C::kOffW), x_base = smem_u32(smem + C::kOffX);
      uint32_t total = 0;
      for (int w = pair; w < p.items; w += pairs) {
        int gb, ge;
        item_groups(w, gb, ge);
        total += (uint32_t)(ge - gb);
      }
      for (uint32_t it = 0; it < total && !failed; ++it) {
        const uint32_t s = it % kStages, b = it % kBufs;
        if (!mbar_wait_cluster(&ready[s], (it / kStages) & 1) || !mbar_wait_cluster(&acc_empty[b], (it / kBufs) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(w_base + s * kTcWBytes);
        const uint64_t db = umma_desc_sw128(x_base + s * C::kXBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_i8_pair(tmem + b * BT, da + 2 * kk, db + 2 * kk, C::kIdesc, kk > 0 ? 1u : 0u);
        umma_commit_pair(&freed[s]);
        umma_commit_pair(&acc_full[b]);
      }
      // every MMA issued above completes before the pair frees its tensor memory
      umma_commit_pair(mma_done);
      mbar_wait(mma_done, 0);
    } else if (warp == 2 && blockIdx.x == 0 && p.zero_after) {
      grid_dep_wait();   // the previous kernel has read them
      for (int i = lane; i < p.zero_n; i += 32) p.zero_after[i] = 0u;
    }
  } else if (warp < 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 88;");
    // expansion: thread t writes weight row t of this CTA's half
    const int t = threadIdx.x - 128;
    const int i = t >> 4, r = t & 15;
    const int sw = t & 7;
    uint32_t it = 0;
    for (int w = pair; w < p.items && !failed; w += pairs) {
    const int nrec = tile_nrec(tile_n0(w / p.splits));
    int gb, ge;
    item_groups(w, gb, ge);
    for (int g = gb; g < ge; ++g, ++it) {
      const uint32_t s = it % kStages;
      if (!mbar_wait(&full[s], (it / kStages) & 1)) {
        failed = true;
        break;
      }
      uint8_t* area = smem + C::kOffW + s * kTcWBytes;
      uint32_t w[4][4];  // [t][j] code words of row t
      uint32_t zz = 0;
      if (i < nrec) {
        const uint8_t* rec = area + i * kRecBytes;
        zz = (uint32_t)rec[kRecZeroOff + r] * 0x01010101u;
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
          const uint4 v = *reinterpret_cast<const uint4*>(rec + r * 64 + tt * 16);
          w[tt][0] = v.x; w[tt][1] = v.y; w[tt][2] = v.z; w[tt][3] = v.w;
        }
      }
      named_barrier(1, 128);  // every record is read before any row is overwritten
      if (i < nrec) {
        uint8_t* row = area + t * 128;
        // 16-channel chunk c < 4 holds the low nibbles of words (t, c) for
        // t = 0..3; chunk c + 4 holds their high nibbles
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4*>(row + ((c ^ sw) << 4)) =
              make_uint4(expand_signed(w[0][c] & 0x0F0F0F0Fu, zz), expand_signed(w[1][c] & 0x0F0F0F0Fu, zz),
                         expand_signed(w[2][c] & 0x0F0F0F0Fu, zz), expand_signed(w[3][c] & 0x0F0F0F0Fu, zz));
          *reinterpret_cast<uint4*>(row + (((c + 4) ^ sw) << 4)) =
              make_uint4(expand_signed((w[0][c] >> 4) & 0x0F0F0F0Fu, zz),
                         expand_signed((w[1][c] >> 4) & 0x0F0F0F0Fu, zz),
                         expand_signed((w[2][c] >> 4) & 0x0F0F0F0Fu, zz),
                         expand_signed((w[3][c] >> 4) & 0x0F0F0F0Fu, zz));
        }
      }
      // rows past the layer's end are left as they are: their outputs are
      // never stored
      fence_proxy_async_smem();  // make the generic-proxy writes visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&ready[s], 0);
    }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 184;");
    // epilogue: warp w reads TMEM lanes 32*(w%4).. (output rows) and token
    // columns kCols*((w-8)/4)..
    constexpr int kCols = C::kCols, kNP = C::kPairs, kChunks = kCols / 16;
    const int q4 = warp & 3, half = (warp - 8) >> 2;
    const int row = q4 * 32 + lane;                       // output row within this CTA's half
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const int col0 = half * kCols;
    // every accumulator buffer starts free
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < kBufs; ++b) mbar_arrive_cluster(&acc_empty[b], 0);
    }
    grid_dep_wait();   // the token scales come from the previous kernel
    uint32_t it = 0;
    for (int w = pair; w < p.items && !failed; w += pairs) {
      const int tile = w / p.splits;
      int gb, ge;
      item_groups(w, gb, ge);
      const int n0 = tile_n0(tile);
      const int64_t m0 = tile_m0(tile);
      const bool row_ok = (row >> 4) < tile_nrec(n0);
      const uint16_t* sp = reinterpret_cast<const uint16_t*>(
          p.packed + rec_offset(n0 / kRecRows + (row_ok ? (row >> 4) : 0), 0, G) + kRecScaleOff) + (row & 15);
      // this row's scale of group g is sp[g * kRecBytes / 2]: its fp16 bits
      // are loaded three groups ahead and converted only where used, so the
      // load's latency never stalls the fold
      auto fetch_bits = [&](int g) -> uint32_t {
        return (row_ok && g < ge) ? ldg_nc_u16(sp + (size_t)g * (kRecBytes / 2)) : 0u;
      };
      uint32_t r0 = fetch_bits(gb), r1 = fetch_bits(gb + 1), r2 = fetch_bits(gb + 2);
      uint64_t y[kNP];
#pragma unroll
      for (int j = 0; j < kNP; ++j) y[j] = 0ull;  // (+0.0f, +0.0f)
      for (int g = gb; g < ge; ++g, ++it) {
        const uint32_t b = it % kBufs;
        const uint32_t r_after = fetch_bits(g + 3);
        if (!mbar_wait(&acc_full[b], (it / kBufs) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const float sc = half_bits_to_f32((uint16_t)r0);
        const uint64_t s2 = pack2(sc, sc);
        // chunk c + 1 is read from tensor memory while chunk c is folded
        const uint32_t tb = tmem + lane_base + b * BT + col0;
        uint32_t va[16], vb[16];
        if constexpr (kChunks == 2) {
          // 64-token tiles: both chunks in flight, one wait (a shorter
          // per-group latency chain: 5-10 % per launch at 64 tokens)
          tmem_ld16(tb, va);
          tmem_ld16(tb + 16, vb);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = fma2(s2, pack2((float)(int)va[2 * j], (float)(int)va[2 * j + 1]), y[j]);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            y[8 + j] = fma2(s2, pack2((float)(int)vb[2 * j], (float)(int)vb[2 * j + 1]), y[8 + j]);
        } else {
          // 256-token tiles: 32-column loads, one round trip each (four per
          // group instead of eight 16-column ones, whose serial latency paced
          // the fold: 2 % more throughput measured on configs[2])
#pragma unroll
          for (int c = 0; c < kChunks; c += 2) {
            uint32_t v[32];
            tmem_ld32(tb + c * 16, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j)
              y[c * 8 + j] = fma2(s2, pack2((float)(int)v[2 * j], (float)(int)v[2 * j + 1]), y[c * 8 + j]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(&acc_empty[b], 0);
        r0 = r1;
        r1 = r2;
        r2 = r_after;
      }
      // token scale, bias, convert, store: this thread holds output row
      // n0 + row for tokens m0 + col0 + (0..kCols-1); the tensor core is
      // already on the next tile.  The warp first stages its token scales in
      // its own slice of shared memory (kCols / 32 per lane).
      float* xs = reinterpret_cast<float*>(smem + C::kOffXs) + (warp - 8) * kCols;
      constexpr int kPerLane = kCols / 32;
#pragma unroll
      for (int q = 0; q < kPerLane; ++q) {
        const int64_t m = m0 + col0 + lane * kPerLane + q;
        xs[lane * kPerLane + q] =
            m < p.M ? ld_dep(p.xscale + tc_set(p, (tile % p.tiles_n) * (2 * kTcRows)) * p.M + m) : 0.f;
      }
      __syncwarp();
      const int n = n0 + row;
      const int64_t mbase = m0 + col0;
      const int valid = (int)(p.M - mbase < kCols ? (p.M - mbase > 0 ? p.M - mbase : 0) : kCols);
      if (p.out_mc) {
        // bf16 through the multicast address (no split-K in this mode)
        const float bn = row_ok ? tc_bias(p.bias, p.bias_dtype, n) : 0.f;
        store_row_mc(y, static_cast<__nv_bfloat16*>(p.out) + mbase * p.N + n, p.N, xs, bn, valid,
                     !failed && row_ok, lane);
      } else if (p.splits == 1) {
        if (!failed && row_ok) {
          const float bn = tc_bias(p.bias, p.bias_dtype, n);
          if (p.out_dtype == PARO_BF16)
            store_row(y, static_cast<__nv_bfloat16*>(p.out) + mbase * p.N + n, p.N, xs, bn, valid);
          else if (p.out_dtype == PARO_F16)
            store_row(y, static_cast<__half*>(p.out) + mbase * p.N + n, p.N, xs, bn, valid);
          else
            store_row(y, static_cast<float*>(p.out) + mbase * p.N + n, p.N, xs, bn, valid);
        }
      } else {
        // split-K: this split's partial sums are added into the workspace
        // as 64-bit fixed point (red_add_fx: integer addition makes the
        // total independent of the order the splits arrive in); the warp
        // that completes the (tile, CTA, warp) count acquires every split's
        // partial for its 32 rows x 128 tokens, stores the outputs and
        // returns the workspace and the counter to zero
        unsigned long long* wp = p.ws + (size_t)mbase * p.N + n;
        if (!failed && row_ok) {
#pragma unroll
          for (int j = 0; j < kNP; ++j) {
            const float2 f = unpack2(y[j]);
            if (2 * j < valid) red_add_fx(wp + (size_t)(2 * j) * p.N, f.x);
            if (2 * j + 1 < valid) red_add_fx(wp + (size_t)(2 * j + 1) * p.N, f.y);
          }
        }
        __syncwarp();
        uint32_t* c = p.cnt + ((size_t)tile * 2 + rank) * 8 + (warp - 8);
        int last = 0;
        if (lane == 0) {
          asm volatile("fence.acq_rel.gpu;" ::: "memory");
          last = atomicAdd(c, 1u) + 1u == (uint32_t)p.splits;
          if (last) asm volatile("fence.acq_rel.gpu;" ::: "memory");
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          if (!failed && row_ok) {
            const float bn = tc_bias(p.bias, p.bias_dtype, n);
            for (int j0 = 0; j0 < valid; j0 += 8) {
              float a[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = j0 + j < valid ? ld_cg_fx(wp + (size_t)(j0 + j) * p.N) : 0.f;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (j0 + j < valid) {
                  const size_t o = (size_t)(j0 + j) * p.N;
                  st_cg_u64(wp + o, 0ull);
                  const float v = a[j] * xs[j0 + j] + bn;
                  if (p.out_dtype == PARO_BF16) static_cast<__nv_bfloat16*>(p.out)[mbase * p.N + n + o] = __float2bfloat16_rn(v);
                  else if (p.out_dtype == PARO_F16) static_cast<__half*>(p.out)[mbase * p.N + n + o] = __float2half_rn(v);
                  else static_cast<float*>(p.out)[mbase * p.N + n + o] = v;
                }
            }
          }
          __syncwarp();
          if (lane == 0) *c = 0u;
        }
      }
      __syncwarp();  // the slice is rewritten for the next tile
    }
  }

  // multicast stores: ordered before whatever follows the kernel at system
  // scope (the caller's cross-rank barrier)
  if (p.out_mc && warp >= 8) __threadfence_system();
  // every role of both CTAs reaches this point; the pair's tensor memory is
  // freed once neither CTA reads it any more
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(C::kTmemCols) : "memory");
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int g_tc_sms = 0;

// The tensor-core kernel handles token counts above the decode range.
static int tc_sms() {
  if (g_tc_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_tc_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_tc_sms <= 1) g_tc_sms = 148;
  }
  return g_tc_sms;
}

static int tc_tiles(int64_t M, int N, int bt) {
  return (int)(((int64_t)N + 2 * kTcRows - 1) / (2 * kTcRows) * ((M + bt - 1) / bt));
}

// Split-K when the tiles fill fewer than all CTA pairs: each tile's groups
// are cut into up to pairs / tiles splits of at least 4 groups, so that
// small layers at mid-size token counts use the whole GPU.
static int tc_splits(int64_t M, int N, int K, int bt) {
  const int pairs = tc_sms() / 2, tiles = tc_tiles(M, N, bt), G = K / kGroup;
  if (tiles >= pairs || M > 0x7FFFFFFF) return 1;
  int s = min(pairs / tiles, G / 4);
  if (s <= 1) return 1;
  const int gper = (G + s - 1) / s;
  return (G + gper - 1) / gper;
}

// Tokens from which the tensor-core kernel (64-token tiles) beats the
// streaming decode kernel, measured per launch in CUDA graphs on B200 with
// weights beyond L2: long rows (down, K = 18944) from 13 tokens (23.6 us
// against 29.6 at 16 tokens, 22.2 against 18.6 at 8); layers with at least
// 0.8 x SMs 256-row tiles (gate_up: 148) from 17 (33.3 against 78.4 us at
// 24, 32.9 against 26.3 at 16); the rest (qkv, o) from 24 (13.6 against
// 13.9 us on qkv, 13.0 against 12.9 on o; 15.1 against 27.2 at 64).
static int tc_min_tokens(int N, int K) {
  if (K >= 8192) return 13;
  if ((int64_t)((N + 2 * kTcRows - 1) / (2 * kTcRows)) * 5 >= (int64_t)tc_sms() * 4) return 17;
  return 24;
}

int gemm_tc_supported(int64_t M, int N, int K) {
  if (N % kRecRows || K % kGroup || M <= 0) return 0;
  return M > 64 || M >= tc_min_tokens(N, K);
}

// Estimated duration (ns) of the kernel with bt-token tiles: waves of work
// items over the CTA pairs, each item's groups at a per-group cost, plus the
// split-K partial sums (64-bit atomic adds into [M][N], then a pass that
// reads them back).  Fitted to graph-timed launches on B200 (0.55 us per
// group of a 64-token tile, 1.0 us of a 256-token tile, whose per-group fold
// of 256 columns bounds it; ~0.75 ns per KB of partial sums); it ranks the
// two tiles within ~15 % of the measured times for qkv, o, gate_up and down
// at 96-256 tokens.
static double tc_estimate_ns(int64_t M, int N, int K, int bt) {
  const int pairs = tc_sms() / 2, G = K / kGroup;
  const int splits = tc_splits(M, N, K, bt);
  const int gper = (G + splits - 1) / splits;
  const int64_t items = (int64_t)tc_tiles(M, N, bt) * splits;
  const int64_t waves = (items + pairs - 1) / pairs;
  double ns = (double)waves * gper * (bt == 64 ? 550.0 : 1000.0);
  if (splits > 1) ns += (double)M * N * 8.0 * splits * 0.00075;
  return ns;
}

// Tokens per tile: 64 up to 64 tokens (a 256-token tile spends most of each
// MMA and of the per-group fold on padding: gate_up at 64 tokens 34 us
// against 55), beyond that the tile the estimate prefers (small layers keep
// 64-token tiles to a few hundred tokens: qkv at 256 tokens 18.9 us against
// 34.9), and 256 from 2048 tokens.
int gemm_tc_tile(int64_t M, int N, int K) {
  if (M <= 64) return 64;
  if (M >= 2048) return 256;
  return tc_estimate_ns(M, N, K, 64) < tc_estimate_ns(M, N, K, 256) ? 64 : 256;
}

static size_t al256_tc(size_t b) { return (b + 255) & ~(size_t)255; }

// Workspace of the kernel with bt-token tiles (0: the tile gemm_tc_tile picks).
size_t gemm_tc_workspace_tile(int64_t M, int N, int K, int bt) {
  if (bt == 0) bt = gemm_tc_tile(M, N, K);
  if (tc_splits(M, N, K, bt) == 1) return 0;
  return al256_tc((size_t)M * N * sizeof(unsigned long long)) + (size_t)tc_tiles(M, N, bt) * 16 * sizeof(uint32_t);
}

size_t gemm_tc_workspace(int64_t M, int N, int K) { return gemm_tc_workspace_tile(M, N, K, 0); }

// Whether T activation sets with these row-block starts can share one
// launch: every table starts on a 256-row tile.
int gemm_tc_sets_ok(int T, const int* tab_nb) {
  if (T < 1 || T > kMaxTables || tab_nb[0] != 0) return 0;
  for (int t = 1; t < T; ++t)
    if ((tab_nb[t] * kRecRows) % (2 * kTcRows) || tab_nb[t] <= tab_nb[t - 1]) return 0;
  return 1;
}

// workspace: gemm_tc_workspace_tile(M, N, K, bt) bytes, zero-filled and
// left so, or NULL (then no split-K).  T activation sets: xq is [T][M][K],
// xscale [T][M], rows from 16 * tab_nb[t] on read set t (gemm_tc_sets_ok).
// bt: tokens per tile, 64 or 256 (0: gemm_tc_tile's choice).
cudaError_t launch_gemm_tc_tile(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, int bt, cudaStream_t st,
                                uint32_t* zero_after, int zero_n, int out_mc) {
  auto encode = get_encode();
  if (!encode) return cudaErrorNotSupported;
  if (bt == 0) bt = gemm_tc_tile(M, N, K);
  if (M > 0x7FFFFFFF || !gemm_tc_sets_ok(T, tab_nb) || (bt != 64 && bt != 256)) return cudaErrorInvalidValue;
  CUtensorMap xmap;
  const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)M, (cuuint64_t)T};
  const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)M * K};
  const cuuint32_t box[3] = {(cuuint32_t)kGroup, (cuuint32_t)(bt / 2), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t*>(xq), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // tile records as a [N/16][G][134 x 8 bytes] tensor; one box = the 8
  // records of one group for 8 consecutive 16-row blocks
  CUtensorMap wmap;
  const int G = K / kGroup;
  const cuuint64_t wdims[3] = {(cuuint64_t)(kRecBytes / 8), (cuuint64_t)G, (cuuint64_t)(N / kRecRows)};
  const cuuint64_t wstrides[2] = {(cuuint64_t)kRecBytes, (cuuint64_t)G * kRecBytes};
  const cuuint32_t wbox[3] = {(cuuint32_t)(kRecBytes / 8), 1, (cuuint32_t)kTcRecs};
  const cuuint32_t westr[3] = {1, 1, 1};
  r = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(packed), wdims, wstrides, wbox, westr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  TcParams p;
  p.xscale = xscale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.packed = static_cast<const uint8_t*>(packed);
  p.bias = bias;
  p.bias_dtype = bias_dtype;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ws = nullptr;
  p.cnt = nullptr;
  p.splits = 1;
  p.tables = T;
  for (int t = 0; t < kMaxTables; ++t) p.tab_nb[t] = t < T ? tab_nb[t] : 0;
  p.zero_after = zero_n > 0 ? zero_after : nullptr;
  p.zero_n = zero_n > 0 ? zero_n : 0;
  p.out_mc = out_mc ? 1 : 0;
  if (out_mc && out_dtype != PARO_BF16) return cudaErrorInvalidValue;
  const size_t wsb = gemm_tc_workspace_tile(M, N, K, bt);
  if (wsb && workspace && workspace_bytes >= wsb && !out_mc) {
    p.splits = tc_splits(M, N, K, bt);
    p.ws = static_cast<unsigned long long*>(workspace);
    p.cnt = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) +
                                        al256_tc((size_t)M * N * sizeof(unsigned long long)));
  }
  p.gper = (G + p.splits - 1) / p.splits;
  const void* fn = bt == 64 ? (const void*)gemm_tc_kernel<64> : (const void*)gemm_tc_kernel<256>;
  const int smem = bt == 64 ? TcTile<64>::kSmem : TcTile<256>::kSmem;
  cudaError_t e = ensure_smem_limit(fn, smem);
  if (e != cudaSuccess) return e;
  p.tiles_n = (N + 2 * kTcRows - 1) / (2 * kTcRows);
  const int64_t tiles = (int64_t)p.tiles_n * ((M + bt - 1) / bt);
  if (tiles > 0x7FFFFFFF) return cudaErrorInvalidValue;
  p.tiles = (int)tiles;
  p.items = p.tiles * p.splits;
  tc_sms();
  const int pairs = (int)(p.items < g_tc_sms / 2 ? p.items : g_tc_sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch: setup and the first weight boxes overlap
  // the previous kernel
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (bt == 64) return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<64>, xmap, wmap, p);
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<256>, xmap, wmap, p);
}

cudaError_t launch_gemm_tc_sets(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, cudaStream_t st) {
  return launch_gemm_tc_tile(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                             workspace_bytes, T, tab_nb, 0, st, nullptr, 0, 0);
}

cudaError_t launch_gemm_tc(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                           const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                           size_t workspace_bytes, cudaStream_t st) {
  const int nb0 = 0;
  return launch_gemm_tc_tile(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                             workspace_bytes, 1, &nb0, 0, st, nullptr, 0, 0);
}

}  // namespace paro
