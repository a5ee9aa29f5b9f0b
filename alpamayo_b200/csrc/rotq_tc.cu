// rotq_tc.cu — the rotation pass of the prefill activation path on the
// tensor cores (tcgen05 kind::f16, fp32 accumulators in tensor memory),
// sm_100a, for bf16 activations.
//
// The eight Givens layers of a 128-channel group, with the channel scales in
// front, are one linear map: y_g = R_g (s_g ⊙ x_g), R_g a 128 x 128
// orthogonal matrix.  Applied layer by layer (rotq_rows.cu) every layer moves
// every value through shared memory, and that exchange bounds the pass; here
// each CTA builds R'_g = R_g diag(s_g) once, and the tensor core applies it to
// 128-row tiles: Y[rows, 128] = X[rows, 128] R'_g^T.
//
//  * Build (256 threads, once per group): thread (half h, row n) carries
//    component n of the 64 unit vectors e_k, k in half h, through the eight
//    layers (the activation kernels' arithmetic: both products and the sum
//    rounded separately, angles from __sincosf), exchanging with the
//    partner's thread through shared memory once per layer; column k is
//    then scaled by s_k.  R' is split into bf16 hi + lo (hi = bf16(R'), lo =
//    bf16(R' - hi)) and written in the UMMA K-major 128-byte-swizzle layout.
//    The first tiles' loads are issued before it.  A table that carries
//    the matrices (paro_prepare_rotation_matrices: the same build, once per
//    group at load time) skips the eight layers: each thread loads its 64
//    entries of R_g and only scales and splits them (bit-identical).
//  * Producer thread: tensor TMA of the 128-row x 128-channel bf16 tile
//    (two 64-channel boxes, 128-byte swizzle), 3 stages.
//  * MMA thread: 8 MMAs (M = 128 rows, N = 128 channels, K = 16) with R'_hi,
//    then 8 with R'_lo, into a 128-column TMEM buffer (two buffers; four in
//    the single-pass mode).  x is exact in bf16, so Y = X hi^T + X lo^T
//    carries R' to about 2^-16 relative: far below the fp16 spacing the
//    result is rounded to.
//  * Two-pass mode (rot_tc_kernel<false>; 8 epilogue warps, TMEM lanes =
//    rows, two warps per lane quarter): each thread reads 64 of its row's
//    128 outputs, rounds them to fp16 — the value the reference's rotate
//    kernel stores (rotation.cuh:333-334) — stores them, and folds their
//    |max| into the row's maximum (atomicMax on the bit pattern).
//    quant_rows_kernel then quantises per token (rotq_rows.cu).
//  * Single-pass mode (rot_tc_kernel<true>, where every group's CTA fits the
//    GPU at once): the kernel quantises its own tiles once every group's
//    maximum of a row tile is in (described above rt_epilogue_quant), so
//    the fp16 rows never leave the SM; same codes bit for bit.
//
// A CTA owns one group and a contiguous range of its row tiles (groups are
// spread over the grid first).  Waits are bounded (kErrMbarTimeout,
// kErrGridWait), tensor memory is freed on every exit.  No load uses
// cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "tc_ptx.cuh"

namespace paro {

PARO_DEFINE_ERROR_ACCESSOR(rtc)

namespace {

constexpr int kRtThreads = 384;   // producer, MMA, 2 idle, 8 epilogue warps
constexpr int kRtStages = 3;
// tiles whose loads go out before R' is in shared memory: the first MMA
// needs R' and one tile, and every CTA starts at once, so the others would
// only compete with the matrix loads for DRAM
constexpr int kRtEarly = 1;
constexpr int kRtRows = 128;                     // rows per tile (MMA M)
constexpr int kRtTileBytes = kRtRows * 128 * 2;  // 32 KB bf16 tile
constexpr int kRtRBytes = 128 * 128 * 2;         // one bf16 128 x 128 matrix
// bit 15 of table word 0 (never set by the table builder): the table carries
// each group's rotation matrix after its 8 x K words
constexpr uint32_t kRotMatricesFlag = 0x8000u;
// shared memory plan (from a 1024-byte aligned base)
constexpr int kOffRhi = 0;
constexpr int kOffRlo = kOffRhi + kRtRBytes;
constexpr int kOffX = kOffRlo + kRtRBytes;
constexpr int kOffEx = kOffX + kRtStages * kRtTileBytes;   // build: [2 halves][32 cols][128 rows] f32 exchange;
                                                            // epilogue: the fp16 output tile (32 KB)
constexpr int kOffTab = kOffEx + 2 * 32 * 128 * 4;          // [8 layers][128] table words
constexpr int kOffBar = kOffTab + 8 * 128 * 4;
constexpr int kOffQ8 = kOffBar + 1024;          // single-pass mode: the int8 tile (16 KB, 1024-aligned)
constexpr int kRtSmem = kOffQ8 + 16384 + 1024;

// kind::f16 instruction descriptor: f32 accumulate, A and B bf16, both
// K-major, N = 128, M = 128
constexpr uint32_t kRtIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kRtIdesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// byte offset of element (row n, column k) of a 128 x 128 bf16 K-major
// matrix in the 128-byte-swizzle layout: two 16 KB halves along k, 8-row
// atoms of 1024 bytes, 16-byte chunks XOR-swizzled by the row within the atom
__device__ __forceinline__ uint32_t sw128_off(int n, int k) {
  const int h = k >> 6, c = (k >> 3) & 7, e = k & 7;
  return (uint32_t)(h * 16384 + (n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4) + e * 2);
}

// Component n of R_g e_k for the 32 columns k = k0 .. k0 + 31, by thread n
// of a 128-thread half h (named barrier 1 + h): v[j] starts as e_{k0+j}[n]
// and goes through the eight layers, exchanging with the partner's thread
// through ex ([32 columns][128 rows] f32) once per layer.  The rotation
// kernel's own build and the load-time kernel below both run this function,
// so a matrix built ahead of time is bit-identical to one built in place.
__device__ __forceinline__ void rt_build_columns(const uint32_t* tab, float* ex, int h, int n, int k0,
                                                 float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = (n == k0 + j) ? 1.f : 0.f;
#pragma unroll 1
  for (int l = 0; l < 8; ++l) {
    const uint32_t w = tab[l * 128 + n];
    const int partner = (int)(w & 0x7F);
    // exchange slots from the table (bits 8-14): every warp's 32 writes
    // and 32 reads fall in 32 different banks
    const int s_me = (int)((w >> 8) & 0x7F), s_pt = (int)((tab[l * 128 + partner] >> 8) & 0x7F);
    float s_, c_;
    __sincosf(half_bits_to_f32((uint16_t)(w >> 16)), &s_, &c_);
    const float cp = ((w >> 7) & 1) ? -s_ : s_;
#pragma unroll
    for (int j = 0; j < 32; ++j) ex[j * 128 + s_me] = v[j];
    named_barrier(1 + h, 128);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = givens(v[j], ex[j * 128 + s_pt], c_, cp);
    named_barrier(1 + h, 128);
  }
}

// Row n, columns k .. k + 7 of R'_g = R_g diag(s_g) from the unscaled r[0..7]:
// scaled in f32, split into bf16 hi = bf16(R'), lo = bf16(R' - hi), written
// at their places in the two swizzled matrices.
__device__ __forceinline__ void rt_store_split(uint8_t* smem, const uint16_t* scales, int g, int n, int k,
                                               const float* r) {
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float a[2];
#pragma unroll
    for (int e = 0; e < 2; ++e)
      a[e] = r[2 * q + e] * (scales ? half_bits_to_f32(scales[g * 128 + k + 2 * q + e]) : 1.f);
    const __nv_bfloat162 bh = __floats2bfloat162_rn(a[0], a[1]);
    const float2 fh = __bfloat1622float2(bh);
    const __nv_bfloat162 bl = __floats2bfloat162_rn(a[0] - fh.x, a[1] - fh.y);
    hi[q] = *reinterpret_cast<const uint32_t*>(&bh);
    lo[q] = *reinterpret_cast<const uint32_t*>(&bl);
  }
  const uint32_t off = sw128_off(n, k);
  *reinterpret_cast<uint4*>(smem + kOffRhi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  *reinterpret_cast<uint4*>(smem + kOffRlo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

}  // namespace

struct RtParams {
  int64_t M;
  int K, G;
  int tiles;        // row tiles of 128
  int splits;       // CTAs per group
  const uint16_t* scales;  // fp16 [K] or null
  const uint32_t* rtab;    // [8, K]
  __half* y;               // [M, K] fp16 out (two-pass mode)
  uint32_t* amax;          // [M] row |max| bits (zero on entry)
  // single-pass mode (quantiser fused): int8 codes, per-token scales, and a
  // counter per row tile of the groups whose maxima are in (zero on entry)
  int8_t* q;               // [M, K]
  float* qscale;           // [M]
  uint32_t* cnt;           // [tiles]
};

// Round half away from zero, for |v| <= 255, as the low byte of the two's
// complement integer, with float adds instead of conversions:
//   s = |v| + 0.5 rounded toward zero lies in [floor(|v| + 0.5), |v| + 0.5]
//     (the floor is an integer, representable, and rounding toward zero
//     never passes it), so floor(s) = floor(|v| + 0.5) = round_half_away(|v|);
//   m = s + 1.5·2^23 rounded toward zero lands in [2^23, 2^24), where the
//     float32 spacing is 1, so m = 1.5·2^23 + floor(s) and the low byte of
//     its bit pattern (0x4B400000 + n) is n;
//   the sign is applied by negating the pattern for negative v (the low
//   byte of -(0x4B400000 + n) is that of -n).
// Equal to (int8) roundf(v) for every such v (the single-pass and
// two-pass quantisers are tested bit-identical, ties included).
__device__ __forceinline__ uint32_t round_half_away_byte(float v) {
  const float s = __fadd_rz(fabsf(v), 0.5f);
  const uint32_t m = __float_as_uint(__fadd_rz(s, 12582912.0f));
  const uint32_t sg = (uint32_t)(__float_as_int(v) >> 31);
  return (m ^ sg) - sg;
}

// Single-pass mode: 16 epilogue warps (warps 2-17), four per TMEM lane
// quarter, thread = row r of the tile and columns 32·j .. 32·j + 31 of group
// g (j = the warp's column slice); a signalling warp (18) and a waiting warp
// (19).  Four TMEM accumulators, so a tile's values stay in tensor memory
// until its codes are written.  Per tile i:
//   epilogue A(i): the row's |max| over the 128 columns (the four slices'
//     maxima combined in shared memory), fp16-rounded, folded into amax
//     (atomicMax on the bit patterns); the combining warps arrive on
//     `maxed`.
//   signalling warp: after `maxed`, one release increment of cnt[tile] for
//     the CTA.
//   waiting warp: once cnt[tile] shows every group of the row range in, the
//     final row maxima are read, 127/a goes to shared memory (and, in group
//     0's CTAs, the per-token scale a/127 to memory); then `amax_ready`.
//   epilogue B(i-2), after A(i): the codes of tile i-2 from its accumulator
//     (fp16-rounded again) and 127/a, staged as an int8 tile (128-byte
//     swizzle) and written by a tensor TMA store; the accumulator is freed.
// The other groups' CTAs run the same tiles at the same pace, so a tile's
// count is complete well before its codes are due and the epilogue never
// waits on memory.  Every CTA counts itself in for a tile before it waits
// for any later one's count, A(k) precedes B(k-2), and all CTAs are
// co-resident (cooperative launch), so the waits always end; each is still
// bounded (kErrMbarTimeout, kErrGridWait), and after a failure the warps
// only pass the barriers.  The quantiser's arithmetic is
// quant_rows_kernel's: a = max(|max|, 1e-10), q = round_half_away(y ·
// 127/a), scale a/127.
constexpr int kRtQuantThreads = 640;   // producer, MMA, 16 epilogue warps, signalling and waiting warps
constexpr int kRtQuantEpi = 512;
constexpr int kRtSignalWarp = 18;
constexpr int kRtWaitWarp = 19;
constexpr int kRtDefer = 2;            // tiles between a tile's maxima and its codes

struct RtQuantBars {
  uint64_t* maxed;        // [4] tile's maxima issued (4 combining warps)
  uint64_t* amax_ready;   // [4] 127/a of the tile in shared memory (waiting warp)
  uint64_t* amax_free;    // [4] the epilogue has read it (16 warps)
};

struct RtQuantCtx {
  const RtParams* p;
  const CUtensorMap* qmap;
  uint8_t* q8;          // the int8 tile being stored (128 rows x 128 B, 128-byte swizzle)
  uint32_t* pm;         // [4 slices][128 rows] row maxima
  const float* inv;     // [4][128] 127/a per row
  RtQuantBars bars;
  uint64_t* acc_full;
  uint64_t* acc_empty;
  volatile uint32_t* wait_failed;
  uint32_t tmem, lane_base;
  int g, tb, ntile, r, j, lane;
  bool issuer;
};

__device__ __forceinline__ void rtq_step(const RtQuantCtx& c, int i, bool& failed) {
  const RtParams& p = *c.p;
  if (i < c.ntile) {
    const int b = i & 3;
    if (!failed && !mbar_wait(&c.acc_full[b], (i >> 2) & 1)) failed = true;
    uint32_t v[32];
    if (!failed) {
      fence_after();
      tmem_ld32(c.tmem + c.lane_base + (uint32_t)(b * 128 + c.j * 32), v);
      tmem_wait_ld();
    }
    // the |max| of the fp16-rounded values is the fp16 rounding of the
    // float32 |max| (rounding is monotonic and symmetric); as float32 bits
    // (non-negative floats order as unsigned integers)
    float mx = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) mx = fmaxf(mx, fabsf(__uint_as_float(v[k])));
    c.pm[c.j * 128 + c.r] = __float_as_uint(__half2float(__float2half_rn(mx)));
    // the int8 tile's previous store has read it before B below writes it
    if (c.issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    named_barrier(3, kRtQuantEpi);
    if (c.j == 0) {
      const uint32_t m = max(max(c.pm[c.r], c.pm[128 + c.r]), max(c.pm[256 + c.r], c.pm[384 + c.r]));
      const int64_t row = (int64_t)(c.tb + i) * kRtRows + c.r;
      if (!failed && row < p.M && m) atomicMax(p.amax + row, m);
      __syncwarp();
      if (c.lane == 0) mbar_arrive(&c.bars.maxed[b]);   // also after a failure
    }
  }
  const int d = i - kRtDefer;
  if (d >= 0 && d < c.ntile) {
    const int tp = c.tb + d, b = d & 3;
    if (!failed && !mbar_wait(&c.bars.amax_ready[b], (d >> 2) & 1)) failed = true;
    if (*c.wait_failed) failed = true;
    const float inv = c.inv[b * 128 + c.r];
    uint32_t v[32];
    if (!failed) {
      tmem_ld32(c.tmem + c.lane_base + (uint32_t)(b * 128 + c.j * 32), v);
      tmem_wait_ld();
    }
    fence_before();
    __syncwarp();
    if (c.lane == 0) {
      mbar_arrive(&c.bars.amax_free[b]);
      if (!failed) mbar_arrive(&c.acc_empty[b]);   // the MMA may reuse the accumulator
    }
    // after the last tile no A phase has waited for the int8 tile's previous
    // store to read it
    if (i >= c.ntile) {
      if (c.issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      named_barrier(3, kRtQuantEpi);
    }
    const int64_t row = (int64_t)tp * kRtRows + c.r;
    if (!failed && row < p.M) {
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float2 f0 = __half22float2(__floats2half2_rn(__uint_as_float(v[4 * k]), __uint_as_float(v[4 * k + 1])));
        const float2 f1 =
            __half22float2(__floats2half2_rn(__uint_as_float(v[4 * k + 2]), __uint_as_float(v[4 * k + 3])));
        const uint32_t q0 = round_half_away_byte(__fmul_rn(f0.x, inv)), q1 = round_half_away_byte(__fmul_rn(f0.y, inv));
        const uint32_t q2 = round_half_away_byte(__fmul_rn(f1.x, inv)), q3 = round_half_away_byte(__fmul_rn(f1.y, inv));
        w[k] = __byte_perm(__byte_perm(q0, q1, 0x0040), __byte_perm(q2, q3, 0x0040), 0x5410);
      }
      // row r's 32 bytes at chunks 2j, 2j + 1, swizzled by the row
      uint8_t* srow = c.q8 + c.r * 128;
      *reinterpret_cast<uint4*>(srow + (((2 * c.j) ^ (c.r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4*>(srow + (((2 * c.j + 1) ^ (c.r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    }
    fence_proxy_async_smem();
    named_barrier(3, kRtQuantEpi);
    // rows past M are clipped by the tensor map
    if (c.issuer && !failed) {
      asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(c.qmap),
                   "r"(c.g * 128), "r"(tp * kRtRows), "r"(smem_u32(c.q8))
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
}

__device__ __forceinline__ void rt_epilogue_quant(const RtQuantCtx& c0, int warp, int lane, bool& failed) {
  RtQuantCtx c = c0;
  const int qd = warp & 3;
  c.lane_base = (uint32_t)(qd * 32) << 16;
  c.r = qd * 32 + lane;
  c.j = (warp - 2) >> 2;
  c.lane = lane;
  c.issuer = warp == 2 && lane == 0;
  for (int i = 0; i < c.ntile + kRtDefer; ++i) rtq_step(c, i, failed);
  if (c.issuer) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// The signalling warp: counts the CTA in for each tile once the tile's
// maxima are issued (the mbarrier orders them before the release).
__device__ __forceinline__ void rt_signal_warp(const RtQuantCtx& c, int lane, bool& failed) {
  const RtParams& p = *c.p;
  for (int i = 0; i < c.ntile; ++i) {
    if (!failed && !mbar_wait(&c.bars.maxed[i & 3], (i >> 2) & 1)) failed = true;
    // counted in even after a failure, so the other CTAs do not wait for it
    if (lane == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.cnt + c.tb + i) : "memory");
  }
}

// The waiting warp: for each tile, waits for the count to complete and
// publishes 127/a of its rows in shared memory.
__device__ __forceinline__ void rt_wait_warp(const RtQuantCtx& c, float* inv, int lane, bool& failed) {
  const RtParams& p = *c.p;
  for (int i = 0; i < c.ntile; ++i) {
    const int b = i & 3, t = c.tb + i;
    if (lane == 0 && !*c.wait_failed) {
      const long long t0 = clock64();
      for (;;) {
        uint32_t n;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(n) : "l"(p.cnt + t) : "memory");
        if (n >= (uint32_t)p.G) break;
        if (clock64() - t0 > 1000000000LL) {
          report_error(kErrGridWait);
          *c.wait_failed = 1u;
          break;
        }
        __nanosleep(32);
      }
    }
    __syncwarp();
    // the epilogue has read this slot's previous values (tile i-4)
    if (!failed && !mbar_wait(&c.bars.amax_free[b], ((i >> 2) & 1) ^ 1)) failed = true;
    if (!failed && !*c.wait_failed) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int rr = lane * 4 + k;
        const int64_t row = (int64_t)t * kRtRows + rr;
        if (row < p.M) {
          uint32_t m;
          asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(m) : "l"(p.amax + row) : "memory");
          const float a = fmaxf(__uint_as_float(m), 1e-10f);
          inv[b * 128 + rr] = __fdiv_rn(127.0f, a);
          if (c.g == 0) p.qscale[row] = __fdiv_rn(a, 127.0f);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&c.bars.amax_ready[b]);
  }
}

template <bool kQuant>
__global__ void __launch_bounds__(kQuant ? kRtQuantThreads : kRtThreads, 1) rot_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                               const __grid_constant__ CUtensorMap ymap,
                                                               const __grid_constant__ CUtensorMap qmap, RtParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);   // [3] tile landed
  uint64_t* freed = full + kRtStages;                               // [3] MMAs done with the tile
  constexpr int kBufs = kQuant ? 4 : 2;                             // TMEM accumulators of 128 columns
  uint64_t* acc_full = freed + kRtStages;                           // [kBufs]
  uint64_t* acc_empty = acc_full + kBufs;                           // [kBufs] the epilogue warps
  uint64_t* mma_done = acc_empty + kBufs;                           // [1]
  uint64_t* qbars = mma_done + 1;                                   // [12] single-pass mode
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qbars + 12);
  volatile uint32_t* wait_failed = tmem_slot + 1;   // single-pass mode: a tile count wait gave up

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = threadIdx.x;
  // the tensor maps' descriptors, fetched while the set-up runs (the first
  // copies would otherwise wait for them)
  if (t == 256) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(kQuant ? &qmap : &ymap) : "memory");
  }
  // this CTA's group and row tiles
  const int part = blockIdx.x / p.G;
  const int g = blockIdx.x - part * p.G;
  const int tb = (int)((int64_t)part * p.tiles / p.splits);
  const int te = (int)((int64_t)(part + 1) * p.tiles / p.splits);
  const int ntile = te - tb;

  if (t == 0) {
    for (int s = 0; s < kRtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&freed[s], 1);
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kQuant ? 16 : 8);   // the epilogue warps
    }
    mbar_init(mma_done, 1);
    if (kQuant) {
      for (int b = 0; b < 4; ++b) {
        mbar_init(&qbars[b], 4);       // maxed: the four combining warps
        mbar_init(&qbars[4 + b], 1);   // amax_ready: the waiting warp
        mbar_init(&qbars[8 + b], 16);  // amax_free: the epilogue warps
      }
    }
    *wait_failed = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kBufs * 128)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // R_g prebuilt at load time (flag in word 0, 16-byte aligned trailer), or
  // the group's table words for the build
  const bool prebuilt =
      (__ldg(p.rtab) & kRotMatricesFlag) != 0 && (reinterpret_cast<uintptr_t>(p.rtab) & 15) == 0;
  uint32_t* tab = reinterpret_cast<uint32_t*>(smem + kOffTab);
  if (!prebuilt)
    for (int i = t; i < 8 * 128; i += (int)blockDim.x) tab[i] = __ldg(p.rtab + (size_t)(i >> 7) * p.K + g * 128 + (i & 127));
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  // the first tile's load goes out before the build, from a thread that
  // takes no part in it
  if (t == 256) {
    for (int i = 0; i < kRtEarly && i < ntile; ++i) {
      mbar_arrive_expect_tx(&full[i], kRtTileBytes);
      const int y0 = (tb + i) * kRtRows;
      tma_load_2d(smem + kOffX + i * kRtTileBytes, &xmap, g * 128, y0, &full[i]);
      tma_load_2d(smem + kOffX + i * kRtTileBytes + 16384, &xmap, g * 128 + 64, y0, &full[i]);
    }
  }

  // ---- R'_g = R_g diag(s_g), split into bf16 hi + lo ---------------------
  if (t < 256) {
    const int h = t >> 7, n = t & 127;   // half h: columns k = 64h .. 64h + 63
    if (prebuilt) {
      // R_g from the table's trailer: row n's 64 columns of half h, eight
      // chunks of 8 (each warp's 32 rows are 1 KB contiguous per chunk)
      const float4* src = reinterpret_cast<const float4*>(p.rtab + (size_t)8 * p.K) + (size_t)g * 4096;
      float r[64];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const size_t i = ((size_t)(8 * h + q) * 128 + n) * 2;
        const float4 u0 = __ldg(src + i), u1 = __ldg(src + i + 1);
        r[8 * q + 0] = u0.x; r[8 * q + 1] = u0.y; r[8 * q + 2] = u0.z; r[8 * q + 3] = u0.w;
        r[8 * q + 4] = u1.x; r[8 * q + 5] = u1.y; r[8 * q + 6] = u1.z; r[8 * q + 7] = u1.w;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) rt_store_split(smem, p.scales, g, n, 64 * h + 8 * q, &r[8 * q]);
    } else {
      float* ex = reinterpret_cast<float*>(smem + kOffEx) + h * (32 * 128);   // [32 cols][128 rows]
      for (int c0 = 0; c0 < 64; c0 += 32) {
        float v[32];
        rt_build_columns(tab, ex, h, n, 64 * h + c0, v);
#pragma unroll
        for (int j = 0; j < 32; j += 8) rt_store_split(smem, p.scales, g, n, 64 * h + c0 + j, &v[j]);
      }
    }
  }
  fence_proxy_async_smem();   // generic-proxy writes of R' -> visible to the tensor core
  __syncthreads();

  bool failed = false;
  if (warp == 0) {
    if (lane == 0) {
      // producer: tiles kRtEarly.. of this CTA's range
      for (int i = kRtEarly; i < ntile; ++i) {
        const int s = i % kRtStages;
        if (i >= kRtStages && !mbar_wait(&freed[s], ((i / kRtStages) - 1) & 1)) break;
        mbar_arrive_expect_tx(&full[s], kRtTileBytes);
        const int y0 = (tb + i) * kRtRows;
        tma_load_2d(smem + kOffX + s * kRtTileBytes, &xmap, g * 128, y0, &full[s]);
        tma_load_2d(smem + kOffX + s * kRtTileBytes + 16384, &xmap, g * 128 + 64, y0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t x_base = smem_u32(smem + kOffX);
      const uint32_t rh = smem_u32(smem + kOffRhi), rl = smem_u32(smem + kOffRlo);
      for (int i = 0; i < ntile; ++i) {
        const int s = i % kRtStages, b = i % kBufs;
        if (!mbar_wait(&full[s], (i / kRtStages) & 1) || !mbar_wait(&acc_empty[b], ((i / kBufs) & 1) ^ 1)) break;
        fence_after();
        const uint32_t d = tmem + (uint32_t)(b * 128);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t koff = (uint32_t)((ks >> 2) * 16384 + (ks & 3) * 32);
          mma_bf16(d, desc_sw128(x_base + s * kRtTileBytes + koff), desc_sw128(rh + koff), ks > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t koff = (uint32_t)((ks >> 2) * 16384 + (ks & 3) * 32);
          mma_bf16(d, desc_sw128(x_base + s * kRtTileBytes + koff), desc_sw128(rl + koff), 1u);
        }
        umma_commit(&freed[s]);
        umma_commit(&acc_full[b]);
      }
      umma_commit(mma_done);
      mbar_wait(mma_done, 0);
    }
  } else if (kQuant) {
    // (the table area is free once R' is built: row maxima and 127/a)
    RtQuantCtx c;
    c.p = &p;
    c.qmap = &qmap;
    c.q8 = smem + kOffQ8;
    c.pm = reinterpret_cast<uint32_t*>(smem + kOffTab);
    float* inv = reinterpret_cast<float*>(smem + kOffTab + 2048);
    c.inv = inv;
    c.bars.maxed = qbars;
    c.bars.amax_ready = qbars + 4;
    c.bars.amax_free = qbars + 8;
    c.acc_full = acc_full;
    c.acc_empty = acc_empty;
    c.wait_failed = wait_failed;
    c.tmem = tmem;
    c.g = g;
    c.tb = tb;
    c.ntile = ntile;
    if (warp == kRtSignalWarp)
      rt_signal_warp(c, lane, failed);
    else if (warp == kRtWaitWarp)
      rt_wait_warp(c, inv, lane, failed);
    else
      rt_epilogue_quant(c, warp, lane, failed);
  } else if (warp >= 4) {
    // epilogue: thread = row within the tile (TMEM lane), warps 4-7 take
    // channels 0-63, warps 8-11 channels 64-127.  The fp16 tile is staged in
    // shared memory (the build's exchange area, 128-byte swizzle) and written
    // by two tensor TMA stores, so each row's 256 bytes leave as whole lines.
    const int q4 = warp & 3, chh = (warp - 4) >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    const bool issuer = warp == 4 && lane == 0;
    uint8_t* stage_out = smem + kOffEx;
    // every epilogue thread passes both named barriers of every tile, also
    // after a timed-out wait (then it only skips the work)
    for (int i = 0; i < ntile; ++i) {
      const int b = i & 1;
      if (!failed && !mbar_wait(&acc_full[b], (i >> 1) & 1)) failed = true;
      uint32_t v[64];
      if (!failed) {
        fence_after();
        tmem_ld32(tmem + lane_base + (uint32_t)(b * 128 + chh * 64), *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tmem + lane_base + (uint32_t)(b * 128 + chh * 64 + 32),
                  *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        fence_before();
      }
      __syncwarp();
      if (!failed && lane == 0) mbar_arrive(&acc_empty[b]);   // the MMA may reuse the buffer
      // the previous tile's stores have read the staging area
      if (issuer) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      named_barrier(3, 256);
      // the row's |max| of the fp16-rounded values: rounding to nearest is
      // monotonic and symmetric, so it is the fp16 rounding of the float32
      // |max| (one conversion instead of one per element); the bit patterns
      // of non-negative floats order as unsigned integers
      uint32_t mx = 0u;
#pragma unroll
      for (int q = 0; q < 8 && !failed; ++q) {
        uint32_t hv[4];
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          const int e = q * 8 + 2 * j2;
          const __half2 hh = __floats2half2_rn(__uint_as_float(v[e]), __uint_as_float(v[e + 1]));
          hv[j2] = *reinterpret_cast<const uint32_t*>(&hh);
          mx = max(mx, max(v[e] & 0x7FFFFFFFu, v[e + 1] & 0x7FFFFFFFu));
        }
        *reinterpret_cast<uint4*>(stage_out + sw128_off(r, chh * 64 + q * 8)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      }
      mx = __float_as_uint(__half2float(__float2half_rn(__uint_as_float(mx))));
      fence_proxy_async_smem();
      named_barrier(3, 256);
      const int y0 = (tb + i) * kRtRows;
      if (issuer && !failed) {
        // rows past M are clipped by the tensor map
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(&ymap),
                     "r"(g * 128), "r"(y0), "r"(smem_u32(stage_out))
                     : "memory");
        asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(&ymap),
                     "r"(g * 128 + 64), "r"(y0), "r"(smem_u32(stage_out + 16384))
                     : "memory");
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      }
      const int64_t row = (int64_t)y0 + r;
      if (!failed && row < p.M && mx) atomicMax(p.amax + row, mx);
    }
    if (issuer) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kBufs * 128) : "memory");
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 rt_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

static int g_rt_sms = 0;
static int g_rt_coresident = -1;   // CTAs of the single-pass kernel that fit the GPU at once

static void rt_init() {
  if (g_rt_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_rt_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_rt_sms <= 0) g_rt_sms = 148;
  }
  if (g_rt_coresident < 0) {
    int per_sm = 0;
    if (ensure_smem_limit((const void*)rot_tc_kernel<true>, kRtSmem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rot_tc_kernel<true>, kRtQuantThreads, kRtSmem) !=
            cudaSuccess)
      per_sm = 0;
    cudaGetLastError();
    g_rt_coresident = per_sm * g_rt_sms;
  }
}

// The single-pass mode needs every CTA resident at once (one group per CTA,
// G <= resident CTAs) and 16-byte aligned int8 rows.
bool rot_tc_single_pass_ok(int K, const void* q) {
  rt_init();
  return K % kGroup == 0 && K / kGroup <= g_rt_coresident && (reinterpret_cast<uintptr_t>(q) & 15) == 0;
}

// The rotation pass for bf16 x [M, K] (K % 128 == 0, 16-byte aligned rows).
// q == nullptr: y fp16 [M, K] and row maxima (amax zeroed by the caller).
// Otherwise the single-pass mode: int8 codes q and per-token scales qscale,
// amax and cnt ([tiles] row-tile counters) zeroed by the caller; launched
// cooperatively, so it either runs with every CTA resident or fails to
// launch (the caller then takes the two-pass mode).
cudaError_t launch_rot_tc(const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab, __half* y,
                          uint32_t* amax, int8_t* q, float* qscale, uint32_t* cnt, cudaStream_t st) {
  if (M <= 0 || M > 0x7FFFFFFF) return cudaErrorInvalidValue;
  auto encode = rt_encode();
  if (!encode) return cudaErrorNotSupported;
  rt_init();
  CUtensorMap xmap;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kRtRows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  CUtensorMap ymap;
  r = encode(&ymap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // int8 codes (single-pass mode): 128-row x 128-byte boxes; else a copy of
  // ymap (unused)
  CUtensorMap qmap = ymap;
  if (q) {
    const cuuint64_t qstr[1] = {(cuuint64_t)K};
    const cuuint32_t qbox[2] = {128, (cuuint32_t)kRtRows};
    r = encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, qstr, qbox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  RtParams p;
  p.M = M;
  p.K = K;
  p.G = K / kGroup;
  p.tiles = (int)((M + kRtRows - 1) / kRtRows);
  const int slots = q ? g_rt_coresident : g_rt_sms;
  int splits = slots / p.G;
  if (splits < 1) splits = 1;
  if (splits > p.tiles) splits = p.tiles;
  p.splits = splits;
  p.scales = scales;
  p.rtab = rtab;
  p.y = y;
  p.amax = amax;
  p.q = q;
  p.qscale = qscale;
  p.cnt = cnt;
  if (q) {
    if (p.G * splits > g_rt_coresident) return cudaErrorCooperativeLaunchTooLarge;
    cudaError_t e = ensure_smem_limit((const void*)rot_tc_kernel<true>, kRtSmem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.G * splits));
    cfg.blockDim = dim3(kRtQuantThreads);
    cfg.dynamicSmemBytes = kRtSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rot_tc_kernel<true>, xmap, ymap, qmap, p);
  }
  cudaError_t e = ensure_smem_limit((const void*)rot_tc_kernel<false>, kRtSmem);
  if (e != cudaSuccess) return e;
  rot_tc_kernel<false><<<(unsigned)(p.G * splits), kRtThreads, kRtSmem, st>>>(xmap, ymap, qmap, p);
  return cudaGetLastError();
}

// Load-time: the rotation matrix R_g of every group of a krot-8, group-128
// table, written after the table's 8 x K words (g * 16384 floats from there,
// element (n, k) at ((k / 8) * 128 + n) * 8 + k % 8), then the flag set in
// word 0.  One CTA per group, the rotation kernel's build arithmetic
// (rt_build_columns); the flag is set by group 0's CTA after it has read
// word 0 (no other CTA reads it).
__global__ void __launch_bounds__(256) rot_matrices_kernel(uint32_t* table, int K) {
  __shared__ uint32_t tab[8 * 128];
  __shared__ float ex_all[2 * 32 * 128];
  const int g = blockIdx.x, t = threadIdx.x, h = t >> 7, n = t & 127;
  for (int i = t; i < 8 * 128; i += 256) tab[i] = table[(size_t)(i >> 7) * K + g * 128 + (i & 127)];
  __syncthreads();
  if (g == 0 && t == 0) atomicOr(table, kRotMatricesFlag);
  float* ex = ex_all + h * (32 * 128);
  float4* dst = reinterpret_cast<float4*>(table + (size_t)8 * K) + (size_t)g * 4096;
  for (int c0 = 0; c0 < 64; c0 += 32) {
    float v[32];
    rt_build_columns(tab, ex, h, n, 64 * h + c0, v);
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      const size_t i = ((size_t)((64 * h + c0 + j) >> 3) * 128 + n) * 2;
      dst[i] = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      dst[i + 1] = make_float4(v[j + 4], v[j + 5], v[j + 6], v[j + 7]);
    }
  }
}

cudaError_t launch_prepare_rotation_matrices(uint32_t* table, int K, cudaStream_t st) {
  if (K <= 0 || K % kGroup) return cudaErrorInvalidValue;
  rot_matrices_kernel<<<(unsigned)(K / kGroup), 256, 0, st>>>(table, K);
  return cudaGetLastError();
}

}  // namespace paro
