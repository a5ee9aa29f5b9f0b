// rotq_rows.cu — channel scale + Givens rotation + per-token int8
// quantisation for many tokens (prefill), sm_100a.
//
// The cluster kernel in rotq_fused.cu keeps a token row in registers across
// all of K, which suits a handful of rows; for thousands of rows its per-row
// overheads dominate.  This path splits the work in two bandwidth-shaped
// passes over a workspace:
//
//  1. rot_rows_kernel: a CTA owns 4 groups (512 channels, one per thread) and
//     16 rows.  Each thread turns its channel's 8 table entries into
//     (partner, coefficient pair) once, in registers, and applies them to all
//     16 rows, 8 at a time (two rows per packed float32 pair), exchanging
//     values through shared memory laid out [row pair][channel]
//     (consecutive threads touch consecutive 8-byte words); the 128 threads
//     of a group synchronise on their own named barrier.  The
//     rotated rows are rounded to fp16 — the value the reference's rotate
//     kernel stores (rotation.cuh:333-334) — and written to the workspace;
//     each row's |max| over the CTA's channels goes to a per-row word with
//     atomicMax (non-negative floats order like their bit patterns).
//  2. quant_rows_kernel: per row, scale = max(|max|, 1e-10) / 127 and
//     q = round_half_away(y * (127 / |max|)), 8 values per thread-step.
//
// The arithmetic is the fused kernel's, operation for operation (products
// and sums rounded separately); the packed pair instructions give the same
// values except, very rarely, in the last bit, so a code may differ from the
// single-pass kernel's by one step about once per million.
#include <type_traits>

#include "tc_ptx.cuh"

namespace paro {

constexpr int kRowsGB = 4;      // groups per CTA
constexpr int kRowsR = 8;       // rows per register chunk
constexpr int kRowsRB = 16;     // rows per CTA

// Workspace: fp16 rows [M, K] (two-pass mode), row maxima [M], row-tile
// counters [ceil(M / 128)] (single-pass mode); maxima and counters adjacent,
// zeroed by one memset.
static size_t rows_y_bytes(int64_t M, int K) { return ((size_t)M * K * sizeof(__half) + 255) & ~(size_t)255; }

size_t rotq_rows_workspace(int64_t M, int K) {
  return rows_y_bytes(M, K) + (size_t)M * sizeof(uint32_t) + (size_t)((M + 127) / 128) * sizeof(uint32_t);
}

template <typename InT>
__global__ void __launch_bounds__(128 * kRowsGB)
rot_rows_kernel(const InT* __restrict__ x, int64_t M, int K, const uint16_t* __restrict__ scales,
                const uint32_t* __restrict__ rtab, __half* __restrict__ y, uint32_t* __restrict__ amax) {
  constexpr int RP = kRowsR / 2;   // row pairs per chunk
  __shared__ float2 buf[2][RP][kRowsGB * 128];
  __shared__ uint32_t cmax[2][kRowsR];   // by chunk parity
  const int t = threadIdx.x, ch = t & 127, gs = t >> 7;
  const int G = K >> 7;
  const int g = blockIdx.x * kRowsGB + gs;
  const bool active = g < G;
  const int c = g * 128 + ch;
  const int slot = gs * 128 + ch;

  // this channel's 8 layers: partner slot and the partner's coefficient
  // (the own coefficient is the cosine for both roles)
  int part[8];
  float cc[8], cp[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const uint32_t tab = active ? __ldg(rtab + (size_t)l * K + c) : 0u;
    part[l] = gs * 128 + (int)(tab & 0x7F);
    float s_, c_;
    __sincosf(half_bits_to_f32((uint16_t)(tab >> 16)), &s_, &c_);
    cc[l] = c_;
    cp[l] = ((tab >> 7) & 1) ? -s_ : s_;
  }
  const float sc = (active && scales) ? half_bits_to_f32(scales[c]) : 1.f;
  if (t < 2 * kRowsR) cmax[t / kRowsR][t % kRowsR] = 0u;
  __syncthreads();

  const int64_t rbeg = (int64_t)blockIdx.y * kRowsRB;
  // the next chunk's inputs are loaded while the current chunk rotates
  InT nx[kRowsR];
  auto load_chunk = [&](int64_t r0) {
#pragma unroll
    for (int r = 0; r < kRowsR; ++r)
      nx[r] = (active && r0 + r < M) ? x[(r0 + r) * (int64_t)K + c] : from_f32<InT>(0.f);
  };
  load_chunk(rbeg);
  for (int chunk = 0; chunk < kRowsRB / kRowsR; ++chunk) {
    const int64_t r0 = rbeg + chunk * kRowsR;
    if (r0 >= M) break;
    const int nrows = M - r0 < kRowsR ? (int)(M - r0) : kRowsR;
    float2 v[RP];
#pragma unroll
    for (int q = 0; q < RP; ++q) v[q] = make_float2(to_f32(nx[2 * q]) * sc, to_f32(nx[2 * q + 1]) * sc);
    if (chunk + 1 < kRowsRB / kRowsR) load_chunk(r0 + kRowsR);
#pragma unroll
    for (int l = 0; l < 8; ++l) {
#pragma unroll
      for (int q = 0; q < RP; ++q) buf[l & 1][q][slot] = v[q];
      // pairs never leave their group: the group's 128 threads sync alone
      named_barrier(1 + gs, 128);
#pragma unroll
      for (int q = 0; q < RP; ++q) v[q] = givens2(v[q], buf[l & 1][q][part[l]], cc[l], cp[l]);
    }
    // fp16 store rounding, rotated rows to the workspace, row maxima (a
    // warp-wide max of the bit patterns, then a shared-memory atomic)
#pragma unroll
    for (int r = 0; r < kRowsR; ++r) {
      const float vr = (r & 1) ? v[r >> 1].y : v[r >> 1].x;
      const __half h = __float2half_rn(vr);
      uint32_t a = 0u;
      if (active && r < nrows) {
        y[(r0 + r) * (int64_t)K + c] = h;
        a = __float_as_uint(fabsf(__half2float(h)));
      }
      a = __reduce_max_sync(0xffffffffu, a);
      if ((t & 31) == 0 && a) atomicMax(&cmax[chunk & 1][r], a);
    }
    __syncthreads();
    if (t < nrows) {
      atomicMax(amax + r0 + t, cmax[chunk & 1][t]);
      cmax[chunk & 1][t] = 0u;
    }
    // this half of cmax is next used two chunks on, after the barrier that
    // ends the next chunk, which this thread reaches only after the reset
  }
}

// A warp per row (8 rows per CTA): the lanes request their share of the
// row, 8 loads in flight each, together with the row's maximum.
__global__ void __launch_bounds__(256)
quant_rows_kernel(const __half* __restrict__ y, const uint32_t* __restrict__ amax, int64_t M, int K, int vec_ok,
                  int8_t* __restrict__ out_q, float* __restrict__ out_scale) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= M) return;
  const __half* yr = y + row * (int64_t)K;
  int8_t* qr = out_q + row * (int64_t)K;
  const int n8 = K / 8;
  constexpr int kBatch = 8;
  for (int i0 = lane; i0 < n8; i0 += kBatch * 32) {
    uint4 u[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = i0 + j * 32;
      if (i < n8) u[j] = *reinterpret_cast<const uint4*>(yr + (size_t)i * 8);
    }
    const float a = fmaxf(__uint_as_float(amax[row]), 1e-10f);
    const float inv = __fdiv_rn(127.0f, a);
    if (i0 == 0) out_scale[row] = __fdiv_rn(a, 127.0f);
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int i = i0 + j * 32;
      if (i < n8) {
        const __half* h = reinterpret_cast<const __half*>(&u[j]);
        int8_t q[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = (int8_t)(int)round_half_away(__half2float(h[e]) * inv);
        if (vec_ok) {
          *reinterpret_cast<uint2*>(qr + (size_t)i * 8) = *reinterpret_cast<const uint2*>(q);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) qr[(size_t)i * 8 + e] = q[e];
        }
      }
    }
  }
}

cudaError_t launch_rot_tc(const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab, __half* y,
                          uint32_t* amax, int8_t* q, float* qscale, uint32_t* cnt, cudaStream_t st);
bool rot_tc_single_pass_ok(int K, const void* q);

template <typename InT>
static cudaError_t launch_rows_t(const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab,
                                 int8_t* q, float* s, void* ws, cudaStream_t st) {
  __half* y = static_cast<__half*>(ws);
  uint32_t* amax = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + rows_y_bytes(M, K));
  uint32_t* cnt = amax + M;
  cudaError_t e = cudaMemsetAsync(amax, 0, rotq_rows_workspace(M, K) - rows_y_bytes(M, K), st);
  if (e != cudaSuccess) return e;
  const int G = K / kGroup;
  if constexpr (std::is_same<InT, __nv_bfloat16>::value) {
    // bf16 rows: the rotation on the tensor cores (rotq_tc.cu), with the
    // quantiser fused where every group's CTA fits the GPU at once
    if (rot_tc_single_pass_ok(K, q)) {
      e = launch_rot_tc(x, M, K, scales, rtab, y, amax, q, s, cnt, st);
      if (e == cudaSuccess) return e;
      cudaGetLastError();   // not launched (e.g. SMs held elsewhere): two passes
    }
    e = launch_rot_tc(x, M, K, scales, rtab, y, amax, nullptr, nullptr, nullptr, st);
  } else {
    dim3 grid1((unsigned)((G + kRowsGB - 1) / kRowsGB), (unsigned)((M + kRowsRB - 1) / kRowsRB));
    rot_rows_kernel<InT><<<grid1, 128 * kRowsGB, 0, st>>>(static_cast<const InT*>(x), M, K, scales, rtab, y, amax);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) return e;
  const int vec_ok = (reinterpret_cast<uintptr_t>(q) & 7) == 0;
  quant_rows_kernel<<<(unsigned)((M + 7) / 8), 256, 0, st>>>(y, amax, M, K, vec_ok, q, s);
  return cudaGetLastError();
}

// Token count from which the two-pass path beats the cluster kernel.
int rotq_rows_min_m() { return 512; }

cudaError_t launch_rotq_rows(int x_dtype, const void* x, int64_t M, int K, const uint16_t* scales,
                             const uint32_t* rtab, int8_t* q, float* s, void* ws, cudaStream_t st) {
  if (M > 0x7FFFFFFF) return cudaErrorInvalidValue;
  switch (x_dtype) {
    case PARO_F32: return launch_rows_t<float>(x, M, K, scales, rtab, q, s, ws, st);
    case PARO_F16: return launch_rows_t<__half>(x, M, K, scales, rtab, q, s, ws, st);
    case PARO_BF16: return launch_rows_t<__nv_bfloat16>(x, M, K, scales, rtab, q, s, ws, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace paro
