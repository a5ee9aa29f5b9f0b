// prepare.cu — load-time conversion kernels (sm_100a).
//
//  * prepare_rotation_kernel : validates that every (layer, group) block of the
//    Givens pair table is a permutation and narrows it to uint8.
//  * prepare_wq_kernel       : WQLinear checkpoint buffers (reference
//    src/alpamayo_r1/utils/quantization/qmodule.py:39-78,149-205) -> tile records.
//  * prepare_awq_kernel      : AWQ int32 buffers (paroquant_marlin_w4a8.py:149-209)
//    -> tile records.
//
// Tile record (one per 16-row block nb and 128-channel group g, 1072 bytes):
//   [0, 1024)    codes: row r's 64 bytes at r*64; word t*4+j (t,j in 0..3) byte b
//                holds code k = 32*(j>>1) + 16*(j&1) + 4t + b in its low nibble
//                and code k + 64 in its high nibble (k relative to the group
//                start), so the low nibbles of a lane's four words are the A
//                fragments of mma k-steps 0-1 and the high nibbles (as 16*q)
//                those of k-steps 2-3;
//   [1024, 1056) fp16 group scales of the 16 rows;
//   [1056, 1072) uint8 zero points of the 16 rows.
#include "paro_common.cuh"

namespace paro {

// One CTA per (layer, group) block.  Entry t of the block is element (t & 1)
// of pair t / 2.  Output, indexed by channel c: the partner channel
// (bits 0-6, group-local), the role (bit 7: 0 = first element i of the pair,
// 1 = second element j), an exchange slot (bits 8-14, 128-channel groups
// only; see below) and the pair's fp16 angle (bits 16-31), so the thread
// owning channel c applies its half of the Givens update
//   i' = c*i + s*j,  j' = -s*i + c*j
// with one 32-bit load.
//
// Exchange slots: a kernel whose thread c (warp c / 32) publishes channel c's
// value in shared memory and reads its partner's would see bank conflicts
// from the pairing's arbitrary permutation.  Publishing at slot(c) instead,
// with slot(c) % 32 a colour such that every warp's 32 writes and every
// warp's 32 reads hit 32 different banks, avoids them.  The colouring always
// exists: channel c is an edge from writer warp c / 32 to reader warp
// partner(c) / 32 in a 32-regular bipartite multigraph on 4 + 4 nodes, which
// splits into 32 perfect matchings (Konig's edge-colouring theorem); colour
// = matching index, slot = colour + 32 * (c / 32).
__global__ void prepare_rotation_kernel(const int16_t* __restrict__ pairs, const uint16_t* __restrict__ theta,
                                        int K, int group, uint32_t* __restrict__ out, int32_t* __restrict__ bad) {
  __shared__ int cnt[128];
  __shared__ uint32_t word[128];
  __shared__ uint8_t slot[128];
  const int blk = blockIdx.x;  // = layer * (K / group) + g
  const int layer = blk / (K / group), g = blk - layer * (K / group);
  const size_t base = (size_t)blk * group;
  const int t = threadIdx.x;
  if (t < group) {
    cnt[t] = 0;
    slot[t] = 0;
  }
  __syncthreads();
  if (t < group) {
    const int v = pairs[base + t];
    const int w = pairs[base + (t ^ 1)];
    if (v >= 0 && v < group) {
      atomicAdd(&cnt[v], 1);
      const uint32_t th = theta[(size_t)layer * (K / 2) + (size_t)g * (group / 2) + (t >> 1)];
      word[v] = (uint32_t)(w & 0x7F) | ((uint32_t)(t & 1) << 7) | (th << 16);
    }
  }
  __syncthreads();
  const int ok = (t >= group) || (cnt[t] == 1);
  const bool valid = __syncthreads_and(ok);
  if (!valid) {
    if (t == 0) atomicAdd(bad, 1);
    return;
  }
  if (group == 128 && t == 0) {
    // channels by (writer warp, reader warp)
    uint8_t lst[4][4][32];
    int n[4][4];
    for (int a = 0; a < 4; ++a)
      for (int b = 0; b < 4; ++b) n[a][b] = 0;
    for (int c = 0; c < 128; ++c) {
      const int a = c >> 5, b = (int)(word[c] & 0x7F) >> 5;
      lst[a][b][n[a][b]++] = (uint8_t)c;
    }
    // peel 32 perfect matchings (writer a -> reader pi[a]); the multigraph
    // stays regular after each, so one of the 24 permutations always fits
    for (int colour = 0; colour < 32; ++colour) {
      int pi[4] = {-1, -1, -1, -1};
      bool found = false;
      for (int p0 = 0; p0 < 4 && !found; ++p0)
        for (int p1 = 0; p1 < 4 && !found; ++p1)
          for (int p2 = 0; p2 < 4 && !found; ++p2) {
            const int p3 = 6 - p0 - p1 - p2;
            if (p0 == p1 || p0 == p2 || p1 == p2 || p3 < 0 || p3 > 3 || p3 == p0 || p3 == p1 || p3 == p2) continue;
            if (n[0][p0] && n[1][p1] && n[2][p2] && n[3][p3]) {
              pi[0] = p0;
              pi[1] = p1;
              pi[2] = p2;
              pi[3] = p3;
              found = true;
            }
          }
      if (!found) {
        // cannot happen for a valid pairing; the identity slots are correct
        // too (each channel its own slot), only not conflict-free
        for (int c = 0; c < 128; ++c) slot[c] = (uint8_t)c;
        break;
      }
      for (int a = 0; a < 4; ++a) {
        const int c = lst[a][pi[a]][--n[a][pi[a]]];
        slot[c] = (uint8_t)(colour + 32 * a);
      }
    }
  }
  __syncthreads();
  if (t < group) out[base + t] = word[t] | ((uint32_t)slot[t] << 8);
}

// Position of code (n, k) inside WQLinear.qweight, inverse of pack_intweight
// (qmodule.py:44-72): returns the int16 element index and the nibble.
__device__ __forceinline__ void wq_locate(int n, int k, int K, size_t& elem, int& nib) {
  const int kb = k >> 5, w = k & 31;
  const int a = w >> 3, b = (w & 7) >> 1, c = w & 1;
  const int p1 = b * 8 + a * 2 + c;                      // after the (4,4,2)->(1,0,2) shuffle
  const int d = p1 >> 3, e = (p1 & 7) >> 1, f = p1 & 1;
  const int p2 = d * 8 + f * 4 + e;                      // after the pair swap
  const int kk = kb * 32 + p2;
  const int nb4 = n >> 2, i = n & 3, kb64 = kk >> 6, j = kk & 63;
  const int flat = i * 64 + j;                           // 4-row x 64-K interleave
  elem = (size_t)nb4 * K + (size_t)kb64 * 64 + (flat >> 2);
  nib = flat & 3;
}

__device__ __forceinline__ uint32_t wq_code(const uint16_t* qw, int n, int k, int K) {
  size_t e;
  int nib;
  wq_locate(n, k, K, e, nib);
  return (qw[e] >> (4 * nib)) & 0xF;
}

// AWQ nibble slot of column n%8 (pack order [0,2,4,6,1,3,5,7],
// paroquant_marlin_w4a8.py:149-164).
__device__ __forceinline__ int awq_slot(int c) {
  const int inv[8] = {0, 4, 1, 5, 2, 6, 3, 7};
  return inv[c];
}

template <bool AWQ>
__global__ void __launch_bounds__(256)
prepare_kernel(const void* __restrict__ qweight, const uint16_t* __restrict__ scales,
               const void* __restrict__ zsrc, int N, int K, uint8_t* __restrict__ packed) {
  const int G = K / kGroup;
  const int nb = blockIdx.x / G, g = blockIdx.x - nb * G;
  uint8_t* rec = packed + rec_offset(nb, g, G);
  const int t = threadIdx.x;
  const int r = t >> 4, wi = t & 15, tt = wi >> 2, j = wi & 3;
  const int n = nb * kRecRows + r;
  uint32_t word = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const int klo = g * kGroup + 32 * (j >> 1) + 16 * (j & 1) + 4 * tt + b, khi = klo + 64;
    uint32_t lo, hi;
    if constexpr (AWQ) {
      const int32_t* aq = static_cast<const int32_t*>(qweight);
      const int sl = awq_slot(n & 7);
      lo = ((uint32_t)aq[(size_t)klo * (N / 8) + (n >> 3)] >> (4 * sl)) & 0xF;
      hi = ((uint32_t)aq[(size_t)khi * (N / 8) + (n >> 3)] >> (4 * sl)) & 0xF;
    } else {
      const uint16_t* qw = static_cast<const uint16_t*>(qweight);
      lo = wq_code(qw, n, klo, K);
      hi = wq_code(qw, n, khi, K);
    }
    word |= (lo | (hi << 4)) << (8 * b);
  }
  reinterpret_cast<uint32_t*>(rec)[r * 16 + wi] = word;
  if (t < kRecRows) {
    const int nn = nb * kRecRows + t;
    const uint16_t sbits = scales[(size_t)g * N + nn];
    uint32_t z;
    if constexpr (AWQ) {
      const int32_t* aqz = static_cast<const int32_t*>(zsrc);
      z = ((uint32_t)aqz[(size_t)g * (N / 8) + (nn >> 3)] >> (4 * awq_slot(nn & 7))) & 0xF;
    } else {
      // zero point recovery of paroquant_marlin_w4a8.py:200-204
      const uint16_t* sz = static_cast<const uint16_t*>(zsrc);
      float s = half_bits_to_f32(sbits);
      if (fabsf(s) < 1e-10f) s = 1.0f;
      const float zf = rintf(__fdiv_rn(-half_bits_to_f32(sz[(size_t)g * N + nn]), s));
      z = (uint32_t)fminf(fmaxf(zf, 0.f), 15.f);
    }
    reinterpret_cast<uint16_t*>(rec + kRecScaleOff)[t] = sbits;
    rec[kRecZeroOff + t] = (uint8_t)z;
  }
}

cudaError_t launch_prepare_rotation(const int16_t* pairs, const uint16_t* theta, int krot, int K, int group,
                                    uint32_t* out, int32_t* bad, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  prepare_rotation_kernel<<<krot * (K / group), 128, 0, st>>>(pairs, theta, K, group, out, bad);
  return cudaGetLastError();
}

cudaError_t launch_prepare_wq(const int16_t* qweight, const uint16_t* scales, const uint16_t* scaled_zeros, int N,
                              int K, void* packed, cudaStream_t st) {
  const int blocks = (N / kRecRows) * (K / kGroup);
  prepare_kernel<false><<<blocks, 256, 0, st>>>(qweight, scales, scaled_zeros, N, K, static_cast<uint8_t*>(packed));
  return cudaGetLastError();
}

cudaError_t launch_prepare_awq(const int32_t* qweight, const uint16_t* scales, const int32_t* qzeros, int N, int K,
                               void* packed, cudaStream_t st) {
  const int blocks = (N / kRecRows) * (K / kGroup);
  prepare_kernel<true><<<blocks, 256, 0, st>>>(qweight, scales, qzeros, N, K, static_cast<uint8_t*>(packed));
  return cudaGetLastError();
}

}  // namespace paro
