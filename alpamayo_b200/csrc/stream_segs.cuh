// stream_segs.cuh — the stream-K walk shared by the decode GEMMs: a
// layer's work units (row tile, 128-channel group), tile-major, are split
// into one contiguous range per CTA, visited one tile segment at a time.
#pragma once

#include <stdint.h>

namespace paro {

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// The order in which a CTA visits its unit range [u0, u1), one row-block
// segment at a time: the head of the last row block, the tail of the first
// (the two segments shared with neighbouring CTAs), then the whole row blocks
// in between.  Two divisions at set-up; a segment is then a few integer
// operations (the producer's loop must stay short: it shares its SM
// sub-partition with consumer warps).
struct Segs {
  int nb0, g0, nbL, gL1, G, n;
  __device__ __forceinline__ Segs(int64_t u0, int64_t u1, int G_) : G(G_) {
    if (u1 <= u0) {
      n = nb0 = g0 = nbL = gL1 = 0;
      return;
    }
    nb0 = (int)(u0 / G);
    g0 = (int)(u0 - (int64_t)nb0 * G);
    nbL = (int)((u1 - 1) / G);
    gL1 = (int)(u1 - (int64_t)nbL * G);
    n = nbL == nb0 ? 1 : nbL - nb0 + 1;
  }
  // segment i (0 <= i < n): row block nb, groups [gb, ge)
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

}  // namespace paro
