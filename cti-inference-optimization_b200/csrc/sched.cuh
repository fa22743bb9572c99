// Persistent tile scheduler over ragged per-expert row segments.
//
// The reference launches cdiv(T,32) x n x E programs per GEMM and lets the
// programs past an expert's row count exit (online_best/infer.py:1316,
// :1376), because it never reads the counts on the host.  Here every CTA of
// a persistent grid reads the device-side group offsets once, builds the
// exclusive prefix of m-tiles per group in shared memory, and maps a linear
// tile index (group-major, then m-tile, then n-tile) back to its coordinates
// with a binary search.  No host synchronisation, no empty CTAs.
#pragma once

#include "common.cuh"

namespace cti {

struct TileCoord {
  int g;      // group (expert) index
  int row0;   // first row of the tile in the packed row space
  int rows;   // rows of the tile that belong to the group (<= BM)
  int n_idx;  // n-tile index
};

template <int MAXG>
struct GroupSchedT {
  static constexpr int kMaxGroups = MAXG;
  __host__ __device__ static constexpr size_t smem_bytes() { return (size_t)2 * (kMaxGroups + 1) * 4 + 8; }

  int32_t* off;   // [G+1] group row offsets
  int32_t* pref;  // [G+1] exclusive prefix of m-tiles per group
  int G;
  int bm;
  int n_tiles;

  // Called by every thread of the CTA (contains __syncthreads).  Groups
  // whose offsets are inconsistent (negative, decreasing, or past
  // rows_total) are reported once and scheduled as empty.
  CTI_DEVICE void init(void* mem, const int32_t* offsets, int G_, int64_t rows_total, int bm_,
                       int n_tiles_, int32_t* status) {
    off = reinterpret_cast<int32_t*>(mem);
    pref = off + kMaxGroups + 1;
    G = G_;
    bm = bm_;
    n_tiles = n_tiles_;
    for (int i = threadIdx.x; i <= G; i += blockDim.x) off[i] = offsets[i];
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      int run = 0;
      for (int base = 0; base < G; base += 32) {
        const int g = base + lane;
        int v = 0;
        if (g < G) {
          const int lo = off[g];
          const int hi = off[g + 1];
          if (lo < 0 || hi < lo || (int64_t)hi > rows_total) {
            if (blockIdx.x == 0) raise_status(status, CTI_ERR_BOUNDS, g);
          } else {
            v = (hi - lo + bm - 1) / bm;
          }
        }
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        if (g < G) pref[g] = run + incl - v;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) pref[G] = run;
    }
    __syncthreads();
  }

  CTI_DEVICE int total_tiles() const { return pref[G] * n_tiles; }

  CTI_DEVICE TileCoord decode(int t) const {
    const int m_lin = t / n_tiles;
    TileCoord c;
    c.n_idx = t - m_lin * n_tiles;
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pref[mid] <= m_lin)
        lo = mid;
      else
        hi = mid - 1;
    }
    c.g = lo;
    c.row0 = off[lo] + (m_lin - pref[lo]) * bm;
    const int left = off[lo + 1] - c.row0;
    c.rows = left < bm ? left : bm;
    return c;
  }
};

using GroupSched = GroupSchedT<1024>;

}  // namespace cti
