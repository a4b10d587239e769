// ep_tiles.h -- the tile order of the expert-parallel expert kernel
// (moe_ep_experts.cu), shared with a host-side check of its invariants:
// the order is a permutation of all (kind, row tile, column tile) triples
// and every down tile of a row tile comes after all of its SwiGLU tiles.
#pragma once

#if defined(__CUDACC__)
#define RB_HD __host__ __device__ __forceinline__
#else
#define RB_HD inline
#endif

namespace rb {
namespace moe {

constexpr int kEpGroupM = 16;  // row tiles per group

struct XTile {
  int down;  // 0: SwiGLU tile, 1: down tile
  int m;     // 128-row tile
  int n;     // column tile
};

// Tile t of the list S0 | S1 D0 | S2 D1 | ... | S_L D_{L-1} | D_L (S_g: the
// SwiGLU tiles of row-tile group g, D_g its down tiles; every group but the
// last holds kEpGroupM row tiles, row tile fastest within a block).
RB_HD XTile x_tile(int t, int total_mt, int tn_s, int tn_d) {
  const int G = (total_mt + kEpGroupM - 1) / kEpGroupM, L = G - 1;
  const int gmL = total_mt - L * kEpGroupM;
  const int fs = kEpGroupM * tn_s, fd = kEpGroupM * tn_d;
  int down, g, rr, gm;
  if (L == 0) {
    down = t >= gmL * tn_s;
    g = 0;
    rr = down ? t - gmL * tn_s : t;
    gm = gmL;
  } else if (t < fs) {
    down = 0;
    g = 0;
    rr = t;
    gm = kEpGroupM;
  } else {
    const int u = t - fs, j = u / (fs + fd) + 1, r = u % (fs + fd);
    if (j < L) {
      down = r >= fs;
      g = down ? j - 1 : j;
      rr = down ? r - fs : r;
      gm = kEpGroupM;
    } else {
      const int tp = t - (fs + (L - 1) * (fs + fd)), sL = gmL * tn_s;
      if (tp < sL) {
        down = 0; g = L; rr = tp; gm = gmL;
      } else if (tp < sL + fd) {
        down = 1; g = L - 1; rr = tp - sL; gm = kEpGroupM;
      } else {
        down = 1; g = L; rr = tp - sL - fd; gm = gmL;
      }
    }
  }
  XTile x;
  x.down = down;
  x.m = g * kEpGroupM + rr % gm;
  x.n = rr / gm;
  return x;
}

// Segment of row tile m: the last q with mt[q] <= m.
RB_HD int seg_of_tile(const int* mt, int S, int m) {
  int lo = 0, hi = S;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (mt[mid] <= m) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace moe
}  // namespace rb
