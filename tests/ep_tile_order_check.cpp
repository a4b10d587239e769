// Host check of the expert-parallel expert kernel's tile order
// (remora_b200/csrc/ep_tiles.h, the same functions the kernel runs):
//  - x_tile is a bijection of [0, total_mt * (tn_s + tn_d)) onto the
//    (kind, row tile, column tile) triples;
//  - every down tile of a row tile comes after all SwiGLU tiles of that row
//    tile, which is what keeps the kernel's waits from forming a cycle;
//  - seg_of_tile returns the last segment whose first row tile is <= m.
// Prints "ok" and exits 0, or names the first failure and exits 1.
#include <cstdio>
#include <vector>

#include "../remora_b200/csrc/ep_tiles.h"

using rb::moe::seg_of_tile;
using rb::moe::x_tile;
using rb::moe::XTile;

static int check_order(int total_mt, int tn_s, int tn_d) {
  const int total = total_mt * (tn_s + tn_d);
  std::vector<int> seen_s((size_t)total_mt * tn_s, -1), seen_d((size_t)total_mt * tn_d, -1);
  std::vector<int> last_s(total_mt, -1), first_d(total_mt, total);
  for (int t = 0; t < total; ++t) {
    const XTile x = x_tile(t, total_mt, tn_s, tn_d);
    const int nmax = x.down ? tn_d : tn_s;
    if (x.m < 0 || x.m >= total_mt || x.n < 0 || x.n >= nmax) {
      std::printf("out of range: total_mt=%d t=%d -> (%d,%d,%d)\n", total_mt, t, x.down, x.m, x.n);
      return 1;
    }
    std::vector<int>& seen = x.down ? seen_d : seen_s;
    int& slot = seen[(size_t)x.m * nmax + x.n];
    if (slot >= 0) {
      std::printf("repeat: total_mt=%d t=%d and t=%d\n", total_mt, slot, t);
      return 1;
    }
    slot = t;
    if (x.down) {
      if (t < first_d[x.m]) first_d[x.m] = t;
    } else if (t > last_s[x.m]) {
      last_s[x.m] = t;
    }
  }
  for (int m = 0; m < total_mt; ++m)
    if (last_s[m] >= first_d[m]) {
      std::printf("down before SwiGLU: total_mt=%d m=%d\n", total_mt, m);
      return 1;
    }
  return 0;
}

static int check_segments() {
  // prefix of row tiles per segment, empty segments included
  const int counts[] = {3, 0, 1, 0, 0, 7, 2, 0, 5};
  const int S = sizeof(counts) / sizeof(counts[0]);
  std::vector<int> mt(S + 1, 0);
  for (int q = 0; q < S; ++q) mt[q + 1] = mt[q] + counts[q];
  for (int m = 0; m < mt[S]; ++m) {
    int want = 0;
    for (int q = 0; q < S; ++q)
      if (mt[q] <= m) want = q;
    const int got = seg_of_tile(mt.data(), S, m);
    if (got != want || m < mt[got] || m >= mt[got + 1]) {
      std::printf("seg_of_tile(%d) = %d, want %d\n", m, got, want);
      return 1;
    }
  }
  return 0;
}

int main() {
  const int shapes[][2] = {{12, 8}, {1, 1}, {3, 5}, {12, 1}, {112, 16}};
  for (int total_mt = 1; total_mt <= 600; ++total_mt)
    for (const auto& sh : shapes)
      if (check_order(total_mt, sh[0], sh[1])) return 1;
  for (int total_mt : {1023, 1024, 1025, 4160, 4161})
    if (check_order(total_mt, 12, 8)) return 1;
  if (check_segments()) return 1;
  std::printf("ok\n");
  return 0;
}
