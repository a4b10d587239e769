// moe_gemm.cu -- persistent grouped GEMMs of the MoE experts on tcgen05.
//
// Expert e owns rows [offsets[e], offsets[e+1]) of the dispatched activation
// matrix (expert-contiguous, written by the dispatch kernels).  Its FFN
// (mixtral_moe_layer.mlir:32-42; the outlined @expert_slot_N of
// compiler/passes/ExpertOutlining.cpp:177-279) runs as two grouped GEMMs:
//   kSwiGLU = true   H[r, :] = silu(X[r] . Wg[e]) * (X[r] . Wu[e])   [rows, F]
//                    gate and up tiles (128 columns each) accumulate side by
//                    side in TMEM; the epilogue applies
//                    silu(g) = g * (1 / (1 + exp(-g))) (:34-41) and stores bf16.
//   kSwiGLU = false  Y[r, :] = H[r] . Wd[e]                           [rows, D]
// Weights are [E, K, N] with N contiguous, consumed MN-major by the smem
// descriptors straight from the reference layout (no interleave pass).
// The tile list (expert, 128-row tile, column tile) is derived on the
// device from the expert offsets[] written by the dispatch scan, so
// variable per-expert row counts need no host round trip.  Rows of a tile
// past its expert's end are computed and discarded (guarded stores).
// Warp roles as in gemm.cu: TMA producer, MMA issuer, 4 epilogue warps,
// double-buffered TMEM accumulators.
#include "runtime.cuh"

namespace rb {
namespace moe {

struct PeerPtrs {
  uint64_t p[8];  // device addresses of a buffer on up to 8 ranks
};

constexpr int GBM = 128, GBK = 64, GStages = 4, GGroupM = 16, GMaxE = 256;
constexpr int GThreads = 192;
constexpr uint32_t GABytes = GBM * GBK * 2;        // 16 KB
constexpr uint32_t GBBytes = 256 * GBK * 2;        // 32 KB: 4 boxes of [64 K x 64 N]
constexpr uint32_t GStageBytes = GABytes + GBBytes;
constexpr uint32_t GBarOffset = GStages * GStageBytes;
constexpr uint32_t GEpiOffset = GBarOffset + ((256 + 7 * (GMaxE + 1) * 4 + 1023) & ~1023u);
constexpr uint32_t GSmemBytes = GEpiOffset + 4 * 32 * 128 + 1024;

struct GroupShape {
  int K, N, E;
  int S;             // row segments (== E when segments are the experts)
  int tiles_n;       // N / (columns per tile)
  int num_kb;
  const int32_t* seg_start;   // [S] device: first row of segment q
  const int32_t* seg_end;     // [S] device: one past its last row (seg_start + 1 for offsets)
  const int32_t* seg_expert;  // [S] device: expert of each segment, or null (segment s = expert s)
  uint16_t* out;              // [rows, N] bf16 (local output when seg_dst_rank is null)
  // Optional remote output: row g of segment q is stored at row
  // seg_dst_row[q] + (g - seg_start[q]) of the [*, N] buffer dst.p[seg_dst_rank[q]]
  // (another GPU's memory, plain stores over NVLink).
  const int32_t* seg_dst_row;
  const int32_t* seg_dst_rank;
  PeerPtrs dst;
};

// The expert-parallel dispatch carried by extra warps of the SwiGLU kernel:
// rows p = 0 .. n-1 of this rank's dispatch order (expert-sorted, so rank q's
// rows are [offsets[q*Epr], offsets[(q+1)*Epr])) are copied from x into
// region `rank` of rank q's recv buffer, visiting the destinations in the
// order rank, rank+1, ... (mod P).  When every row of global expert e is
// stored, the last warp to finish one of them publishes `epoch` in
// ready.p[e / Epr][rank * Epr + e % Epr].
struct ScatterArgs {
  const uint16_t* x;        // [T_local, D] this rank's tokens
  const int32_t* perm;      // [n] dispatch order -> slot (token * k + j)
  const int32_t* offsets;   // [E + 1] expert offsets of the dispatch order
  int64_t n, cap;
  int k, D, Epr, P, rank, epoch;
  PeerPtrs recv;            // recv [P][cap][D] bf16 on every rank
  PeerPtrs ready;           // ready [P * Epr] int32 on every rank
  int32_t* done;            // [E] rows stored per expert (zero at launch)
};

struct GSmem {
  uint64_t full[GStages], empty[GStages];
  uint64_t tmem_full[2], tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
};

struct TileInfo {
  int e, r0, r_end, n, seg;
};

__device__ __forceinline__ TileInfo group_tile(const GroupShape& s, const int* mt, const int* st,
                                               const int* en, const int* sexp, int total_mt,
                                               int t) {
  const int span = GGroupM * s.tiles_n;
  const int grp = t / span;
  const int first = grp * GGroupM;
  const int gm = min(total_mt - first, GGroupM);
  const int rr = t - grp * span;
  const int g = first + rr % gm;
  TileInfo ti;
  ti.n = rr / gm;
  int lo = 0, hi = s.S;  // last segment with mt[seg] <= g
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (mt[mid] <= g) lo = mid; else hi = mid;
  }
  ti.e = sexp[lo];
  ti.seg = lo;
  ti.r0 = st[lo] + (g - mt[lo]) * GBM;
  ti.r_end = en[lo];
  return ti;
}

// Bounded acquire-wait until *f >= v (wrapping compare); false after the limit.
__device__ __forceinline__ bool wait_flag_geq(const int32_t* f, int v) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    int32_t x;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(x) : "l"(f) : "memory");
    if (x - v >= 0) return true;
    if ((it & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) return false;
    __nanosleep(32);
  }
}

__device__ __forceinline__ void st_release_sys(int32_t* f, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t* ep_ready_slot(const ScatterArgs& a, int e) {
  return reinterpret_cast<int32_t*>(a.ready.p[e / a.Epr]) + a.rank * a.Epr + e % a.Epr;
}

// Copy warps of the expert-parallel expert kernel (see ScatterArgs).
// Each warp copies chunks of two consecutive rows (16-byte pieces, up to 16
// in flight per lane); chunks are spread over all scatter warps of the grid,
// so the grid sweeps the rows in order and experts complete one after
// another.  A warp counts the rows it stored per expert and keeps the
// (expert, count) pairs it has finished in a pending list, one entry per
// lane.  When the list reaches its limit (and at the end) the warp fences
// its stores at system scope once and each pending lane adds its count to
// done[e]; the add that completes done[e] publishes the flag.  One fence
// per kPending experts keeps the warp from waiting on NVLink
// acknowledgements after every chunk; the limit starts at 1 and doubles
// after each flush, so the first experts' flags (the ones the GEMM needs
// first) rise without waiting for later experts.
constexpr int kPending = 4;

__device__ __forceinline__ void ep_scatter_warp(const ScatterArgs& a, int64_t gw, int64_t GW,
                                                int lane) {
  const int64_t n = a.n;
  const int32_t* off = a.offsets;
  const int E = a.P * a.Epr;
  if (gw == 0) {  // experts that get no rows are complete at once
    for (int e = lane; e < E; e += 32)
      if (off[e + 1] == off[e]) st_release_sys(ep_ready_slot(a, e), a.epoch);
  }
  if (n == 0) return;
  const int64_t base = off[a.rank * a.Epr];
  const int D8 = a.D / 8;
  int cur = -1, cnt = 0;         // expert being copied, rows of it stored so far
  int pend_e = -1, pend_c = 0;    // this lane's entry of the pending list
  int npend = 0;                  // warp-uniform length of the pending list
  int limit = 1;                  // warp-uniform: flush at this length
  auto flush = [&]() {
    if (npend == 0) return;
    __threadfence_system();
    __syncwarp();
    if (lane < npend) {
      const int total = off[pend_e + 1] - off[pend_e];
      const int old = atomicAdd(a.done + pend_e, pend_c);
      if (old + pend_c == total) {
        __threadfence_system();
        st_release_sys(ep_ready_slot(a, pend_e), a.epoch);
      }
    }
    __syncwarp();
    npend = 0;
  };
  auto retire = [&]() {  // move (cur, cnt) to the pending list
    if (cur < 0 || cnt == 0) return;
    if (lane == npend) {
      pend_e = cur;
      pend_c = cnt;
    }
    if (++npend >= limit) {
      flush();
      limit = min(2 * limit, kPending);
    }
  };
  for (int64_t c = 2 * gw; c < n; c += 2 * GW) {
    const uint4* src[2];
    uint4* dst[2];
    int ee[2];
    bool ok[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      ok[u] = c + u < n;
      int64_t p = c + u + base;
      if (p >= n) p -= n;
      if (!ok[u]) p = 0;
      int lo = 0, hi = E;  // expert of p: the last e with off[e] <= p
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off[mid] <= p) lo = mid; else hi = mid;
      }
      ee[u] = lo;
      const int q = lo / a.Epr;
      src[u] = reinterpret_cast<const uint4*>(a.x + (int64_t)(a.perm[p] / a.k) * a.D);
      dst[u] = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.recv.p[q]) +
                                        ((int64_t)a.rank * a.cap + (p - off[q * a.Epr])) * a.D);
    }
    for (int c0 = 0; c0 < D8; c0 += 8 * 32) {
      uint4 v[2][8];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int cc = c0 + j * 32 + lane;
          if (ok[u] && cc < D8) v[u][j] = __ldg(src[u] + cc);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int cc = c0 + j * 32 + lane;
          if (ok[u] && cc < D8) dst[u][cc] = v[u][j];
        }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!ok[u]) continue;
      if (ee[u] != cur) {
        retire();
        cur = ee[u];
        cnt = 0;
      }
      ++cnt;
    }
  }
  retire();
  flush();
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-g * 1.4426950408889634f));
  return (g * __frcp_rn(1.0f + e)) * u;
}

template <bool kSwiGLU>
__global__ void __launch_bounds__(GThreads, 1)
    k_grouped_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmB1, GroupShape s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  GSmem* sm = reinterpret_cast<GSmem*>(smem + GBarOffset);
  int* s_mt = reinterpret_cast<int*>(smem + GBarOffset + 256);
  int* s_st = s_mt + (GMaxE + 1);
  int* s_en = s_st + (GMaxE + 1);
  int* s_exp = s_en + (GMaxE + 1);
  int* s_drow = s_exp + (GMaxE + 1);
  int* s_drank = s_drow + (GMaxE + 1);
  // per epilogue warp: one [32 rows][128 B] staging tile, 1024-byte aligned
  uint8_t* epi_stage_base = smem + GEpiOffset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i <= s.S; i += blockDim.x) {
    if (i < s.S) {
      s_st[i] = s.seg_start[i];
      s_en[i] = s.seg_end[i];
      s_drow[i] = s.seg_dst_row ? s.seg_dst_row[i] : 0;
      s_drank[i] = s.seg_dst_rank ? s.seg_dst_rank[i] : 0;
      const int e = s.seg_expert ? s.seg_expert[i] : i;
      s_exp[i] = (e >= 0 && e < s.E) ? e : 0;
      if (e < 0 || e >= s.E) atomicExch(&g_device_error, 2);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // m-tile prefix: segment q owns tiles [s_mt[q], s_mt[q+1]) of GBM rows
    int mt = 0;
    for (int q = 0; q < s.S; ++q) {
      s_mt[q] = mt;
      mt += max(s_en[q] - s_st[q], 0) / GBM + ((max(s_en[q] - s_st[q], 0) % GBM) ? 1 : 0);
    }
    s_mt[s.S] = mt;
    for (int i = 0; i < GStages; ++i) {
      mbar_init(&sm->full[i], 1);
      mbar_init(&sm->empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm->tmem_full[i], 1);
      mbar_init(&sm->tmem_empty[i], 4);
    }
    mbar_init(&sm->drain, 1);
    sm->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sm->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sm->tmem_base;
  volatile int* abort_flag = &sm->abort_flag;
  const int total_mt = s_mt[s.S];
  const int total_tiles = total_mt * s.tiles_n;
  constexpr int kColsPerTile = kSwiGLU ? 128 : 256;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB0);
      if (kSwiGLU) tma_prefetch_desc(&tmB1);
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const TileInfo ti = group_tile(s, s_mt, s_st, s_en, s_exp, total_mt, t);
        const int n0 = ti.n * kColsPerTile;
        for (int kb = 0; kb < s.num_kb; ++kb) {
          if (!mbar_wait(&sm->empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * GStageBytes;
          uint8_t* sb = sa + GABytes;
          mbar_arrive_expect_tx(&sm->full[stage], GStageBytes);
          tma_load_2d(sa, &tmA, &sm->full[stage], kb * GBK, ti.r0);
          if (kSwiGLU) {
            for (int c = 0; c < 2; ++c) {
              tma_load_3d(sb + c * 8192, &tmB0, &sm->full[stage], n0 + c * 64, kb * GBK, ti.e);
              tma_load_3d(sb + 16384 + c * 8192, &tmB1, &sm->full[stage], n0 + c * 64, kb * GBK,
                          ti.e);
            }
          } else {
            for (int c = 0; c < 4; ++c)
              tma_load_3d(sb + c * 8192, &tmB0, &sm->full[stage], n0 + c * 64, kb * GBK, ti.e);
          }
          ++issued;
          if (++stage == GStages) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
        int st = stage, ph = phase;
        for (int i = 0; i < GStages && i < issued; ++i) {
          if (--st < 0) { st = GStages - 1; ph ^= 1; }
          mbar_wait(&sm->full[st], ph);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idesc = kSwiGLU ? idesc_bf16_f32(GBM, 128, 0, 1)
                                         : idesc_bf16_f32(GBM, 256, 0, 1);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(&sm->tmem_empty[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * 256;
        for (int kb = 0; kb < s.num_kb; ++kb) {
          if (!mbar_wait(&sm->full[stage], phase)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * GStageBytes);
          const uint32_t sb = sa + GABytes;
#pragma unroll
          for (int k = 0; k < GBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (kSwiGLU) {
              mma_bf16_ss(d0, adesc, smem_desc_sw128(sb + k * 2048, 8192, 1024), idesc, accum);
              mma_bf16_ss(d0 + 128, adesc, smem_desc_sw128(sb + 16384 + k * 2048, 8192, 1024),
                          idesc, accum);
            } else {
              mma_bf16_ss(d0, adesc, smem_desc_sw128(sb + k * 2048, 8192, 1024), idesc, accum);
            }
          }
          issued_any = true;
          mma_commit(&sm->empty[stage]);
          if (++stage == GStages) { stage = 0; phase ^= 1; }
        }
        if (*abort_flag) break;
        mma_commit(&sm->tmem_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      if (*abort_flag && issued_any) {
        mma_commit(&sm->drain);
        mbar_wait(&sm->drain, 0);
      }
    }
  } else {
    const int lg = warp & 3;
    uint8_t* epi_stage = epi_stage_base + (warp - 2) * 32 * 128;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const TileInfo ti = group_tile(s, s_mt, s_st, s_en, s_exp, total_mt, t);
      bool got = !*abort_flag && mbar_wait(&sm->tmem_full[acc], acc_phase);
      if (!__all_sync(0xffffffffu, got)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * 256;
      // Output rows of this warp: tile rows lg*32 .. lg*32+31.  Each 64-column
      // block is packed to bf16, staged in a 128-byte-swizzled [32][64] smem
      // tile, then copied out with 8 lanes per row: every store instruction
      // writes four full 128-byte row segments (local HBM, or a peer GPU's
      // memory over NVLink when the segment names a destination rank).
      const int n_base = ti.n * kColsPerTile;
      const int row_base = ti.r0 + lg * 32;
      uint16_t* seg_base =
          s.seg_dst_rank ? reinterpret_cast<uint16_t*>(s.dst.p[s_drank[ti.seg]]) : s.out;
      const int64_t row_shift = s.seg_dst_rank ? (int64_t)s_drow[ti.seg] - s_st[ti.seg] : 0;
      const uint32_t stage = smem_u32(epi_stage);
      constexpr int kBlocks = kColsPerTile / 64;
#pragma unroll 1
      for (int c = 0; c < kBlocks; ++c) {
        uint32_t pk[32];
        if (kSwiGLU) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t g[32], u[32];
            tmem_ld32(t_row + c * 64 + h2 * 32, g);
            tmem_ld32(t_row + 128 + c * 64 + h2 * 32, u);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[h2 * 16 + i] =
                  pack_bf16x2(silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i])),
                              silu_mul(__uint_as_float(g[2 * i + 1]),
                                       __uint_as_float(u[2 * i + 1])));
          }
        } else {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t v[32];
            tmem_ld32(t_row + c * 64 + h2 * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i)
              pk[h2 * 16 + i] =
                  pack_bf16x2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
          }
        }
        if (c == kBlocks - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm->tmem_empty[acc]);
        }
        __syncwarp();  // the previous block's copy-out has read the stage
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(stage + lane * 128 + ((j ^ (lane & 7)) << 4), pk[4 * j], pk[4 * j + 1],
                       pk[4 * j + 2], pk[4 * j + 3]);
        __syncwarp();
        const int col0 = n_base + c * 64;
        if (col0 < s.N) {  // N % 32 == 0: a block is either in range or half in range
          const int j = lane & 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3);
            const int grow = row_base + r;
            if (grow < ti.r_end && col0 + j * 8 < s.N) {
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(stage + r * 128 + ((j ^ (r & 7)) << 4)));
              *reinterpret_cast<uint4*>(seg_base + (grow + row_shift) * (int64_t)s.N + col0 +
                                        j * 8) = v;
            }
          }
        }
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace moe
}  // namespace rb
