// moe_ep_experts.cu -- the whole expert side of an expert-parallel MoE layer
// in one persistent tcgen05 kernel per rank:
//
//   scatter warps   this rank's dispatched rows -> the owners' recv buffers
//                   over NVLink (ep_scatter_warp, moe_gemm.cu), raising one
//                   ready flag per (source, expert) on the owner;
//   SwiGLU tiles    h[r, n0:n0+128] = silu(X[r] . Wg[e]) * (X[r] . Wu[e]) over the
//                   received rows, each segment's first tile waiting for its
//                   ready flag; every finished tile adds 1 per epilogue warp to
//                   mt_done[m] of its 128-row tile m;
//   down tiles      Y[r, n0:n0+256] = h[r] . Wd[e], stored straight into the
//                   source rank's y; a down tile of row tile m starts once
//                   mt_done[m] shows all SwiGLU tiles of m finished.
//
// Tiles are taken round-robin by the 148 resident CTAs from one list in
// which the SwiGLU tiles of row-tile group g+1 come before the down tiles
// of group g (groups of 16 row tiles).  So the NVLink stores of the down
// epilogues overlap the tensor work of later SwiGLU tiles instead of
// following it, and every down tile comes after all SwiGLU tiles it reads:
// the unfinished tile with the smallest index can always proceed, so the
// waits cannot form a cycle (all CTAs are resident: cooperative launch).
// Warp roles as in k_grouped_gemm: TMA producer, MMA issuer, 4 epilogue
// warps (TMEM accumulators double-buffered), then the scatter warps.
#include "runtime.cuh"
#include "ep_tiles.h"

namespace rb {
namespace moe {

static_assert(GGroupM == kEpGroupM, "the tile order assumes groups of GGroupM row tiles");

struct ExpertsShape {
  int D, F, E;                // model width, FFN width, experts on this rank
  int S;                      // segments (source rank, local expert)
  int tn_s, tn_d;             // column tiles: ceil(F / 128) SwiGLU, ceil(D / 256) down
  int kb_s, kb_d;             // k blocks of 64: ceil(D / 64), ceil(F / 64)
  const int32_t* seg_start;   // [S] first received row
  const int32_t* seg_end;     // [S] one past the last
  const int32_t* seg_expert;  // [S] local expert
  const int32_t* seg_dst_row; // [S] row of the segment's first output in its source's y
  const int32_t* seg_src;     // [S] source rank
  uint16_t* h;                // [rows, F] local SwiGLU output
  PeerPtrs y;                 // [*, D] expert outputs on every rank
  const int32_t* ready;       // [P * E] this rank's ready flags (slot src * E + e)
  int epoch;                  // value the ready flags reach this layer
  int32_t* mt_done;           // [row tiles] zero at launch
};

__device__ __forceinline__ bool wait_gpu_geq(const int32_t* f, int v) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    int32_t x;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(x) : "l"(f) : "memory");
    if (x >= v) return true;
    if ((it & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) return false;
    __nanosleep(64);
  }
}

template <int kScatterWarps>
__global__ void __launch_bounds__(GThreads + 32 * kScatterWarps, 1)
    k_ep_experts(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
                 const __grid_constant__ CUtensorMap tmU, const __grid_constant__ CUtensorMap tmH,
                 const __grid_constant__ CUtensorMap tmW, ExpertsShape s, ScatterArgs sc) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  GSmem* sm = reinterpret_cast<GSmem*>(smem + GBarOffset);
  int* s_mt = reinterpret_cast<int*>(smem + GBarOffset + 256);
  int* s_st = s_mt + (GMaxE + 1);
  int* s_en = s_st + (GMaxE + 1);
  int* s_exp = s_en + (GMaxE + 1);
  int* s_drow = s_exp + (GMaxE + 1);
  int* s_src = s_drow + (GMaxE + 1);
  int* s_wait = s_src + (GMaxE + 1);  // producer only: 1 once the segment's flag was seen
  uint8_t* epi_stage_base = smem + GEpiOffset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int i = threadIdx.x; i < s.S; i += blockDim.x) {
    s_st[i] = s.seg_start[i];
    s_en[i] = s.seg_end[i];
    s_drow[i] = s.seg_dst_row[i];
    s_src[i] = s.seg_src[i];
    s_wait[i] = 0;
    const int e = s.seg_expert[i];
    s_exp[i] = (e >= 0 && e < s.E) ? e : 0;
    if (e < 0 || e >= s.E) atomicExch(&g_device_error, 2);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int mt = 0;
    for (int q = 0; q < s.S; ++q) {
      s_mt[q] = mt;
      const int n = max(s_en[q] - s_st[q], 0);
      mt += n / GBM + ((n % GBM) ? 1 : 0);
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
  const int total_tiles = total_mt * (s.tn_s + s.tn_d);
  const int done_target = 4 * s.tn_s;  // epilogue warps x SwiGLU column tiles

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmX);
      tma_prefetch_desc(&tmG);
      tma_prefetch_desc(&tmU);
      tma_prefetch_desc(&tmH);
      tma_prefetch_desc(&tmW);
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const XTile x = x_tile(t, total_mt, s.tn_s, s.tn_d);
        const int q = seg_of_tile(s_mt, s.S, x.m);
        const int e = s_exp[q];
        const int r0 = s_st[q] + (x.m - s_mt[q]) * GBM;
        bool ok = true;
        if (!x.down) {
          if (!s_wait[q]) {
            ok = wait_flag_geq(s.ready + s_src[q] * s.E + e, s.epoch);
            s_wait[q] = 1;
          }
        } else {
          ok = wait_gpu_geq(s.mt_done + x.m, done_target);
        }
        if (!ok) {
          atomicExch(&g_device_error, 1);
          *abort_flag = 1;
          break;
        }
        // rows written through the generic proxy (scatter warps, epilogues)
        // are read below by TMA (the async proxy)
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const int nkb = x.down ? s.kb_d : s.kb_s;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&sm->empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * GStageBytes;
          uint8_t* sb = sa + GABytes;
          mbar_arrive_expect_tx(&sm->full[stage], GStageBytes);
          if (!x.down) {
            const int n0 = x.n * 128;
            tma_load_2d(sa, &tmX, &sm->full[stage], kb * GBK, r0);
            for (int c = 0; c < 2; ++c) {
              tma_load_3d(sb + c * 8192, &tmG, &sm->full[stage], n0 + c * 64, kb * GBK, e);
              tma_load_3d(sb + 16384 + c * 8192, &tmU, &sm->full[stage], n0 + c * 64, kb * GBK, e);
            }
          } else {
            const int n0 = x.n * 256;
            tma_load_2d(sa, &tmH, &sm->full[stage], kb * GBK, r0);
            for (int c = 0; c < 4; ++c)
              tma_load_3d(sb + c * 8192, &tmW, &sm->full[stage], n0 + c * 64, kb * GBK, e);
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
      constexpr uint32_t idesc_s = idesc_bf16_f32(GBM, 128, 0, 1);
      constexpr uint32_t idesc_d = idesc_bf16_f32(GBM, 256, 0, 1);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const XTile x = x_tile(t, total_mt, s.tn_s, s.tn_d);
        if (!mbar_wait(&sm->tmem_empty[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * 256;
        const int nkb = x.down ? s.kb_d : s.kb_s;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&sm->full[stage], phase)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * GStageBytes);
          const uint32_t sb = sa + GABytes;
#pragma unroll
          for (int k = 0; k < GBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
            if (!x.down) {
              mma_bf16_ss(d0, adesc, smem_desc_sw128(sb + k * 2048, 8192, 1024), idesc_s, accum);
              mma_bf16_ss(d0 + 128, adesc, smem_desc_sw128(sb + 16384 + k * 2048, 8192, 1024),
                          idesc_s, accum);
            } else {
              mma_bf16_ss(d0, adesc, smem_desc_sw128(sb + k * 2048, 8192, 1024), idesc_d, accum);
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
  } else if (warp >= 6) {
    if (kScatterWarps > 0)
      ep_scatter_warp(sc, (int64_t)blockIdx.x * kScatterWarps + (warp - 6),
                      (int64_t)gridDim.x * kScatterWarps, lane);
  } else {
    const int lg = warp & 3;
    uint8_t* epi_stage = epi_stage_base + (warp - 2) * 32 * 128;
    const uint32_t stage = smem_u32(epi_stage);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const XTile x = x_tile(t, total_mt, s.tn_s, s.tn_d);
      const int q = seg_of_tile(s_mt, s.S, x.m);
      const int r0 = s_st[q] + (x.m - s_mt[q]) * GBM;
      const int r_end = s_en[q];
      bool got = !*abort_flag && mbar_wait(&sm->tmem_full[acc], acc_phase);
      if (!__all_sync(0xffffffffu, got)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * 256;
      // SwiGLU tiles: h (local), 128 columns = 2 blocks of 64; down tiles: the
      // source rank's y over NVLink, 256 columns = 4 blocks.  Each 64-column
      // block is packed to bf16, staged in a 128-byte-swizzled [32][64] smem
      // tile and copied out with 8 lanes per row (full 128-byte row segments).
      const int N = x.down ? s.D : s.F;
      const int n_base = x.down ? x.n * 256 : x.n * 128;
      const int row_base = r0 + lg * 32;
      uint16_t* base = x.down ? reinterpret_cast<uint16_t*>(s.y.p[s_src[q]]) : s.h;
      const int64_t row_shift = x.down ? (int64_t)s_drow[q] - s_st[q] : 0;
      const int nblocks = x.down ? 4 : 2;
#pragma unroll 1
      for (int c = 0; c < nblocks; ++c) {
        uint32_t pk[32];
        if (!x.down) {
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
        if (c == nblocks - 1) {
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
        if (col0 < N) {  // N % 32 == 0: a block is either in range or half in range
          const int j = lane & 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3);
            const int grow = row_base + r;
            if (grow < r_end && col0 + j * 8 < N) {
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(stage + r * 128 + ((j ^ (r & 7)) << 4)));
              *reinterpret_cast<uint4*>(base + (grow + row_shift) * (int64_t)N + col0 + j * 8) = v;
            }
          }
        }
      }
      if (!x.down) {
        // this warp's h rows of tile (m, n) are stored: count it for the down tiles
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(s.mt_done + x.m, 1);
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
