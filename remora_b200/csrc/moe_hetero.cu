// moe_hetero.cu -- the MoE layer whose experts have different FFN widths
// (mlir/stablehlo/heterogeneous_moe_layer.mlir:66-212: 8 experts of
// d_model 4096 with F = 14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048,
// top-1 routing, one-hot dispatch and combine).  No single [E, D, F] weight
// tensor can hold these experts (the program passes one [1, D, F_e] tensor
// per expert, :66-100), so the grouped GEMMs here take one tensor map per
// expert and a tile list whose column count (N) and contraction length (K)
// are per expert:
//   kSwiGLU = true   h[r, :F_e] = silu(xs[r] . Wg_e) * (xs[r] . Wu_e)   K = D,   N = F_e
//   kSwiGLU = false  y[r, :]    = h[r, :F_e] . Wd_e                      K = F_e, N = D
// Expert e owns rows [offsets[e], offsets[e+1]) (the dispatch order); its
// tiles are (128-row tile m, column tile n) with m fastest, so CTAs that run
// neighbouring tiles share the expert's weight slab in L2.  All experts'
// tiles run in one persistent launch: the wide experts' many column tiles
// and the narrow experts' few fill the GPU together instead of one launch
// per expert.  Warp roles, pipeline and epilogue as k_grouped_gemm.
#include "runtime.cuh"

namespace rb {
namespace moe {

constexpr int kVarMaxE = 16;
constexpr int64_t kSplitRows = 2048;  // down-GEMM K splits only for batches of <= this many rows
constexpr int kMaxSplits = 8;

// Per-expert weight tensor maps (2-D, [K_e rows x N_e columns], N contiguous).
// Passed as one __grid_constant__ parameter (4 KB): TMA reads the maps where
// the launch put them.
struct VarMaps {
  CUtensorMap b0[kVarMaxE];  // Wg_e (SwiGLU) or Wd_e (down)
  CUtensorMap b1[kVarMaxE];  // Wu_e (SwiGLU only)
};

struct VarShape {
  int E;
  int K[kVarMaxE];         // contraction length of expert e
  int N[kVarMaxE];         // output columns of expert e
  int ks[kVarMaxE];        // K splits of expert e (1: no split)
  int64_t ldo;             // output row stride (elements)
  const int32_t* offsets;  // [E + 1] device: expert row ranges
  uint16_t* out;
  float* partial;          // [max ks][prows][ldo] fp32 partial sums of split experts
  int64_t prows;
};

struct VarTile {
  int e, r0, r_end, n, sp;
};

// Tile t -> (expert, row tile, column tile, K split).  tp: tile prefix per
// expert, mt: row tiles per expert, tn: column tiles per expert, st / en:
// row range per expert.  Row tile fastest, then column tile, then split.
__device__ __forceinline__ VarTile var_tile(int E, const int* tp, const int* mt, const int* tn,
                                            const int* st, const int* en, int t) {
  int e = 0;
  while (e + 1 < E && tp[e + 1] <= t) ++e;
  const int l = t - tp[e];
  const int rest = l / mt[e];
  VarTile v;
  v.e = e;
  v.r0 = st[e] + (l % mt[e]) * GBM;
  v.n = rest % tn[e];
  v.sp = rest / tn[e];
  v.r_end = en[e];
  return v;
}

// k blocks [kb0, kb1) of split sp of a K of nkb blocks in ks splits
__device__ __forceinline__ void split_range(int nkb, int ks, int sp, int* kb0, int* kb1) {
  const int per = (nkb + ks - 1) / ks;
  *kb0 = min(nkb, sp * per);
  *kb1 = min(nkb, *kb0 + per);
}

template <bool kSwiGLU>
__global__ void __launch_bounds__(GThreads, 1)
    k_grouped_var(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ VarMaps maps,
                  VarShape s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  GSmem* sm = reinterpret_cast<GSmem*>(smem + GBarOffset);
  int* s_tp = reinterpret_cast<int*>(smem + GBarOffset + 256);  // [E + 1]
  int* s_mt = s_tp + (kVarMaxE + 1);
  int* s_tn = s_mt + kVarMaxE;
  int* s_st = s_tn + kVarMaxE;
  int* s_en = s_st + kVarMaxE;
  uint8_t* epi_stage_base = smem + GEpiOffset;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kCols = kSwiGLU ? 128 : 256;

  if (threadIdx.x == 0) {
    int tp = 0;
    for (int e = 0; e < s.E; ++e) {
      const int a = s.offsets[e], b = s.offsets[e + 1];
      const int rows = b > a ? b - a : 0;
      s_st[e] = a;
      s_en[e] = b;
      s_mt[e] = (rows + GBM - 1) / GBM;
      s_tn[e] = (s.N[e] + kCols - 1) / kCols;
      s_tp[e] = tp;
      tp += s_mt[e] * s_tn[e] * s.ks[e];
    }
    s_tp[s.E] = tp;
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
  const int total_tiles = s_tp[s.E];

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
        const VarTile ti = var_tile(s.E, s_tp, s_mt, s_tn, s_st, s_en, t);
        const int n0 = ti.n * kCols;
        int kb0, kb1;
        split_range((s.K[ti.e] + GBK - 1) / GBK, s.ks[ti.e], ti.sp, &kb0, &kb1);
        const CUtensorMap* b0 = &maps.b0[ti.e];
        const CUtensorMap* b1 = &maps.b1[ti.e];
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&sm->empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * GStageBytes;
          uint8_t* sb = sa + GABytes;
          mbar_arrive_expect_tx(&sm->full[stage], GStageBytes);
          tma_load_2d(sa, &tmA, &sm->full[stage], kb * GBK, ti.r0);
          if (kSwiGLU) {
            for (int c = 0; c < 2; ++c) {
              tma_load_2d(sb + c * 8192, b0, &sm->full[stage], n0 + c * 64, kb * GBK);
              tma_load_2d(sb + 16384 + c * 8192, b1, &sm->full[stage], n0 + c * 64, kb * GBK);
            }
          } else {
            for (int c = 0; c < 4; ++c)
              tma_load_2d(sb + c * 8192, b0, &sm->full[stage], n0 + c * 64, kb * GBK);
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
        const VarTile ti = var_tile(s.E, s_tp, s_mt, s_tn, s_st, s_en, t);
        int kb0, kb1;
        split_range((s.K[ti.e] + GBK - 1) / GBK, s.ks[ti.e], ti.sp, &kb0, &kb1);
        if (!mbar_wait(&sm->tmem_empty[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * 256;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&sm->full[stage], phase)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * GStageBytes);
          const uint32_t sb = sa + GABytes;
#pragma unroll
          for (int k = 0; k < GBK / 16; ++k) {
            const uint64_t adesc = smem_desc_sw128(sa + k * 32, 16, 1024);
            const uint32_t accum = (kb > kb0 || k > 0) ? 1u : 0u;
            mma_bf16_ss(d0, adesc, smem_desc_sw128(sb + k * 2048, 8192, 1024), idesc, accum);
            if (kSwiGLU)
              mma_bf16_ss(d0 + 128, adesc, smem_desc_sw128(sb + 16384 + k * 2048, 8192, 1024),
                          idesc, accum);
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
      const VarTile ti = var_tile(s.E, s_tp, s_mt, s_tn, s_st, s_en, t);
      bool got = !*abort_flag && mbar_wait(&sm->tmem_full[acc], acc_phase);
      if (!__all_sync(0xffffffffu, got)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * 256;
      const int n_base = ti.n * kCols;
      const int row_base = ti.r0 + lg * 32;
      const int ncols = s.N[ti.e];
      if (!kSwiGLU && s.ks[ti.e] > 1) {
        // split tile: this thread's row of fp32 partial sums, 128 bytes per store run
        const int grow = row_base + lane;
        float* prow = s.partial + ((int64_t)ti.sp * s.prows + grow) * s.ldo;
#pragma unroll 1
        for (int c = 0; c < kCols; c += 32) {
          uint32_t v[32];
          tmem_ld32(t_row + c, v);
          tmem_ld_wait();
          const int col0 = n_base + c;
          if (grow < ti.r_end && col0 < ncols) {
            float4* dst = reinterpret_cast<float4*>(prow + col0);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                   __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm->tmem_empty[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        continue;
      }
      const uint32_t stage = smem_u32(epi_stage);
      constexpr int kBlocks = kCols / 64;
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
        if (col0 < ncols) {  // N_e % 32 == 0: a block is either in range or half in range
          const int j = lane & 7;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3);
            const int grow = row_base + r;
            if (grow < ti.r_end && col0 + j * 8 < ncols) {
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(stage + r * 128 + ((j ^ (r & 7)) << 4)));
              *reinterpret_cast<uint4*>(s.out + grow * s.ldo + col0 + j * 8) = v;
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

// Launches one variable-extent grouped GEMM.  a: [rows, lda] bf16 (lda >=
// every K_e); w0 (and w1 for SwiGLU): E host-side device pointers of
// [K_e, N_e] bf16 weights; out [rows, ldo].
// Sums the fp32 partials of the K-split experts in split order and stores
// bf16; rows of unsplit experts were stored by the GEMM itself.  One thread
// per 4 columns of a row, all of its splits' loads issued before the sum.
__global__ void k_var_reduce(const float* __restrict__ partial, int64_t prows, int64_t ldo,
                             const int32_t* __restrict__ offsets, VarShape s, int64_t rows,
                             uint16_t* __restrict__ out) {
  __shared__ int off[kVarMaxE + 1];
  if (threadIdx.x <= s.E) off[threadIdx.x] = offsets[threadIdx.x];
  __syncthreads();
  const int64_t groups = ldo / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * groups;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / groups, c = (i - r * groups) * 4;
    int e = 0;
    while (e + 1 < s.E && off[e + 1] <= r) ++e;
    const int ks = s.ks[e];
    if (ks <= 1 || c >= s.N[e]) continue;
    float4 v[kMaxSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      if (sp < ks) v[sp] = *reinterpret_cast<const float4*>(partial + (sp * prows + r) * ldo + c);
    float4 acc = v[0];
#pragma unroll
    for (int sp = 1; sp < kMaxSplits; ++sp)
      if (sp < ks) {
        acc.x += v[sp].x;
        acc.y += v[sp].y;
        acc.z += v[sp].z;
        acc.w += v[sp].w;
      }
    uint2 o;
    o.x = pack_bf16x2(acc.x, acc.y);
    o.y = pack_bf16x2(acc.z, acc.w);
    *reinterpret_cast<uint2*>(out + r * ldo + c) = o;
  }
}

// K splits of expert e for the down GEMM of a small batch: with few rows the
// grid would otherwise run each wide expert's long-K tiles on a few SMs.
// Splits bring every expert's tiles near the shortest K; none when the rows
// alone fill the GPU.  ks[e] = 1 means no split.
inline int plan_splits(int64_t rows, const int64_t* K, int E, int* ks) {
  int64_t kmin = K[0];
  for (int e = 1; e < E; ++e) kmin = std::min(kmin, K[e]);
  int kmax = 1;
  for (int e = 0; e < E; ++e) {
    ks[e] = 1;
    if (rows <= kSplitRows && kmin > 0) {
      const int64_t nkb = (K[e] + GBK - 1) / GBK;
      const int64_t want = std::min<int64_t>(kMaxSplits, std::max<int64_t>(1, K[e] / kmin));
      const int64_t per = (nkb + want - 1) / want;
      ks[e] = (int)((nkb + per - 1) / per);  // every split gets at least one k block
    }
    kmax = std::max(kmax, ks[e]);
  }
  return kmax;
}

int var_launch(bool swiglu, const void* a, int64_t lda, const void* const* w0,
               const void* const* w1, void* out, int64_t ldo, const int32_t* offsets,
               int64_t rows, const int64_t* K, const int64_t* N, int E, cudaStream_t st,
               float* partial = nullptr) {
  RB_CHECK_ARG(E >= 1 && E <= kVarMaxE, "grouped_gemm_var: E=%d unsupported (1..%d)", E,
               kVarMaxE);
  RB_CHECK_ARG(rows >= 0 && rows < (1ll << 31), "grouped_gemm_var: bad row count");
  if (rows == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(a && w0 && out && offsets && K && N && (!swiglu || w1),
               "grouped_gemm_var: null pointer");
  RB_CHECK_ARG(lda > 0 && lda % 8 == 0 && ldo % 8 == 0 && aligned16(a) && aligned16(out),
               "grouped_gemm_var: leading dimensions must be multiples of 8 elements and the "
               "matrices 16-byte aligned");
  VarShape sh;
  VarMaps maps;
  memset(&maps, 0, sizeof(maps));
  int64_t max_tn = 1;
  const int cols = swiglu ? 128 : 256;
  int rc;
  for (int e = 0; e < E; ++e) {
    RB_CHECK_ARG(K[e] > 0 && K[e] <= lda && N[e] > 0 && N[e] % 32 == 0 && N[e] <= ldo &&
                     N[e] < (1ll << 31),
                 "grouped_gemm_var: expert %d has K=%lld N=%lld (need K <= lda, N %% 32 == 0, "
                 "N <= ldo)", e, (long long)K[e], (long long)N[e]);
    RB_CHECK_ARG(swiglu || K[e] % GBK == 0 || K[e] == lda,
                 "grouped_gemm_var: expert %d: K=%lld must be a multiple of %d below lda", e,
                 (long long)K[e], GBK);
    RB_CHECK_ARG(w0[e] && aligned16(w0[e]) && (!swiglu || (w1[e] && aligned16(w1[e]))),
                 "grouped_gemm_var: expert %d weights null or not 16-byte aligned", e);
    sh.K[e] = (int)K[e];
    sh.N[e] = (int)N[e];
    uint64_t d[2] = {(uint64_t)N[e], (uint64_t)K[e]};
    uint64_t s1[1] = {(uint64_t)N[e] * 2};
    uint32_t box[2] = {64, GBK};
    if ((rc = make_tmap(&maps.b0[e], w0[e], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, s1, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    if (swiglu && (rc = make_tmap(&maps.b1[e], w1[e], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, s1,
                                  box, CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
    max_tn = std::max<int64_t>(max_tn, (N[e] + cols - 1) / cols);
  }
  // A: rows x lda; a K_e below lda stops at a whole k block (checked above),
  // so no column past an expert's K is ever read
  CUtensorMap tA;
  {
    uint64_t d[2] = {(uint64_t)lda, (uint64_t)rows};
    uint64_t s1[1] = {(uint64_t)lda * 2};
    uint32_t box[2] = {GBK, GBM};
    if ((rc = make_tmap(&tA, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, s1, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  sh.E = E;
  sh.ldo = ldo;
  sh.offsets = offsets;
  sh.out = static_cast<uint16_t*>(out);
  sh.partial = partial;
  sh.prows = rows;
  int max_ks = 1;
  if (!swiglu && partial)
    max_ks = plan_splits(rows, K, E, sh.ks);
  else
    for (int e = 0; e < E; ++e) sh.ks[e] = 1;
  const int64_t max_tiles = (rows / GBM + E) * max_tn * max_ks;
  const int grid = (int)std::min<int64_t>(num_sms(), max_tiles);
  if (swiglu) {
    RB_CUDA(cudaFuncSetAttribute(k_grouped_var<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GSmemBytes));
    k_grouped_var<true><<<grid, GThreads, GSmemBytes, st>>>(tA, maps, sh);
  } else {
    RB_CUDA(cudaFuncSetAttribute(k_grouped_var<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, GSmemBytes));
    k_grouped_var<false><<<grid, GThreads, GSmemBytes, st>>>(tA, maps, sh);
    RB_LAUNCH_CHECK();
    if (max_ks > 1) {
      RB_CHECK_ARG(ldo % 4 == 0, "grouped_gemm_var: split output stride must be a multiple of 4");
      const int64_t want = (rows * (ldo / 4) + 255) / 256;
      k_var_reduce<<<(unsigned)std::min<int64_t>(want, (int64_t)num_sms() * 8), 256, 0, st>>>(
          partial, rows, ldo, offsets, sh, rows, static_cast<uint16_t*>(out));
    }
  }
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

struct HeteroWs {
  int32_t *idx, *counts, *offsets, *perm, *inv, *block_counts;
  float *w, *partial;
  uint16_t *xs, *h, *y;
  size_t bytes;
};

inline HeteroWs hetero_ws(void* base, int64_t T, int64_t D, int64_t Fmax, int E, int k) {
  HeteroWs L;
  const int64_t n = T * k;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += align256(bytes);
    return static_cast<uint8_t*>(base) + at;
  };
  L.idx = reinterpret_cast<int32_t*>(take(n * 4));
  L.w = reinterpret_cast<float*>(take(n * 4));
  L.counts = reinterpret_cast<int32_t*>(take(E * 4));
  L.offsets = reinterpret_cast<int32_t*>(take((E + 1) * 4));
  L.perm = reinterpret_cast<int32_t*>(take(n * 4));
  L.inv = reinterpret_cast<int32_t*>(take(n * 4));
  L.block_counts = reinterpret_cast<int32_t*>(take(dispatch_ws_bytes(T, k, E)));
  L.xs = reinterpret_cast<uint16_t*>(take(n * D * 2));
  L.h = reinterpret_cast<uint16_t*>(take(n * Fmax * 2));
  L.y = reinterpret_cast<uint16_t*>(take(n * D * 2));
  // fp32 partial sums of the split down GEMM (small batches only)
  L.partial = n <= kSplitRows ? reinterpret_cast<float*>(take(kMaxSplits * n * D * 4)) : nullptr;
  L.bytes = o;
  return L;
}

inline int64_t max_ffn(const int64_t* F, int E) {
  int64_t m = 0;
  for (int e = 0; e < E; ++e) m = std::max(m, F[e]);
  return (m + 63) / 64 * 64;  // h rows padded to whole k blocks
}

}  // namespace moe
}  // namespace rb

using namespace rb;
using namespace rb::moe;

extern "C" int remora_b200_grouped_gemm_swiglu_var_bf16(const void* xs, const void* const* wg,
                                                        const void* const* wu, void* h,
                                                        int64_t ldh, const int32_t* offsets,
                                                        int64_t rows, int64_t D,
                                                        const int64_t* F, int E, void* stream) {
  clear_error();
  RB_CHECK_ARG(E >= 1 && E <= kVarMaxE && D > 0 && D % 8 == 0 && F,
               "grouped_gemm_swiglu_var: bad sizes");
  int64_t K[kVarMaxE];
  for (int e = 0; e < E; ++e) K[e] = D;
  return var_launch(true, xs, D, wg, wu, h, ldh, offsets, rows, K, F, E, as_stream(stream));
}

extern "C" int remora_b200_grouped_gemm_var_bf16(const void* h, int64_t ldh,
                                                 const void* const* wd, void* y,
                                                 const int32_t* offsets, int64_t rows,
                                                 const int64_t* F, int64_t D, int E,
                                                 void* stream) {
  clear_error();
  RB_CHECK_ARG(E >= 1 && E <= kVarMaxE && D > 0 && F, "grouped_gemm_var: bad sizes");
  int64_t N[kVarMaxE];
  for (int e = 0; e < E; ++e) N[e] = D;
  return var_launch(false, h, ldh, wd, nullptr, y, D, offsets, rows, F, N, E, as_stream(stream));
}

extern "C" size_t remora_b200_moe_hetero_workspace_bytes(int64_t T, int64_t D, const int64_t* F,
                                                         int E, int k) {
  if (T < 0 || D <= 0 || !F || E < 1 || E > kVarMaxE || k < 1 || k > E || T > INT32_MAX / k)
    return 0;
  return hetero_ws(nullptr, T, D, max_ffn(F, E), E, k).bytes;
}

extern "C" int remora_b200_moe_hetero_layer_bf16(const void* x, const void* wr,
                                                 const void* const* wg, const void* const* wu,
                                                 const void* const* wd, const int64_t* F,
                                                 void* out, int64_t T, int64_t D, int E, int k,
                                                 void* workspace, size_t workspace_bytes,
                                                 void* stream) {
  clear_error();
  RB_CHECK_ARG(T >= 0 && D > 0 && D % 32 == 0 && E >= 1 && E <= kVarMaxE && k >= 1 && k <= E &&
                   F,
               "moe_hetero_layer: bad sizes (D %% 32 == 0, 1 <= E <= %d, k <= E)", kVarMaxE);
  RB_CHECK_ARG(T <= INT32_MAX / k, "moe_hetero_layer: T*k exceeds the int32 range");
  if (T == 0) return REMORA_B200_OK;
  for (int e = 0; e < E; ++e)
    RB_CHECK_ARG(F[e] > 0 && F[e] % 64 == 0, "moe_hetero_layer: F[%d]=%lld must be a positive "
                 "multiple of 64", e, (long long)F[e]);
  RB_CHECK_ARG(x && wr && wg && wu && wd && out && workspace, "moe_hetero_layer: null pointer");
  const int64_t ldh = max_ffn(F, E);
  HeteroWs L = hetero_ws(workspace, T, D, ldh, E, k);
  RB_CHECK_ARG(workspace_bytes >= L.bytes, "moe_hetero_layer: workspace of %zu bytes, %zu needed",
               workspace_bytes, L.bytes);
  RB_CHECK_ARG(aligned16(workspace), "moe_hetero_layer: workspace must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int64_t n = T * k;
  int64_t K[kVarMaxE], N[kVarMaxE];
  for (int e = 0; e < E; ++e) {
    K[e] = D;
    N[e] = D;
  }
  int rc;
  if ((rc = router_launch(x, wr, T, D, E, k, L.idx, L.w, st))) return rc;
  if ((rc = dispatch_launch(L.idx, T, k, E, L.counts, L.offsets, L.perm, L.inv, L.block_counts,
                            st)))
    return rc;
  if ((rc = gather_launch(x, L.perm, n, k, D, L.xs, st))) return rc;
  if ((rc = var_launch(true, L.xs, D, wg, wu, L.h, ldh, L.offsets, n, K, F, E, st))) return rc;
  if ((rc = var_launch(false, L.h, ldh, wd, nullptr, L.y, D, L.offsets, n, F, N, E, st,
                       L.partial)))
    return rc;
  return combine_launch(L.y, L.inv, L.w, T, k, D, out, st);
}
