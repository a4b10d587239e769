// gemm.cu -- stablehlo.dot_general on sm_100a tensor cores.
//
// C[b] = A[b] * B[b], bf16 in, fp32 accumulate in TMEM, bf16 out.
//
// Persistent, warp-specialised kernel, one CTA per SM (192 threads):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [64 x 256] (or
//               [256 x 64] for a K-contiguous B) per k-block into a
//               kStages-deep shared-memory ring, 128-byte swizzle.
//   warp 1      TMEM owner + MMA issuer: one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=256, K=16) x4
//               per k-block into one of two 256-column fp32 accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 64 columns, round to bf16,
//               write a 128-byte-swizzled staging tile, TMA store.  The two
//               accumulators let the epilogue of tile i overlap the MMAs of
//               tile i+1.
// Tiles are walked in groups of kGroupM row-tiles so that the operands a
// wave of CTAs touches stay resident in the 126 MB L2.
// The B operand of dot_general ([K, N], N contiguous) is consumed MN-major
// straight from its natural layout: no transpose pass.
#include "runtime.cuh"

namespace rb {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64, kStages = 4, kGroupM = 16;
constexpr int kThreads = 192;
constexpr uint32_t kABytes = BM * BK * 2;          // 16 KB
constexpr uint32_t kBBytes = BN * BK * 2;          // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kEpiBuf = 32 * 128;             // 32 rows x 64 bf16
constexpr uint32_t kEpiBytes = 4 * 2 * kEpiBuf;    // 4 warps x double buffer
constexpr uint32_t kBarOffset = kStages * kStageBytes + kEpiBytes;
constexpr uint32_t kSmemBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
constexpr uint32_t kTmemCols = 2 * BN;

struct Shape {
  int M, N, K, batch;
  int tiles_m, tiles_n, num_kb;
  int total_tiles;
};

struct Smem {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void tile_coords(const Shape& s, int t, int& b, int& m, int& n) {
  int per_batch = s.tiles_m * s.tiles_n;
  b = t / per_batch;
  int r = t - b * per_batch;
  int group_span = kGroupM * s.tiles_n;
  int g = r / group_span;
  int first_m = g * kGroupM;
  int gm = min(s.tiles_m - first_m, kGroupM);
  int rr = r - g * group_span;
  m = first_m + rr % gm;
  n = rr / gm;
}

template <bool kBKN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, Shape s) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  Smem* sm = reinterpret_cast<Smem*>(smem + kBarOffset);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
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
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(&sm->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = sm->tmem_base;
  volatile int* abort_flag = &sm->abort_flag;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < s.total_tiles && !*abort_flag; t += gridDim.x) {
        int b, tm, tn;
        tile_coords(s, t, b, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = 0; kb < s.num_kb; ++kb) {
          if (!mbar_wait(&sm->empty[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          mbar_arrive_expect_tx(&sm->full[stage], kStageBytes);
          tma_load_3d(sa, &tmA, &sm->full[stage], kb * BK, m0, b);
          if (kBKN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(sb + c * (64 * BK * 2), &tmB, &sm->full[stage], n0 + c * 64, kb * BK, b);
          } else {
            tma_load_3d(sb, &tmB, &sm->full[stage], kb * BK, n0, b);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
        // Let the loads already issued land before the CTA exits.
        int st = stage, ph = phase;
        for (int i = 0; i < kStages && i < issued; ++i) {
          if (--st < 0) { st = kStages - 1; ph ^= 1; }
          mbar_wait(&sm->full[st], ph);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, 0, kBKN ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued_any = false;
      for (int t = blockIdx.x; t < s.total_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(&sm->tmem_empty[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < s.num_kb; ++kb) {
          if (!mbar_wait(&sm->full[stage], phase)) { *abort_flag = 1; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t adesc = smem_desc_sw128(sa + k * 32, 16, 1024);
            uint64_t bdesc = kBKN ? smem_desc_sw128(sb + k * 2048, 64 * BK * 2, 1024)
                                  : smem_desc_sw128(sb + k * 32, 16, 1024);
            mma_bf16_ss(d_tmem, adesc, bdesc, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          issued_any = true;
          mma_commit(&sm->empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
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
    // ------------------------------------------------------------ epilogue
    const int lg = warp & 3;  // TMEM lane group this warp may access
    uint8_t* epi = smem + kStages * kStageBytes + (warp - 2) * 2 * kEpiBuf;
    int acc = 0;
    uint32_t acc_phase = 0;
    int nbuf = 0;
    for (int t = blockIdx.x; t < s.total_tiles; t += gridDim.x) {
      if (*abort_flag) break;
      int b, tm, tn;
      tile_coords(s, t, b, tm, tn);
      if (!mbar_wait(&sm->tmem_full[acc], acc_phase)) { *abort_flag = 1; break; }
      tc_fence_after();
      const uint32_t t_row = tmem_base + ((uint32_t)(lg * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 64; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld32(t_row + c * 64, r0);
        tmem_ld32(t_row + c * 64 + 32, r1);
        tmem_ld_wait();
        if (c == BN / 64 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm->tmem_empty[acc]);
        }
        uint32_t p[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          p[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
          p[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
        }
        uint8_t* buf = epi + (nbuf & 1) * kEpiBuf;
        if (lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
        const uint32_t row = smem_u32(buf) + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(row + ((j ^ (lane & 7)) << 4), p[4 * j], p[4 * j + 1], p[4 * j + 2],
                       p[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmC, buf, tn * BN + c * 64, tm * BM + lg * 32, b);
          bulk_commit_group();
        }
        ++nbuf;
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

__global__ void k_zero_bf16(uint16_t* c, int64_t batch, int64_t M, int64_t N, int64_t ldc,
                            int64_t stride_c) {
  int64_t total = batch * M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t b = i / (M * N), r = (i / N) % M, col = i % N;
    c[b * stride_c + r * ldc + col] = 0;
  }
}

}  // namespace gemm

// Host launcher shared by the dense and batched entry points.
static int gemm_bf16_launch(const void* A, const void* B, void* C, int64_t batch, int64_t M,
                            int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                            int64_t sa, int64_t sb, int64_t sc, int b_layout,
                            cudaStream_t st) {
  using namespace gemm;
  RB_CHECK_ARG(batch >= 1 && M >= 0 && N >= 0 && K >= 0, "gemm_bf16: bad sizes");
  RB_CHECK_ARG(b_layout == REMORA_B200_B_KN || b_layout == REMORA_B200_B_NK,
               "gemm_bf16: bad b_layout %d", b_layout);
  RB_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31) && batch < (1ll << 31),
               "gemm_bf16: sizes exceed 2^31");
  if (M == 0 || N == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(C && (K == 0 || (A && B)), "gemm_bf16: null pointer");
  const bool kn = b_layout == REMORA_B200_B_KN;
  RB_CHECK_ARG(lda >= K && ldc >= N && ldb >= (kn ? N : K), "gemm_bf16: leading dims too small");
  if (K == 0) {
    k_zero_bf16<<<num_sms() * 4, 256, 0, st>>>(static_cast<uint16_t*>(C), batch, M, N, ldc, sc);
    RB_LAUNCH_CHECK();
    return REMORA_B200_OK;
  }
  RB_CHECK_ARG(aligned16(A) && aligned16(B) && aligned16(C),
               "gemm_bf16: A, B and C must be 16-byte aligned");
  RB_CHECK_ARG(lda % 8 == 0 && ldb % 8 == 0 && ldc % 8 == 0,
               "gemm_bf16: leading dimensions must be multiples of 8 elements");
  if (batch > 1)
    RB_CHECK_ARG(sa % 8 == 0 && sb % 8 == 0 && sc % 8 == 0 && sa > 0 && sb > 0 && sc > 0,
                 "gemm_bf16: batch strides must be positive multiples of 8 elements");
  else {
    sa = M * lda;
    sb = kn ? K * ldb : N * ldb;
    sc = M * ldc;
  }

  CUtensorMap tA, tB, tC;
  {
    uint64_t d[3] = {(uint64_t)K, (uint64_t)M, (uint64_t)batch};
    uint64_t s[2] = {(uint64_t)lda * 2, (uint64_t)sa * 2};
    uint32_t box[3] = {BK, BM, 1};
    int rc = make_tmap(&tA, A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (kn) {
    uint64_t d[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)batch};
    uint64_t s[2] = {(uint64_t)ldb * 2, (uint64_t)sb * 2};
    uint32_t box[3] = {64, BK, 1};
    int rc = make_tmap(&tB, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    uint64_t d[3] = {(uint64_t)K, (uint64_t)N, (uint64_t)batch};
    uint64_t s[2] = {(uint64_t)ldb * 2, (uint64_t)sb * 2};
    uint32_t box[3] = {BK, BN, 1};
    int rc = make_tmap(&tB, B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    uint64_t d[3] = {(uint64_t)N, (uint64_t)M, (uint64_t)batch};
    uint64_t s[2] = {(uint64_t)ldc * 2, (uint64_t)sc * 2};
    uint32_t box[3] = {64, 32, 1};
    int rc = make_tmap(&tC, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }

  Shape sh;
  sh.M = (int)M;
  sh.N = (int)N;
  sh.K = (int)K;
  sh.batch = (int)batch;
  sh.tiles_m = (int)((M + BM - 1) / BM);
  sh.tiles_n = (int)((N + BN - 1) / BN);
  sh.num_kb = (int)((K + BK - 1) / BK);
  int64_t total = (int64_t)sh.tiles_m * sh.tiles_n * batch;
  RB_CHECK_ARG(total < (1ll << 31), "gemm_bf16: too many tiles");
  sh.total_tiles = (int)total;

  int grid = num_sms();
  if (grid > sh.total_tiles) grid = sh.total_tiles;
  if (kn) {
    RB_CUDA(cudaFuncSetAttribute(k_gemm_bf16<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes));
    k_gemm_bf16<true><<<grid, kThreads, kSmemBytes, st>>>(tA, tB, tC, sh);
  } else {
    RB_CUDA(cudaFuncSetAttribute(k_gemm_bf16<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes));
    k_gemm_bf16<false><<<grid, kThreads, kSmemBytes, st>>>(tA, tB, tC, sh);
  }
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

}  // namespace rb

extern "C" int remora_b200_gemm_bf16(const void* A, const void* B, void* C, int64_t batch,
                                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                     int64_t ldc, int64_t stride_a, int64_t stride_b,
                                     int64_t stride_c, int b_layout, void* stream) {
  rb::clear_error();
  return rb::gemm_bf16_launch(A, B, C, batch, M, N, K, lda, ldb, ldc, stride_a, stride_b,
                              stride_c, b_layout, rb::as_stream(stream));
}
