// gemm_f32.cu -- the f32 projection (--test=projection) with the reference
// CPU path's exact arithmetic.
//
// remora's CPU path lowers the dot_general of
// mlir/stablehlo/simple_attention_projection.mlir:4-6 to
// linalg.fill(0) + a reduction linalg.generic
// (mlir/linalg/attention_projection_lowered_to_linalg.mlir:8-12) and then to
// scalar loops (compiler/cpu.cpp:50-55): out = out + a*b, k increasing, a
// separately rounded product and sum.  Each output here runs that exact
// sequence (__fmul_rn / __fadd_rn, no contraction), so results are
// bit-identical to it; the parallelism is across outputs only.  CUDA cores:
// a tensor-core f32 path cannot reproduce the per-product rounding.
#include "runtime.cuh"

namespace rb {

constexpr int F32_TM = 64, F32_TN = 64, F32_TK = 16;

template <bool kBKN>
__global__ void __launch_bounds__(256) k_gemm_f32_exact(const float* __restrict__ A,
                                                        const float* __restrict__ B,
                                                        float* __restrict__ C, int M, int N,
                                                        int K, int64_t lda, int64_t ldb,
                                                        int64_t ldc) {
  __shared__ float sA[F32_TK][F32_TM + 4];
  __shared__ float sB[F32_TK][F32_TN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * F32_TM, n0 = blockIdx.x * F32_TN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  for (int k0 = 0; k0 < K; k0 += F32_TK) {
    for (int e = threadIdx.x; e < F32_TM * F32_TK; e += 256) {
      int r = e / F32_TK, kk = e % F32_TK;
      int gm = m0 + r, gk = k0 + kk;
      sA[kk][r] = (gm < M && gk < K) ? A[(int64_t)gm * lda + gk] : 0.0f;
    }
    for (int e = threadIdx.x; e < F32_TN * F32_TK; e += 256) {
      int c, kk;
      if (kBKN) { kk = e / F32_TN; c = e % F32_TN; } else { c = e / F32_TK; kk = e % F32_TK; }
      int gn = n0 + c, gk = k0 + kk;
      float v = 0.0f;
      if (gn < N && gk < K) v = kBKN ? B[(int64_t)gk * ldb + gn] : B[(int64_t)gn * ldb + gk];
      sB[kk][c] = v;
    }
    __syncthreads();
    const int kend = min(F32_TK, K - k0);
    for (int kk = 0; kk < kend; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sA[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sB[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int gm = m0 + ty + 16 * i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int gn = n0 + tx + 16 * j;
      if (gn < N) C[(int64_t)gm * ldc + gn] = acc[i][j];
    }
  }
}

}  // namespace rb

extern "C" int remora_b200_gemm_f32_exact(const float* A, const float* B, float* C, int64_t M,
                                          int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                          int64_t ldc, int b_layout, void* stream) {
  using namespace rb;
  clear_error();
  RB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0 && M < (1 << 30) && N < (1 << 30) && K < (1 << 30),
               "gemm_f32_exact: bad sizes");
  RB_CHECK_ARG(b_layout == REMORA_B200_B_KN || b_layout == REMORA_B200_B_NK,
               "gemm_f32_exact: bad b_layout %d", b_layout);
  const bool kn = b_layout == REMORA_B200_B_KN;
  RB_CHECK_ARG(lda >= K && ldc >= N && ldb >= (kn ? N : K),
               "gemm_f32_exact: leading dims too small");
  if (M == 0 || N == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(C && (K == 0 || (A && B)), "gemm_f32_exact: null pointer");
  dim3 grid((unsigned)((N + F32_TN - 1) / F32_TN), (unsigned)((M + F32_TM - 1) / F32_TM));
  RB_CHECK_ARG(grid.y < 65536, "gemm_f32_exact: M too large");
  cudaStream_t st = as_stream(stream);
  if (kn)
    k_gemm_f32_exact<true><<<grid, 256, 0, st>>>(A, B, C, (int)M, (int)N, (int)K, lda, ldb, ldc);
  else
    k_gemm_f32_exact<false><<<grid, 256, 0, st>>>(A, B, C, (int)M, (int)N, (int)K, lda, ldb, ldc);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}
