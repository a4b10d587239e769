// moe.cu -- the MoE layer's routing, dispatch and combine kernels.
//
// Reference semantics (mlir/stablehlo/mixtral_moe_layer.mlir):
//   :12     logits = tokens . router_w            (dot_general, f32)
//   :13     mhlo.topk k                           (descending, stable)
//   :14-24  softmax over the k selected logits    (max, subtract, exp, sum, divide)
//   :28-31  one-hot dispatch of tokens to experts (dense [E, T, D] in the reference)
//   :43-46  weighted combine over the k slots     (0 + w0*y0, then + w1*y1, ...)
// Here dispatch is sparse: each (token, slot) row goes to its expert's
// contiguous segment, experts in order, rows of one expert in (token, slot)
// order, so the permutation is deterministic.
#include "runtime.cuh"

namespace rb {
namespace moe {

// ------------------------------------------------------------------ router
// Logits accumulate over d in increasing order from +0.0 in fp32, one
// (token, expert) pair per serial chain: the order of remora's lowered
// loop nest (linalg.fill + reduction, convert-linalg-to-loops), so the
// top-k indices are bit-identical to it.  A bf16 x bf16 product is exact in
// fp32, so fmaf(a, b, acc) == acc + a*b here.
constexpr int kRouterThreads = 256;
constexpr int kRouterDC = 64;           // d per shared-memory chunk
constexpr int kRowPad = kRouterDC + 8;  // bf16 elements per padded token row

__device__ __forceinline__ bool topk_before(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  if (a != b) return a > b;
  return ia < ib;
}

// G token groups x E experts threads; each thread owns R tokens (R
// independent chains).  Shared memory per d-chunk: the block's tokens
// [TPB][kRowPad] and the router chunk in its natural [kRouterDC][E] layout
// (a warp then reads consecutive experts: no bank conflicts, no transpose).
template <int R>
__global__ void __launch_bounds__(kRouterThreads)
    k_router_topk(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, int T, int D,
                  int E, int k, int G, int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  const int TPB = G * R;
  uint16_t* xs = reinterpret_cast<uint16_t*>(sm_raw);                 // [TPB][kRowPad]
  uint16_t* ws = xs + TPB * kRowPad;                                  // [kRouterDC][E]
  float* lg = reinterpret_cast<float*>(ws + ((kRouterDC * E + 7) & ~7));  // [TPB][E]
  const int tid = threadIdx.x;
  const int e = tid % E, g = tid / E;
  const bool active = g < G;
  const int t0 = blockIdx.x * TPB;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.0f;

  for (int d0 = 0; d0 < D; d0 += kRouterDC) {
    const int dc = min(kRouterDC, D - d0);
    // tokens chunk: TPB rows x dc bf16, 16-byte pieces (D % 8 == 0)
    for (int i = tid; i < TPB * (kRouterDC / 8); i += blockDim.x) {
      const int row = i / (kRouterDC / 8), c8 = (i % (kRouterDC / 8)) * 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t0 + row < T && c8 < dc)
        v = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + row) * D + d0 + c8);
      *reinterpret_cast<uint4*>(xs + row * kRowPad + c8) = v;
    }
    // router chunk rows d0 .. d0+dc-1 (contiguous in global memory)
    if ((E & 7) == 0) {
      const int n8 = kRouterDC * E / 8;
      for (int i = tid; i < n8; i += blockDim.x) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (i * 8 < dc * E) v = *reinterpret_cast<const uint4*>(wr + (int64_t)d0 * E + i * 8);
        *reinterpret_cast<uint4*>(ws + i * 8) = v;
      }
    } else {
      for (int i = tid; i < kRouterDC * E; i += blockDim.x)
        ws[i] = i < dc * E ? wr[(int64_t)d0 * E + i] : (uint16_t)0;
    }
    __syncthreads();
    if (active) {
#pragma unroll 2
      for (int dd = 0; dd < kRouterDC; dd += 8) {
        float wv[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) wv[q] = __uint_as_float((uint32_t)ws[(dd + q) * E + e] << 16);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + (g * R + r) * kRowPad + dd);
          const uint32_t xq[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[r] = fmaf(__uint_as_float(xq[q] << 16), wv[2 * q], acc[r]);
            acc[r] = fmaf(__uint_as_float(xq[q] & 0xffff0000u), wv[2 * q + 1], acc[r]);
          }
        }
      }
    }
    __syncthreads();
  }
  if (active) {
#pragma unroll
    for (int r = 0; r < R; ++r) lg[(g * R + r) * E + e] = acc[r];
  }
  __syncthreads();

  // warp-shuffle top-k over each token's E logits, then softmax over the k
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const int per_lane = (E + 31) / 32;  // <= 8
  for (int tok = warp; tok < TPB; tok += nwarps) {
    const int t = t0 + tok;
    if (t >= T) break;
    float v[8];
    int vi[8];
    uint32_t used = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ei = lane + 32 * i;
      vi[i] = ei;
      v[i] = (i < per_lane && ei < E) ? lg[tok * E + ei] : 0.0f;
      if (!(i < per_lane && ei < E)) used |= 1u << i;
    }
    float sel_v[16];
    int sel_i[16];
    for (int j = 0; j < k; ++j) {
      float bv = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (!(used >> i & 1u) && (bi == 0x7fffffff || topk_before(v[i], vi[i], bv, bi))) {
          bv = v[i];
          bi = vi[i];
        }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || topk_before(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      sel_v[j] = bv;
      sel_i[j] = bi;
      if ((bi & 31) == lane) used |= 1u << (bi >> 5);
    }
    if (lane == 0) {
      // stablehlo.reduce maximum (init -inf), exp, reduce add (init 0), divide
      float m = -INFINITY;
      for (int j = 0; j < k; ++j) m = (sel_v[j] != sel_v[j] || sel_v[j] > m) ? sel_v[j] : m;
      float ex[16], s = 0.0f;
      for (int j = 0; j < k; ++j) {
        ex[j] = expf(__fsub_rn(sel_v[j], m));
        s = __fadd_rn(s, ex[j]);
      }
      for (int j = 0; j < k; ++j) {
        idx_out[(int64_t)t * k + j] = sel_i[j];
        w_out[(int64_t)t * k + j] = __fdiv_rn(ex[j], s);
      }
    }
  }
}

// ---------------------------------------------------------------- dispatch
constexpr int kDispThreads = 1024;  // entries per dispatch block (32 warps x 32)

// Per-block expert histogram of the routed (token, slot) entries.
__global__ void __launch_bounds__(kDispThreads)
    k_dispatch_count(const int32_t* __restrict__ idx, int64_t n, int E,
                     int32_t* __restrict__ block_counts) {
  extern __shared__ int cnt[];  // [E]
  for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * kDispThreads + threadIdx.x;
  if (r < n) {
    const int e = idx[r];
    if (e >= 0 && e < E)
      atomicAdd(&cnt[e], 1);
    else
      atomicExch(&g_device_error, 2);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x)
    block_counts[(int64_t)blockIdx.x * E + i] = cnt[i];
}

// Per-expert exclusive scan over blocks, then the expert offsets.
__global__ void k_dispatch_scan(int32_t* __restrict__ block_counts, int nblocks, int E,
                                int32_t* __restrict__ counts, int32_t* __restrict__ offsets) {
  extern __shared__ int tot[];  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nblocks; ++b) {
      const int c = block_counts[(int64_t)b * E + e];
      block_counts[(int64_t)b * E + e] = run;  // becomes the block's base within e
      run += c;
    }
    tot[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = o;
      o += tot[e];
    }
    offsets[E] = o;
  }
}

// Stable positions: expert offset + earlier blocks + earlier warps + rank
// among same-expert lanes of this warp.
__global__ void __launch_bounds__(kDispThreads)
    k_dispatch_scatter(const int32_t* __restrict__ idx, int64_t n, int E,
                       const int32_t* __restrict__ block_base, const int32_t* __restrict__ offsets,
                       int32_t* __restrict__ perm, int32_t* __restrict__ inv) {
  extern __shared__ int wc[];  // [32 warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * kDispThreads + threadIdx.x;
  const int e = (r < n) ? idx[r] : -1;
  const bool valid = e >= 0 && e < E;
  const uint32_t same = __match_any_sync(0xffffffffu, valid ? e : -1);
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (valid && rank == 0) wc[warp * E + e] = __popc(same);
  __syncthreads();
  for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wc[w * E + ee];
      wc[w * E + ee] = run;
      run += c;
    }
  }
  __syncthreads();
  if (valid) {
    const int pos = offsets[e] + block_base[(int64_t)blockIdx.x * E + e] + wc[warp * E + e] + rank;
    perm[pos] = (int32_t)r;
    inv[r] = pos;
  }
}

// xs[pos, :] = x[perm[pos] / k, :]; one warp per row, 16-byte pieces.
__global__ void k_gather_rows(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm,
                              int64_t rows, int k, int D, uint16_t* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  for (int64_t row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * wpb) {
    const int64_t t = perm[row] / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
    uint4* dst = reinterpret_cast<uint4*>(xs + row * D);
    for (int c = lane; c < D / 8; c += 32) dst[c] = __ldg(src + c);
  }
}

// ----------------------------------------------------------------- combine
// out[t, :] = bf16( (((0 + w0*y0) + w1*y1) + ...) ) in slot order, each
// product and sum rounded separately as the reference ops are.
__global__ void k_combine(const uint16_t* __restrict__ y, const int32_t* __restrict__ inv,
                          const float* __restrict__ w, int64_t T, int k, int D,
                          uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  for (int64_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < T; t += (int64_t)gridDim.x * wpb) {
    int32_t rows[16];
    float ws[16];
    for (int j = 0; j < k; ++j) {
      rows[j] = inv[t * k + j];
      ws[j] = w[t * k + j];
    }
    for (int c = lane; c < D / 8; c += 32) {
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
      for (int j = 0; j < k; ++j) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(y + (int64_t)rows[j] * D) + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(ws[j], __uint_as_float(u[q] << 16)));
          acc[2 * q + 1] =
              __fadd_rn(acc[2 * q + 1], __fmul_rn(ws[j], __uint_as_float(u[q] & 0xffff0000u)));
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + t * D)[c] = o;
    }
  }
}

}  // namespace moe
}  // namespace rb
