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

__device__ __forceinline__ bool topk_before(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  if (a != b) return a > b;
  return ia < ib;
}

// Register-blocked router.  Thread (token group tg, expert group eg) owns an
// RT x 8 block of (token, expert) accumulators: tokens tg*RT .. +RT-1 of the
// block, experts eg*8 .. eg*8+7.  Each accumulator is still one serial fp32
// chain over d in increasing order (bit-exact), but a 4-d step costs RT + 8
// shared loads for 32*RT FMAs.  Tokens and router chunks are converted to f32
// once while staging.  NG = expert groups per token, a power of two <= 32:
// the NG lanes of a token are adjacent, so top-k is a segmented shuffle.
constexpr int kRouterDCh = 32;             // d per chunk
constexpr int kRowPadF = kRouterDCh + 4;   // padded f32 row (conflict-free 16-byte loads)

template <int RT, int NG>
__global__ void __launch_bounds__(kRouterThreads, 1)
    k_router_topk(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, int T, int D,
                  int E, int k, int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  constexpr int TG = kRouterThreads / NG;  // token groups per block
  constexpr int TPB = TG * RT;             // tokens per block
  constexpr int EP = NG * 8;               // padded expert count
  float* xs = reinterpret_cast<float*>(sm_raw);  // [TPB][kRowPadF]
  float* ws = xs + TPB * kRowPadF;               // [EP][kRowPadF] (transposed chunk)
  const int tid = threadIdx.x;
  const int eg = tid % NG, tg = tid / NG;
  const int t0 = blockIdx.x * TPB;
  float acc[RT][8];
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[r][i] = 0.0f;

  // The next chunk's global loads are issued into registers before the
  // current chunk is computed, so their latency overlaps the FMAs.
  constexpr int XPT = (TPB * (kRouterDCh / 8) + kRouterThreads - 1) / kRouterThreads;
  constexpr int WPT = (kRouterDCh * EP + kRouterThreads - 1) / kRouterThreads;
  uint4 xpre[XPT];
  uint16_t wpre[WPT];
  auto load_chunk = [&](int d0) {
    const int dc = min(kRouterDCh, D - d0);
#pragma unroll
    for (int j = 0; j < XPT; ++j) {
      const int i = tid + j * kRouterThreads;
      const int row = i / (kRouterDCh / 8), c8 = (i % (kRouterDCh / 8)) * 8;
      xpre[j] = make_uint4(0, 0, 0, 0);
      if (i < TPB * (kRouterDCh / 8) && t0 + row < T && c8 < dc)
        xpre[j] = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + row) * D + d0 + c8);
    }
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
      const int i = tid + j * kRouterThreads;
      const int dd = i / EP, ee = i % EP;
      wpre[j] = (i < kRouterDCh * EP && dd < dc && ee < E) ? wr[(int64_t)(d0 + dd) * E + ee]
                                                             : (uint16_t)0;
    }
  };
  auto store_chunk = [&]() {
#pragma unroll
    for (int j = 0; j < XPT; ++j) {
      const int i = tid + j * kRouterThreads;
      if (i >= TPB * (kRouterDCh / 8)) break;
      const int row = i / (kRouterDCh / 8), c8 = (i % (kRouterDCh / 8)) * 8;
      // token q = tg*RT + r lives in smem row r*TG + tg: the token groups of a
      // warp then read adjacent rows (conflict-free 16-byte loads)
      const int srow = (row % RT) * TG + row / RT;
      const uint4 v = xpre[j];
      float4* dst = reinterpret_cast<float4*>(xs + srow * kRowPadF + c8);
      dst[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
      dst[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u),
                           __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xffff0000u));
    }
#pragma unroll
    for (int j = 0; j < WPT; ++j) {
      const int i = tid + j * kRouterThreads;
      if (i >= kRouterDCh * EP) break;
      const int dd = i / EP, ee = i % EP;
      // expert ee = eg*8 + q lives in row q*NG + eg (adjacent rows across eg)
      ws[((ee & 7) * NG + (ee >> 3)) * kRowPadF + dd] = __uint_as_float((uint32_t)wpre[j] << 16);
    }
  };

  load_chunk(0);
  for (int d0 = 0; d0 < D; d0 += kRouterDCh) {
    store_chunk();
    __syncthreads();
    if (d0 + kRouterDCh < D) load_chunk(d0 + kRouterDCh);
#pragma unroll 2
    for (int dd = 0; dd < kRouterDCh; dd += 4) {
      float4 wv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        wv[i] = *reinterpret_cast<const float4*>(ws + (i * NG + eg) * kRowPadF + dd);
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + (r * TG + tg) * kRowPadF + dd);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[r][i] = fmaf(xv.x, wv[i].x, acc[r][i]);
          acc[r][i] = fmaf(xv.y, wv[i].y, acc[r][i]);
          acc[r][i] = fmaf(xv.z, wv[i].z, acc[r][i]);
          acc[r][i] = fmaf(xv.w, wv[i].w, acc[r][i]);
        }
      }
    }
    __syncthreads();
  }

  // top-k per token over the NG lanes of its group (8 candidates per lane)
  const int lane = tid & 31;
  const unsigned gmask = (NG == 32) ? 0xffffffffu : (((1u << NG) - 1u) << (lane & ~(NG - 1)));
#pragma unroll
  for (int r = 0; r < RT; ++r) {  // unrolled: acc[r][i] stays in registers
    const int t = t0 + tg * RT + r;
    uint32_t used = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (eg * 8 + i >= E) used |= 1u << i;
    float sel_v[16];
    int sel_i[16];
    for (int j = 0; j < k; ++j) {
      float bv = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (!(used >> i & 1u) &&
            (bi == 0x7fffffff || topk_before(acc[r][i], eg * 8 + i, bv, bi))) {
          bv = acc[r][i];
          bi = eg * 8 + i;
        }
#pragma unroll
      for (int off = NG / 2; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(gmask, bv, off, NG);
        const int oi = __shfl_xor_sync(gmask, bi, off, NG);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || topk_before(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      sel_v[j] = bv;
      sel_i[j] = bi;
      if (bi >> 3 == eg) used |= 1u << (bi & 7);
    }
    if (eg == 0 && t < T) {
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
