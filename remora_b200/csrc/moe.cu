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
constexpr int kRouterDCh = 32;             // d per shared-memory chunk (default)

__device__ __forceinline__ bool topk_before(float a, int ia, float b, int ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  if (a != b) return a > b;
  return ia < ib;
}

// Router, expert-lane form.  A warp is LT = 32/LE token groups of LE lanes
// (LE a power of two, 1..32, chosen by the host).  Lane (tg, le) owns RT
// tokens of its group and the experts le, le+LE, ..., le+(EPL-1)*LE, one
// accumulator each.  Every accumulator is one serial fp32 chain over d in
// increasing order (bit-exact).  Per 4-d step a lane loads EPL rows of the
// staged router chunk (one row per expert, the same row for all token
// groups of a warp) and RT token rows (one address per token group: the LE
// lanes of a group read it as a broadcast), then issues 4*RT*EPL FMAs, so
// the shared-memory traffic per FMA falls as RT and EPL grow.  Tokens and
// router chunks are converted to f32 once while staging; the next chunk's
// global loads are issued into registers before the current chunk is used.
// Top-k: per token, a segmented butterfly over the LE lanes of its group.
// WARPS warps per block: fewer warps per block give more blocks (every SM
// busy) when there are few tokens and the register block RT x EPL is large.
// Host contract: RT <= LE (so at most WARPS * 32 tokens per block),
// E % 8 == 0 or E <= 128, k <= 16.
template <int RT, int EPL, int WARPS, int DCH = kRouterDCh>
__global__ void __launch_bounds__(WARPS * 32)
    k_router_topk(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, int T, int D,
                  int E, int k, int LE, int32_t* __restrict__ idx_out,
                  float* __restrict__ w_out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  constexpr int kRouterThreads = WARPS * 32;
  constexpr int kChunk = DCH;      // d per shared-memory chunk
  constexpr int kPad = DCH + 4;    // padded f32 row (16-byte aligned rows)
  constexpr int kWarps = WARPS;
  constexpr int kDC8 = kChunk / 8;
  const int LT = 32 / LE;              // token groups per warp
  const int TGB = kWarps * LT;         // token groups per block
  const int TPB = TGB * RT;            // tokens per block
  const int EP = LE * EPL;             // staged router rows (>= E)
  float* xs = reinterpret_cast<float*>(sm_raw);  // [TPB][kPad]
  float* ws = xs + TPB * kPad;               // [EP][kPad] (router chunk, transposed)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tg = lane / LE, le = lane % LE;
  const int gtg = warp * LT + tg;      // token group within the block
  const int t0 = blockIdx.x * TPB;
  float acc[RT][EPL];
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int j = 0; j < EPL; ++j) acc[r][j] = 0.0f;
  // rows beyond E stay zero (their experts are never selected)
  for (int i = tid; i < (EP - E) * kPad; i += kRouterThreads) ws[E * kPad + i] = 0.0f;

  // Block token q = g*RT + r (token group g) lives in smem row r*TGB + g: the
  // LT token groups of a warp read LT adjacent rows for a given r.
  // Router chunk: with E % 8 == 0 each thread moves 8 experts x 1 d (one
  // 16-byte load; the lanes of a warp take consecutive d, so the transposed
  // shared stores are conflict-free); otherwise single values.
  const bool vec_w = (E % 8) == 0;
  const int nx = TPB * kDC8;                              // x pieces of 8 per chunk
  const int nw = vec_w ? kChunk * (E / 8) : kChunk * E;
  // pieces per thread: TPB <= WARPS*32 (RT <= LE) and E <= 32*EPL (LE <= 32)
  constexpr int kXPT = kDC8;
  constexpr int kWPT = (4 * kChunk * EPL + kRouterThreads - 1) / kRouterThreads;   // 16-byte
  constexpr int kWPS = (32 * kChunk * EPL + kRouterThreads - 1) / kRouterThreads;  // single
  uint4 xpre[kXPT];
  uint32_t wreg[4 * kWPT > kWPS ? 4 * kWPT : kWPS];
  auto load_chunk = [&](int d0) {
    const int dc = min(kChunk, D - d0);
#pragma unroll
    for (int j = 0; j < kXPT; ++j) {
      const int i = tid + j * kRouterThreads;
      const int row = i / kDC8, c8 = (i % kDC8) * 8;
      xpre[j] = make_uint4(0, 0, 0, 0);
      if (i < nx && t0 + row < T && c8 < dc)
        xpre[j] = *reinterpret_cast<const uint4*>(x + (int64_t)(t0 + row) * D + d0 + c8);
    }
    if (vec_w) {
#pragma unroll
      for (int j = 0; j < kWPT; ++j) {
        const int i = tid + j * kRouterThreads;
        const int dd = i % kChunk, e0 = (i / kChunk) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (i < nw && dd < dc) v = *reinterpret_cast<const uint4*>(wr + (int64_t)(d0 + dd) * E + e0);
        wreg[4 * j] = v.x;
        wreg[4 * j + 1] = v.y;
        wreg[4 * j + 2] = v.z;
        wreg[4 * j + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < kWPS; ++j) {
        const int i = tid + j * kRouterThreads;
        const int dd = i % kChunk, e = i / kChunk;
        wreg[j] = (i < nw && dd < dc) ? wr[(int64_t)(d0 + dd) * E + e] : 0u;
      }
    }
  };
  auto store_chunk = [&]() {
#pragma unroll
    for (int j = 0; j < kXPT; ++j) {
      const int i = tid + j * kRouterThreads;
      if (i >= nx) break;
      const int row = i / kDC8, c8 = (i % kDC8) * 8;
      const int srow = (row % RT) * TGB + row / RT;
      const uint4 v = xpre[j];
      float4* dst = reinterpret_cast<float4*>(xs + srow * kPad + c8);
      dst[0] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
      dst[1] = make_float4(__uint_as_float(v.z << 16), __uint_as_float(v.z & 0xffff0000u),
                           __uint_as_float(v.w << 16), __uint_as_float(v.w & 0xffff0000u));
    }
    if (vec_w) {
#pragma unroll
      for (int j = 0; j < kWPT; ++j) {
        const int i = tid + j * kRouterThreads;
        if (i >= nw) break;
        float* col = ws + (i / kChunk) * 8 * kPad + i % kChunk;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          col[(2 * q) * kPad] = __uint_as_float(wreg[4 * j + q] << 16);
          col[(2 * q + 1) * kPad] = __uint_as_float(wreg[4 * j + q] & 0xffff0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < kWPS; ++j) {
        const int i = tid + j * kRouterThreads;
        if (i >= nw) break;
        ws[(i / kChunk) * kPad + i % kChunk] = __uint_as_float(wreg[j] << 16);
      }
    }
  };

  const float* wrow = ws + le * kPad;
  const float* xrow = xs + gtg * kPad;
  load_chunk(0);
  for (int d0 = 0; d0 < D; d0 += kChunk) {
    store_chunk();
    __syncthreads();
    if (d0 + kChunk < D) load_chunk(d0 + kChunk);
#pragma unroll 2
    for (int dd = 0; dd < kChunk; dd += 4) {
      float4 wv[EPL];
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        wv[j] = *reinterpret_cast<const float4*>(wrow + j * LE * kPad + dd);
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(xrow + r * TGB * kPad + dd);
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
          acc[r][j] = fmaf(xv.x, wv[j].x, acc[r][j]);
          acc[r][j] = fmaf(xv.y, wv[j].y, acc[r][j]);
          acc[r][j] = fmaf(xv.z, wv[j].z, acc[r][j]);
          acc[r][j] = fmaf(xv.w, wv[j].w, acc[r][j]);
        }
      }
    }
    __syncthreads();
  }

  // top-k per token over the LE lanes of its group (EPL candidates per lane)
#pragma unroll
  for (int r = 0; r < RT; ++r) {  // unrolled: acc[r][j] stays in registers
    const int t = t0 + gtg * RT + r;
    uint32_t used = 0;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (le + j * LE >= E) used |= 1u << j;
    float sel_v[16];
    int sel_i[16];
    for (int s = 0; s < k; ++s) {
      float bv = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (!(used >> j & 1u) &&
            (bi == 0x7fffffff || topk_before(acc[r][j], le + j * LE, bv, bi))) {
          bv = acc[r][j];
          bi = le + j * LE;
        }
      for (int off = LE / 2; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off, LE);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off, LE);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || topk_before(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      sel_v[s] = bv;
      sel_i[s] = bi;
      if (bi % LE == le) used |= 1u << (bi / LE);
    }
    if (le == 0 && t < T) {
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

// Router, bf16-ring form (E % 8 == 0, E <= LE * EPL).  Same arithmetic as
// k_router_topk (one serial fp32 chain per (token, expert), increasing d,
// from +0.0), different data movement and issue:
//   * bf16 tiles of x ([TPB tokens][C d]) and of the router ([C d][E]) stream
//     through an S-stage shared-memory ring by cp.async, S-1 chunks in flight
//     ahead of the one being multiplied (one __syncthreads per chunk);
//   * operands stay bf16 in shared memory (a 16-byte read carries 8 d of a
//     token, an 8-byte read 4 experts of one d) and are widened to f32 in
//     registers (a bf16 is the high half of its f32);
//   * two adjacent experts of a token advance together with one
//     fma.rn.f32x2 (two independent fmaf's, each rounded once: the chains are
//     the same as with scalar fmaf);
//   * the operands of the next 8-d step are read before the current step's
//     FMAs are issued.
// Shared-memory bandwidth to the registers, not the FMA pipe, bounds the
// f32-staged forms: a 16-byte shared read costs four wavefronts for a warp
// even when its lanes share addresses, so halving the bytes per operand
// (bf16) and the FMA instructions (f32x2) is what moves the kernel.
// Lane (token group tg of LE lanes, le) owns RT tokens (block rows
// r*TGB + gtg) and the EPL experts e = g*4*LE + 4*le + jj (g < EPL/4,
// jj < 4).  Router columns E..EP-1 are zero and never selected; rows past T
// and d past D are zero-filled by cp.async (a +0.0 product leaves a chain
// unchanged: no chain is ever -0.0).  Measured on B200 against
// k_router_topk, indices and weights bit-identical: (65536, 2048, 64)
// 660 -> 471 us; (8192, 2048, 64) 126 -> 105 us; (1000, 2056, 64) 127 ->
// 50 us; (8192, 4096, 8) 68 -> 49 us; (512, 4096, 8) 56 -> 47 us.
// {d0, d1} = fma.rn({a, a}, {b0, b1}, {d0, d1}): two fmaf's in one instruction.
__device__ __forceinline__ void fma2_bcast(float& d0, float& d1, float a, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %2};\n\t"
      "mov.b64 rb, {%3, %4};\n\t"
      "mov.b64 rc, {%0, %1};\n\t"
      "fma.rn.f32x2 rc, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <int LE, int EPL, int RT, int WARPS, int C, int S>
struct RouterRing {
  static constexpr int kThreads = WARPS * 32;
  static constexpr int LT = 32 / LE;          // token groups per warp
  static constexpr int TGB = WARPS * LT;      // token groups per block
  static constexpr int TPB = TGB * RT;        // tokens per block
  static constexpr int EP = LE * EPL;         // router columns covered (>= E)
  static constexpr int XP = C + 8;            // bf16 token-row pitch (16-byte rows)
  static constexpr int WP = EP + 8;           // bf16 router-row pitch
  static constexpr int C8 = C / 8;
  static constexpr int kStage = TPB * XP + C * WP;  // bf16 elements per ring stage
  static constexpr size_t smem_bytes() { return (size_t)S * kStage * 2; }
  static_assert(EPL % 4 == 0 && C % 16 == 0 && S >= 2 && 32 % LE == 0, "router ring shape");
};

template <int LE, int EPL, int RT, int WARPS, int C, int S>
__global__ void __launch_bounds__(WARPS * 32)
    k_router_ring(const uint16_t* __restrict__ x, const uint16_t* __restrict__ wr, int T, int D,
                  int E, int k, int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  using P = RouterRing<LE, EPL, RT, WARPS, C, S>;
  constexpr int NT = P::kThreads, TGB = P::TGB, TPB = P::TPB, EP = P::EP, XP = P::XP,
                WP = P::WP, C8 = P::C8, LT = P::LT, G = EPL / 4;
  extern __shared__ __align__(16) uint8_t sm_raw[];
  uint16_t* ring = reinterpret_cast<uint16_t*>(sm_raw);  // [S][TPB*XP + C*WP]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tg = lane / LE, le = lane % LE;
  const int gtg = warp * LT + tg;
  const int t0 = blockIdx.x * TPB;
  const int E8 = E / 8;
  const int nch = (D + C - 1) / C;

  // router columns E..EP-1 of every stage stay zero (the copies never write them)
  for (int i = tid; i < S * C * (EP - E); i += NT) {
    const int st = i / (C * (EP - E)), r = i % (C * (EP - E));
    ring[st * P::kStage + TPB * XP + (r / (EP - E)) * WP + E + r % (EP - E)] = 0;
  }
  auto issue = [&](int c) {  // chunk c into ring stage c % S (one commit group)
    if (c < nch) {
      const int d0 = c * C;
      uint16_t* rx = ring + (c % S) * P::kStage;
      uint16_t* rw = rx + TPB * XP;
#pragma unroll
      for (int j = 0; j < (TPB * C8 + NT - 1) / NT; ++j) {
        const int p = tid + j * NT;
        if ((TPB * C8) % NT != 0 && p >= TPB * C8) break;
        const int row = p / C8, c8 = (p % C8) * 8;
        const bool ok = t0 + row < T && d0 + c8 < D;
        cp_async16(rx + row * XP + c8, ok ? x + (int64_t)(t0 + row) * D + d0 + c8 : x, ok);
      }
      for (int p = tid; p < C * E8; p += NT) {
        const int dd = p / E8, e8 = (p % E8) * 8;
        const bool ok = d0 + dd < D;
        cp_async16(rw + dd * WP + e8, ok ? wr + (int64_t)(d0 + dd) * E + e8 : wr, ok);
      }
    }
    cp_async_commit();
  };

  float acc[RT][EPL];
#pragma unroll
  for (int r = 0; r < RT; ++r)
#pragma unroll
    for (int j = 0; j < EPL; ++j) acc[r][j] = 0.0f;

#pragma unroll 1
  for (int c = 0; c < S - 1; ++c) issue(c);
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    cp_async_wait<S - 2>();  // chunk c landed (this thread's copies) ...
    __syncthreads();         // ... and everyone's; chunk c-1's stage is free again
    issue(c + S - 1);
    const uint16_t* bx = ring + (c % S) * P::kStage + gtg * XP;
    const uint16_t* bw = ring + (c % S) * P::kStage + TPB * XP + 4 * le;
    // operands of 8 d: RT token pieces (8 bf16 each) and, per d, G groups
    // of 4 adjacent experts (4 bf16 each)
    auto load = [&](uint4 (&xv)[RT], uint2 (&wv)[8][G], int dd) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
        xv[r] = *reinterpret_cast<const uint4*>(bx + r * TGB * XP + dd);
#pragma unroll
      for (int q = 0; q < 8; ++q)
#pragma unroll
        for (int g = 0; g < G; ++g)
          wv[q][g] = *reinterpret_cast<const uint2*>(bw + (dd + q) * WP + g * 4 * LE);
    };
    auto mac = [&](const uint4 (&xv)[RT], const uint2 (&wv)[8][G]) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {  // d = dd + q, in increasing order
        float wq[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          wq[g][0] = bf16_lo(wv[q][g].x);
          wq[g][1] = bf16_hi(wv[q][g].x);
          wq[g][2] = bf16_lo(wv[q][g].y);
          wq[g][3] = bf16_hi(wv[q][g].y);
        }
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const uint32_t pair = (q >> 1) == 0 ? xv[r].x
                                : (q >> 1) == 1 ? xv[r].y
                                : (q >> 1) == 2 ? xv[r].z
                                                : xv[r].w;
          const float xq = (q & 1) ? bf16_hi(pair) : bf16_lo(pair);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            fma2_bcast(acc[r][4 * g + 0], acc[r][4 * g + 1], xq, wq[g][0], wq[g][1]);
            fma2_bcast(acc[r][4 * g + 2], acc[r][4 * g + 3], xq, wq[g][2], wq[g][3]);
          }
        }
      }
    };
    uint4 xa[RT], xb[RT];
    uint2 wa[8][G], wb[8][G];
    load(xa, wa, 0);
#pragma unroll 1
    for (int dd = 0; dd < C; dd += 16) {
      load(xb, wb, dd + 8);
      mac(xa, wa);
      if (dd + 16 < C) load(xa, wa, dd + 16);
      mac(xb, wb);
    }
  }
  cp_async_wait<0>();

  // top-k per token over the LE lanes of its group (EPL candidates per lane)
  auto expert_of = [&](int j) { return (j >> 2) * 4 * LE + 4 * le + (j & 3); };
#pragma unroll
  for (int r = 0; r < RT; ++r) {
    const int t = t0 + r * TGB + gtg;
    uint32_t used = 0;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (expert_of(j) >= E) used |= 1u << j;
    float sel_v[16];
    int sel_i[16];
    for (int s = 0; s < k; ++s) {
      float bv = 0.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (!(used >> j & 1u) &&
            (bi == 0x7fffffff || topk_before(acc[r][j], expert_of(j), bv, bi))) {
          bv = acc[r][j];
          bi = expert_of(j);
        }
      for (int off = LE / 2; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off, LE);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off, LE);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || topk_before(ov, oi, bv, bi))) {
          bv = ov;
          bi = oi;
        }
      }
      sel_v[s] = bv;
      sel_i[s] = bi;
      if (((bi % (4 * LE)) >> 2) == le) used |= 1u << ((bi / (4 * LE)) * 4 + (bi & 3));
    }
    if (le == 0 && t < T) {
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

// Per-expert exclusive scan over the dispatch blocks, then the expert
// offsets.  Lanes run over experts (a warp reads 32 consecutive counts of
// one block row: coalesced) and the blocks are split into W contiguous
// parts, one warp each, for the 32 experts of its group: each warp sums its
// part, the part sums are scanned in shared memory, and each warp rewrites
// its part in place as the blocks' bases within each expert.  (One thread
// per expert walking the blocks with dependent loads took 121 us at 512
// blocks x 64 experts; one warp per expert reading a column, 42 us, bound
// by uncoalesced L1 wavefronts.)
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads)
    k_dispatch_scan(int32_t* __restrict__ block_counts, int nblocks, int E,
                    int32_t* __restrict__ counts, int32_t* __restrict__ offsets) {
  __shared__ int part_sum[32][33], part_base[32][33];
  __shared__ int tot[256];  // E <= 256 (the dispatch entry points reject more)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (E + 31) / 32;          // expert groups of 32 lanes (E <= 256: G <= 8)
  const int W = 32 / G;                 // warps (block parts) per group
  const int g = warp / W, part = warp % W;
  const int e = g * 32 + lane;
  const bool act = g < G && e < E;
  const int per = (nblocks + W - 1) / W;
  const int b_lo = min(nblocks, part * per), b_hi = min(nblocks, b_lo + per);
  int sum = 0;
  if (act) {
    int b = b_lo;
    for (; b + 8 <= b_hi; b += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = block_counts[(int64_t)(b + j) * E + e];
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[j];
    }
    for (; b < b_hi; ++b) sum += block_counts[(int64_t)b * E + e];
  }
  if (g < G) part_sum[warp][lane] = sum;
  __syncthreads();
  if (g < G && part == 0) {
    int run = 0;
    for (int p = 0; p < W; ++p) {
      part_base[g * W + p][lane] = run;
      run += part_sum[g * W + p][lane];
    }
    if (act) {
      tot[e] = run;
      counts[e] = run;
    }
  }
  __syncthreads();
  if (act) {
    int run = part_base[warp][lane];
    int b = b_lo;
    for (; b + 8 <= b_hi; b += 8) {
      int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = block_counts[(int64_t)(b + j) * E + e];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        block_counts[(int64_t)(b + j) * E + e] = run;  // the block's base within e
        run += v[j];
      }
    }
    for (; b < b_hi; ++b) {
      const int c = block_counts[(int64_t)b * E + e];
      block_counts[(int64_t)b * E + e] = run;
      run += c;
    }
  }
  if (warp == 0) {  // offsets: exclusive scan of the totals, 32 experts at a time
    int carry = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int v = e0 + lane < E ? tot[e0 + lane] : 0;
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
      }
      if (e0 + lane < E) offsets[e0 + lane] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) offsets[E] = carry;
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

// xs[pos, :] = x[perm[pos] / k, :]; one warp per row, 16-byte pieces, up
// to 8 pieces per lane loaded before they are stored (loads in flight).
__global__ void k_gather_rows(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm,
                              int64_t rows, int k, int D, uint16_t* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  const int D8 = D / 8;
  for (int64_t row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows;
       row += (int64_t)gridDim.x * wpb) {
    const int64_t t = perm[row] / k;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
    uint4* dst = reinterpret_cast<uint4*>(xs + row * D);
    for (int c0 = 0; c0 < D8; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < D8) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < D8) dst[c] = v[u];
      }
    }
  }
}

// xs[inv[t*k + j], :] = x[t, :] for j < k: the same copy as k_gather_rows,
// driven by tokens instead of destination rows, so each token row is read
// from HBM once and written k times ((1 + k) * D * 2 bytes per token against
// 2 * k * D * 2 for the gather).  One warp per token, up to 8 16-byte pieces
// per lane loaded before the k stores of each.
__global__ void k_scatter_rows(const uint16_t* __restrict__ x, const int32_t* __restrict__ inv,
                               int64_t T, int k, int D, uint16_t* __restrict__ xs) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  const int D8 = D / 8;
  for (int64_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < T; t += (int64_t)gridDim.x * wpb) {
    const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
    for (int c0 = 0; c0 < D8; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < D8) v[u] = __ldg(src + c);
      }
      for (int j = 0; j < k; ++j) {
        uint4* dst = reinterpret_cast<uint4*>(xs + (int64_t)inv[t * k + j] * D);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < D8) dst[c] = v[u];
        }
      }
    }
  }
}

// ----------------------------------------------------------------- combine
// out[t, :] = bf16( (((0 + w0*y0) + w1*y1) + ...) ) in slot order, each
// product and sum rounded separately as the reference ops are.  One warp
// per token; KMAX >= k is a compile-time bound, so the slot rows and
// weights sit in registers and, for each 16-byte column piece, the k row
// loads are issued before the slot-order accumulation.
template <int KMAX>
__global__ void k_combine(const uint16_t* __restrict__ y, const int32_t* __restrict__ inv,
                          const float* __restrict__ w, int64_t T, int k, int D,
                          uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  for (int64_t t = blockIdx.x * wpb + (threadIdx.x >> 5); t < T; t += (int64_t)gridDim.x * wpb) {
    const uint4* rows[KMAX];
    float ws[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; ++j) {
      rows[j] = reinterpret_cast<const uint4*>(y + (int64_t)(j < k ? inv[t * k + j] : 0) * D);
      ws[j] = j < k ? w[t * k + j] : 0.0f;
    }
    for (int c = lane; c < D / 8; c += 32) {
      uint4 v[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j)
        if (j < k) v[j] = __ldg(rows[j] + c);
      float acc[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        if (j < k) {
          const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[2 * q] = __fadd_rn(acc[2 * q], __fmul_rn(ws[j], __uint_as_float(u[q] << 16)));
            acc[2 * q + 1] =
                __fadd_rn(acc[2 * q + 1], __fmul_rn(ws[j], __uint_as_float(u[q] & 0xffff0000u)));
          }
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
