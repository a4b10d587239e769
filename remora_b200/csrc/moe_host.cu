// moe_host.cu -- C ABI launchers of the MoE layer (router, dispatch, gather,
// grouped expert GEMMs, combine) and the fused layer entry point.
#include <algorithm>

#include "runtime.cuh"

namespace rb {
namespace moe {

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline int64_t dispatch_blocks(int64_t n) { return (n + kDispThreads - 1) / kDispThreads; }

// Router tile: lanes per token group LE, experts per lane EPL, tokens per
// lane RT, warps per block, and the launch geometry that follows.  ring > 0
// selects a k_router_ring instantiation (E % 8 == 0, E <= 64), 0 the
// f32-staged k_router_topk.
struct RouterPlan {
  int le, epl, rt, warps, dch;
  int64_t tpb, grid;
  size_t smem;
  int ring;
  char name[64];
};

// k_router_ring instantiations (LE, EPL, RT, WARPS, C, S), chosen from a
// B200 sweep of the ring kernel (every variant bit-identical):
//   1: E <= 8            <2,4,1,4,128,3>  (8192, 4096, 8) 49 us; (512, 4096, 8) 47 us
//   2: E <= 16           <4,4,1,4,64,4>
//   3: E <= 32           <8,4,2,4,64,4>
//   4: E <= 64, T < 4096 <16,4,2,4,64,4>  (1000, 2056, 64) 50 us (16 tokens per block)
//   5: E <= 64, T < 16K  <16,4,4,4,64,4>  (8192, 2048, 64) 105 us
//   6: E <= 64, larger   <8,8,4,4,64,4>   (65536, 2048, 64) 471 us
using RingA = RouterRing<2, 4, 1, 4, 128, 3>;
using RingB = RouterRing<4, 4, 1, 4, 64, 4>;
using RingC = RouterRing<8, 4, 2, 4, 64, 4>;
using RingD = RouterRing<16, 4, 2, 4, 64, 4>;
using RingE = RouterRing<16, 4, 4, 4, 64, 4>;
using RingF = RouterRing<8, 8, 4, 4, 64, 4>;

template <class R>
void ring_plan(RouterPlan& p, int64_t T, int id, int le, int epl, int rt, int warps, int c,
               int st) {
  p.ring = id;
  p.le = le;
  p.epl = epl;
  p.rt = rt;
  p.warps = warps;
  p.dch = c;
  p.tpb = R::TPB;
  p.smem = R::smem_bytes();
  p.grid = (T + p.tpb - 1) / p.tpb;
  snprintf(p.name, sizeof(p.name), "k_router_ring<%d,%d,%d,%d,%d,%d>", le, epl, rt, warps, c, st);
}

RouterPlan router_plan(int64_t T, int E) {
  RouterPlan p;
  if (E % 8 == 0 && E <= 64) {
    if (E <= 8) ring_plan<RingA>(p, T, 1, 2, 4, 1, 4, 128, 3);
    else if (E <= 16) ring_plan<RingB>(p, T, 2, 4, 4, 1, 4, 64, 4);
    else if (E <= 32) ring_plan<RingC>(p, T, 3, 8, 4, 2, 4, 64, 4);
    else if (T < 4096) ring_plan<RingD>(p, T, 4, 16, 4, 2, 4, 64, 4);
    else if (T < 16384) ring_plan<RingE>(p, T, 5, 16, 4, 4, 4, 64, 4);
    else ring_plan<RingF>(p, T, 6, 8, 8, 4, 4, 64, 4);
    return p;
  }
  // Lanes per token group LE (a power of two) and experts per lane EPL with
  // LE * EPL >= E; tokens per lane RT as large as still leaves at least 3/4
  // of the SMs a block (RT <= LE, RT * EPL <= 32 accumulators).  The shared
  // memory delivers 16 (RT + EPL) bytes per 4 RT EPL FMAs, so larger blocks
  // of (tokens x experts) per lane are faster until the grid runs short.
  // Measured on B200 (T, D, E): (8192, 2048, 64) 134 us with LE 16, EPL 4,
  // RT 4; (65536, 2048, 64) 660 us with RT 8.  A sweep of RT, EPL and warps
  // per block found nothing faster for 64 experts (LE 32 with EPL 2 and RT
  // 16, the largest register block, is 1.4-2x slower).  With 5-8 experts
  // (LE 8, EPL 1) blocks of 2 warps with RT 2 are fastest: (8192, 4096, 8)
  // 84 us against 104 us with 8-warp blocks.  With few blocks each 32-d
  // chunk costs about one global-load latency, so the latency-bound shapes
  // take 64-d chunks: (8192, 4096, 8) 68 us, (512, 4096, 8) 56 us (86 us with
  // 32-d chunks), (8192, 2048, 64) 126 us; with many tokens 32-d chunks stay
  // best ((65536, 2048, 64): 660 us against 826 us with 64-d chunks).
  int epl = 1, le = 1;
  if (E > 128) {
    epl = 8;
    le = 32;
  } else if (E > 64) {
    epl = 4;
    le = 32;
  } else if (E > 32) {
    epl = 4;
    le = 16;
  } else {
    while (le < E) le *= 2;
  }
  const int warps = (le == 8 && epl == 1) ? 2 : 8;
  auto tokens_per_block = [&](int rt) { return (int64_t)warps * (32 / le) * rt; };
  int rt = 1;
  int dch = kRouterDCh;
  if (warps == 2) {
    rt = 2;
    dch = 64;
  } else if (le == 16 && epl == 4) {  // 33-64 experts: swept at 8192 to 65536 tokens
    rt = T > 16384 ? 8 : 4;
    dch = T <= 8192 ? 64 : kRouterDCh;
  } else {
    for (int c = 16; c > 1; c /= 2)
      if (c <= le && c * epl <= 32 &&
          4 * ((T + tokens_per_block(c) - 1) / tokens_per_block(c)) >= 3 * (int64_t)num_sms()) {
        rt = c;
        break;
      }
  }
  p.ring = 0;
  p.le = le;
  p.epl = epl;
  p.rt = rt;
  p.warps = warps;
  p.dch = dch;
  p.tpb = tokens_per_block(rt);
  p.smem = (size_t)(p.tpb + le * epl) * (p.dch + 4) * 4;
  p.grid = (T + p.tpb - 1) / p.tpb;
  snprintf(p.name, sizeof(p.name), "k_router_topk<%d,%d,%d,%d>", rt, epl, warps, dch);
  return p;
}

int router_launch(const void* x, const void* wr, int64_t T, int64_t D, int E, int k,
                  int32_t* idx, float* w, cudaStream_t st) {
  RB_CHECK_ARG(T >= 0 && D > 0 && E >= 1 && E <= GMaxE && k >= 1 && k <= 16 && k <= E,
               "router: unsupported sizes (T=%lld D=%lld E=%d k=%d)", (long long)T,
               (long long)D, E, k);
  RB_CHECK_ARG(D % 8 == 0, "router: d_model must be a multiple of 8");
  if (T == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(x && wr && idx && w, "router: null pointer");
  RB_CHECK_ARG(aligned16(x), "router: x must be 16-byte aligned");
  RB_CHECK_ARG(E % 8 != 0 || aligned16(wr),
               "router: wr must be 16-byte aligned (its rows are read 8 experts at a time)");
  RB_CHECK_ARG(T < (1ll << 31) && D < (1ll << 31), "router: sizes exceed 2^31");
  RB_CHECK_ARG(E % 8 == 0 || E <= 128, "router: E=%d must be a multiple of 8 above 128", E);
  const RouterPlan pl = router_plan(T, E);
  const int le = pl.le, epl = pl.epl, rt = pl.rt, warps = pl.warps;
  const size_t smem = pl.smem;
  const int64_t grid = pl.grid;
  auto launch = [&](auto kern) -> int {
    if (smem > 48 * 1024)
      RB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<(unsigned)grid, warps * 32, smem, st>>>(static_cast<const uint16_t*>(x),
                                                       static_cast<const uint16_t*>(wr), (int)T,
                                                       (int)D, E, k, le, idx, w);
    return REMORA_B200_OK;
  };
  auto launch_ring = [&](auto kern) -> int {
    RB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<(unsigned)grid, warps * 32, smem, st>>>(static_cast<const uint16_t*>(x),
                                                       static_cast<const uint16_t*>(wr), (int)T,
                                                       (int)D, E, k, idx, w);
    return REMORA_B200_OK;
  };
  int rc;
  if (pl.ring) {
    switch (pl.ring) {
      case 1: rc = launch_ring(k_router_ring<2, 4, 1, 4, 128, 3>); break;
      case 2: rc = launch_ring(k_router_ring<4, 4, 1, 4, 64, 4>); break;
      case 3: rc = launch_ring(k_router_ring<8, 4, 2, 4, 64, 4>); break;
      case 4: rc = launch_ring(k_router_ring<16, 4, 2, 4, 64, 4>); break;
      case 5: rc = launch_ring(k_router_ring<16, 4, 4, 4, 64, 4>); break;
      default: rc = launch_ring(k_router_ring<8, 8, 4, 4, 64, 4>); break;
    }
    if (rc) return rc;
    RB_LAUNCH_CHECK();
    return REMORA_B200_OK;
  }
  switch (warps == 2 ? -1 : (pl.dch == 64 ? -2 : epl * 100 + rt)) {
    case -1: rc = launch(k_router_topk<2, 1, 2, 64>); break;
    case -2: rc = launch(k_router_topk<4, 4, 8, 64>); break;
    case 101: rc = launch(k_router_topk<1, 1, 8>); break;
    case 102: rc = launch(k_router_topk<2, 1, 8>); break;
    case 104: rc = launch(k_router_topk<4, 1, 8>); break;
    case 108: rc = launch(k_router_topk<8, 1, 8>); break;
    case 116: rc = launch(k_router_topk<16, 1, 8>); break;
    case 201: rc = launch(k_router_topk<1, 2, 8>); break;
    case 202: rc = launch(k_router_topk<2, 2, 8>); break;
    case 204: rc = launch(k_router_topk<4, 2, 8>); break;
    case 208: rc = launch(k_router_topk<8, 2, 8>); break;
    case 216: rc = launch(k_router_topk<16, 2, 8>); break;
    case 401: rc = launch(k_router_topk<1, 4, 8>); break;
    case 402: rc = launch(k_router_topk<2, 4, 8>); break;
    case 404: rc = launch(k_router_topk<4, 4, 8>); break;
    case 408: rc = launch(k_router_topk<8, 4, 8>); break;
    case 801: rc = launch(k_router_topk<1, 8, 8>); break;
    case 802: rc = launch(k_router_topk<2, 8, 8>); break;
    default: rc = launch(k_router_topk<4, 8, 8>); break;
  }
  if (rc) return rc;
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

size_t dispatch_ws_bytes(int64_t T, int k, int E) {
  return align256((size_t)dispatch_blocks(T * k) * E * 4);
}

int dispatch_launch(const int32_t* idx, int64_t T, int k, int E, int32_t* counts,
                    int32_t* offsets, int32_t* perm, int32_t* inv, int32_t* block_counts,
                    cudaStream_t st) {
  const int64_t n = T * k;
  const int64_t nb = dispatch_blocks(n);
  RB_CHECK_ARG(nb < (1 << 30), "dispatch: too many entries");
  if (n == 0) {
    RB_CHECK_ARG(counts && offsets, "dispatch: null pointer");
    RB_CUDA(cudaMemsetAsync(counts, 0, sizeof(int32_t) * E, st));
    RB_CUDA(cudaMemsetAsync(offsets, 0, sizeof(int32_t) * (E + 1), st));
    return REMORA_B200_OK;
  }
  k_dispatch_count<<<(unsigned)nb, kDispThreads, E * sizeof(int), st>>>(idx, n, E, block_counts);
  RB_LAUNCH_CHECK();
  k_dispatch_scan<<<1, kScanThreads, 0, st>>>(block_counts, (int)nb, E, counts, offsets);
  RB_LAUNCH_CHECK();
  k_dispatch_scatter<<<(unsigned)nb, kDispThreads, 32 * E * sizeof(int), st>>>(
      idx, n, E, block_counts, offsets, perm, inv);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

int gather_launch(const void* x, const int32_t* perm, int64_t rows, int k, int64_t D, void* xs,
                  cudaStream_t st) {
  RB_CHECK_ARG(rows >= 0 && k >= 1 && D > 0 && D % 8 == 0, "gather: bad sizes");
  if (rows == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(x && perm && xs && aligned16(x) && aligned16(xs),
               "gather: null or unaligned pointer");
  const int64_t want = (rows + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  k_gather_rows<<<(unsigned)(want < cap ? want : cap), 256, 0, st>>>(
      static_cast<const uint16_t*>(x), perm, rows, k, (int)D, static_cast<uint16_t*>(xs));
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

int scatter_launch(const void* x, const int32_t* inv, int64_t T, int k, int64_t D, void* xs,
                   cudaStream_t st) {
  RB_CHECK_ARG(T >= 0 && k >= 1 && D > 0 && D % 8 == 0, "scatter: bad sizes");
  if (T == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(x && inv && xs && aligned16(x) && aligned16(xs),
               "scatter: null or unaligned pointer");
  const int64_t want = (T + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  k_scatter_rows<<<(unsigned)(want < cap ? want : cap), 256, 0, st>>>(
      static_cast<const uint16_t*>(x), inv, T, k, (int)D, static_cast<uint16_t*>(xs));
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

// Grouped GEMM over expert row segments.  a [rows, K]; b0 (and b1 for the
// SwiGLU form) [E, K, N]; out [rows, N].  offsets [E+1] on the device.
int grouped_launch(bool swiglu, const void* a, const void* b0, const void* b1, void* out,
                   const int32_t* offsets, int64_t rows, int64_t K, int64_t N, int E,
                   cudaStream_t st, const int32_t* seg_expert = nullptr, int n_seg = -1,
                   const int32_t* seg_start = nullptr, const int32_t* seg_end = nullptr,
                   const int32_t* dst_row = nullptr, const int32_t* dst_rank = nullptr,
                   const PeerPtrs* dst = nullptr) {
  const int cols = swiglu ? 128 : 256;
  const int S = n_seg < 0 ? E : n_seg;
  RB_CHECK_ARG(E >= 1 && E <= GMaxE, "grouped_gemm: E=%d unsupported (1..%d)", E, GMaxE);
  RB_CHECK_ARG(S >= 1 && S <= GMaxE, "grouped_gemm: %d segments unsupported (1..%d)", S, GMaxE);
  RB_CHECK_ARG(rows >= 0 && K > 0 && N > 0 && K % 8 == 0 && N % 32 == 0,
               "grouped_gemm: need K %% 8 == 0 and N %% 32 == 0 (K=%lld N=%lld)", (long long)K,
               (long long)N);
  RB_CHECK_ARG(rows < (1ll << 31) && K < (1ll << 31) && N < (1ll << 31),
               "grouped_gemm: sizes exceed 2^31");
  if (rows == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(a && b0 && (out || dst) && (offsets || (seg_start && seg_end)) &&
                   (!swiglu || b1),
               "grouped_gemm: null pointer");
  RB_CHECK_ARG(aligned16(a) && aligned16(b0) && (!out || aligned16(out)) &&
                   (!swiglu || aligned16(b1)),
               "grouped_gemm: pointers must be 16-byte aligned");
  CUtensorMap tA, tB0, tB1;
  int rc;
  {
    uint64_t d[2] = {(uint64_t)K, (uint64_t)rows};
    uint64_t s[1] = {(uint64_t)K * 2};
    uint32_t box[2] = {GBK, GBM};
    if ((rc = make_tmap(&tA, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, s, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  uint64_t d[3] = {(uint64_t)N, (uint64_t)K, (uint64_t)E};
  uint64_t s[2] = {(uint64_t)N * 2, (uint64_t)K * N * 2};
  uint32_t box[3] = {64, GBK, 1};
  if ((rc = make_tmap(&tB0, b0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  if ((rc = make_tmap(&tB1, swiglu ? b1 : b0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, s, box,
                      CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc;
  GroupShape sh;
  sh.K = (int)K;
  sh.N = (int)N;
  sh.E = E;
  sh.S = S;
  sh.seg_expert = seg_expert;
  sh.tiles_n = (int)((N + cols - 1) / cols);
  sh.num_kb = (int)((K + GBK - 1) / GBK);
  sh.seg_start = seg_start ? seg_start : offsets;
  sh.seg_end = seg_end ? seg_end : offsets + 1;
  sh.seg_dst_row = dst ? dst_row : nullptr;
  sh.seg_dst_rank = dst ? dst_rank : nullptr;
  sh.dst = dst ? *dst : PeerPtrs{};
  sh.out = static_cast<uint16_t*>(out);
  // upper bound of the tile count: sum over experts of ceil(n_e / 128)
  const int64_t max_tiles = (rows / GBM + S) * (int64_t)sh.tiles_n;
  int grid = num_sms();
  if (grid > max_tiles) grid = (int)max_tiles;
  if (swiglu) {
    RB_CUDA(cudaFuncSetAttribute(k_grouped_gemm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 GSmemBytes));
    k_grouped_gemm<true><<<grid, GThreads, GSmemBytes, st>>>(tA, tB0, tB1, sh);
  } else {
    RB_CUDA(cudaFuncSetAttribute(k_grouped_gemm<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, GSmemBytes));
    k_grouped_gemm<false><<<grid, GThreads, GSmemBytes, st>>>(tA, tB0, tB1, sh);
  }
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

int combine_launch(const void* y, const int32_t* inv, const float* w, int64_t T, int k,
                   int64_t D, void* out, cudaStream_t st) {
  RB_CHECK_ARG(T >= 0 && k >= 1 && k <= 16 && D > 0 && D % 8 == 0, "combine: bad sizes");
  if (T == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(y && inv && w && out && aligned16(y) && aligned16(out),
               "combine: null or unaligned pointer");
  const int64_t want = (T + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  const uint16_t* yy = static_cast<const uint16_t*>(y);
  uint16_t* oo = static_cast<uint16_t*>(out);
  if (k <= 2)
    k_combine<2><<<grid, 256, 0, st>>>(yy, inv, w, T, k, (int)D, oo);
  else if (k <= 4)
    k_combine<4><<<grid, 256, 0, st>>>(yy, inv, w, T, k, (int)D, oo);
  else if (k <= 8)
    k_combine<8><<<grid, 256, 0, st>>>(yy, inv, w, T, k, (int)D, oo);
  else
    k_combine<16><<<grid, 256, 0, st>>>(yy, inv, w, T, k, (int)D, oo);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

// Workspace layout of the fused layer (each piece 256-byte aligned).
struct LayerWs {
  int32_t *idx, *counts, *offsets, *perm, *inv, *block_counts;
  float* w;
  uint16_t *xs, *h, *y;  // dispatched rows [T*k, D], SwiGLU [T*k, F], expert outputs [T*k, D]
  size_t bytes;
};

inline LayerWs layer_ws(void* base, int64_t T, int64_t D, int64_t F, int E, int k) {
  LayerWs L;
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
  L.h = reinterpret_cast<uint16_t*>(take(n * F * 2));
  L.y = reinterpret_cast<uint16_t*>(take(n * D * 2));
  L.bytes = o;
  return L;
}

// The layer's launches on one stream over a carved workspace (sizes checked
// by the callers).
int layer_run(const void* x, const void* wr, const void* wg, const void* wu, const void* wd,
              void* out, int64_t T, int64_t D, int64_t F, int E, int k, const LayerWs& L,
              cudaStream_t st) {
  const int64_t n = T * k;
  int rc;
  if ((rc = router_launch(x, wr, T, D, E, k, L.idx, L.w, st))) return rc;
  if ((rc = dispatch_launch(L.idx, T, k, E, L.counts, L.offsets, L.perm, L.inv, L.block_counts,
                            st)))
    return rc;
  if ((rc = scatter_launch(x, L.inv, T, k, D, L.xs, st))) return rc;
  if ((rc = grouped_launch(true, L.xs, wg, wu, L.h, L.offsets, n, D, F, E, st))) return rc;
  if ((rc = grouped_launch(false, L.h, wd, nullptr, L.y, L.offsets, n, F, D, E, st))) return rc;
  return combine_launch(L.y, L.inv, L.w, T, k, D, out, st);
}

int layer_check(const void* x, const void* wr, const void* wg, const void* wu, const void* wd,
                const void* out, int64_t T, int64_t D, int64_t F, int E, int k) {
  RB_CHECK_ARG(T >= 0 && D > 0 && F > 0 && E >= 1 && E <= GMaxE && k >= 1 && k <= 16 && k <= E,
               "moe_layer: bad sizes");
  RB_CHECK_ARG(T <= INT32_MAX / k, "moe_layer: T*k exceeds the int32 range of the routing tables");
  RB_CHECK_ARG(T == 0 || (x && wr && wg && wu && wd && out), "moe_layer: null pointer");
  return REMORA_B200_OK;
}

// Copy streams and events of the host-buffer layer, one set per (thread,
// device), created on first use and kept for the life of the thread; made
// again when the device's context has changed (after a cudaDeviceReset the
// old handles belong to a destroyed context).
struct HostPipe {
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t start = nullptr, h2d[2] = {}, done[2] = {}, d2h[2] = {};
  unsigned long long ctx_id = 0;
};

int host_pipe(HostPipe** out) {
  static thread_local HostPipe pipes[16];
  int dev = 0;
  RB_CUDA(cudaGetDevice(&dev));
  RB_CHECK_ARG(dev >= 0 && dev < 16, "moe_layer_host: device %d out of range", dev);
  HostPipe& p = pipes[dev];
  const unsigned long long ctx = current_ctx_id();
  if (p.up && ctx != p.ctx_id) p = HostPipe{};
  if (!p.up) {  // built whole before it is kept, so a failed call leaves no half set
    HostPipe q;
    RB_CUDA(cudaStreamCreateWithFlags(&q.up, cudaStreamNonBlocking));
    RB_CUDA(cudaStreamCreateWithFlags(&q.down, cudaStreamNonBlocking));
    RB_CUDA(cudaEventCreateWithFlags(&q.start, cudaEventDisableTiming));
    for (int i = 0; i < 2; ++i) {
      RB_CUDA(cudaEventCreateWithFlags(&q.h2d[i], cudaEventDisableTiming));
      RB_CUDA(cudaEventCreateWithFlags(&q.done[i], cudaEventDisableTiming));
      RB_CUDA(cudaEventCreateWithFlags(&q.d2h[i], cudaEventDisableTiming));
    }
    q.ctx_id = current_ctx_id();  // the context exists now
    p = q;
  }
  *out = &p;
  return REMORA_B200_OK;
}

constexpr int64_t kHostChunkTokens = 16384;

int64_t host_chunk(int64_t T, int64_t chunk_tokens) {
  const int64_t c = chunk_tokens > 0 ? chunk_tokens : kHostChunkTokens;
  return T < c ? (T > 0 ? T : 1) : c;
}

// Workspace of the host-buffer layer: the layer workspace of one chunk, then
// two token buffers and two output buffers of one chunk each.
size_t host_ws_bytes(int64_t chunk, int64_t D, int64_t F, int E, int k) {
  return layer_ws(nullptr, chunk, D, F, E, k).bytes + 4 * align256((size_t)chunk * D * 2);
}

}  // namespace moe
}  // namespace rb

using namespace rb;
using namespace rb::moe;

extern "C" int remora_b200_moe_router_topk_bf16(const void* x, const void* wr, int64_t T,
                                                int64_t D, int E, int k, int32_t* idx, float* w,
                                                void* stream) {
  clear_error();
  return router_launch(x, wr, T, D, E, k, idx, w, as_stream(stream));
}

extern "C" size_t remora_b200_moe_dispatch_workspace_bytes(int64_t T, int k, int E) {
  if (T < 0 || k < 1 || E < 1 || T > INT32_MAX / k) return 0;  // the dispatch rejects these
  return dispatch_ws_bytes(T, k, E);
}

extern "C" int remora_b200_moe_dispatch(const int32_t* idx, int64_t T, int k, int E,
                                        int32_t* counts, int32_t* offsets, int32_t* perm,
                                        int32_t* inv, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  clear_error();
  RB_CHECK_ARG(T >= 0 && k >= 1 && E >= 1 && E <= GMaxE, "dispatch: bad sizes");
  RB_CHECK_ARG(T <= INT32_MAX / k,
               "dispatch: T*k = %lld*%d exceeds the int32 range of perm and inv", (long long)T,
               k);
  RB_CHECK_ARG(T * k == 0 || (idx && counts && offsets && perm && inv && workspace),
               "dispatch: null pointer");
  RB_CHECK_ARG(workspace_bytes >= dispatch_ws_bytes(T, k, E) || T * k == 0,
               "dispatch: workspace of %zu bytes, %zu needed", workspace_bytes,
               dispatch_ws_bytes(T, k, E));
  return dispatch_launch(idx, T, k, E, counts, offsets, perm, inv,
                         static_cast<int32_t*>(workspace), as_stream(stream));
}

extern "C" int remora_b200_moe_gather(const void* x, const int32_t* perm, int64_t rows, int k,
                                      int64_t D, void* xs, void* stream) {
  clear_error();
  return gather_launch(x, perm, rows, k, D, xs, as_stream(stream));
}

extern "C" int remora_b200_moe_scatter(const void* x, const int32_t* inv, int64_t T, int k,
                                       int64_t D, void* xs, void* stream) {
  clear_error();
  return scatter_launch(x, inv, T, k, D, xs, as_stream(stream));
}

extern "C" int remora_b200_grouped_gemm_swiglu_bf16(const void* xs, const void* wg,
                                                    const void* wu, void* h,
                                                    const int32_t* offsets, int64_t rows,
                                                    int64_t D, int64_t F, int E, void* stream) {
  clear_error();
  return grouped_launch(true, xs, wg, wu, h, offsets, rows, D, F, E, as_stream(stream));
}

extern "C" int remora_b200_grouped_gemm_bf16(const void* a, const void* w, void* y,
                                             const int32_t* offsets, int64_t rows, int64_t K,
                                             int64_t N, int E, void* stream) {
  clear_error();
  return grouped_launch(false, a, w, nullptr, y, offsets, rows, K, N, E, as_stream(stream));
}

extern "C" int remora_b200_grouped_gemm_swiglu_segments_bf16(
    const void* xs, const void* wg, const void* wu, void* h, const int32_t* seg_offsets,
    const int32_t* seg_expert, int n_seg, int64_t rows, int64_t D, int64_t F, int E,
    void* stream) {
  clear_error();
  RB_CHECK_ARG(seg_expert, "grouped_gemm_segments: null seg_expert");
  return grouped_launch(true, xs, wg, wu, h, seg_offsets, rows, D, F, E, as_stream(stream),
                        seg_expert, n_seg);
}

extern "C" int remora_b200_grouped_gemm_segments_bf16(const void* a, const void* w, void* y,
                                                      const int32_t* seg_offsets,
                                                      const int32_t* seg_expert, int n_seg,
                                                      int64_t rows, int64_t K, int64_t N, int E,
                                                      void* stream) {
  clear_error();
  RB_CHECK_ARG(seg_expert, "grouped_gemm_segments: null seg_expert");
  return grouped_launch(false, a, w, nullptr, y, seg_offsets, rows, K, N, E, as_stream(stream),
                        seg_expert, n_seg);
}

extern "C" int remora_b200_moe_combine_bf16(const void* y, const int32_t* inv, const float* w,
                                            int64_t T, int k, int64_t D, void* out,
                                            void* stream) {
  clear_error();
  return combine_launch(y, inv, w, T, k, D, out, as_stream(stream));
}

extern "C" size_t remora_b200_moe_workspace_bytes(int64_t T, int64_t D, int64_t F, int E, int k) {
  return layer_ws(nullptr, T, D, F, E, k).bytes;
}

extern "C" int remora_b200_moe_layer_bf16(const void* x, const void* wr, const void* wg,
                                          const void* wu, const void* wd, void* out, int64_t T,
                                          int64_t D, int64_t F, int E, int k, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  clear_error();
  int rc;
  if ((rc = layer_check(x, wr, wg, wu, wd, out, T, D, F, E, k))) return rc;
  if (T == 0) return REMORA_B200_OK;
  RB_CHECK_ARG(workspace, "moe_layer: null workspace");
  LayerWs L = layer_ws(workspace, T, D, F, E, k);
  RB_CHECK_ARG(workspace_bytes >= L.bytes, "moe_layer: workspace of %zu bytes, %zu needed",
               workspace_bytes, L.bytes);
  RB_CHECK_ARG(aligned16(workspace), "moe_layer: workspace must be 16-byte aligned");
  return layer_run(x, wr, wg, wu, wd, out, T, D, F, E, k, L, as_stream(stream));
}

extern "C" size_t remora_b200_moe_layer_host_workspace_bytes(int64_t T, int64_t D, int64_t F,
                                                             int E, int k, int64_t chunk_tokens) {
  if (T < 0 || D <= 0 || F <= 0 || E < 1 || E > GMaxE || k < 1 || k > 16 || k > E ||
      chunk_tokens < 0 || T > INT32_MAX / k)
    return 0;
  return host_ws_bytes(host_chunk(T, chunk_tokens), D, F, E, k);
}

extern "C" int remora_b200_moe_layer_host_bf16(const void* x_host, const void* wr, const void* wg,
                                               const void* wu, const void* wd, void* out_host,
                                               int64_t T, int64_t D, int64_t F, int E, int k,
                                               int64_t chunk_tokens, void* workspace,
                                               size_t workspace_bytes, void* stream) {
  clear_error();
  int rc;
  if ((rc = layer_check(x_host, wr, wg, wu, wd, out_host, T, D, F, E, k))) return rc;
  RB_CHECK_ARG(chunk_tokens >= 0, "moe_layer_host: chunk_tokens must be >= 0");
  if (T == 0) return REMORA_B200_OK;
  const int64_t C = host_chunk(T, chunk_tokens);
  RB_CHECK_ARG(workspace && aligned16(workspace), "moe_layer_host: null or unaligned workspace");
  RB_CHECK_ARG(workspace_bytes >= host_ws_bytes(C, D, F, E, k),
               "moe_layer_host: workspace of %zu bytes, %zu needed", workspace_bytes,
               host_ws_bytes(C, D, F, E, k));
  LayerWs L = layer_ws(workspace, C, D, F, E, k);
  uint8_t* bufs = static_cast<uint8_t*>(workspace) + L.bytes;
  const size_t cb = align256((size_t)C * D * 2);
  uint8_t* xb[2] = {bufs, bufs + cb};
  uint8_t* ob[2] = {bufs + 2 * cb, bufs + 3 * cb};
  HostPipe* p = nullptr;
  if ((rc = host_pipe(&p))) return rc;
  cudaStream_t st = as_stream(stream);
  // Copies start after the caller's earlier work on `stream`; chunk c's
  // tokens go up on one stream while chunk c-1 computes on `stream` and chunk
  // c-2's output comes down on another; buffers are reused two chunks later.
  RB_CUDA(cudaEventRecord(p->start, st));
  RB_CUDA(cudaStreamWaitEvent(p->up, p->start, 0));
  RB_CUDA(cudaStreamWaitEvent(p->down, p->start, 0));
  // Chunk sizes: with T >= 2C the first two chunks are C/4 and C/2 and the last
  // two C/2 and C/4, so the copy in of the first chunk and the copy out of the
  // last one, which nothing overlaps, are short; the rest is split into
  // near-equal chunks of at most C.
  int64_t sizes[64];
  int nc = 0;
  const int64_t mid = T - 2 * (C / 4 + C / 2);
  const int64_t nm = (mid + C - 1) / C;
  if (T >= 2 * C && C >= 4 && nm <= 60) {
    const int64_t head[2] = {C / 4, C / 2};
    sizes[nc++] = head[0];
    sizes[nc++] = head[1];
    for (int64_t i = 0; i < nm; ++i) sizes[nc++] = mid / nm + (i < mid % nm ? 1 : 0);
    sizes[nc++] = head[1];
    sizes[nc++] = head[0];
  }
  int64_t t0 = 0;
  int last = 0;
  for (int c = 0; t0 < T; ++c) {
    const int b = c & 1;
    const int64_t tc = c < nc ? sizes[c] : std::min<int64_t>(C, T - t0);
    const size_t bytes = (size_t)tc * D * 2;
    if (c >= 2) RB_CUDA(cudaStreamWaitEvent(p->up, p->done[b], 0));
    RB_CUDA(cudaMemcpyAsync(xb[b], static_cast<const uint8_t*>(x_host) + (size_t)t0 * D * 2,
                            bytes, cudaMemcpyHostToDevice, p->up));
    RB_CUDA(cudaEventRecord(p->h2d[b], p->up));
    RB_CUDA(cudaStreamWaitEvent(st, p->h2d[b], 0));
    if (c >= 2) RB_CUDA(cudaStreamWaitEvent(st, p->d2h[b], 0));
    if ((rc = layer_run(xb[b], wr, wg, wu, wd, ob[b], tc, D, F, E, k, L, st))) return rc;
    RB_CUDA(cudaEventRecord(p->done[b], st));
    RB_CUDA(cudaStreamWaitEvent(p->down, p->done[b], 0));
    RB_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(out_host) + (size_t)t0 * D * 2, ob[b], bytes,
                            cudaMemcpyDeviceToHost, p->down));
    RB_CUDA(cudaEventRecord(p->d2h[b], p->down));
    t0 += tc;
    last = b;
  }
  // the call is complete on `stream` once the last output chunk is down
  RB_CUDA(cudaStreamWaitEvent(st, p->d2h[last], 0));
  return REMORA_B200_OK;
}

