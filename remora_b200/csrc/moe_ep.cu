// moe_ep.cu -- expert-parallel dispatch and combine over NVLink peer memory.
//
// Each rank owns, in memory every peer can address (remora_b200_peer_alloc):
//   recv  [P][cap][D] bf16  region s receives the rows rank s routes here
//   meta  [P][Epr+1]  int32 region s: rows per local expert, then the row
//                            of rank s's dispatch order they start at
//   y     [T_local*k][D]    the expert outputs of this rank's own rows,
//                            written back by the ranks that computed them
//   flags [P]         int32 barrier epochs, slot s written by rank s
// A layer: scatter (this rank's dispatched rows -> peers' recv, no local
// gather copy, no host round trip) -> barrier -> grouped GEMMs over
// (source, local expert) segments, the down GEMM storing each output row
// straight into its source rank's y -> barrier -> local combine.
// Plain loads and stores to peer addresses only (no TMA, no multicast).
// The barrier's waits are bounded: after the limit the kernel records
// error 1 in the device error word and returns.
#include "runtime.cuh"

namespace rb {
namespace moe {

// Rows of this rank in dispatch order p = 0 .. n-1 (expert-sorted); the
// destination rank is e / Epr, the row index inside region `rank` of that
// peer is p - offsets[q * Epr].  Token row = perm[p] / k.
__global__ void k_ep_scatter(const uint16_t* __restrict__ x, const int32_t* __restrict__ perm,
                             const int32_t* __restrict__ offsets, int64_t n, int k, int D,
                             int Epr, int P, int rank, int64_t cap, PeerPtrs recv,
                             PeerPtrs meta) {
  // metadata first (block 0): counts per local expert and the base row
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < P * (Epr + 1); i += blockDim.x) {
      const int q = i / (Epr + 1), j = i % (Epr + 1);
      const int v = j < Epr ? offsets[q * Epr + j + 1] - offsets[q * Epr + j] : offsets[q * Epr];
      reinterpret_cast<int32_t*>(meta.p[q])[rank * (Epr + 1) + j] = v;
    }
  }
  const int lane = threadIdx.x & 31;
  const int64_t wpb = blockDim.x >> 5;
  for (int64_t p = blockIdx.x * wpb + (threadIdx.x >> 5); p < n; p += (int64_t)gridDim.x * wpb) {
    // destination rank: the last q with offsets[q * Epr] <= p
    int q = 0;
    while (q + 1 < P && offsets[(q + 1) * Epr] <= p) ++q;
    const int64_t i = p - offsets[q * Epr];
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)(perm[p] / k) * D);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(recv.p[q]) +
                                          ((int64_t)rank * cap + i) * D);
    // up to 8 pieces of 16 bytes in flight per lane before they are stored
    for (int c0 = 0; c0 < D / 8; c0 += 8 * 32) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < D / 8) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < D / 8) dst[c] = v[u];
      }
    }
  }
}

// Barrier over P ranks: publish `epoch` in every peer's flag slot `rank`,
// then wait (bounded) until every slot of this rank's flags holds >= epoch.
__global__ void k_ep_barrier(int32_t* flags, PeerPtrs peer_flags, int P, int rank, int epoch) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  __threadfence_system();  // this rank's earlier stores (previous kernels) first
  if (lane < P) {
    int32_t* f = reinterpret_cast<int32_t*>(peer_flags.p[lane]) + rank;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
  if (lane < P) {
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
      int32_t v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + lane) : "memory");
      if (v - epoch >= 0) break;
      if ((it & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) {
        atomicExch(&g_device_error, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncwarp();
  __threadfence_system();
}

// Segments of the received rows, (source s, local expert e) in that order:
// start = s*cap + rows of s for experts < e, end = start + count, expert e,
// output row in s's y = base_s + rows of s for experts < e.
__global__ void k_ep_segments(const int32_t* __restrict__ meta, int P, int Epr, int64_t cap,
                              int32_t* seg_start, int32_t* seg_end, int32_t* seg_expert,
                              int32_t* seg_dst_row, int32_t* seg_dst_rank) {
  for (int s = threadIdx.x; s < P; s += blockDim.x) {
    const int32_t* m = meta + s * (Epr + 1);
    int32_t run = 0;
    for (int e = 0; e < Epr; ++e) {
      const int q = s * Epr + e;
      seg_start[q] = (int32_t)(s * cap) + run;
      seg_end[q] = seg_start[q] + m[e];
      seg_expert[q] = e;
      seg_dst_row[q] = m[Epr] + run;
      seg_dst_rank[q] = s;
      run += m[e];
    }
  }
}

// Metadata exchange of the fused path, one warp: publish this rank's
// per-expert row counts (and its base row) in region `rank` of every peer's
// meta, zero the scatter completion counters done[E], barrier on `epoch`, then build
// the segment table from the received meta with the sources in the order
// the fused scatter delivers them: rank, rank-1, ..., rank-P+1 (mod P).
// Segment j*Epr + e is (source s = rank - j, local expert e); the source
// doubles as the rank whose ready flag the SwiGLU producer waits for and
// the rank the down GEMM's output rows go to.  If the barrier runs out of
// time, error 1 is recorded and every segment is left empty.
__global__ void k_ep_meta(const int32_t* __restrict__ offsets, int P, int Epr, int rank,
                          int64_t cap, PeerPtrs meta, const int32_t* meta_local, int32_t* flags,
                          PeerPtrs peer_flags, int epoch, int32_t* done, int32_t* seg_start,
                          int32_t* seg_end, int32_t* seg_expert, int32_t* seg_dst_row,
                          int32_t* seg_src) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  for (int i = lane; i < P * (Epr + 1); i += 32) {
    const int q = i / (Epr + 1), j = i % (Epr + 1);
    const int v = j < Epr ? offsets[q * Epr + j + 1] - offsets[q * Epr + j] : offsets[q * Epr];
    reinterpret_cast<int32_t*>(meta.p[q])[rank * (Epr + 1) + j] = v;
  }
  for (int e = lane; e < P * Epr; e += 32) done[e] = 0;
  __threadfence_system();
  __syncwarp();
  bool ok = true;
  if (lane < P) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(
                     reinterpret_cast<int32_t*>(peer_flags.p[lane]) + rank),
                 "r"(epoch)
                 : "memory");
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
      int32_t v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + lane) : "memory");
      if (v - epoch >= 0) break;
      if ((it & 63u) == 63u && globaltimer() - t0 > kWaitLimitNs) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  if (!ok && lane == 0) atomicExch(&g_device_error, 1);
  if (lane < P) {
    const int s = lane;
    const int j = (rank - s + P) % P;
    const int32_t* m = meta_local + s * (Epr + 1);
    int32_t run = 0;
    for (int e = 0; e < Epr; ++e) {
      const int q = j * Epr + e;
      const int32_t c = ok ? m[e] : 0;
      seg_start[q] = (int32_t)(s * cap) + run;
      seg_end[q] = seg_start[q] + c;
      seg_expert[q] = e;
      seg_dst_row[q] = (ok ? m[Epr] : 0) + run;
      seg_src[q] = s;
      run += c;
    }
  }
}

}  // namespace moe
}  // namespace rb

using namespace rb;
using namespace rb::moe;

namespace {

int peer_ptrs(const uint64_t* host, int P, PeerPtrs* out, const char* what) {
  RB_CHECK_ARG(host, "moe_ep: null %s address list", what);
  *out = PeerPtrs{};
  for (int i = 0; i < P; ++i) {
    RB_CHECK_ARG(host[i] != 0 && (host[i] & 15u) == 0, "moe_ep: %s address of rank %d is null "
                 "or not 16-byte aligned", what, i);
    out->p[i] = host[i];
  }
  return REMORA_B200_OK;
}

}  // namespace

extern "C" int remora_b200_moe_ep_scatter_bf16(const void* x, const int32_t* perm,
                                               const int32_t* offsets, int64_t n, int k,
                                               int64_t D, int E, int P, int rank, int64_t cap,
                                               const uint64_t* recv_ptrs,
                                               const uint64_t* meta_ptrs, void* stream) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && P <= 8 && rank >= 0 && rank < P && E % P == 0 && E <= GMaxE,
               "moe_ep_scatter: bad P=%d rank=%d E=%d", P, rank, E);
  RB_CHECK_ARG(n >= 0 && k >= 1 && D > 0 && D % 8 == 0 && cap >= 0 && n <= cap,
               "moe_ep_scatter: bad sizes");
  RB_CHECK_ARG((int64_t)P * cap < (1ll << 31), "moe_ep_scatter: P*cap exceeds 2^31 rows");
  PeerPtrs rp, mp;
  int rc;
  if ((rc = peer_ptrs(recv_ptrs, P, &rp, "recv")) || (rc = peer_ptrs(meta_ptrs, P, &mp, "meta")))
    return rc;
  RB_CHECK_ARG(offsets && (n == 0 || (x && perm && aligned16(x))),
               "moe_ep_scatter: null or unaligned pointer");
  const int64_t want = (n + 7) / 8 + 1;
  const int64_t cap_blocks = (int64_t)num_sms() * 16;
  k_ep_scatter<<<(unsigned)(want < cap_blocks ? want : cap_blocks), 256, 0, as_stream(stream)>>>(
      static_cast<const uint16_t*>(x), perm, offsets, n, k, (int)D, E / P, P, rank, cap, rp, mp);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

extern "C" int remora_b200_moe_ep_barrier(int32_t* flags, const uint64_t* flag_ptrs, int P,
                                          int rank, int epoch, void* stream) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && P <= 8 && rank >= 0 && rank < P && flags,
               "moe_ep_barrier: bad arguments");
  PeerPtrs fp = PeerPtrs{};
  RB_CHECK_ARG(flag_ptrs, "moe_ep_barrier: null flag address list");
  for (int i = 0; i < P; ++i) {
    RB_CHECK_ARG(flag_ptrs[i] != 0 && (flag_ptrs[i] & 3u) == 0, "moe_ep_barrier: bad address");
    fp.p[i] = flag_ptrs[i];
  }
  k_ep_barrier<<<1, 32, 0, as_stream(stream)>>>(flags, fp, P, rank, epoch);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

extern "C" int remora_b200_moe_ep_segments(const int32_t* meta, int P, int Epr, int64_t cap,
                                           int32_t* seg, void* stream) {
  clear_error();
  RB_CHECK_ARG(meta && seg && P >= 1 && P <= 8 && Epr >= 1 && P * Epr <= GMaxE,
               "moe_ep_segments: bad arguments");
  const int S = P * Epr;
  k_ep_segments<<<1, 32, 0, as_stream(stream)>>>(meta, P, Epr, cap, seg, seg + S, seg + 2 * S,
                                                 seg + 3 * S, seg + 4 * S);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

// The local experts over the received rows: SwiGLU grouped GEMM into h
// (same row layout as recv), then the down GEMM storing every output row
// into its source rank's y (seg = the 5*S table of remora_b200_moe_ep_segments).
extern "C" int remora_b200_moe_ep_experts_bf16(const void* recv, const void* wg, const void* wu,
                                               const void* wd, void* h, const int32_t* seg,
                                               int P, int Epr, int64_t cap, int64_t D,
                                               int64_t F, const uint64_t* y_ptrs,
                                               void* stream) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && P <= 8 && Epr >= 1 && P * Epr <= GMaxE && seg,
               "moe_ep_experts: bad arguments");
  PeerPtrs yp;
  int rc;
  if ((rc = peer_ptrs(y_ptrs, P, &yp, "y"))) return rc;
  const int S = P * Epr;
  const int64_t rows = (int64_t)P * cap;
  cudaStream_t st = as_stream(stream);
  if ((rc = grouped_launch(true, recv, wg, wu, h, nullptr, rows, D, F, Epr, st, seg + 2 * S, S,
                           seg, seg + S)))
    return rc;
  return grouped_launch(false, h, wd, nullptr, nullptr, nullptr, rows, F, D, Epr, st,
                        seg + 2 * S, S, seg, seg + S, seg + 3 * S, seg + 4 * S, &yp);
}

// Fused path, step 1: metadata exchange + barrier + segment table + zeroed
// completion counters (one small kernel).
extern "C" int remora_b200_moe_ep_meta(const int32_t* offsets, int P, int E, int rank,
                                       int64_t cap, const uint64_t* meta_ptrs,
                                       const int32_t* meta_local, int32_t* flags,
                                       const uint64_t* flag_ptrs, int epoch, int32_t* done,
                                       int32_t* seg, void* stream) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && P <= 8 && rank >= 0 && rank < P && E % P == 0 && E <= GMaxE && cap >= 0,
               "moe_ep_meta: bad P=%d rank=%d E=%d", P, rank, E);
  RB_CHECK_ARG(offsets && meta_local && flags && done && seg, "moe_ep_meta: null pointer");
  RB_CHECK_ARG((int64_t)P * cap < (1ll << 31), "moe_ep_meta: P*cap exceeds 2^31 rows");
  PeerPtrs mp, fp;
  int rc;
  if ((rc = peer_ptrs(meta_ptrs, P, &mp, "meta")) || (rc = peer_ptrs(flag_ptrs, P, &fp, "flag")))
    return rc;
  const int Epr = E / P, S = E;
  k_ep_meta<<<1, 32, 0, as_stream(stream)>>>(offsets, P, Epr, rank, cap, mp, meta_local, flags, fp,
                                             epoch, done, seg, seg + S, seg + 2 * S, seg + 3 * S,
                                             seg + 4 * S);
  RB_LAUNCH_CHECK();
  return REMORA_B200_OK;
}

// Fused path, steps 2 and 3 in one kernel: scatter + SwiGLU + down (see
// moe_ep_experts.cu).  mt_done: [P*cap/128 + E + 1] int32 scratch (zeroed
// here, stream-ordered).
extern "C" int remora_b200_moe_ep_experts_fused_bf16(
    const void* x, const int32_t* perm, const int32_t* offsets, int64_t n, int k, int64_t D,
    int64_t F, int E, int P, int rank, int64_t cap, const uint64_t* recv_ptrs,
    const uint64_t* ready_ptrs, const int32_t* ready_local, int32_t* done, int epoch,
    const void* recv_local, const void* wg, const void* wu, const void* wd, void* h,
    const int32_t* seg, int32_t* mt_done, const uint64_t* y_ptrs, void* stream) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && P <= 8 && rank >= 0 && rank < P && E % P == 0 && E <= GMaxE,
               "moe_ep_experts_fused: bad P=%d rank=%d E=%d", P, rank, E);
  RB_CHECK_ARG(n >= 0 && n <= cap && k >= 1 && cap > 0 && D > 0 && F > 0 && D % 32 == 0 &&
                   F % 32 == 0,
               "moe_ep_experts_fused: bad sizes (D, F multiples of 32)");
  RB_CHECK_ARG((int64_t)P * cap < (1ll << 31) && D < (1 << 30) && F < (1 << 30),
               "moe_ep_experts_fused: sizes exceed 2^31");
  RB_CHECK_ARG(offsets && ready_local && done && seg && mt_done && recv_local && wg && wu && wd &&
                   h && (n == 0 || (x && perm)),
               "moe_ep_experts_fused: null pointer");
  RB_CHECK_ARG(aligned16(recv_local) && aligned16(wg) && aligned16(wu) && aligned16(wd) &&
                   aligned16(h) && (n == 0 || aligned16(x)),
               "moe_ep_experts_fused: pointers must be 16-byte aligned");
  PeerPtrs rp, rdp, yp;
  int rc;
  if ((rc = peer_ptrs(recv_ptrs, P, &rp, "recv")) || (rc = peer_ptrs(ready_ptrs, P, &rdp, "ready")) ||
      (rc = peer_ptrs(y_ptrs, P, &yp, "y")))
    return rc;
  const int Epr = E / P, S = E;
  const int64_t rows = (int64_t)P * cap;
  CUtensorMap tX, tG, tU, tH, tW;
  {
    uint64_t d[2] = {(uint64_t)D, (uint64_t)rows};
    uint64_t st[1] = {(uint64_t)D * 2};
    uint32_t box[2] = {GBK, GBM};
    if ((rc = make_tmap(&tX, recv_local, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, st, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  {
    uint64_t d[2] = {(uint64_t)F, (uint64_t)rows};
    uint64_t st[1] = {(uint64_t)F * 2};
    uint32_t box[2] = {GBK, GBM};
    if ((rc = make_tmap(&tH, h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, st, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  {
    uint64_t d[3] = {(uint64_t)F, (uint64_t)D, (uint64_t)Epr};
    uint64_t st[2] = {(uint64_t)F * 2, (uint64_t)D * F * 2};
    uint32_t box[3] = {64, GBK, 1};
    if ((rc = make_tmap(&tG, wg, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, st, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)) ||
        (rc = make_tmap(&tU, wu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, st, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  {
    uint64_t d[3] = {(uint64_t)D, (uint64_t)F, (uint64_t)Epr};
    uint64_t st[2] = {(uint64_t)D * 2, (uint64_t)F * D * 2};
    uint32_t box[3] = {64, GBK, 1};
    if ((rc = make_tmap(&tW, wd, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, d, st, box,
                        CU_TENSOR_MAP_SWIZZLE_128B)))
      return rc;
  }
  ExpertsShape sh;
  sh.D = (int)D;
  sh.F = (int)F;
  sh.E = Epr;
  sh.S = S;
  sh.tn_s = (int)((F + 127) / 128);
  sh.tn_d = (int)((D + 255) / 256);
  sh.kb_s = (int)((D + GBK - 1) / GBK);
  sh.kb_d = (int)((F + GBK - 1) / GBK);
  sh.seg_start = seg;
  sh.seg_end = seg + S;
  sh.seg_expert = seg + 2 * S;
  sh.seg_dst_row = seg + 3 * S;
  sh.seg_src = seg + 4 * S;
  sh.h = static_cast<uint16_t*>(h);
  sh.y = yp;
  sh.ready = ready_local;
  sh.epoch = epoch;
  sh.mt_done = mt_done;
  ScatterArgs sc;
  sc.x = static_cast<const uint16_t*>(x);
  sc.perm = perm;
  sc.offsets = offsets;
  sc.n = n;
  sc.cap = cap;
  sc.k = k;
  sc.D = (int)D;
  sc.Epr = Epr;
  sc.P = P;
  sc.rank = rank;
  sc.epoch = epoch;
  sc.recv = rp;
  sc.ready = rdp;
  sc.done = done;
  RB_CUDA(cudaMemsetAsync(mt_done, 0, sizeof(int32_t) * (size_t)(rows / GBM + S + 1),
                          as_stream(stream)));
  constexpr int kSW = 2;
  auto kern = k_ep_experts<kSW>;
  RB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GSmemBytes));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms());
  cfg.blockDim = dim3(GThreads + 32 * kSW);
  cfg.dynamicSmemBytes = GSmemBytes;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RB_CUDA(cudaLaunchKernelEx(&cfg, kern, tX, tG, tU, tH, tW, sh, sc));
  return REMORA_B200_OK;
}

// ------------------------------------------------------------------------
// Peer-addressable buffers.  Plain cudaMalloc memory shared through CUDA IPC:
// no NVLink multicast object is created or bound, so a rank that exits (or
// dies) leaves its peers' GPUs with nothing but an unmapped range.
// ------------------------------------------------------------------------

static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");

extern "C" int remora_b200_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  clear_error();
  RB_CHECK_ARG(bytes > 0 && ptr && ipc_handle, "peer_alloc: bad arguments");
  void* p = nullptr;
  RB_CUDA(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(REMORA_B200_ERR_CUDA, "peer_alloc: cudaIpcGetMemHandle: %s",
                cudaGetErrorString(e));
  }
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(REMORA_B200_ERR_CUDA, "peer_alloc: cudaMemset: %s", cudaGetErrorString(e));
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return REMORA_B200_OK;
}

extern "C" int remora_b200_peer_open(const void* ipc_handle, void** ptr) {
  clear_error();
  RB_CHECK_ARG(ipc_handle && ptr, "peer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  RB_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return REMORA_B200_OK;
}

extern "C" int remora_b200_peer_close(void* ptr) {
  clear_error();
  RB_CHECK_ARG(ptr, "peer_close: null pointer");
  RB_CUDA(cudaIpcCloseMemHandle(ptr));
  return REMORA_B200_OK;
}

extern "C" int remora_b200_peer_free(void* ptr) {
  clear_error();
  if (!ptr) return REMORA_B200_OK;
  RB_CUDA(cudaFree(ptr));
  return REMORA_B200_OK;
}
