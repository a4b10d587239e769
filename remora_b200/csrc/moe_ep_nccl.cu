// moe_ep_nccl.cu -- expert-parallel MoE layer with the token exchange done by
// NCCL send/recv (an all-to-all-v), for callers that hold an ncclComm_t:
// one process (or host thread) per GPU, P ranks, E/P experts per rank.
//
// One layer on rank r, stream-ordered on the caller's stream:
//   router + top-k over all E experts, dispatch, gather   (library kernels;
//     the gathered rows are grouped by expert, so the rows for rank q are
//     one contiguous block ordered by q's local experts)
//   counts exchange: q receives r's per-local-expert row counts  (NCCL)
//   ONE host read of the split sizes (offsets and received counts, 2E+1
//     int32): NCCL's send/recv sizes are host values.  This synchronises
//     the stream once per layer -- the stated cost of this path; the
//     peer-memory path (moe_ep.cu) keeps every size on the device.
//   rows exchange: xs block q -> rank q; received blocks ordered by source
//     then local expert                                      (NCCL)
//   SwiGLU and down grouped GEMMs over the (source, local expert) segments
//   output rows back to their source ranks                   (NCCL)
//   combine in slot order                                    (kernel)
// Every row's expert output depends only on the row and its expert's
// weights, so the result equals the single-GPU layer bit for bit.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the copy already in
// the process if there is one) so that the library has no link-time NCCL
// dependency and shares the caller's NCCL.  Host waits are bounded: the
// wait on the stream polls cudaStreamQuery and ncclCommGetAsyncError until
// a wall-clock limit, then aborts the communicator (ncclCommAbort ends its
// kernels) and returns REMORA_B200_ERR_TIMEOUT; a non-blocking communicator
// (config.blocking = 0) is polled the same way whenever a call returns
// ncclInProgress.  An aborted communicator cannot be used again.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <thread>
#include <vector>

#include "runtime.cuh"

namespace rb {
namespace ncclx {

struct Api {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommFinalize)(ncclComm_t);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommCount)(const ncclComm_t, int*);
  ncclResult_t (*CommUserRank)(const ncclComm_t, int*);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
  bool ok;
};

static const Api* api() {
  static Api a = {};
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the caller's NCCL, if loaded
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    bool ok = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      ok = ok && fn != nullptr;
    };
    get(a.GetUniqueId, "ncclGetUniqueId");
    get(a.CommInitRankConfig, "ncclCommInitRankConfig");
    get(a.CommFinalize, "ncclCommFinalize");
    get(a.CommDestroy, "ncclCommDestroy");
    get(a.CommAbort, "ncclCommAbort");
    get(a.CommGetAsyncError, "ncclCommGetAsyncError");
    get(a.CommCount, "ncclCommCount");
    get(a.CommUserRank, "ncclCommUserRank");
    get(a.GroupStart, "ncclGroupStart");
    get(a.GroupEnd, "ncclGroupEnd");
    get(a.Send, "ncclSend");
    get(a.Recv, "ncclRecv");
    get(a.GetErrorString, "ncclGetErrorString");
    a.ok = ok;
  });
  return a.ok ? &a : nullptr;
}

using Clock = std::chrono::steady_clock;

inline Clock::time_point deadline_after(int64_t timeout_ms) {
  return Clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 60000);
}

inline int nccl_fail(const Api* A, ncclResult_t r, const char* what) {
  return fail(REMORA_B200_ERR_NCCL, "%s: %s (%d)", what, A->GetErrorString(r), (int)r);
}

// Every NCCL failure inside the layer aborts the communicator, so that a
// caller can rely on it: ERR_NCCL or ERR_TIMEOUT from the layer means the
// communicator is gone.
inline int abort_fail(const Api* A, ncclComm_t comm, ncclResult_t r, const char* what) {
  A->CommAbort(comm);
  return nccl_fail(A, r, what);
}

// First failure among the calls enqueued inside one group.
struct GroupErr {
  ncclResult_t first = ncclSuccess;
  void operator()(ncclResult_t r) {
    if (r != ncclSuccess && r != ncclInProgress && first == ncclSuccess) first = r;
  }
};

// After an NCCL call: success, or (non-blocking communicator) poll until the
// call has been enqueued, bounded by `until`; on expiry abort the communicator.
int settle(const Api* A, ncclComm_t comm, ncclResult_t r, Clock::time_point until,
           const char* what) {
  if (r != ncclSuccess && r != ncclInProgress) {
    A->CommAbort(comm);
    return nccl_fail(A, r, what);
  }
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = A->CommGetAsyncError(comm, &st);
    if (q != ncclSuccess) {
      A->CommAbort(comm);
      return nccl_fail(A, q, "ncclCommGetAsyncError");
    }
    if (st == ncclSuccess) return REMORA_B200_OK;
    if (st != ncclInProgress) {
      A->CommAbort(comm);
      return nccl_fail(A, st, what);
    }
    if (Clock::now() > until) {
      A->CommAbort(comm);
      return fail(REMORA_B200_ERR_TIMEOUT, "%s: NCCL did not finish in time; communicator "
                  "aborted", what);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Waits for the stream (bounded), watching the communicator for errors; on
// expiry or error the communicator is aborted, which ends its kernels.
int wait_stream(const Api* A, ncclComm_t comm, cudaStream_t st, Clock::time_point until,
                const char* what) {
  for (uint32_t it = 0;; ++it) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return REMORA_B200_OK;
    if (e != cudaErrorNotReady)
      return fail(REMORA_B200_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    ncclResult_t as = ncclSuccess;
    if (A->CommGetAsyncError(comm, &as) == ncclSuccess && as != ncclSuccess &&
        as != ncclInProgress) {
      A->CommAbort(comm);
      return nccl_fail(A, as, what);
    }
    if (Clock::now() > until) {
      A->CommAbort(comm);
      return fail(REMORA_B200_ERR_TIMEOUT, "%s: the stream did not drain in time (a peer "
                  "missing?); communicator aborted", what);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(it < 1000 ? 2 : 50));
  }
}

__global__ void k_nccl_segments(const int32_t* __restrict__ recv_counts, int n, int Epr,
                                int32_t* seg_off, int32_t* seg_expert) {
  if (threadIdx.x != 0) return;
  int32_t run = 0;
  for (int q = 0; q < n; ++q) {
    seg_off[q] = run;
    seg_expert[q] = q % Epr;
    run += recv_counts[q];
  }
  seg_off[n] = run;
}

struct EpWs {
  int32_t *idx, *counts, *offsets, *perm, *inv, *block_counts, *recv_counts, *seg_off, *seg_exp;
  float* w;
  uint16_t *xs, *xr, *h;  // y aliases xs, yr aliases xr
  size_t bytes;
};

inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

inline EpWs ep_ws(void* base, int64_t T, int64_t D, int64_t F, int E, int k, int P) {
  EpWs L;
  const int64_t n = T * k, cap = (int64_t)P * n;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t at = o;
    o += a256(bytes);
    return static_cast<uint8_t*>(base) + at;
  };
  L.idx = reinterpret_cast<int32_t*>(take(n * 4));
  L.w = reinterpret_cast<float*>(take(n * 4));
  L.counts = reinterpret_cast<int32_t*>(take(E * 4));
  L.offsets = reinterpret_cast<int32_t*>(take((E + 1) * 4));
  L.perm = reinterpret_cast<int32_t*>(take(n * 4));
  L.inv = reinterpret_cast<int32_t*>(take(n * 4));
  L.block_counts = reinterpret_cast<int32_t*>(take(moe::dispatch_ws_bytes(T, k, E)));
  L.recv_counts = reinterpret_cast<int32_t*>(take(E * 4));
  L.seg_off = reinterpret_cast<int32_t*>(take((E + 1) * 4));
  L.seg_exp = reinterpret_cast<int32_t*>(take(E * 4));
  L.xs = reinterpret_cast<uint16_t*>(take(n * D * 2));
  L.xr = reinterpret_cast<uint16_t*>(take(cap * D * 2));
  L.h = reinterpret_cast<uint16_t*>(take(cap * F * 2));
  L.bytes = o;
  return L;
}

}  // namespace ncclx
}  // namespace rb

using namespace rb;
using namespace rb::ncclx;

extern "C" int remora_b200_moe_ep_splits(const int32_t* offsets, const int32_t* recv_counts,
                                         int P, int E, int64_t* send_off, int64_t* send_rows,
                                         int64_t* recv_off, int64_t* recv_rows) {
  clear_error();
  RB_CHECK_ARG(P >= 1 && E >= P && E % P == 0 && offsets && recv_counts && send_off &&
                   send_rows && recv_off && recv_rows,
               "moe_ep_splits: bad arguments (P=%d E=%d)", P, E);
  const int Epr = E / P;
  int64_t run = 0;
  for (int q = 0; q < P; ++q) {
    RB_CHECK_ARG(offsets[(q + 1) * Epr] >= offsets[q * Epr], "moe_ep_splits: offsets decrease");
    send_off[q] = offsets[q * Epr];
    send_rows[q] = offsets[(q + 1) * Epr] - offsets[q * Epr];
    int64_t r = 0;
    for (int e = 0; e < Epr; ++e) {
      RB_CHECK_ARG(recv_counts[q * Epr + e] >= 0, "moe_ep_splits: negative count");
      r += recv_counts[q * Epr + e];
    }
    recv_off[q] = run;
    recv_rows[q] = r;
    run += r;
  }
  return REMORA_B200_OK;
}

extern "C" int remora_b200_nccl_unique_id(void* id) {
  clear_error();
  RB_CHECK_ARG(id, "nccl_unique_id: null argument");
  const Api* A = api();
  if (!A) return fail(REMORA_B200_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  ncclResult_t r = A->GetUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail(A, r, "ncclGetUniqueId");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  memcpy(id, &u, sizeof(u));
  return REMORA_B200_OK;
}

extern "C" int remora_b200_nccl_comm_init(void** comm, int nranks, const void* id, int rank,
                                          int blocking, int64_t timeout_ms) {
  clear_error();
  RB_CHECK_ARG(comm && id && nranks >= 1 && rank >= 0 && rank < nranks,
               "nccl_comm_init: bad arguments");
  const Api* A = api();
  if (!A) return fail(REMORA_B200_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = blocking ? 1 : 0;
  ncclComm_t c = nullptr;
  ncclResult_t r = A->CommInitRankConfig(&c, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(A, r, "ncclCommInitRankConfig");
  if (c == nullptr) return fail(REMORA_B200_ERR_NCCL, "ncclCommInitRankConfig gave no comm");
  int rc = settle(A, c, r, deadline_after(timeout_ms), "ncclCommInitRankConfig");
  if (rc) return rc;  // the communicator was aborted
  *comm = c;
  return REMORA_B200_OK;
}

extern "C" int remora_b200_nccl_comm_destroy(void* comm, int64_t timeout_ms) {
  clear_error();
  if (!comm) return REMORA_B200_OK;
  const Api* A = api();
  if (!A) return fail(REMORA_B200_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int rc = settle(A, c, A->CommFinalize(c), deadline_after(timeout_ms), "ncclCommFinalize");
  if (rc) return rc;  // aborted (which frees it)
  ncclResult_t r = A->CommDestroy(c);
  return r == ncclSuccess ? REMORA_B200_OK : nccl_fail(A, r, "ncclCommDestroy");
}

extern "C" int remora_b200_nccl_comm_abort(void* comm) {
  clear_error();
  if (!comm) return REMORA_B200_OK;
  const Api* A = api();
  if (!A) return fail(REMORA_B200_ERR_NCCL, "libnccl.so.2 could not be loaded");
  ncclResult_t r = A->CommAbort(static_cast<ncclComm_t>(comm));
  return r == ncclSuccess ? REMORA_B200_OK : nccl_fail(A, r, "ncclCommAbort");
}

extern "C" size_t remora_b200_moe_ep_nccl_workspace_bytes(int64_t T, int64_t D, int64_t F, int E,
                                                          int k, int P) {
  if (T < 0 || D <= 0 || F <= 0 || E < 1 || k < 1 || P < 1 || T > INT32_MAX / k / P) return 0;
  return ep_ws(nullptr, T, D, F, E, k, P).bytes;
}

extern "C" int remora_b200_moe_ep_nccl_bf16(const void* x, const void* wr, const void* wg,
                                            const void* wu, const void* wd, void* out, int64_t T,
                                            int64_t D, int64_t F, int E, int k, void* comm,
                                            int64_t timeout_ms, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  using namespace rb::moe;
  clear_error();
  const Api* A = api();
  if (!A) return fail(REMORA_B200_ERR_NCCL, "libnccl.so.2 could not be loaded");
  RB_CHECK_ARG(comm, "moe_ep_nccl: null communicator");
  ncclComm_t c = static_cast<ncclComm_t>(comm);
  int P = 0, rank = 0;
  ncclResult_t r;
  if (A->CommCount(c, &P) != ncclSuccess || A->CommUserRank(c, &rank) != ncclSuccess)
    return fail(REMORA_B200_ERR_INVALID, "moe_ep_nccl: not a usable communicator");
  RB_CHECK_ARG(T >= 1 && D > 0 && F > 0 && E >= 1 && E <= GMaxE && k >= 1 && k <= 16 && k <= E &&
                   E % P == 0,
               "moe_ep_nccl: bad sizes (T=%lld E=%d k=%d over %d ranks)", (long long)T, E, k, P);
  RB_CHECK_ARG(D % 32 == 0 && F % 32 == 0, "moe_ep_nccl: D and F must be multiples of 32");
  RB_CHECK_ARG(T <= INT32_MAX / k / P, "moe_ep_nccl: P*T*k exceeds the int32 row range");
  RB_CHECK_ARG(x && wr && wg && wu && wd && out && workspace, "moe_ep_nccl: null pointer");
  EpWs L = ep_ws(workspace, T, D, F, E, k, P);
  RB_CHECK_ARG(workspace_bytes >= L.bytes, "moe_ep_nccl: workspace of %zu bytes, %zu needed",
               workspace_bytes, L.bytes);
  RB_CHECK_ARG(aligned16(workspace), "moe_ep_nccl: workspace must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const Clock::time_point until = deadline_after(timeout_ms);
  const int Epr = E / P;
  const int64_t n = T * k;
  int rc;
  if ((rc = router_launch(x, wr, T, D, E, k, L.idx, L.w, st))) return rc;
  if ((rc = dispatch_launch(L.idx, T, k, E, L.counts, L.offsets, L.perm, L.inv, L.block_counts,
                            st)))
    return rc;
  if ((rc = scatter_launch(x, L.inv, T, k, D, L.xs, st))) return rc;  // rows in dispatch order

  // per-local-expert counts: rank q gets counts[q*Epr .. (q+1)*Epr)
  if ((r = A->GroupStart()) != ncclSuccess) return abort_fail(A, c, r, "ncclGroupStart");
  GroupErr ge;
  for (int q = 0; q < P; ++q) {
    ge(A->Send(L.counts + q * Epr, Epr, ncclInt32, q, c, st));
    ge(A->Recv(L.recv_counts + q * Epr, Epr, ncclInt32, q, c, st));
  }
  if ((rc = settle(A, c, A->GroupEnd(), until, "counts exchange"))) return rc;
  if (ge.first != ncclSuccess) return abort_fail(A, c, ge.first, "counts exchange");
  // the one host read of the split sizes
  std::vector<int32_t> h_off(E + 1), h_recv(E);
  RB_CUDA(cudaMemcpyAsync(h_off.data(), L.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost, st));
  RB_CUDA(cudaMemcpyAsync(h_recv.data(), L.recv_counts, E * 4, cudaMemcpyDeviceToHost, st));
  if ((rc = wait_stream(A, c, st, until, "split sizes"))) return rc;
  std::vector<int64_t> s_off(P), s_rows(P), r_off(P), r_rows(P);
  if ((rc = remora_b200_moe_ep_splits(h_off.data(), h_recv.data(), P, E, s_off.data(),
                                      s_rows.data(), r_off.data(), r_rows.data())))
    return rc;
  const int64_t recv_total = r_off[P - 1] + r_rows[P - 1];
  RB_CHECK_ARG(recv_total <= (int64_t)P * n,
               "moe_ep_nccl: %lld rows received, more than P*T*k (do all ranks pass the same T?)",
               (long long)recv_total);
  k_nccl_segments<<<1, 32, 0, st>>>(L.recv_counts, E, Epr, L.seg_off, L.seg_exp);
  RB_LAUNCH_CHECK();

  // rows out to their experts' ranks
  if ((r = A->GroupStart()) != ncclSuccess) return abort_fail(A, c, r, "ncclGroupStart");
  for (int q = 0; q < P; ++q) {
    if (s_rows[q]) ge(A->Send(L.xs + s_off[q] * D, (size_t)(s_rows[q] * D), ncclBfloat16, q, c, st));
    if (r_rows[q]) ge(A->Recv(L.xr + r_off[q] * D, (size_t)(r_rows[q] * D), ncclBfloat16, q, c, st));
  }
  if ((rc = settle(A, c, A->GroupEnd(), until, "rows exchange"))) return rc;
  if (ge.first != ncclSuccess) return abort_fail(A, c, ge.first, "rows exchange");

  // local experts over the (source, local expert) segments; yr aliases xr
  if (recv_total > 0) {
    if ((rc = grouped_launch(true, L.xr, wg, wu, L.h, L.seg_off, recv_total, D, F, Epr, st,
                             L.seg_exp, E)))
      return rc;
    if ((rc = grouped_launch(false, L.h, wd, nullptr, L.xr, L.seg_off, recv_total, F, D, Epr, st,
                             L.seg_exp, E)))
      return rc;
  }

  // outputs back to their source ranks, into y (aliases xs) in dispatch order
  if ((r = A->GroupStart()) != ncclSuccess) return abort_fail(A, c, r, "ncclGroupStart");
  for (int q = 0; q < P; ++q) {
    if (r_rows[q]) ge(A->Send(L.xr + r_off[q] * D, (size_t)(r_rows[q] * D), ncclBfloat16, q, c, st));
    if (s_rows[q]) ge(A->Recv(L.xs + s_off[q] * D, (size_t)(s_rows[q] * D), ncclBfloat16, q, c, st));
  }
  if ((rc = settle(A, c, A->GroupEnd(), until, "outputs exchange"))) return rc;
  if (ge.first != ncclSuccess) return abort_fail(A, c, ge.first, "outputs exchange");
  (void)rank;
  return combine_launch(L.xs, L.inv, L.w, T, k, D, out, st);
}
