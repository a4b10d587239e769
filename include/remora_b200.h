/*
 * remora_b200.h -- C ABI of the B200 (sm_100a) execution backend for remora.
 *
 * remora's GPU harness, `int launchOnGpu(const std::vector<std::string>&
 * ptxModules, llvm::StringRef test)` (compiler/gpu_tests.h:6-9,
 * compiler/gpu_tests.cpp:101-125), loads NVVM-generated sm_89 PTX and
 * launches it with the MLIR memref-descriptor argument list
 * (compiler/gpu_tests.cpp:58-79).  This library replaces what sits below
 * that call for the programs it recognises: `launchOnGpu` asks
 * remora_b200_recognise(test) and, if recognised, calls
 * remora_b200_run_test() instead of loading the PTX.  The per-op entry
 * points take caller-owned device pointers, plain sizes and a CUDA stream.
 *
 * Conventions
 *   - Every function returns an int status: REMORA_B200_OK (0) or a negative
 *     REMORA_B200_ERR_* code; remora_b200_last_error() gives the text
 *     (thread-local).  remora's CUDA_CHECK returned 1 on any failure
 *     (gpu_tests.cpp:11-20); a caller that wants that convention maps
 *     "status != 0" to 1.  A failed parity check IS an error here, unlike
 *     gpu_tests.cpp:91-94.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream).  Launches are stream-ordered and asynchronous unless stated.
 *   - bf16 tensors are passed as void* to 16-bit storage.  Row-major unless
 *     stated.  Leading dimensions are in elements.
 *   - The per-op entry points never allocate or free caller memory.
 */
#ifndef REMORA_B200_H
#define REMORA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define REMORA_B200_OK 0
#define REMORA_B200_ERR_INVALID (-1)     /* bad argument, shape or alignment */
#define REMORA_B200_ERR_CUDA (-2)        /* CUDA runtime / driver error */
#define REMORA_B200_ERR_NCCL (-3)        /* NCCL error */
#define REMORA_B200_ERR_TIMEOUT (-4)     /* a bounded device or host wait expired */
#define REMORA_B200_ERR_PARITY (-5)      /* run_test: results outside tolerance */
#define REMORA_B200_ERR_UNSUPPORTED (-6) /* test kind not recognised */

/* B operand layouts of the GEMM entry points. */
#define REMORA_B200_B_KN 0 /* B is [K, N], N contiguous (dot_general rhs [K,N]) */
#define REMORA_B200_B_NK 1 /* B is [N, K], K contiguous (transposed rhs)        */

/* Text of the last error raised on the calling thread ("" if none). */
const char* remora_b200_last_error(void);

/* Library version, major*10000 + minor*100 + patch. */
int remora_b200_version(void);

/* Synchronises the current device and reports (then clears) an error a
 * kernel recorded on the device since the last check: REMORA_B200_ERR_TIMEOUT
 * for a bounded device wait that expired, REMORA_B200_ERR_INVALID for a bad
 * value seen by a kernel (an expert id outside [0, E)). */
int remora_b200_device_status(void);

/* ------------------------------------------------------------------------
 * Dispatcher (replaces the body of launchOnGpu, gpu_tests.cpp:101-125)
 * --------------------------------------------------------------------- */

/* Options of one run_test call.  Zero-initialise, then set what you need. */
typedef struct remora_b200_opts {
  int device;       /* CUDA device ordinal (remora uses device 0, gpu_tests.cpp:103) */
  uint64_t seed;    /* base seed of the input generator; 0 means 42 */
  int iters;        /* timed iterations (0 = 1) */
  int warmup;       /* untimed warm-up iterations */
  int validate;     /* 1 = check the result (known answer or sampled self-check) */
  const char* config; /* optional named configuration, NULL = the reference program's shape */
} remora_b200_opts;

typedef struct remora_b200_report {
  double ms_per_iter;   /* CUDA-event time per iteration */
  double work;          /* algorithmic FLOPs or bytes per iteration */
  double rate;          /* work / time, in FLOP/s or B/s */
  double max_abs_err;   /* validation: worst absolute error */
  double max_rel_err;   /* validation: worst relative error */
  int64_t checked;      /* number of output elements checked */
  int passed;           /* 1 if validation passed (or was not requested) */
  char detail[256];     /* one-line human readable summary */
} remora_b200_report;

/* 1 if `test` (the --test= kind) is handled by this library, else 0.
 * Kinds: "elementwise" (gpu_tests.cpp:35-95), "projection"
 * (cpu_tests.cpp:65-97), "elementwise_chain", "gemm", "attention", "moe"
 * (configs "4", "5", "mixtral" = mixtral_moe_layer.mlir:8, "simple" =
 * simple_moe.mlir:16, "hetero" = heterogeneous_moe_layer.mlir:66, with
 * bf16 operands). */
int remora_b200_recognise(const char* test);

/* The launch plan of a recognised program, written to out (NUL-terminated,
 * at most out_bytes): the entry points it calls and, for each, its kernels
 * with grid x block, dynamic shared memory and argument shapes.  This is
 * what `remora-b200 --emit-ptx` prints in place of the NVVM PTX that
 * remora's --emit-ptx prints (compiler/gpu.cpp:222-224): the kernels here
 * are hand-written sm_100a code, not generated.  Needs no GPU (the SM count
 * defaults to 148 when no device is visible). */
int remora_b200_launch_plan(const char* test, const char* config, char* out, size_t out_bytes);

/* Runs the recognised program end to end on `o->device`: allocates its own
 * buffers, fills the inputs, launches, times and validates.  Replaces
 * launchElementwiseOnGpu (gpu_tests.cpp:35-95), which allocated, filled
 * x = 1 and bias = -0.5, launched and checked |v - 0.5| <= 1e-5. */
int remora_b200_run_test(const char* test, const remora_b200_opts* o, remora_b200_report* r);

/* ------------------------------------------------------------------------
 * Elementwise attention epilogue
 * --------------------------------------------------------------------- */

/* out[r, j] = maximumf(x[r, j] + bias[j], 0) for r < rows, j < d.
 * The fused linalg.generic of
 * mlir/linalg/attention_elementwise_lowered_to_linalg.mlir:7-11 (the
 * --test=elementwise program, mlir/stablehlo/simple_attention_elementwise.mlir:5-17).
 * NaN propagates; -0 becomes +0. */
int remora_b200_relu_bias_f32(const float* x, const float* bias, float* out, int64_t rows,
                              int64_t d, void* stream);

/* out[i] = exp(s[i] * scale + b[i]) for i < n: stablehlo.multiply by a
 * scalar, stablehlo.add, stablehlo.exponential, one HBM round trip.  The
 * product and the sum are rounded separately (no contraction). */
int remora_b200_scale_add_exp_f32(const float* s, const float* b, float* out, int64_t n,
                                  float scale, void* stream);

/* ------------------------------------------------------------------------
 * stablehlo.dot_general GEMM (contracting lhs dim 1 x rhs dim 0)
 * --------------------------------------------------------------------- */

/* C[b] = A[b] * B[b] for b < batch: bf16 inputs, fp32 accumulation in
 * tensor memory, bf16 output (round to nearest even).
 * A: [M, K] (lda), B: [K, N] (ldb) if b_layout == REMORA_B200_B_KN else
 * [N, K], C: [M, N] (ldc).  stride_a/b/c: elements between batches.
 * Requires K % 8 == 0, N % 8 == 0, lda/ldb/ldc % 8 == 0 and 16-byte
 * aligned base pointers (TMA rules); M, N, K need not be tile multiples.
 * Replaces the two NVVM modules (fill + reduction) that remora emits for
 * mlir/linalg/attention_projection_lowered_to_linalg.mlir:8-12
 * (compiler/gpu.cpp:159-160), which gpu_tests.cpp:119 never launches. */
int remora_b200_gemm_bf16(const void* A, const void* B, void* C, int64_t batch, int64_t M,
                          int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                          int64_t stride_a, int64_t stride_b, int64_t stride_c, int b_layout,
                          void* stream);

/* f32 dot_general with the reference CPU path's exact arithmetic: for each
 * output, fill 0 then out = out + a*b over k in increasing order, each
 * product and sum rounded separately (cpu.cpp:50-55 convert-linalg-to-loops
 * of attention_projection_lowered_to_linalg.mlir:8-12).  Results are
 * bit-identical to that loop nest.  The --test=projection program. */
int remora_b200_gemm_f32_exact(const float* A, const float* B, float* C, int64_t M, int64_t N,
                               int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int b_layout,
                               void* stream);

/* ------------------------------------------------------------------------
 * Softmax attention (no counterpart program in the reference: README.md:12
 * lists FlashAttention as in progress; this is the backend's fused form)
 * --------------------------------------------------------------------- */

/* out = softmax(q k^T * scale [+ causal mask]) v per (batch, head), bf16
 * q, k, v, out [batch, heads, seq, head_dim] contiguous; fp32 softmax
 * statistics, P rounded to bf16 for the second product.  head_dim must be
 * 128; seq is arbitrary (rows past seq are masked).  causal != 0 masks key
 * j > query i. */
int remora_b200_attention_fwd_bf16(const void* q, const void* k, const void* v, void* out,
                                   int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                   int causal, float scale, void* stream);

/* ------------------------------------------------------------------------
 * MoE layer (mlir/stablehlo/mixtral_moe_layer.mlir:8-68; simple_moe.mlir:16-35)
 * T tokens, D d_model, F ffn dim, E experts, k slots per token.
 * --------------------------------------------------------------------- */

/* Router: logits[t, e] = sum_d x[t, d] * wr[d, e], accumulated in fp32 in
 * increasing d from +0.0 (the loop order of the lowered dot_general,
 * mixtral_moe_layer.mlir:12), so idx is bit-identical to that loop nest;
 * top-k (:13, mhlo.topk: larger first, NaN first, ties to the lower
 * expert), then w = softmax over the k selected logits (:14-24).
 * x bf16 [T, D], wr bf16 [D, E]; idx int32 [T, k], w f32 [T, k].
 * E <= 256, k <= min(E, 16), D % 8 == 0. */
int remora_b200_moe_router_topk_bf16(const void* x, const void* wr, int64_t T, int64_t D, int E,
                                     int k, int32_t* idx, float* w, void* stream);

/* Bytes of device workspace remora_b200_moe_dispatch needs. */
size_t remora_b200_moe_dispatch_workspace_bytes(int64_t T, int k, int E);

/* Dispatch: the sparse form of the one-hot scatter of
 * mixtral_moe_layer.mlir:28-31 / :70-78.  counts[E], offsets[E+1]
 * (exclusive scan), perm[T*k] = t*k + j of the row at each position (rows
 * grouped by expert, each expert's rows in (token, slot) order),
 * inv[t*k + j] = its position.  Deterministic.  An expert id outside
 * [0, E) is reported as a device error by the next synchronising call. */
int remora_b200_moe_dispatch(const int32_t* idx, int64_t T, int k, int E, int32_t* counts,
                             int32_t* offsets, int32_t* perm, int32_t* inv, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Same dispatch as remora_b200_moe_dispatch, for callers that cannot
 * allocate device memory when they dispatch (code running inside a memory
 * pool it does not own, embedders that fix their memory use at start-up,
 * latency-critical paths that must not take the allocator's lock).  No
 * counterpart in the reference.  It allocates nothing: its scratch is a
 * fixed 1 MiB array inside the library, held by every GPU that loads the
 * library until the process exits.  A call needing more than
 * 262144 scratch slots (ceil(T*k / 1024) * E) fails with
 * REMORA_B200_ERR_INVALID.  All calls on a device share the array, so calls
 * that overlap on the GPU race; serialise them (e.g. one stream).  The first
 * call on a device looks up the array's device address; make it before any
 * stream capture. */
int remora_b200_moe_dispatch_noalloc(const int32_t* idx, int64_t T, int k, int E,
                                     int32_t* counts, int32_t* offsets, int32_t* perm,
                                     int32_t* inv, void* stream);

/* xs[p, :] = x[perm[p] / k, :] for p < rows (bf16 rows, D % 8 == 0). */
int remora_b200_moe_gather(const void* x, const int32_t* perm, int64_t rows, int k, int64_t D,
                           void* xs, void* stream);

/* The same rows written token by token: xs[inv[t*k + j], :] = x[t, :] for
 * t < T, j < k (inv from remora_b200_moe_dispatch).  Each token row is read
 * once, so it moves (1 + k) * D * 2 bytes per token instead of 2 * k * D * 2;
 * the fused layer uses this form for the one-hot dispatch of
 * mixtral_moe_layer.mlir:28-31. */
int remora_b200_moe_scatter(const void* x, const int32_t* inv, int64_t T, int k, int64_t D,
                            void* xs, void* stream);

/* Grouped expert GEMM with the SwiGLU epilogue (mixtral_moe_layer.mlir:32-41;
 * the outlined @expert_slot_N body, compiler/passes/ExpertOutlining.cpp:177-279):
 * for rows r of expert e (offsets[e] <= r < offsets[e+1]),
 * h[r, :] = silu(xs[r] . wg[e]) * (xs[r] . wu[e]), silu(g) = g / (1 + exp(-g)).
 * xs bf16 [rows, D]; wg, wu bf16 [E, D, F]; h bf16 [rows, F].
 * D % 8 == 0, F % 32 == 0; offsets on the device. */
int remora_b200_grouped_gemm_swiglu_bf16(const void* xs, const void* wg, const void* wu, void* h,
                                         const int32_t* offsets, int64_t rows, int64_t D,
                                         int64_t F, int E, void* stream);

/* Grouped expert GEMM (the down projection, mixtral_moe_layer.mlir:42):
 * y[r, :] = a[r] . w[e] for the rows of expert e.  a bf16 [rows, K],
 * w bf16 [E, K, N], y bf16 [rows, N]; K % 8 == 0, N % 32 == 0. */
int remora_b200_grouped_gemm_bf16(const void* a, const void* w, void* y, const int32_t* offsets,
                                  int64_t rows, int64_t K, int64_t N, int E, void* stream);

/* The two grouped GEMMs over row segments that name their expert: segment q
 * owns rows [seg_offsets[q], seg_offsets[q+1]) and uses expert
 * seg_expert[q] (0 <= seg_expert[q] < E, n_seg <= 256).  This is the layout
 * of the rows an expert-parallel rank receives from its peers: ordered by
 * source rank, then by local expert.  Same arithmetic as the forms above. */
int remora_b200_grouped_gemm_swiglu_segments_bf16(const void* xs, const void* wg, const void* wu,
                                                  void* h, const int32_t* seg_offsets,
                                                  const int32_t* seg_expert, int n_seg,
                                                  int64_t rows, int64_t D, int64_t F, int E,
                                                  void* stream);
int remora_b200_grouped_gemm_segments_bf16(const void* a, const void* w, void* y,
                                           const int32_t* seg_offsets, const int32_t* seg_expert,
                                           int n_seg, int64_t rows, int64_t K, int64_t N, int E,
                                           void* stream);

/* Combine (mixtral_moe_layer.mlir:43-46, :52-55): out[t, :] =
 * bf16(0 + w[t,0]*y[inv[t,0]] + w[t,1]*y[inv[t,1]] + ...), slot order, each
 * product and sum rounded separately.  y bf16 [T*k, D]; out bf16 [T, D]. */
int remora_b200_moe_combine_bf16(const void* y, const int32_t* inv, const float* w, int64_t T,
                                 int k, int64_t D, void* out, void* stream);

/* Bytes of device workspace remora_b200_moe_layer_bf16 needs. */
size_t remora_b200_moe_workspace_bytes(int64_t T, int64_t D, int64_t F, int E, int k);

/* The whole MoE layer: router -> dispatch -> row copy -> SwiGLU grouped GEMM
 * -> down grouped GEMM -> combine, stream-ordered, no host synchronisation.
 * x bf16 [T, D]; wr bf16 [D, E]; wg, wu bf16 [E, D, F]; wd bf16 [E, F, D];
 * out bf16 [T, D].  F % 32 == 0, D % 32 == 0.  The workspace (caller
 * owned, 16-byte aligned) holds the routing tables and the dispatched
 * activations. */
int remora_b200_moe_layer_bf16(const void* x, const void* wr, const void* wg, const void* wu,
                               const void* wd, void* out, int64_t T, int64_t D, int64_t F, int E,
                               int k, void* workspace, size_t workspace_bytes, void* stream);

/* The same layer with the tokens and the output in HOST memory, for callers
 * whose activations live on the host (remora's harness fills host vectors,
 * compiler/gpu_tests.cpp:48-56): the tokens go up and the output comes back
 * in chunks of chunk_tokens (0 = 16384) on two copy streams of the library's
 * own, overlapped with the layer's kernels on `stream` (chunk c computes
 * while chunk c+1 goes up and chunk c-1 comes down; from T >= 2 chunks the
 * first two and last two chunks are a quarter and a half of the others, so
 * the copies nothing overlaps are short; tokens are independent, so the
 * output is bit-identical to remora_b200_moe_layer_bf16).  Weights
 * and router are device pointers.  x_host and out_host should be pinned
 * (cudaHostAlloc / cudaHostRegister); pageable memory is correct but its
 * copies do not overlap.  The call only enqueues work: out_host is complete
 * once `stream` has reached this point (synchronise it before reading).
 * The copy streams and events are created once per (thread, device). */
size_t remora_b200_moe_layer_host_workspace_bytes(int64_t T, int64_t D, int64_t F, int E, int k,
                                                  int64_t chunk_tokens);
int remora_b200_moe_layer_host_bf16(const void* x_host, const void* wr, const void* wg,
                                    const void* wu, const void* wd, void* out_host, int64_t T,
                                    int64_t D, int64_t F, int E, int k, int64_t chunk_tokens,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Heterogeneous MoE: experts of different FFN widths
 * (mlir/stablehlo/heterogeneous_moe_layer.mlir:66-212, one [1, D, F_e] weight
 * tensor per expert, :66-100).  E <= 16 experts; wg, wu, wd are host arrays
 * of E device pointers (expert e: wg[e], wu[e] bf16 [D, F_e], wd[e] bf16
 * [F_e, D]); F is a host array of the E widths.
 * --------------------------------------------------------------------- */

/* h[r, :F_e] = silu(xs[r] . wg[e]) * (xs[r] . wu[e]) for the rows of expert e
 * (offsets[e] <= r < offsets[e+1], offsets on the device).  h [rows, ldh],
 * ldh >= every F_e; F_e % 32 == 0, D % 8 == 0.  All experts' tiles run in
 * one persistent launch: the tile list carries each expert's own column
 * count and weight tensor map. */
int remora_b200_grouped_gemm_swiglu_var_bf16(const void* xs, const void* const* wg,
                                             const void* const* wu, void* h, int64_t ldh,
                                             const int32_t* offsets, int64_t rows, int64_t D,
                                             const int64_t* F, int E, void* stream);

/* y[r, :] = h[r, :F_e] . wd[e] for the rows of expert e: the contraction
 * length is each expert's own F_e (a multiple of 64, or equal to ldh). */
int remora_b200_grouped_gemm_var_bf16(const void* h, int64_t ldh, const void* const* wd, void* y,
                                      const int32_t* offsets, int64_t rows, const int64_t* F,
                                      int64_t D, int E, void* stream);

/* Bytes of device workspace remora_b200_moe_hetero_layer_bf16 needs (0 for
 * sizes it rejects). */
size_t remora_b200_moe_hetero_workspace_bytes(int64_t T, int64_t D, const int64_t* F, int E,
                                              int k);

/* The heterogeneous layer: router (bit-exact top-k as the uniform layer),
 * dispatch, gather, the two variable-width grouped GEMMs, combine.  With
 * k = 1 the combine weight is softmax over one logit = 1, so out[t] is the
 * selected expert's output, as the program's one-hot combine gives
 * (:210-225).  D % 32 == 0; every F_e a positive multiple of 64. */
int remora_b200_moe_hetero_layer_bf16(const void* x, const void* wr, const void* const* wg,
                                      const void* const* wu, const void* const* wd,
                                      const int64_t* F, void* out, int64_t T, int64_t D, int E,
                                      int k, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* ------------------------------------------------------------------------
 * Expert-parallel MoE over NVLink peer memory (P <= 8 ranks, one per GPU).
 * The reference has no multi-GPU path (one device, gpu_tests.cpp:102-104);
 * these replace an NCCL all-to-all for the token exchange.  Every rank holds
 * buffers its peers can address (remora_b200_peer_alloc below): recv
 * [P][cap][D] bf16, meta [P][E/P+1] int32, y [T_local*k][D] bf16 and flags
 * [P] int32 (zero-initialised once).  *_ptrs are host arrays of the P
 * ranks' device addresses of that buffer.  Only plain loads and stores
 * reach peer memory.
 * --------------------------------------------------------------------- */

/* Peer-addressable buffers for the entry points below, one process per GPU.
 * remora_b200_peer_alloc cudaMallocs `bytes` on the current device, zeroes
 * them and writes the 64-byte CUDA IPC handle of the allocation to
 * ipc_handle; the caller hands the handles to its peers (any channel: a
 * process-group all-gather, MPI, a file) and each peer maps them with
 * remora_b200_peer_open (cudaIpcOpenMemHandle with lazy peer access; the
 * owner itself uses its own pointer).  Plain device memory: no NVLink
 * multicast object is created, so a rank that exits leaves its peers only
 * an unmapped range.  Teardown: every rank stops using the buffers (e.g. a
 * barrier), closes the peers' mappings with remora_b200_peer_close, then
 * frees its own with remora_b200_peer_free.  The reference has no
 * counterpart (single device, compiler/gpu_tests.cpp:102-104). */
int remora_b200_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int remora_b200_peer_open(const void* ipc_handle, void** ptr);
int remora_b200_peer_close(void* ptr);
int remora_b200_peer_free(void* ptr);

/* Copies this rank's n dispatched rows (x[perm[p]/k], dispatch order of
 * remora_b200_moe_dispatch over all E experts) into region `rank` of the
 * owning rank's recv buffer, and writes that rank's meta[rank] (rows per
 * local expert, then the first dispatch position of those rows).
 * n <= cap; cap = the most rows one rank can send (T_local * k). */
int remora_b200_moe_ep_scatter_bf16(const void* x, const int32_t* perm, const int32_t* offsets,
                                    int64_t n, int k, int64_t D, int E, int P, int rank,
                                    int64_t cap, const uint64_t* recv_ptrs,
                                    const uint64_t* meta_ptrs, void* stream);

/* Stream-ordered barrier: publishes `epoch` (increasing per call) in every
 * peer's flags[rank], then waits until all of this rank's flags reach it.
 * Bounded: a wait longer than 2 s records a timeout that
 * remora_b200_device_status() reports (REMORA_B200_ERR_TIMEOUT). */
int remora_b200_moe_ep_barrier(int32_t* flags, const uint64_t* flag_ptrs, int P, int rank,
                               int epoch, void* stream);

/* Builds the 5*(P*Epr) int32 segment table of the received rows from this
 * rank's meta: start, end, local expert, destination row, source rank. */
int remora_b200_moe_ep_segments(const int32_t* meta, int P, int Epr, int64_t cap, int32_t* seg,
                                void* stream);

/* The local experts over the received rows: SwiGLU grouped GEMM into h
 * ([P*cap, F], recv's row layout), then the down grouped GEMM, each output
 * row stored into its source rank's y at the row it was dispatched from.
 * wg, wu [Epr, D, F]; wd [Epr, F, D] (this rank's experts). */
int remora_b200_moe_ep_experts_bf16(const void* recv, const void* wg, const void* wu,
                                    const void* wd, void* h, const int32_t* seg, int P, int Epr,
                                    int64_t cap, int64_t D, int64_t F, const uint64_t* y_ptrs,
                                    void* stream);

/* Fused form of the exchange (three calls per layer instead of scatter,
 * barrier, segments, experts).  It needs, beside the buffers above, a
 * peer-addressable ready[E] int32 (slot s*(E/P)+e: source s, local expert
 * e; zero-initialised once) and a local done[E] int32 scratch.
 *
 * Step 1: publishes this rank's per-expert row counts in every peer's meta,
 * zeroes done, barriers on `epoch` (as remora_b200_moe_ep_barrier) and
 * builds the 5*E segment table from the received meta with the sources in
 * delivery order rank, rank-1, ... (start, end, local expert, destination
 * row, source rank). */
int remora_b200_moe_ep_meta(const int32_t* offsets, int P, int E, int rank, int64_t cap,
                            const uint64_t* meta_ptrs, const int32_t* meta_local,
                            int32_t* flags, const uint64_t* flag_ptrs, int epoch,
                            int32_t* done, int32_t* seg, void* stream);

/* Step 2: one cooperative kernel (one CTA per SM) that does the whole
 * expert side.  Two extra warps per CTA copy this rank's n dispatched rows
 * into region `rank` of their owners' recv (destinations in the order rank,
 * rank+1, ...) and publish `epoch` (the layer count, increasing) in the
 * owner's ready slot of an expert once all of the expert's rows are stored.
 * The tcgen05 pipeline meanwhile runs two kinds of tile from one list:
 * SwiGLU tiles over the received segments (recv_local -> h [P*cap, F]; a
 * segment's first tile waits, bounded, for its ready slot) and down tiles
 * (h -> the source rank's y over NVLink; a down tile waits, bounded, until
 * every SwiGLU tile of its 128-row tile is stored).  The SwiGLU tiles of a
 * group of 16 row tiles come before the down tiles of the previous group,
 * so the down epilogues' NVLink stores overlap later SwiGLU tensor work.
 * wg, wu [E/P, D, F], wd [E/P, F, D]: this rank's experts.  mt_done: local
 * int32 scratch of P*cap/128 + E + 1 entries (zeroed by the call).  D and F
 * multiples of 32.  Step 3 is remora_b200_moe_ep_barrier, then the local
 * remora_b200_moe_combine_bf16 of y. */
int remora_b200_moe_ep_experts_fused_bf16(
    const void* x, const int32_t* perm, const int32_t* offsets, int64_t n, int k, int64_t D,
    int64_t F, int E, int P, int rank, int64_t cap, const uint64_t* recv_ptrs,
    const uint64_t* ready_ptrs, const int32_t* ready_local, int32_t* done, int epoch,
    const void* recv_local, const void* wg, const void* wu, const void* wd, void* h,
    const int32_t* seg, int32_t* mt_done, const uint64_t* y_ptrs, void* stream);

/* ------------------------------------------------------------------------
 * Expert-parallel MoE over NCCL (the all-to-all form).  One process or host
 * thread per GPU; `comm` is an ncclComm_t (passed as void*) over the P ranks
 * of the layer, created by the caller (or remora_b200_nccl_comm_init).
 * NCCL is loaded at run time (libnccl.so.2, the copy the process already
 * has if any), so the library has no link-time NCCL dependency.  The
 * reference has no multi-GPU path (one device, compiler/gpu_tests.cpp:102-104);
 * these serve the mixtral_moe_layer.mlir:8-68 program with its experts
 * split over the ranks.
 * --------------------------------------------------------------------- */

/* Bytes of device workspace remora_b200_moe_ep_nccl_bf16 needs (0 for sizes
 * it rejects).  Sized for the worst case: P*T*k rows may arrive. */
size_t remora_b200_moe_ep_nccl_workspace_bytes(int64_t T, int64_t D, int64_t F, int E, int k,
                                               int P);

/* The whole layer on this rank: x bf16 [T, D] (this rank's tokens; every
 * rank passes the same T), wr bf16 [D, E] (the full router), wg, wu bf16
 * [E/P, D, F] and wd [E/P, F, D] (this rank's experts: global experts
 * rank*E/P ...), out bf16 [T, D].  Router, dispatch and gather run locally;
 * the per-expert counts and then the rows go to the experts' ranks by
 * ncclSend/ncclRecv; the local grouped SwiGLU and down GEMMs run over the
 * (source rank, local expert) segments; the outputs return the same way and
 * are combined in slot order.  The result equals the single-GPU layer bit
 * for bit.  The split sizes are read on the host once per call (2E+1
 * int32), which synchronises `stream` once.  Host waits are bounded by
 * timeout_ms (0 = 60 s): on expiry or on an NCCL error the communicator is
 * aborted (ncclCommAbort, which ends its kernels) and the call returns
 * REMORA_B200_ERR_TIMEOUT or REMORA_B200_ERR_NCCL.  Either code means the
 * communicator has been aborted (and freed): do not use or destroy it again.  Works with blocking and non-blocking
 * (config.blocking = 0) communicators.  D, F multiples of 32. */
int remora_b200_moe_ep_nccl_bf16(const void* x, const void* wr, const void* wg, const void* wu,
                                 const void* wd, void* out, int64_t T, int64_t D, int64_t F,
                                 int E, int k, void* comm, int64_t timeout_ms, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* Host-side split bookkeeping of the exchange (no GPU needed): from this
 * rank's dispatch offsets[E+1] and the received counts recv_counts[P][E/P]
 * (rows source s routes to local expert e), the row block this rank sends
 * to each rank q (send_off[q], send_rows[q]: dispatch rows of q's experts)
 * and the block it receives from each (recv_off[q], recv_rows[q]: sources in
 * rank order, each source's rows in local-expert order). */
int remora_b200_moe_ep_splits(const int32_t* offsets, const int32_t* recv_counts, int P, int E,
                              int64_t* send_off, int64_t* send_rows, int64_t* recv_off,
                              int64_t* recv_rows);

/* Communicator helpers for callers without their own NCCL bootstrap:
 * rank 0 makes a 128-byte unique id and shares it with the others (any
 * channel); every rank then calls remora_b200_nccl_comm_init with its
 * device current.  blocking = 0 makes a non-blocking communicator whose
 * initialisation is polled until timeout_ms (0 = 60 s), then aborted.
 * remora_b200_nccl_comm_destroy finalises (bounded the same way) and frees;
 * remora_b200_nccl_comm_abort ends a communicator at once. */
int remora_b200_nccl_unique_id(void* id);
int remora_b200_nccl_comm_init(void** comm, int nranks, const void* id, int rank, int blocking,
                               int64_t timeout_ms);
int remora_b200_nccl_comm_destroy(void* comm, int64_t timeout_ms);
int remora_b200_nccl_comm_abort(void* comm);

/* ------------------------------------------------------------------------
 * Seeded input generator (device side of the counter-based generator the
 * tests and benchmarks use; one stream key per tensor)
 * --------------------------------------------------------------------- */

/* out[i] = mean + sigma * N(0,1) draw i (Box-Muller in double), as f32
 * (dtype 0) or bf16 (dtype 1, f32 then round to nearest even). */
int remora_b200_fill_normal(void* out, int64_t n, int dtype, uint64_t key, double mean,
                            double sigma, void* stream);

/* out[i] = lo + (hi - lo) * U(0,1) draw i, as f32 (dtype 0) or bf16 (1). */
int remora_b200_fill_uniform(void* out, int64_t n, int dtype, uint64_t key, double lo,
                             double hi, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* REMORA_B200_H */
