// dispatch.cu -- the --test=<kind> dispatcher that replaces the body of
// remora's launchOnGpu (compiler/gpu_tests.cpp:101-125) for recognised
// programs.  Each kind owns its buffers end to end, fills its inputs,
// launches through the per-op C ABI, times with CUDA events and validates on
// the host, as launchElementwiseOnGpu (gpu_tests.cpp:35-95) did -- except
// that a validation failure is a non-zero status here.
#include <algorithm>
#include <cmath>
#include <string>
#include <vector>

#include "runtime.cuh"

namespace rb {

struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int alloc(size_t bytes) {
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
      return fail(REMORA_B200_ERR_CUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
    return REMORA_B200_OK;
  }
};

struct Timer {
  cudaEvent_t a = nullptr, b = nullptr;
  ~Timer() {
    if (a) cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
  }
};

static uint64_t host_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Stream key of tensor `stream` under `seed` (the generator's key schedule).
static uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return host_mix64(seed * 0x9E3779B97F4A7C15ull + stream);
}

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

// Relative error as |g - r| / max(|r|, floor), floor = 1e-3 * max|r|.
struct ErrStat {
  double max_abs = 0, max_rel = 0;
  int64_t n = 0;
  void add(double g, double r, double floor) {
    double a = std::fabs(g - r);
    double d = std::max(std::fabs(r), floor);
    if (!(a <= max_abs)) max_abs = a;
    double rel = d > 0 ? a / d : a;
    if (!(rel <= max_rel)) max_rel = rel;
    ++n;
  }
};

template <class F>
static int time_iters(const remora_b200_opts* o, cudaStream_t st, F&& launch, double* ms) {
  Timer t;
  RB_CUDA(cudaEventCreate(&t.a));
  RB_CUDA(cudaEventCreate(&t.b));
  int iters = o && o->iters > 0 ? o->iters : 1;
  int warm = o ? o->warmup : 0;
  for (int i = 0; i < warm; ++i) {
    int rc = launch();
    if (rc) return rc;
  }
  RB_CUDA(cudaEventRecord(t.a, st));
  for (int i = 0; i < iters; ++i) {
    int rc = launch();
    if (rc) return rc;
  }
  RB_CUDA(cudaEventRecord(t.b, st));
  RB_CUDA(cudaEventSynchronize(t.b));
  float f = 0;
  RB_CUDA(cudaEventElapsedTime(&f, t.a, t.b));
  *ms = (double)f / iters;
  return collect_device_error(st);
}

static void finish(remora_b200_report* r, double ms, double work, const ErrStat& e, double tol,
                   bool validate, const char* what, const char* unit) {
  r->ms_per_iter = ms;
  r->work = work;
  r->rate = ms > 0 ? work / (ms * 1e-3) : 0;
  r->max_abs_err = e.max_abs;
  r->max_rel_err = e.max_rel;
  r->checked = e.n;
  r->passed = !validate || (e.n > 0 && e.max_rel <= tol);
  snprintf(r->detail, sizeof(r->detail), "%s: %.4f ms/iter, %.3f %s, checked %lld, max rel %.3g (tol %.1g) %s",
           what, ms, r->rate * 1e-12, unit, (long long)e.n, e.max_rel, tol,
           validate ? (r->passed ? "PASS" : "FAIL") : "");
}

// --test=elementwise: relu(x + bias) on f32 [1,512,768], x = 1, bias = -0.5,
// expected 0.5 everywhere within 1e-5 (gpu_tests.cpp:36, :53-56, :88-91).
static int run_elementwise(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  const int64_t N = 1, T = 512, D = 768, n = N * T * D;
  DevBuf x, b, out;
  int rc;
  if ((rc = x.alloc(n * 4)) || (rc = b.alloc(D * 4)) || (rc = out.alloc(n * 4))) return rc;
  std::vector<float> hx(n, 1.0f), hb(D, -0.5f), ho(n);
  RB_CUDA(cudaMemcpyAsync(x.p, hx.data(), n * 4, cudaMemcpyHostToDevice, st));
  RB_CUDA(cudaMemcpyAsync(b.p, hb.data(), D * 4, cudaMemcpyHostToDevice, st));
  double ms = 0;
  rc = time_iters(o, st, [&] {
    return remora_b200_relu_bias_f32((const float*)x.p, (const float*)b.p, (float*)out.p, N * T,
                                     D, st);
  }, &ms);
  if (rc) return rc;
  RB_CUDA(cudaMemcpy(ho.data(), out.p, n * 4, cudaMemcpyDeviceToHost));
  ErrStat e;
  for (float v : ho) e.add(v, 0.5, 0.0);
  finish(r, ms, (double)(2 * n * 4 + D * 4), e, 1e-5 / 0.5, true, "elementwise relu(x+bias)",
         "TB/s");
  return REMORA_B200_OK;
}

// --test=projection: x = 1 [1,512,768] . w = 1/768 [768,768] -> 1.0
// (cpu_tests.cpp:65-97), through the exact f32 path.
static int run_projection(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  const int64_t M = 512, K = 768, N = 768;
  DevBuf x, w, out;
  int rc;
  if ((rc = x.alloc(M * K * 4)) || (rc = w.alloc(K * N * 4)) || (rc = out.alloc(M * N * 4)))
    return rc;
  std::vector<float> hx(M * K, 1.0f), hw(K * N, 1.0f / 768.0f), ho(M * N);
  RB_CUDA(cudaMemcpyAsync(x.p, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice, st));
  RB_CUDA(cudaMemcpyAsync(w.p, hw.data(), hw.size() * 4, cudaMemcpyHostToDevice, st));
  double ms = 0;
  rc = time_iters(o, st, [&] {
    return remora_b200_gemm_f32_exact((const float*)x.p, (const float*)w.p, (float*)out.p, M, N,
                                      K, K, N, N, REMORA_B200_B_KN, st);
  }, &ms);
  if (rc) return rc;
  RB_CUDA(cudaMemcpy(ho.data(), out.p, ho.size() * 4, cudaMemcpyDeviceToHost));
  // The loop nest's own value: fill 0, then 768 separately rounded adds.
  float expect = 0.0f;
  {
    volatile float a = 0.0f;
    for (int k = 0; k < 768; ++k) {
      volatile float p = 1.0f * (1.0f / 768.0f);
      a = a + p;
    }
    expect = a;
  }
  ErrStat e;
  for (float v : ho) e.add(v, expect, 0.0);
  finish(r, ms, 2.0 * M * N * K, e, 1e-5, true, "projection f32 exact", "TFLOP/s");
  return REMORA_B200_OK;
}

// The scale -> add -> exp chain on f32 [1,8,128,128] seeded N(0,1).
static int run_chain(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  const int64_t n = 1 * 8 * 128 * 128;
  const uint64_t seed = o && o->seed ? o->seed : 42;
  DevBuf s, b, out;
  int rc;
  if ((rc = s.alloc(n * 4)) || (rc = b.alloc(n * 4)) || (rc = out.alloc(n * 4))) return rc;
  if ((rc = remora_b200_fill_normal(s.p, n, 0, stream_key(seed, 1), 0.0, 1.0, st))) return rc;
  if ((rc = remora_b200_fill_normal(b.p, n, 0, stream_key(seed, 2), 0.0, 1.0, st))) return rc;
  const float scale = 0.125f;  // 1/sqrt(64)
  double ms = 0;
  rc = time_iters(o, st, [&] {
    return remora_b200_scale_add_exp_f32((const float*)s.p, (const float*)b.p, (float*)out.p, n,
                                         scale, st);
  }, &ms);
  if (rc) return rc;
  std::vector<float> hs(n), hb(n), ho(n);
  RB_CUDA(cudaMemcpy(hs.data(), s.p, n * 4, cudaMemcpyDeviceToHost));
  RB_CUDA(cudaMemcpy(hb.data(), b.p, n * 4, cudaMemcpyDeviceToHost));
  RB_CUDA(cudaMemcpy(ho.data(), out.p, n * 4, cudaMemcpyDeviceToHost));
  ErrStat e;
  for (int64_t i = 0; i < n; ++i) {
    volatile float t = hs[i] * scale;
    volatile float u = t + hb[i];
    e.add(ho[i], (double)expf(u), 0.0);
  }
  finish(r, ms, (double)n * 12, e, 1e-5, o ? o->validate : 0, "scale-add-exp chain", "TB/s");
  return REMORA_B200_OK;
}

// dot_general bf16 [M,K] x [K,N], U(-1,1) inputs; config "8192" (default),
// "batched" (8 x 4096^3) or "MxNxK".  Validation samples 4096 outputs.
static int run_gemm(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  int64_t batch = 1, M = 8192, N = 8192, K = 8192;
  if (o && o->config && *o->config) {
    std::string c = o->config;
    long long a = 0, b2 = 0, k = 0;
    if (c == "batched") {
      batch = 8; M = N = K = 4096;
    } else if (sscanf(c.c_str(), "%lldx%lldx%lld", &a, &b2, &k) == 3) {
      M = a; N = b2; K = k;
    } else if (c != "8192") {
      return fail(REMORA_B200_ERR_INVALID, "gemm: unknown config '%s'", c.c_str());
    }
  }
  const uint64_t seed = o && o->seed ? o->seed : 42;
  DevBuf A, B, C;
  int rc;
  if ((rc = A.alloc(batch * M * K * 2)) || (rc = B.alloc(batch * K * N * 2)) ||
      (rc = C.alloc(batch * M * N * 2)))
    return rc;
  if ((rc = remora_b200_fill_uniform(A.p, batch * M * K, 1, stream_key(seed, 10), -1, 1, st)))
    return rc;
  if ((rc = remora_b200_fill_uniform(B.p, batch * K * N, 1, stream_key(seed, 11), -1, 1, st)))
    return rc;
  double ms = 0;
  rc = time_iters(o, st, [&] {
    return remora_b200_gemm_bf16(A.p, B.p, C.p, batch, M, N, K, K, N, N, M * K, K * N, M * N,
                                 REMORA_B200_B_KN, st);
  }, &ms);
  if (rc) return rc;
  ErrStat e;
  if (o && o->validate) {
    std::vector<uint16_t> hA(batch * M * K), hB(batch * K * N), hC(batch * M * N);
    RB_CUDA(cudaMemcpy(hA.data(), A.p, hA.size() * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hB.data(), B.p, hB.size() * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hC.data(), C.p, hC.size() * 2, cudaMemcpyDeviceToHost));
    const double floor = 1e-3 * std::sqrt((double)K);  // |C| scales as sqrt(K)/3
    uint64_t key = stream_key(seed, 99);
    for (int s2 = 0; s2 < 4096; ++s2) {
      uint64_t h = host_mix64(key + (uint64_t)s2 * 0x9E3779B97F4A7C15ull);
      int64_t b = (int64_t)(h % (uint64_t)batch);
      int64_t i = (int64_t)((h >> 16) % (uint64_t)M), j = (int64_t)((h >> 40) % (uint64_t)N);
      float acc = 0.0f;
      for (int64_t k = 0; k < K; ++k)
        acc += bf16_to_f32(hA[b * M * K + i * K + k]) * bf16_to_f32(hB[b * K * N + k * N + j]);
      e.add(bf16_to_f32(hC[b * M * N + i * N + j]), acc, floor);
    }
  }
  finish(r, ms, 2.0 * batch * M * N * K, e, 2e-2, o ? o->validate : 0, "gemm bf16", "TFLOP/s");
  return REMORA_B200_OK;
}

// Causal softmax attention, bf16 [B,H,S,128] N(0,1); config "4x32x4096"
// (default) or "BxHxS"; validation: 64 (head, row) samples, full rows of
// the output against a double-precision softmax on the host, normwise
// relative error per row (max |g - r| / max |r|).
static int run_attention(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  long long B = 4, H = 32, S = 4096;
  const int64_t Dh = 128;
  if (o && o->config && *o->config) {
    if (sscanf(o->config, "%lldx%lldx%lld", &B, &H, &S) != 3)
      return fail(REMORA_B200_ERR_INVALID, "attention: unknown config '%s'", o->config);
  }
  const uint64_t seed = o && o->seed ? o->seed : 42;
  const int64_t n = B * H * S * Dh;
  DevBuf q, k, v, out;
  int rc;
  if ((rc = q.alloc(n * 2)) || (rc = k.alloc(n * 2)) || (rc = v.alloc(n * 2)) ||
      (rc = out.alloc(n * 2)))
    return rc;
  if ((rc = remora_b200_fill_normal(q.p, n, 1, stream_key(seed, 20), 0, 1, st)) ||
      (rc = remora_b200_fill_normal(k.p, n, 1, stream_key(seed, 21), 0, 1, st)) ||
      (rc = remora_b200_fill_normal(v.p, n, 1, stream_key(seed, 22), 0, 1, st)))
    return rc;
  const float scale = 1.0f / sqrtf((float)Dh);
  double ms = 0;
  rc = time_iters(o, st, [&] {
    return remora_b200_attention_fwd_bf16(q.p, k.p, v.p, out.p, B, H, S, Dh, 1, scale, st);
  }, &ms);
  if (rc) return rc;
  ErrStat e;
  if (o && o->validate) {
    std::vector<uint16_t> hq(n), hk(n), hv(n), ho(n);
    RB_CUDA(cudaMemcpy(hq.data(), q.p, n * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hk.data(), k.p, n * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hv.data(), v.p, n * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(ho.data(), out.p, n * 2, cudaMemcpyDeviceToHost));
    std::vector<double> pr(S), acc(Dh);
    uint64_t key = stream_key(seed, 98);
    for (int s2 = 0; s2 < 64; ++s2) {
      uint64_t h = host_mix64(key + (uint64_t)s2 * 0x9E3779B97F4A7C15ull);
      int64_t bh = (int64_t)(h % (uint64_t)(B * H)), i = (int64_t)((h >> 20) % (uint64_t)S);
      const uint16_t* Q = hq.data() + (bh * S + i) * Dh;
      double m = -1e300;
      for (int64_t j = 0; j <= i; ++j) {
        const uint16_t* Kr = hk.data() + (bh * S + j) * Dh;
        double d = 0;
        for (int64_t c = 0; c < Dh; ++c) d += (double)bf16_to_f32(Q[c]) * bf16_to_f32(Kr[c]);
        pr[j] = d * scale;
        m = std::max(m, pr[j]);
      }
      double l = 0;
      for (int64_t j = 0; j <= i; ++j) { pr[j] = std::exp(pr[j] - m); l += pr[j]; }
      std::fill(acc.begin(), acc.end(), 0.0);
      for (int64_t j = 0; j <= i; ++j) {
        const uint16_t* Vr = hv.data() + (bh * S + j) * Dh;
        for (int64_t c = 0; c < Dh; ++c) acc[c] += pr[j] / l * bf16_to_f32(Vr[c]);
      }
      double mx = 0;
      for (int64_t c = 0; c < Dh; ++c) mx = std::max(mx, std::fabs(acc[c]));
      for (int64_t c = 0; c < Dh; ++c)
        e.add(bf16_to_f32(ho[(bh * S + i) * Dh + c]), acc[c], std::max(mx, 1e-6));  // normwise per row
    }
  }
  const double flops = 4.0 * B * H * (double)S * S * Dh / 2.0;  // causal half
  finish(r, ms, flops, e, 2e-2, o ? o->validate : 0, "attention causal bf16", "TFLOP/s");
  return REMORA_B200_OK;
}

// --test=moe: the MoE layer of mlir/stablehlo/mixtral_moe_layer.mlir:8-68
// with bf16 operands.  config "4" (default: T=8192 D=4096 F=14336 E=8 top-2),
// "5" (T=65536 D=2048 F=1536 E=64 top-8), "mixtral" (the program's own
// T=512 D=4096 F=14336 E=8 top-2) or "simple" (simple_moe.mlir:16:
// T=8 D=32 F=64 E=2 top-1).  Tokens N(0,1), weights N(0,0.02), seeded.
// Validation on up to 16 sampled tokens: router indices exactly as the
// increasing-d fp32 loop nest gives them, layer output normwise <= 2e-2.
// config "hetero": heterogeneous_moe_layer.mlir:66-212 (T=512, D=4096,
// experts of F 14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048, top-1)
// through remora_b200_moe_hetero_layer_bf16; expert e's weights follow
// expert e-1's in one buffer per kind.
static int run_moe(const remora_b200_opts* o, remora_b200_report* r, cudaStream_t st) {
  int64_t T = 8192, D = 4096, F = 14336;
  int E = 8, k = 2;
  std::string c = o && o->config ? o->config : "4";
  std::vector<int64_t> Fe;
  if (c == "5") { T = 65536; D = 2048; F = 1536; E = 64; k = 8; }
  else if (c == "mixtral") { T = 512; }
  else if (c == "simple") { T = 8; D = 32; F = 64; E = 2; k = 1; }
  else if (c == "hetero") {
    T = 512; k = 1;
    Fe = {14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048};
  }
  else if (c != "4") return fail(REMORA_B200_ERR_INVALID, "moe: unknown config '%s'", c.c_str());
  const bool hetero = !Fe.empty();
  if (!hetero) Fe.assign(E, F);
  std::vector<int64_t> off(E + 1, 0);  // element offset of expert e's weights
  for (int e = 0; e < E; ++e) off[e + 1] = off[e] + D * Fe[e];
  const int64_t wtot = off[E];
  const uint64_t seed = o && o->seed ? o->seed : 42;
  DevBuf x, wr, wg, wu, wd, out, ws, idx, w;
  const size_t wsb = hetero ? remora_b200_moe_hetero_workspace_bytes(T, D, Fe.data(), E, k)
                            : remora_b200_moe_workspace_bytes(T, D, F, E, k);
  int rc;
  if ((rc = x.alloc(T * D * 2)) || (rc = wr.alloc(D * E * 2)) || (rc = wg.alloc(wtot * 2)) ||
      (rc = wu.alloc(wtot * 2)) || (rc = wd.alloc(wtot * 2)) ||
      (rc = out.alloc(T * D * 2)) || (rc = ws.alloc(wsb)) || (rc = idx.alloc(T * k * 4)) ||
      (rc = w.alloc(T * k * 4)))
    return rc;
  if ((rc = remora_b200_fill_normal(x.p, T * D, 1, stream_key(seed, 30), 0, 1, st)) ||
      (rc = remora_b200_fill_normal(wr.p, D * E, 1, stream_key(seed, 31), 0, 0.02, st)) ||
      (rc = remora_b200_fill_normal(wg.p, wtot, 1, stream_key(seed, 32), 0, 0.02, st)) ||
      (rc = remora_b200_fill_normal(wu.p, wtot, 1, stream_key(seed, 33), 0, 0.02, st)) ||
      (rc = remora_b200_fill_normal(wd.p, wtot, 1, stream_key(seed, 34), 0, 0.02, st)))
    return rc;
  std::vector<const void*> pg(E), pu(E), pd(E);
  for (int e = 0; e < E; ++e) {
    pg[e] = (const uint16_t*)wg.p + off[e];
    pu[e] = (const uint16_t*)wu.p + off[e];
    pd[e] = (const uint16_t*)wd.p + off[e];
  }
  double ms = 0;
  rc = time_iters(o, st, [&] {
    if (hetero)
      return remora_b200_moe_hetero_layer_bf16(x.p, wr.p, pg.data(), pu.data(), pd.data(),
                                               Fe.data(), out.p, T, D, E, k, ws.p, wsb, st);
    return remora_b200_moe_layer_bf16(x.p, wr.p, wg.p, wu.p, wd.p, out.p, T, D, F, E, k, ws.p,
                                      wsb, st);
  }, &ms);
  if (rc) return rc;
  ErrStat e;
  bool idx_ok = true;
  if (o && o->validate) {
    if ((rc = remora_b200_moe_router_topk_bf16(x.p, wr.p, T, D, E, k, (int32_t*)idx.p,
                                               (float*)w.p, st)))
      return rc;
    RB_CUDA(cudaStreamSynchronize(st));
    std::vector<uint16_t> hx(T * D), hwr(D * E), ho(T * D);
    std::vector<int32_t> hidx(T * k);
    RB_CUDA(cudaMemcpy(hx.data(), x.p, hx.size() * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hwr.data(), wr.p, hwr.size() * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(ho.data(), out.p, ho.size() * 2, cudaMemcpyDeviceToHost));
    RB_CUDA(cudaMemcpy(hidx.data(), idx.p, hidx.size() * 4, cudaMemcpyDeviceToHost));
    const int ns = (int)std::min<int64_t>(T, 16);
    std::vector<std::vector<uint16_t>> eg(E), eu(E), ed(E);
    const int64_t Fmax = *std::max_element(Fe.begin(), Fe.end());
    std::vector<double> ref(D), hrow(Fmax), g(Fmax), u(Fmax);
    double worst = 0, scale = 0;
    for (int si = 0; si < ns; ++si) {
      const int64_t t = (int64_t)(host_mix64(stream_key(seed, 97) + si) % (uint64_t)T);
      const uint16_t* xr = hx.data() + t * D;
      std::vector<float> lg(E, 0.0f);
      for (int64_t d = 0; d < D; ++d)
        for (int ee = 0; ee < E; ++ee) lg[ee] = lg[ee] + bf16_to_f32(xr[d]) * bf16_to_f32(hwr[d * E + ee]);
      std::vector<int> sel;
      std::vector<float> sv;
      std::vector<char> used(E, 0);
      for (int j = 0; j < k; ++j) {
        int best = -1;
        for (int ee = 0; ee < E; ++ee)
          if (!used[ee] && (best < 0 || lg[ee] > lg[best])) best = ee;  // ties -> lower index
        used[best] = 1;
        sel.push_back(best);
        sv.push_back(lg[best]);
        if (hidx[t * k + j] != best) idx_ok = false;
      }
      float m = -INFINITY, ssum = 0.0f;
      for (float v : sv) m = v > m ? v : m;
      std::vector<float> ex(k);
      for (int j = 0; j < k; ++j) { ex[j] = expf(sv[j] - m); ssum = ssum + ex[j]; }
      std::fill(ref.begin(), ref.end(), 0.0);
      for (int j = 0; j < k; ++j) {
        const int ee = sel[j];
        const int64_t F = Fe[ee];
        if (eg[ee].empty()) {
          eg[ee].resize(D * F); eu[ee].resize(D * F); ed[ee].resize(F * D);
          RB_CUDA(cudaMemcpy(eg[ee].data(), pg[ee], D * F * 2, cudaMemcpyDeviceToHost));
          RB_CUDA(cudaMemcpy(eu[ee].data(), pu[ee], D * F * 2, cudaMemcpyDeviceToHost));
          RB_CUDA(cudaMemcpy(ed[ee].data(), pd[ee], F * D * 2, cudaMemcpyDeviceToHost));
        }
        std::fill(g.begin(), g.end(), 0.0);
        std::fill(u.begin(), u.end(), 0.0);
        for (int64_t d = 0; d < D; ++d) {
          const double a = bf16_to_f32(xr[d]);
          const uint16_t* gr = eg[ee].data() + d * F;
          const uint16_t* ur = eu[ee].data() + d * F;
          for (int64_t f = 0; f < F; ++f) { g[f] += a * bf16_to_f32(gr[f]); u[f] += a * bf16_to_f32(ur[f]); }
        }
        for (int64_t f = 0; f < F; ++f) hrow[f] = g[f] / (1.0 + std::exp(-g[f])) * u[f];
        const double wj = ex[j] / ssum;
        for (int64_t f = 0; f < F; ++f) {
          const uint16_t* dr = ed[ee].data() + f * D;
          const double hv = wj * hrow[f];
          for (int64_t d = 0; d < D; ++d) ref[d] += hv * bf16_to_f32(dr[d]);
        }
      }
      for (int64_t d = 0; d < D; ++d) {
        worst = std::max(worst, std::fabs(bf16_to_f32(ho[t * D + d]) - ref[d]));
        scale = std::max(scale, std::fabs(ref[d]));
      }
      e.n += D;
    }
    e.max_abs = worst;
    e.max_rel = scale > 0 ? worst / scale : worst;
  }
  double fsum = 0;  // expert FLOP as if the rows spread evenly over the experts
  for (int64_t f : Fe) fsum += (double)f;
  finish(r, ms, 6.0 * D * (fsum / E) * T * k, e, 2e-2, o ? o->validate : 0,
         hetero ? "heterogeneous moe layer bf16" : "moe layer bf16", "TFLOP/s");
  if (o && o->validate && !idx_ok) {
    r->passed = 0;
    snprintf(r->detail, sizeof(r->detail), "moe layer: router indices differ from the loop nest");
  }
  return REMORA_B200_OK;
}

}  // namespace rb

extern "C" const char* remora_b200_last_error(void) { return rb::t_last_error; }

extern "C" int remora_b200_version(void) { return 100; }

extern "C" int remora_b200_device_status(void) {
  rb::clear_error();
  int v = 0, zero = 0;
  RB_CUDA(cudaDeviceSynchronize());
  RB_CUDA(cudaMemcpyFromSymbol(&v, rb::g_device_error, sizeof(int)));
  if (v == 0) return REMORA_B200_OK;
  RB_CUDA(cudaMemcpyToSymbol(rb::g_device_error, &zero, sizeof(int)));
  if (v == 1) return rb::fail(REMORA_B200_ERR_TIMEOUT, "a device-side wait timed out");
  if (v == 2) return rb::fail(REMORA_B200_ERR_INVALID, "an expert index was outside [0, E)");
  return rb::fail(REMORA_B200_ERR_INVALID, "device reported error %d", v);
}

extern "C" int remora_b200_recognise(const char* test) {
  if (!test) return 0;
  std::string t = test;
  return t == "elementwise" || t == "projection" || t == "elementwise_chain" || t == "gemm" ||
         t == "attention" || t == "moe";
}

extern "C" int remora_b200_run_test(const char* test, const remora_b200_opts* o,
                                    remora_b200_report* r) {
  using namespace rb;
  clear_error();
  RB_CHECK_ARG(test && r, "run_test: null argument");
  memset(r, 0, sizeof(*r));
  RB_CUDA(cudaSetDevice(o ? o->device : 0));
  cudaStream_t st;
  RB_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  std::string t = test;
  int rc;
  if (t == "elementwise")
    rc = run_elementwise(o, r, st);
  else if (t == "projection")
    rc = run_projection(o, r, st);
  else if (t == "elementwise_chain")
    rc = run_chain(o, r, st);
  else if (t == "gemm")
    rc = run_gemm(o, r, st);
  else if (t == "attention")
    rc = run_attention(o, r, st);
  else if (t == "moe")
    rc = run_moe(o, r, st);
  else
    rc = fail(REMORA_B200_ERR_UNSUPPORTED, "--run-gpu for test '%s' not recognised", test);
  cudaStreamDestroy(st);
  if (rc == REMORA_B200_OK && !r->passed)
    rc = fail(REMORA_B200_ERR_PARITY, "%s", r->detail);
  return rc;
}
