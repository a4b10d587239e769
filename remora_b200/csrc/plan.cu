// plan.cu -- the launch plan of a recognised program, in place of the PTX that
// remora's --emit-ptx prints (compiler/gpu.cpp:222-224 prints the NVVM PTX
// modules).  This backend ships hand-written sm_100a kernels, so what it can
// show is which entry points a --test kind calls and, for each, the kernels
// with their launch geometry (grid x block, dynamic shared memory) and
// argument shapes, computed by the same host rules the entry points use.
#include <string>

#include "runtime.cuh"

namespace rb {
namespace plan {

struct Text {
  std::string s;
  void add(const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    s += buf;
  }
};

void gemm_plan(Text& t, int64_t batch, int64_t M, int64_t N, int64_t K) {
  const int64_t tiles = batch * ((M + gemm::BM - 1) / gemm::BM) * ((N + gemm::BN - 1) / gemm::BN);
  t.add("remora_b200_gemm_bf16(A bf16[%lld,%lld,%lld], B bf16[%lld,%lld,%lld] (KN), "
        "C bf16[%lld,%lld,%lld])\n",
        (long long)batch, (long long)M, (long long)K, (long long)batch, (long long)K,
        (long long)N, (long long)batch, (long long)M, (long long)N);
  t.add("  rb::gemm::k_gemm_bf16  grid %lld x block %d, smem %u B; %lld tiles of %dx%d, "
        "K step %d, %d-stage TMA ring, tcgen05 M128 N256 K16, TMEM accumulators\n",
        (long long)std::min<int64_t>(num_sms(), tiles), gemm::kThreads, gemm::kSmemBytes,
        (long long)tiles, gemm::BM, gemm::BN, gemm::BK, gemm::kStages);
}

void moe_plan(Text& t, int64_t T, int64_t D, int64_t F, int E, int k) {
  using namespace moe;
  const int64_t n = T * k, nb = dispatch_blocks(n);
  const RouterPlan rp = router_plan(T, E);
  t.add("remora_b200_moe_layer_bf16(x bf16[%lld,%lld], wr bf16[%lld,%d], wg/wu bf16[%d,%lld,%lld], "
        "wd bf16[%d,%lld,%lld], out bf16[%lld,%lld]), top-%d, workspace %zu B\n",
        (long long)T, (long long)D, (long long)D, E, E, (long long)D, (long long)F, E,
        (long long)F, (long long)D, (long long)T, (long long)D, k,
        remora_b200_moe_workspace_bytes(T, D, F, E, k));
  t.add("  rb::moe::%s  grid %lld x block %d, smem %zu B (LE %d lanes per token group)\n",
        rp.name, (long long)rp.grid, rp.warps * 32, rp.smem, rp.le);
  t.add("  rb::moe::k_dispatch_count  grid %lld x block %d, smem %d B\n", (long long)nb,
        kDispThreads, E * 4);
  t.add("  rb::moe::k_dispatch_scan  grid 1 x block %d\n", kScanThreads);
  t.add("  rb::moe::k_dispatch_scatter  grid %lld x block %d, smem %d B\n", (long long)nb,
        kDispThreads, 32 * E * 4);
  const int64_t scatter_grid = std::min<int64_t>((T + 7) / 8, (int64_t)num_sms() * 16);
  t.add("  rb::moe::k_scatter_rows  grid %lld x block 256 (%lld token rows of %lld bf16, %d "
        "copies each)\n",
        (long long)scatter_grid, (long long)T, (long long)D, k);
  const int64_t up_tiles = (n / GBM + E) * ((F + 127) / 128);
  const int64_t dn_tiles = (n / GBM + E) * ((D + 255) / 256);
  t.add("  rb::moe::k_grouped_gemm<true>  grid %lld x block %d, smem %u B (SwiGLU: gate|up "
        "128+128 TMEM columns per 128-row tile)\n",
        (long long)std::min<int64_t>(num_sms(), up_tiles), GThreads, GSmemBytes);
  t.add("  rb::moe::k_grouped_gemm<false>  grid %lld x block %d, smem %u B (down: 256-column "
        "tiles)\n",
        (long long)std::min<int64_t>(num_sms(), dn_tiles), GThreads, GSmemBytes);
  const int kmax = k <= 2 ? 2 : k <= 4 ? 4 : k <= 8 ? 8 : 16;
  t.add("  rb::moe::k_combine<%d>  grid %lld x block 256\n", kmax,
        (long long)std::min<int64_t>((T + 7) / 8, (int64_t)num_sms() * 16));
}

void hetero_plan(Text& t) {
  using namespace moe;
  const int64_t T = 512, D = 4096;
  const int64_t F[8] = {14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048};
  const RouterPlan rp = router_plan(T, 8);
  t.add("remora_b200_moe_hetero_layer_bf16(x bf16[512,4096], wr bf16[4096,8], wg[e]/wu[e] "
        "bf16[4096,F_e], wd[e] bf16[F_e,4096], F_e = 14336 14336 8192 8192 4096 4096 2048 2048, "
        "out bf16[512,4096]), top-1, workspace %zu B\n",
        remora_b200_moe_hetero_workspace_bytes(T, D, F, 8, 1));
  t.add("  rb::moe::%s  grid %lld x block %d, smem %zu B\n", rp.name, (long long)rp.grid,
        rp.warps * 32, rp.smem);
  t.add("  rb::moe::k_dispatch_count / k_dispatch_scan / k_dispatch_scatter  grid 1 / 1 / 1\n");
  t.add("  rb::moe::k_gather_rows  grid 64 x block 256 (512 rows of 4096 bf16)\n");
  t.add("  rb::moe::k_grouped_var<true>  grid %d x block %d, smem %u B (per-expert tensor maps; "
        "column tiles of 128 up to each F_e)\n", num_sms(), GThreads, GSmemBytes);
  t.add("  rb::moe::k_grouped_var<false>  grid %d x block %d, smem %u B (K = F_e per expert)\n",
        num_sms(), GThreads, GSmemBytes);
  t.add("  rb::moe::k_combine<2>  grid 64 x block 256\n");
}

}  // namespace plan
}  // namespace rb

extern "C" int remora_b200_launch_plan(const char* test, const char* config, char* out,
                                       size_t out_bytes) {
  using namespace rb;
  using namespace rb::plan;
  clear_error();
  RB_CHECK_ARG(test && out && out_bytes > 0, "launch_plan: null argument");
  const std::string kind = test, c = config ? config : "";
  Text t;
  if (kind == "elementwise") {
    const int64_t n = 512 * 768;
    t.add("remora_b200_relu_bias_f32(x f32[1,512,768], bias f32[768], out f32[1,512,768])\n");
    t.add("  rb::k_relu_bias_v4  grid %d x block 256 (%lld float4, grid-stride)\n",
          ew_grid(n / 4, 256), (long long)(n / 4));
  } else if (kind == "elementwise_chain") {
    const int64_t n4 = 8 * 128 * 128 / 4;
    t.add("remora_b200_scale_add_exp_f32(s f32[1,8,128,128], b f32[1,8,128,128], scale 0.125, "
          "out f32[1,8,128,128])\n");
    t.add("  rb::k_scale_add_exp_v4  grid %d x block 256 (%lld float4, two per thread)\n",
          ew_grid((n4 + 1) / 2, 256), (long long)n4);
  } else if (kind == "projection") {
    t.add("remora_b200_gemm_f32_exact(x f32[512,768], w f32[768,768] (KN), out f32[512,768])\n");
    t.add("  rb::k_gemm_f32_exact  grid %d x %d x block 256 (%dx%d output tiles, serial "
          "increasing-k fp32 chains)\n",
          (768 + F32_TN - 1) / F32_TN, (512 + F32_TM - 1) / F32_TM, F32_TM, F32_TN);
  } else if (kind == "gemm") {
    long long a = 0, b = 0, kk = 0;
    if (c.empty() || c == "8192")
      gemm_plan(t, 1, 8192, 8192, 8192);
    else if (c == "batched")
      gemm_plan(t, 8, 4096, 4096, 4096);
    else if (sscanf(c.c_str(), "%lldx%lldx%lld", &a, &b, &kk) == 3)
      gemm_plan(t, 1, a, b, kk);
    else
      return fail(REMORA_B200_ERR_INVALID, "launch_plan: unknown gemm config '%s'", c.c_str());
  } else if (kind == "attention") {
    long long B = 4, H = 32, S = 4096;
    if (!c.empty() && sscanf(c.c_str(), "%lldx%lldx%lld", &B, &H, &S) != 3)
      return fail(REMORA_B200_ERR_INVALID, "launch_plan: unknown attention config '%s'",
                  c.c_str());
    const int64_t chunks = (S + 2 * attn::BQ - 1) / (2 * attn::BQ);
    t.add("remora_b200_attention_fwd_bf16(q, k, v, out bf16[%lld,%lld,%lld,128], causal)\n", B, H,
          S);
    const long long items = (long long)(chunks * B * H);
    t.add("  rb::attnp::k_attention_persist  grid %lld x block %d, smem %u B (persistent: %lld "
          "work items of one (b,h) and 256 query rows)\n",
          std::min<long long>(items, num_sms()), attnp::kThreads, attn::kSmemBytes, items);
  } else if (kind == "moe") {
    if (c.empty() || c == "4")
      moe_plan(t, 8192, 4096, 14336, 8, 2);
    else if (c == "5")
      moe_plan(t, 65536, 2048, 1536, 64, 8);
    else if (c == "mixtral")
      moe_plan(t, 512, 4096, 14336, 8, 2);
    else if (c == "simple")
      moe_plan(t, 8, 32, 64, 2, 1);
    else if (c == "hetero")
      hetero_plan(t);
    else
      return fail(REMORA_B200_ERR_INVALID, "launch_plan: unknown moe config '%s'", c.c_str());
  } else {
    return fail(REMORA_B200_ERR_UNSUPPORTED, "launch_plan: test '%s' not recognised", test);
  }
  const size_t m = std::min(out_bytes - 1, t.s.size());
  memcpy(out, t.s.data(), m);
  out[m] = '\0';
  return t.s.size() < out_bytes ? REMORA_B200_OK
                                 : fail(REMORA_B200_ERR_INVALID, "launch_plan: buffer too small");
}
