// cli.cpp -- `remora-b200`, a standalone driver with remora's argv grammar
// (compiler/main.cpp:19-50):
//
//   remora-b200 <input.mlir> [--test=<kind>] [--run-gpu] [--emit-ptx]
//               [--no-execute] [--config=<name>] [--seed=<n>] [--iters=<n>]
//               [--warmup=<n>] [--device=<n>]
//
// It recognises the shipped StableHLO programs by their @main signature text
// (remora parses them with MLIR, main.cpp:74-79, which is not available
// here), maps them to a --test kind, and hands them to the library's
// dispatcher exactly as the patched launchOnGpu does.  Exit status follows
// remora: 0 on success, 1 on any failure (main.cpp:19-27, gpu_tests.cpp:11-20).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>

#include "../../include/remora_b200.h"

namespace {

struct Program {
  const char* kind;
  const char* config;
  const char* what;
};

// The @main signature of each program in mlir/stablehlo/ (file:line cited).
Program recognise_program(const std::string& text) {
  const size_t at = text.find("@main(");
  const std::string sig = at == std::string::npos ? text : text.substr(at, 1200);
  auto has = [&](const char* s) { return sig.find(s) != std::string::npos; };
  // simple_attention_elementwise.mlir:5
  if (has("tensor<1x512x768xf32>") && has("tensor<768xf32>"))
    return {"elementwise", nullptr, "relu(x + bias), f32 [1,512,768]"};
  // simple_attention_projection.mlir:4
  if (has("tensor<1x512x768xf32>") && has("tensor<768x768xf32>"))
    return {"projection", nullptr, "dot_general x . w, f32 [1,512,768] x [768,768]"};
  // heterogeneous_moe_layer.mlir:66-100: one [1, D, F_e] weight per expert
  if (has("tensor<512x4096xf32>") && has("tensor<1x4096x14336xf32>") &&
      has("tensor<1x4096x2048xf32>"))
    return {"moe", "hetero", "heterogeneous MoE layer T=512 D=4096 F=14336/8192/4096/2048 E=8 top-1"};
  // mixtral_moe_layer.mlir:8
  if (has("tensor<512x4096xf32>") && has("tensor<8x4096x14336xf32>"))
    return {"moe", "mixtral", "MoE layer T=512 D=4096 F=14336 E=8 top-2"};
  // simple_moe.mlir:16
  if (has("tensor<8x32xf32>") && has("tensor<2x32x64xf32>"))
    return {"moe", "simple", "MoE layer T=8 D=32 F=64 E=2 top-1"};
  return {nullptr, nullptr, nullptr};
}

bool read_file(const char* path, std::string* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::stringstream ss;
  ss << f.rdbuf();
  *out = ss.str();
  return true;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr,
                 "Usage: remora-b200 <input.mlir> [--test=<kind>] [--run-gpu] [--emit-ptx] "
                 "[--no-execute] [--config=<name>] [--seed=<n>] [--iters=<n>] [--warmup=<n>] "
                 "[--device=<n>]\n");
    return 1;
  }
  std::string test, config;
  bool run_gpu = false, emit_ptx = false, no_execute = false;
  remora_b200_opts o;
  std::memset(&o, 0, sizeof(o));
  o.iters = 1;
  o.validate = 1;
  for (int i = 2; i < argc; ++i) {
    const char* a = argv[i];
    if (!std::strcmp(a, "--run-gpu")) run_gpu = true;
    else if (!std::strcmp(a, "--emit-ptx")) emit_ptx = true;
    else if (!std::strcmp(a, "--no-execute")) no_execute = true;
    else if (!std::strncmp(a, "--test=", 7)) test = a + 7;
    else if (!std::strncmp(a, "--config=", 9)) config = a + 9;
    else if (!std::strncmp(a, "--seed=", 7)) o.seed = std::strtoull(a + 7, nullptr, 10);
    else if (!std::strncmp(a, "--iters=", 8)) o.iters = std::atoi(a + 8);
    else if (!std::strncmp(a, "--warmup=", 9)) o.warmup = std::atoi(a + 9);
    else if (!std::strncmp(a, "--device=", 9)) o.device = std::atoi(a + 9);
    // remora's IR-tracing flags (--mlir-print-ir-after-all, --pass-pipeline=,
    // --dump-compilation-phases-to=) concern its compiler and are ignored here
  }
  std::string text;
  if (!read_file(argv[1], &text)) {
    std::fprintf(stderr, "Failed to parse: %s\n", argv[1]);
    return 1;
  }
  const Program prog = recognise_program(text);
  if (test.empty() && prog.kind) test = prog.kind;
  if (config.empty() && prog.config && test == (prog.kind ? prog.kind : "")) config = prog.config;
  if (prog.what) std::printf("program: %s\n", prog.what);

  if (!run_gpu && !emit_ptx) {
    // remora's CPU/LLVM ExecutionEngine path (compiler/cpu.cpp) belongs to remora.
    std::fprintf(stderr,
                 "remora-b200 runs the GPU path only (--run-gpu); the CPU path is remora's "
                 "own ExecutionEngine\n");
    return 1;
  }
  if (!remora_b200_recognise(test.c_str())) {
    std::fprintf(stderr, "--run-gpu for test '%s' not recognised by remora-b200\n",
                 test.c_str());
    return 1;
  }
  if (emit_ptx) {
    // remora prints the NVVM PTX here (gpu.cpp:222-224); this backend's kernels are
    // hand-written, so it prints the launch plan: entry points, kernels, geometry
    static char plan[16384];
    if (remora_b200_launch_plan(test.c_str(), config.empty() ? nullptr : config.c_str(), plan,
                                sizeof(plan)) != REMORA_B200_OK) {
      std::fprintf(stderr, "remora_b200: %s\n", remora_b200_last_error());
      return 1;
    }
    std::printf("%s", plan);
    if (!run_gpu) return 0;
  }
  if (no_execute) return 0;
  o.config = config.empty() ? nullptr : config.c_str();
  remora_b200_report r;
  const int rc = remora_b200_run_test(test.c_str(), &o, &r);
  std::printf("%s\n", r.detail);
  if (rc != REMORA_B200_OK) {
    std::fprintf(stderr, "remora_b200: %s\n", remora_b200_last_error());
    std::printf("Validation: FAIL\n");
    return 1;
  }
  std::printf("Validation: PASS\n");
  return 0;
}
