"""The remora-b200 driver: remora's argv grammar (compiler/main.cpp:19-50),
programs recognised by their @main signature, exit status 0 / 1."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "remora_b200", "remora-b200")

# @main signatures of the programs in remora's mlir/stablehlo/ (types only)
SIGS = {
    "elementwise": "func.func public @main(%arg0: tensor<1x512x768xf32>, %arg1: tensor<768xf32>)",
    "projection": "func.func public @main(%arg0: tensor<1x512x768xf32>, %arg1: tensor<768x768xf32>)",
    "moe_simple": "func.func public @main(%arg0: tensor<8x32xf32>, %arg1: tensor<32x2xf32>, "
                  "%arg2: tensor<2x32x64xf32>, %arg3: tensor<2x32x64xf32>, %arg4: tensor<2x64x32xf32>)",
    "moe_mixtral": "func.func public @main(%arg0: tensor<512x4096xf32>, %arg1: tensor<4096x8xf32>, "
                   "%arg2: tensor<8x4096x14336xf32>, %arg3: tensor<8x4096x14336xf32>)",
    "moe_hetero": "func.func public @main(%tokens : tensor<512x4096xf32>, %router_w : "
                  "tensor<4096x8xf32>, %wg_0 : tensor<1x4096x14336xf32>, %wg_6 : "
                  "tensor<1x4096x2048xf32>)",
}


@pytest.fixture(scope="module")
def cli():
    from remora_b200 import build

    build.build()
    return CLI


def _run(cli, *args, tmp_path=None, sig=None):
    argv = [cli]
    if sig is not None:
        p = tmp_path / "prog.mlir"
        p.write_text(SIGS[sig] + "\n")
        argv.append(str(p))
    argv += list(args)
    return subprocess.run(argv, capture_output=True, text=True, timeout=600)


def test_usage_and_missing_file(cli, tmp_path):
    assert _run(cli).returncode == 1
    r = _run(cli, str(tmp_path / "nope.mlir"), "--run-gpu")
    assert r.returncode == 1 and "Failed to parse" in r.stderr


@pytest.mark.parametrize("sig,entry,kernels", [
    ("elementwise", "remora_b200_relu_bias_f32", ["k_relu_bias_v4"]),
    ("projection", "remora_b200_gemm_f32_exact", ["k_gemm_f32_exact"]),
    ("moe_simple", "remora_b200_moe_layer_bf16(x bf16[8,32]",
     ["k_router_topk", "k_dispatch_scan", "k_grouped_gemm<true>", "k_combine<2>"]),
    ("moe_mixtral", "remora_b200_moe_layer_bf16(x bf16[512,4096]",
     ["k_router_ring<2,4,1,4,128,3>", "k_scatter_rows", "k_grouped_gemm<false>"]),
    ("moe_hetero", "remora_b200_moe_hetero_layer_bf16",
     ["k_grouped_var<true>", "k_grouped_var<false>", "F_e = 14336 14336 8192"])])
def test_emit_ptx_prints_the_launch_plan_without_gpu(cli, tmp_path, sig, entry, kernels):
    """--emit-ptx (compiler/gpu.cpp:222-224 prints the NVVM PTX) prints the
    recognised program's entry points and kernels with their geometry."""
    r = _run(cli, "--emit-ptx", tmp_path=tmp_path, sig=sig)
    assert r.returncode == 0, r.stderr
    assert entry in r.stdout and all(k in r.stdout for k in kernels), r.stdout
    assert "grid" in r.stdout and "block" in r.stdout


def test_launch_plan_rejects_unknown_kind_and_small_buffer():
    import ctypes

    import remora_b200 as rb

    buf = ctypes.create_string_buffer(16)
    assert rb.lib().remora_b200_launch_plan(b"softmax_v2", None, buf, 16) == rb.ERR_UNSUPPORTED
    assert rb.lib().remora_b200_launch_plan(b"moe", b"5", buf, 16) == rb.ERR_INVALID
    assert "gemm_bf16" in rb.launch_plan("gemm", "1024x512x256")


def test_unknown_kind_fails(cli, tmp_path):
    r = _run(cli, "--run-gpu", "--test=softmax_v2", tmp_path=tmp_path, sig="elementwise")
    assert r.returncode == 1 and "not recognised" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("sig", ["elementwise", "projection", "moe_simple", "moe_hetero"])
def test_run_gpu_known_programs(cli, tmp_path, sig):
    r = _run(cli, "--run-gpu", tmp_path=tmp_path, sig=sig)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Validation: PASS" in r.stdout


@pytest.mark.gpu
def test_run_gpu_gemm_config(cli, tmp_path):
    r = _run(cli, "--run-gpu", "--test=gemm", "--config=1024x512x256", tmp_path=tmp_path,
             sig="elementwise")
    assert r.returncode == 0 and "Validation: PASS" in r.stdout
