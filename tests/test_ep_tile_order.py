"""The tile order of the expert-parallel expert kernel, checked on the host:
tests/ep_tile_order_check.cpp includes the header the kernel uses
(remora_b200/csrc/ep_tiles.h), so the functions checked are the ones the
GPU runs.  A down tile must follow every SwiGLU tile of its row tile; with
that, the kernel's bounded waits cannot form a cycle."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def test_tile_order_is_a_permutation_with_down_after_swiglu(tmp_path):
    exe = tmp_path / "ep_tile_order_check"
    env = {k: v for k, v in os.environ.items() if k not in ("CC", "CXX")}
    subprocess.run(["g++", "-std=c++17", "-O1", "-o", str(exe),
                    os.path.join(HERE, "ep_tile_order_check.cpp")], check=True, env=env)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
