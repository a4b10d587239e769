"""Builds libremora_b200.so in-tree with nvcc for sm_100a.

Usage: python -m remora_b200.build   (or remora_b200.build.build()).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libremora_b200.so")
CLI = os.path.join(HERE, "remora-b200")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-ffp-contract=off",
    "-Xptxas", "-warn-spills",
    "-shared",
]


def sources() -> list[str]:
    out = []
    for d in (CSRC, os.path.join(HERE, "..", "include")):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cu", ".cuh", ".h", ".cpp")):
                out.append(os.path.join(d, f))
    return out


def needs_build() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(CLI):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [NVCC, *NVCC_FLAGS, os.path.join(CSRC, "lib.cu"), "-o", LIB + ".tmp", "-lcudart", "-ldl"]
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed building libremora_b200.so")
    os.replace(LIB + ".tmp", LIB)
    build_cli(verbose=verbose)
    return LIB


def build_cli(verbose: bool = False) -> str:
    """The standalone `remora-b200` driver (remora's argv grammar), linked
    against the in-tree library."""
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", os.path.join(CSRC, "cli.cpp"), "-o", CLI,
           "-L" + HERE, "-lremora_b200", "-Wl,-rpath,$ORIGIN"]
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if verbose or r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError("g++ failed building remora-b200")
    return CLI


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
