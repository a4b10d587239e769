"""GPU test of remora_b200_moe_dispatch_noalloc, the dispatch entry point
that allocates nothing (its scratch is a fixed array inside the library),
for callers that cannot allocate device memory when they dispatch.

It is called through the C ABI and must match remora_b200_moe_dispatch
(which takes a caller-allocated workspace) exactly -- dispatch is integer
work, so the tolerance is zero -- on two calls in a row, since the shared
array keeps the previous call's contents.  This file sorts last so that a
run stopping at its first failure has run every other test already."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dispatch_outputs(T, k, E, dev):
    return [torch.full((n,), -7, dtype=torch.int32, device=dev)
            for n in (E, E + 1, T * k, T * k)]


def _call_noalloc(rb, idx, T, k, E, outs):
    stream = torch.cuda.current_stream().cuda_stream
    rc = rb.lib().remora_b200_moe_dispatch_noalloc(
        ctypes.c_void_p(idx.data_ptr()), T, k, E, *(ctypes.c_void_p(o.data_ptr()) for o in outs),
        ctypes.c_void_p(stream))
    assert rc == 0, rb.last_error()


def _call_with_workspace(rb, idx, T, k, E, outs):
    stream = torch.cuda.current_stream().cuda_stream
    nws = rb.lib().remora_b200_moe_dispatch_workspace_bytes(T, k, E)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=idx.device)
    rc = rb.lib().remora_b200_moe_dispatch(
        ctypes.c_void_p(idx.data_ptr()), T, k, E, *(ctypes.c_void_p(o.data_ptr()) for o in outs),
        ctypes.c_void_p(ws.data_ptr()), nws, ctypes.c_void_p(stream))
    assert rc == 0, rb.last_error()


@pytest.mark.parametrize("T,k,E", [(65536, 8, 64), (8192, 2, 8), (777, 4, 32)])
def test_dispatch_noalloc_matches_workspace_dispatch_twice(rb, T, k, E):
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(T * 31 + E)
    for call in range(2):  # two calls in a row on different routing tables
        idx_np = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        idx = torch.from_numpy(idx_np).to(dev)
        ref = _dispatch_outputs(T, k, E, dev)
        got = _dispatch_outputs(T, k, E, dev)
        _call_with_workspace(rb, idx, T, k, E, ref)
        _call_noalloc(rb, idx, T, k, E, got)
        torch.cuda.synchronize(dev)
        for r, g, name in zip(ref, got, ("counts", "offsets", "perm", "inv")):
            assert torch.equal(r, g), f"call {call}: {name} differs"


@pytest.mark.parametrize("T,k,E,words", [
    (1 << 20, 8, 64, "scratch"),    # needs 8192 * 64 slots > 262144
    ((1 << 62) + 3, 4, 8, "int32"),  # T*k wraps around int64; perm/inv are int32
    (1 << 31, 1, 8, "int32"),
])
def test_dispatch_noalloc_rejects_oversize(rb, T, k, E, words):
    dev = torch.device("cuda", 0)
    idx = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = _dispatch_outputs(1, 1, E, dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = rb.lib().remora_b200_moe_dispatch_noalloc(
        ctypes.c_void_p(idx.data_ptr()), T, k, E, *(ctypes.c_void_p(o.data_ptr()) for o in outs),
        ctypes.c_void_p(stream))
    assert rc == rb.ERR_INVALID and words in rb.last_error()


_RESET_CHILD = r"""
import ctypes, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import remora_b200 as rb
L = rb.lib()
rt = ctypes.CDLL("libcudart.so.12")  # the runtime instance the library itself uses
rt.cudaMalloc.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_size_t]
rt.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
rt.cudaFree.argtypes = [ctypes.c_void_p]
T, k, E = 4096, 4, 16
rng = np.random.default_rng(5)

def buf(n):
    p = ctypes.c_void_p()
    assert rt.cudaMalloc(ctypes.byref(p), n) == 0
    return p

def run_once(call):
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    d_idx = buf(idx.nbytes)
    assert rt.cudaMemcpy(d_idx, idx.ctypes.data, idx.nbytes, 1) == 0
    sizes = (E, E + 1, T * k, T * k)
    got = [buf(4 * n) for n in sizes]
    ref = [buf(4 * n) for n in sizes]
    nws = L.remora_b200_moe_dispatch_workspace_bytes(T, k, E)
    ws = buf(nws)
    assert L.remora_b200_moe_dispatch(d_idx, T, k, E, *ref, ws, nws, None) == 0
    assert L.remora_b200_moe_dispatch_noalloc(d_idx, T, k, E, *got, None) == 0, rb.last_error()
    for n, g, r in zip(sizes, got, ref):
        hg, hr = np.empty(n, np.int32), np.empty(n, np.int32)
        assert rt.cudaMemcpy(hg.ctypes.data, g, 4 * n, 2) == 0
        assert rt.cudaMemcpy(hr.ctypes.data, r, 4 * n, 2) == 0
        assert np.array_equal(hg, hr), f"{call}: outputs differ"
    for p in (d_idx, ws, *got, *ref):
        rt.cudaFree(p)

run_once("before reset")
assert rt.cudaDeviceReset() == 0  # ends this process's context only
run_once("after reset")
print("ok")
"""


def test_dispatch_noalloc_after_device_reset(rb, tmp_path):
    """A cudaDeviceReset replaces the device's context, and with it the
    scratch array's device address: the next call must look the address up
    again.  Run in a child process (no torch there), whose reset ends only
    its own context."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "reset_child.py"
    script.write_text(_RESET_CHILD)
    r = subprocess.run([sys.executable, str(script), root], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
