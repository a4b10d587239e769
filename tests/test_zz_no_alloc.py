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


def test_dispatch_noalloc_rejects_oversize(rb):
    dev = torch.device("cuda", 0)
    T, k, E = 1 << 20, 8, 64  # needs 8192 * 64 slots > 262144
    idx = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = _dispatch_outputs(1, 1, E, dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = rb.lib().remora_b200_moe_dispatch_noalloc(
        ctypes.c_void_p(idx.data_ptr()), T, k, E, *(ctypes.c_void_p(o.data_ptr()) for o in outs),
        ctypes.c_void_p(stream))
    assert rc == rb.ERR_INVALID and "scratch" in rb.last_error()
