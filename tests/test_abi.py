"""CPU tests of the C ABI: the library builds for sm_100a, loads, and exports
every entry point that include/remora_b200.h declares.  No compute calls."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(remora_b200_\w+)\s*\(", text))
    return sorted(names)


def test_library_builds_and_exports_every_declared_symbol():
    from remora_b200 import build

    path = build.build()
    lib = ctypes.CDLL(path)
    syms = declared_symbols()
    assert len(syms) >= 10
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_mirror_binds_every_declared_symbol():
    import remora_b200

    remora_b200.lib()
    assert set(declared_symbols()) <= set(remora_b200._SIGNATURES)


def test_recognise_and_errors_without_gpu():
    import remora_b200 as rb

    assert rb.recognise("elementwise") and rb.recognise("projection") and rb.recognise("gemm")
    assert not rb.recognise("softmax_v2")
    # argument validation happens before any CUDA call
    rc = rb.lib().remora_b200_gemm_bf16(None, None, None, 1, 8, 8, 8, 8, 8, 8, 0, 0, 0, 0, None)
    assert rc == rb.ERR_INVALID and "null" in rb.last_error()
    rc = rb.lib().remora_b200_relu_bias_f32(None, None, None, 1, 0, None)
    assert rc == rb.ERR_INVALID


def test_stream_keys_agree_with_oracle():
    import oracle
    import remora_b200 as rb

    for s in (1, 10, 34):
        for seed in (42, 7):
            assert rb.stream_key(s, seed) == oracle.stream_key(s, seed)


def test_expert_parallel_entry_points_validate_before_cuda():
    """Bad rank counts, sizes and null or misaligned peer addresses are
    rejected on the host, before any CUDA call (works without a GPU)."""
    import remora_b200 as rb

    L = rb.lib()
    P = 2
    good = (ctypes.c_uint64 * P)(1 << 20, 2 << 20)
    null = (ctypes.c_uint64 * P)(1 << 20, 0)
    odd = (ctypes.c_uint64 * P)(1 << 20, (2 << 20) + 8)
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)

    def experts(P_, rank, E, D, F, recv, ready, y, x=p):
        return L.remora_b200_moe_ep_experts_fused_bf16(
            x, p, p, 16, 2, D, F, E, P_, rank, 16, recv, ready, p, p, 1, p, p, p, p, p, p, p, y,
            None)

    assert experts(9, 0, 64, 256, 256, good, good, good) == rb.ERR_INVALID   # P > 8
    assert experts(2, 2, 64, 256, 256, good, good, good) == rb.ERR_INVALID   # rank >= P
    assert experts(2, 0, 63, 256, 256, good, good, good) == rb.ERR_INVALID   # E % P
    assert experts(2, 0, 64, 200, 256, good, good, good) == rb.ERR_INVALID   # D % 32
    assert experts(2, 0, 64, 256, 256, null, good, good) == rb.ERR_INVALID   # null peer
    assert "null" in rb.last_error()
    assert experts(2, 0, 64, 256, 256, good, good, odd) == rb.ERR_INVALID    # misaligned peer
    assert experts(2, 0, 64, 256, 256, good, good, good, x=0) == rb.ERR_INVALID  # null x
    rc = L.remora_b200_moe_ep_meta(p, P, 64, 5, 16, good, p, p, good, 1, p, p, None)
    assert rc == rb.ERR_INVALID                                              # rank >= P
    rc = L.remora_b200_moe_ep_barrier(p, null, P, 0, 1, None)
    assert rc == rb.ERR_INVALID


def test_heterogeneous_and_nccl_entry_points_validate_without_gpu():
    """The heterogeneous-layer, NCCL expert-parallel and peer-buffer entry
    points reject bad arguments on the host, before any CUDA or NCCL call."""
    import remora_b200 as rb

    L = rb.lib()
    F = (ctypes.c_int64 * 8)(14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048)
    assert L.remora_b200_moe_hetero_workspace_bytes(512, 4096, F, 8, 1) > 0
    assert L.remora_b200_moe_hetero_workspace_bytes(512, 4096, F, 17, 1) == 0   # E > 16
    assert L.remora_b200_moe_hetero_workspace_bytes(512, 4096, F, 8, 9) == 0    # k > E
    assert L.remora_b200_moe_hetero_workspace_bytes(512, 4096, None, 8, 1) == 0
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf)
    ptrs = (ctypes.c_void_p * 8)(*([p] * 8))
    bad = (ctypes.c_int64 * 8)(14336, 96, 8192, 8192, 4096, 4096, 2048, 2048)  # 96 % 64 != 0
    rc = L.remora_b200_moe_hetero_layer_bf16(p, p, ptrs, ptrs, ptrs, bad, p, 512, 4096, 8, 1, p,
                                             1 << 30, None)
    assert rc == rb.ERR_INVALID and "F[1]" in rb.last_error()
    rc = L.remora_b200_moe_hetero_layer_bf16(p, p, ptrs, ptrs, ptrs, F, p, 512, 4040, 8, 1, p,
                                             1 << 30, None)
    assert rc == rb.ERR_INVALID                                                # D % 32
    rc = L.remora_b200_moe_hetero_layer_bf16(p, p, ptrs, ptrs, ptrs, F, p, 512, 4096, 8, 1, p,
                                             16, None)
    assert rc == rb.ERR_INVALID and "workspace" in rb.last_error()
    # NCCL expert parallelism: a null communicator is rejected before NCCL is used
    rc = L.remora_b200_moe_ep_nccl_bf16(p, p, p, p, p, p, 512, 4096, 14336, 8, 2, None, 1000, p,
                                        1 << 30, None)
    assert rc in (rb.ERR_INVALID, rb.ERR_NCCL)
    assert L.remora_b200_moe_ep_nccl_workspace_bytes(1 << 40, 2048, 1536, 64, 8, 8) == 0
    # peer buffers: null arguments
    out = ctypes.c_void_p()
    assert L.remora_b200_peer_alloc(0, ctypes.byref(out), p) == rb.ERR_INVALID
    assert L.remora_b200_peer_open(None, ctypes.byref(out)) == rb.ERR_INVALID
    assert L.remora_b200_peer_close(None) == rb.ERR_INVALID
    assert L.remora_b200_peer_free(None) == rb.OK


def test_host_buffer_layer_validates_before_cuda():
    import remora_b200 as rb

    L = rb.lib()
    assert L.remora_b200_moe_layer_host_workspace_bytes(65536, 2048, 1536, 64, 8, 0) > 0
    # one chunk's workspace, whatever T is
    assert (L.remora_b200_moe_layer_host_workspace_bytes(65536, 2048, 1536, 64, 8, 4096) ==
            L.remora_b200_moe_layer_host_workspace_bytes(8192, 2048, 1536, 64, 8, 4096))
    assert L.remora_b200_moe_layer_host_workspace_bytes(100, 256, 128, 8, 9, 0) == 0   # k > E
    assert L.remora_b200_moe_layer_host_workspace_bytes(100, 256, 128, 8, 2, -1) == 0
    p = ctypes.c_void_p(16)
    rc = L.remora_b200_moe_layer_host_bf16(p, p, p, p, p, p, 100, 256, 128, 8, 2, -5, p, 1 << 30,
                                           None)
    assert rc == rb.ERR_INVALID and "chunk" in rb.last_error()
    rc = L.remora_b200_moe_layer_host_bf16(p, p, p, p, p, p, 100, 256, 128, 8, 2, 0, None, 0, None)
    assert rc == rb.ERR_INVALID and "workspace" in rb.last_error()
    rc = L.remora_b200_moe_layer_host_bf16(p, p, p, p, p, p, 100, 256, 128, 8, 2, 0, p, 16, None)
    assert rc == rb.ERR_INVALID and "workspace" in rb.last_error()


def test_router_rejects_unaligned_operands_before_cuda():
    import remora_b200 as rb

    L = rb.lib()
    a = ctypes.c_void_p(4096)
    odd = ctypes.c_void_p(4096 + 2)
    # x and (with E % 8 == 0) the router rows are read 16 bytes at a time
    rc = L.remora_b200_moe_router_topk_bf16(odd, a, 64, 256, 64, 8, a, a, None)
    assert rc == rb.ERR_INVALID and "x must be 16-byte aligned" in rb.last_error()
    rc = L.remora_b200_moe_router_topk_bf16(a, odd, 64, 256, 64, 8, a, a, None)
    assert rc == rb.ERR_INVALID and "wr must be 16-byte aligned" in rb.last_error()
