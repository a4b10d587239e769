"""remora_b200 -- B200 (sm_100a) execution backend for remora's recognised
data-parallel programs.

The product is ``libremora_b200.so`` (CUDA kernels + the C ABI declared in
``include/remora_b200.h``).  This module is the host-side mirror of that ABI
for Python callers: it loads the library with ctypes and passes torch CUDA
tensors as raw device pointers on the current CUDA stream.  There is no CPU
path: if the library is missing, or a tensor is not on a CUDA device, the
call raises.

remora's own harness entry point is ``launchOnGpu(ptxModules, test)``
(compiler/gpu_tests.h:6-9); ``recognise`` / ``run_test`` mirror the
dispatcher that replaces its body.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libremora_b200.so")
_lib = None

OK = 0
ERR_INVALID = -1
ERR_CUDA = -2
ERR_NCCL = -3
ERR_TIMEOUT = -4
ERR_PARITY = -5
ERR_UNSUPPORTED = -6

B_KN = 0
B_NK = 1


class RemoraError(RuntimeError):
    """A non-zero status from the C ABI, with remora_b200_last_error() text."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"remora_b200 error {code}: {msg}")
        self.code = code


class Opts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("seed", ctypes.c_uint64), ("iters", ctypes.c_int),
                ("warmup", ctypes.c_int), ("validate", ctypes.c_int), ("config", ctypes.c_char_p)]


class Report(ctypes.Structure):
    _fields_ = [("ms_per_iter", ctypes.c_double), ("work", ctypes.c_double),
                ("rate", ctypes.c_double), ("max_abs_err", ctypes.c_double),
                ("max_rel_err", ctypes.c_double), ("checked", ctypes.c_int64),
                ("passed", ctypes.c_int), ("detail", ctypes.c_char * 256)]


P, I64, I, F, D, U64 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float,
                        ctypes.c_double, ctypes.c_uint64)

_SIGNATURES = {
    "remora_b200_last_error": ([], ctypes.c_char_p),
    "remora_b200_version": ([], I),
    "remora_b200_recognise": ([ctypes.c_char_p], I),
    "remora_b200_run_test": ([ctypes.c_char_p, ctypes.POINTER(Opts), ctypes.POINTER(Report)], I),
    "remora_b200_launch_plan": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                 ctypes.c_size_t], I),
    "remora_b200_relu_bias_f32": ([P, P, P, I64, I64, P], I),
    "remora_b200_scale_add_exp_f32": ([P, P, P, I64, F, P], I),
    "remora_b200_gemm_bf16": ([P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I, P], I),
    "remora_b200_gemm_f32_exact": ([P, P, P, I64, I64, I64, I64, I64, I64, I, P], I),
    "remora_b200_attention_fwd_bf16": ([P, P, P, P, I64, I64, I64, I64, I, F, P], I),
    "remora_b200_moe_router_topk_bf16": ([P, P, I64, I64, I, I, P, P, P], I),
    "remora_b200_moe_dispatch_workspace_bytes": ([I64, I, I], ctypes.c_size_t),
    "remora_b200_moe_dispatch": ([P, I64, I, I, P, P, P, P, P, ctypes.c_size_t, P], I),
    "remora_b200_moe_dispatch_noalloc": ([P, I64, I, I, P, P, P, P, P], I),
    "remora_b200_moe_gather": ([P, P, I64, I, I64, P, P], I),
    "remora_b200_moe_scatter": ([P, P, I64, I, I64, P, P], I),
    "remora_b200_grouped_gemm_swiglu_bf16": ([P, P, P, P, P, I64, I64, I64, I, P], I),
    "remora_b200_grouped_gemm_bf16": ([P, P, P, P, I64, I64, I64, I, P], I),
    "remora_b200_grouped_gemm_swiglu_segments_bf16": ([P, P, P, P, P, P, I, I64, I64, I64, I, P],
                                                      I),
    "remora_b200_grouped_gemm_segments_bf16": ([P, P, P, P, P, I, I64, I64, I64, I, P], I),
    "remora_b200_moe_combine_bf16": ([P, P, P, I64, I, I64, P, P], I),
    "remora_b200_moe_workspace_bytes": ([I64, I64, I64, I, I], ctypes.c_size_t),
    "remora_b200_moe_layer_bf16": ([P, P, P, P, P, P, I64, I64, I64, I, I, P, ctypes.c_size_t, P],
                                   I),
    "remora_b200_moe_layer_host_workspace_bytes": ([I64, I64, I64, I, I, I64], ctypes.c_size_t),
    "remora_b200_moe_layer_host_bf16": ([P, P, P, P, P, P, I64, I64, I64, I, I, I64, P,
                                         ctypes.c_size_t, P], I),
    "remora_b200_moe_ep_scatter_bf16": ([P, P, P, I64, I, I64, I, I, I, I64, P, P, P], I),
    "remora_b200_moe_ep_barrier": ([P, P, I, I, I, P], I),
    "remora_b200_moe_ep_segments": ([P, I, I, I64, P, P], I),
    "remora_b200_moe_ep_experts_bf16": ([P, P, P, P, P, P, I, I, I64, I64, I64, P, P], I),
    "remora_b200_moe_ep_meta": ([P, I, I, I, I64, P, P, P, P, I, P, P, P], I),
    "remora_b200_moe_ep_experts_fused_bf16": ([P, P, P, I64, I, I64, I64, I, I, I, I64, P, P, P,
                                               P, I, P, P, P, P, P, P, P, P, P], I),
    "remora_b200_peer_alloc": ([ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), P], I),
    "remora_b200_peer_open": ([P, ctypes.POINTER(ctypes.c_void_p)], I),
    "remora_b200_peer_close": ([P], I),
    "remora_b200_peer_free": ([P], I),
    "remora_b200_moe_ep_nccl_workspace_bytes": ([I64, I64, I64, I, I, I], ctypes.c_size_t),
    "remora_b200_moe_ep_nccl_bf16": ([P, P, P, P, P, P, I64, I64, I64, I, I, P, I64, P,
                                      ctypes.c_size_t, P], I),
    "remora_b200_moe_ep_splits": ([P, P, I, I, P, P, P, P], I),
    "remora_b200_nccl_unique_id": ([P], I),
    "remora_b200_nccl_comm_init": ([ctypes.POINTER(ctypes.c_void_p), I, P, I, I, I64], I),
    "remora_b200_nccl_comm_destroy": ([P, I64], I),
    "remora_b200_nccl_comm_abort": ([P], I),
    "remora_b200_grouped_gemm_swiglu_var_bf16": ([P, P, P, P, I64, P, I64, I64, P, I, P], I),
    "remora_b200_grouped_gemm_var_bf16": ([P, I64, P, P, P, I64, P, I64, I, P], I),
    "remora_b200_moe_hetero_workspace_bytes": ([I64, I64, P, I, I], ctypes.c_size_t),
    "remora_b200_moe_hetero_layer_bf16": ([P, P, P, P, P, P, P, I64, I64, I, I, P,
                                           ctypes.c_size_t, P], I),
    "remora_b200_device_status": ([], I),
    "remora_b200_fill_normal": ([P, I64, I, U64, D, D, P], I),
    "remora_b200_fill_uniform": ([P, I64, I, U64, D, D, P], I),
}


def lib() -> ctypes.CDLL:
    """The loaded C ABI.  Raises if libremora_b200.so has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m remora_b200.build` "
                "(remora_b200 has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def last_error() -> str:
    return lib().remora_b200_last_error().decode()


def _check(rc: int) -> None:
    if rc != OK:
        raise RemoraError(rc, last_error())


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dev(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("remora_b200 operates on CUDA tensors only (no CPU fallback)")


def _bf16(*ts: torch.Tensor) -> None:
    for t in ts:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"expected a bfloat16 tensor, got {t.dtype}")


# --------------------------------------------------------------- dispatcher
def recognise(test: str) -> bool:
    return bool(lib().remora_b200_recognise(test.encode()))


def run_test(test: str, device: int = 0, seed: int = 42, iters: int = 1, warmup: int = 0,
             validate: bool = True, config: str | None = None) -> dict:
    """Runs a recognised --test=<kind> program end to end; raises on failure."""
    o = Opts(device, seed, iters, warmup, int(validate), config.encode() if config else None)
    r = Report()
    rc = lib().remora_b200_run_test(test.encode(), ctypes.byref(o), ctypes.byref(r))
    rep = {k: getattr(r, k) for k, _ in Report._fields_ if k != "detail"}
    rep["detail"] = r.detail.decode()
    if rc != OK:
        raise RemoraError(rc, last_error())
    return rep


def launch_plan(test: str, config: str | None = None) -> str:
    """The kernels a recognised program launches, with their geometry
    (what `remora-b200 --emit-ptx` prints)."""
    buf = ctypes.create_string_buffer(8192)
    _check(lib().remora_b200_launch_plan(test.encode(), config.encode() if config else None,
                                         buf, len(buf)))
    return buf.value.decode()


# -------------------------------------------------------------- elementwise
def relu_bias(x: torch.Tensor, bias: torch.Tensor, out: torch.Tensor | None = None):
    """maximumf(x + bias, 0), bias broadcast over the last dim (f32)."""
    _dev(x, bias)
    if x.dtype != torch.float32 or bias.dtype != torch.float32:
        raise TypeError("relu_bias takes float32 tensors")
    if bias.dim() != 1 or x.shape[-1] != bias.shape[0]:
        raise ValueError("bias must be 1-D and match x's last dim")
    x = x.contiguous()
    out = torch.empty_like(x) if out is None else out
    d = bias.shape[0]
    _check(lib().remora_b200_relu_bias_f32(x.data_ptr(), bias.contiguous().data_ptr(),
                                           out.data_ptr(), x.numel() // d, d, _stream(x)))
    return out


def scale_add_exp(s: torch.Tensor, b: torch.Tensor, scale: float,
                  out: torch.Tensor | None = None):
    """exp(s * scale + b), f32, elementwise."""
    _dev(s, b)
    if s.shape != b.shape or s.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("scale_add_exp takes two float32 tensors of one shape")
    s, b = s.contiguous(), b.contiguous()
    out = torch.empty_like(s) if out is None else out
    _check(lib().remora_b200_scale_add_exp_f32(s.data_ptr(), b.data_ptr(), out.data_ptr(),
                                               s.numel(), float(scale), _stream(s)))
    return out


# --------------------------------------------------------------------- GEMM
def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
         b_layout: int = B_KN) -> torch.Tensor:
    """dot_general: a [.., M, K] x b [.., K, N] (or [.., N, K] with B_NK), bf16."""
    _dev(a, b)
    _bf16(a, b)
    batched = a.dim() == 3
    a3 = a if batched else a.unsqueeze(0)
    b3 = b if b.dim() == 3 else b.unsqueeze(0)
    if a3.stride(-1) != 1 or b3.stride(-1) != 1:
        raise ValueError("gemm operands must have a unit innermost stride")
    batch, M, K = a3.shape
    if b3.shape[0] != batch:
        raise ValueError("batch mismatch")
    if b_layout == B_KN:
        Kb, N = b3.shape[1], b3.shape[2]
    else:
        N, Kb = b3.shape[1], b3.shape[2]
    if Kb != K:
        raise ValueError(f"contracting dims differ: {K} vs {Kb}")
    if out is None:
        out = torch.empty((batch, M, N) if batched else (M, N), dtype=torch.bfloat16,
                          device=a.device)
    c3 = out if out.dim() == 3 else out.unsqueeze(0)
    _check(lib().remora_b200_gemm_bf16(
        a3.data_ptr(), b3.data_ptr(), c3.data_ptr(), batch, M, N, K, a3.stride(1), b3.stride(1),
        c3.stride(1), a3.stride(0), b3.stride(0), c3.stride(0), b_layout, _stream(a)))
    return out


def gemm_f32_exact(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
                   b_layout: int = B_KN) -> torch.Tensor:
    """f32 dot_general with the reference loop nest's exact rounding sequence."""
    _dev(a, b)
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise TypeError("gemm_f32_exact takes float32 tensors")
    M, K = a.shape
    N = b.shape[1] if b_layout == B_KN else b.shape[0]
    a, b = a.contiguous(), b.contiguous()
    out = torch.empty((M, N), dtype=torch.float32, device=a.device) if out is None else out
    _check(lib().remora_b200_gemm_f32_exact(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
                                            a.stride(0), b.stride(0), out.stride(0), b_layout,
                                            _stream(a)))
    return out


# ---------------------------------------------------------------- attention
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
              scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale [+ causal mask]) v; q, k, v bf16 [B, H, S, 128]."""
    _dev(q, k, v)
    _bf16(q, k, v)
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must be [B, H, S, D] of one shape")
    B, H, S, Dh = q.shape
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    out = torch.empty_like(q) if out is None else out
    if scale is None:
        scale = Dh ** -0.5
    _check(lib().remora_b200_attention_fwd_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                out.data_ptr(), B, H, S, Dh, int(causal),
                                                float(scale), _stream(q)))
    return out


# ---------------------------------------------------------------------- MoE
def _i32(*ts):
    for t in ts:
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise TypeError("expected a contiguous int32 tensor")


def moe_router_topk(x: torch.Tensor, wr: torch.Tensor, k: int, idx: torch.Tensor | None = None,
                    w: torch.Tensor | None = None):
    """Router logits (increasing-d fp32), top-k indices and softmax weights."""
    _dev(x, wr)
    _bf16(x, wr)
    T, D = x.shape
    E = wr.shape[1]
    x, wr = x.contiguous(), wr.contiguous()
    idx = torch.empty((T, k), dtype=torch.int32, device=x.device) if idx is None else idx
    w = torch.empty((T, k), dtype=torch.float32, device=x.device) if w is None else w
    _check(lib().remora_b200_moe_router_topk_bf16(x.data_ptr(), wr.data_ptr(), T, D, E, k,
                                                  idx.data_ptr(), w.data_ptr(), _stream(x)))
    return idx, w


def moe_dispatch(idx: torch.Tensor, E: int):
    """counts[E], offsets[E+1], perm[T*k], inv[T*k] (stable by expert)."""
    _dev(idx)
    _i32(idx)
    T, k = idx.shape
    dev = idx.device
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    inv = torch.empty(T * k, dtype=torch.int32, device=dev)
    nws = lib().remora_b200_moe_dispatch_workspace_bytes(T, k, E)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=dev)
    _check(lib().remora_b200_moe_dispatch(idx.data_ptr(), T, k, E, counts.data_ptr(),
                                          offsets.data_ptr(), perm.data_ptr(), inv.data_ptr(),
                                          ws.data_ptr(), nws, _stream(idx)))
    return counts, offsets, perm, inv


def moe_scatter(x: torch.Tensor, inv: torch.Tensor, k: int) -> torch.Tensor:
    """xs[inv[t, j]] = x[t]: the dispatched rows, written token by token."""
    _dev(x, inv)
    _i32(inv)
    T, D = x.shape
    xs = torch.empty((T * k, D), dtype=x.dtype, device=x.device)
    _check(lib().remora_b200_moe_scatter(x.contiguous().data_ptr(), inv.data_ptr(), T, k, D,
                                         xs.data_ptr(), _stream(x)))
    return xs


def moe_gather(x: torch.Tensor, perm: torch.Tensor, k: int) -> torch.Tensor:
    _dev(x, perm)
    _i32(perm)
    T, D = x.shape
    rows = perm.numel()
    xs = torch.empty((rows, D), dtype=x.dtype, device=x.device)
    _check(lib().remora_b200_moe_gather(x.contiguous().data_ptr(), perm.data_ptr(), rows, k, D,
                                        xs.data_ptr(), _stream(x)))
    return xs


def grouped_gemm_swiglu(xs: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor,
                        offsets: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """h = silu(xs . wg[e]) * (xs . wu[e]) over each expert's row segment."""
    _dev(xs, wg, wu, offsets)
    _bf16(xs, wg, wu)
    _i32(offsets)
    rows, D = xs.shape
    E, _, F = wg.shape
    h = torch.empty((rows, F), dtype=torch.bfloat16, device=xs.device) if out is None else out
    _check(lib().remora_b200_grouped_gemm_swiglu_bf16(
        xs.contiguous().data_ptr(), wg.contiguous().data_ptr(), wu.contiguous().data_ptr(),
        h.data_ptr(), offsets.data_ptr(), rows, D, F, E, _stream(xs)))
    return h


def grouped_gemm(a: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """y = a . w[e] over each expert's row segment (w [E, K, N])."""
    _dev(a, w, offsets)
    _bf16(a, w)
    _i32(offsets)
    rows, K = a.shape
    E, _, N = w.shape
    y = torch.empty((rows, N), dtype=torch.bfloat16, device=a.device) if out is None else out
    _check(lib().remora_b200_grouped_gemm_bf16(a.contiguous().data_ptr(), w.contiguous().data_ptr(),
                                               y.data_ptr(), offsets.data_ptr(), rows, K, N, E,
                                               _stream(a)))
    return y


def grouped_gemm_swiglu_segments(xs, wg, wu, seg_offsets, seg_expert) -> torch.Tensor:
    """SwiGLU grouped GEMM over row segments that name their expert."""
    _dev(xs, wg, wu, seg_offsets, seg_expert)
    _bf16(xs, wg, wu)
    _i32(seg_offsets, seg_expert)
    rows, D = xs.shape
    E, _, F = wg.shape
    h = torch.empty((rows, F), dtype=torch.bfloat16, device=xs.device)
    _check(lib().remora_b200_grouped_gemm_swiglu_segments_bf16(
        xs.contiguous().data_ptr(), wg.contiguous().data_ptr(), wu.contiguous().data_ptr(),
        h.data_ptr(), seg_offsets.data_ptr(), seg_expert.data_ptr(), seg_expert.numel(), rows, D,
        F, E, _stream(xs)))
    return h


def grouped_gemm_segments(a, w, seg_offsets, seg_expert) -> torch.Tensor:
    """Grouped GEMM over row segments that name their expert (w [E, K, N])."""
    _dev(a, w, seg_offsets, seg_expert)
    _bf16(a, w)
    _i32(seg_offsets, seg_expert)
    rows, K = a.shape
    E, _, N = w.shape
    y = torch.empty((rows, N), dtype=torch.bfloat16, device=a.device)
    _check(lib().remora_b200_grouped_gemm_segments_bf16(
        a.contiguous().data_ptr(), w.contiguous().data_ptr(), y.data_ptr(), seg_offsets.data_ptr(),
        seg_expert.data_ptr(), seg_expert.numel(), rows, K, N, E, _stream(a)))
    return y


def moe_combine(y: torch.Tensor, inv: torch.Tensor, w: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    _dev(y, inv, w)
    _i32(inv)
    T, k = w.shape
    D = y.shape[1]
    if out is None:
        out = torch.empty((T, D), dtype=torch.bfloat16, device=y.device)
    elif out.shape != (T, D) or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("moe_combine: out must be a contiguous bf16 [T, D] tensor")
    _check(lib().remora_b200_moe_combine_bf16(y.contiguous().data_ptr(), inv.data_ptr(),
                                              w.contiguous().data_ptr(), T, k, D, out.data_ptr(),
                                              _stream(y)))
    return out


def moe_workspace_bytes(T: int, D: int, F: int, E: int, k: int) -> int:
    return int(lib().remora_b200_moe_workspace_bytes(T, D, F, E, k))


def moe_layer(x: torch.Tensor, wr: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor,
              wd: torch.Tensor, k: int, out: torch.Tensor | None = None,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The whole MoE layer (router, dispatch, SwiGLU experts, combine), bf16."""
    _dev(x, wr, wg, wu, wd)
    _bf16(x, wr, wg, wu, wd)
    T, D = x.shape
    E, _, F = wg.shape
    need = moe_workspace_bytes(T, D, F, E, k)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    out = torch.empty((T, D), dtype=torch.bfloat16, device=x.device) if out is None else out
    _check(lib().remora_b200_moe_layer_bf16(
        x.contiguous().data_ptr(), wr.contiguous().data_ptr(), wg.contiguous().data_ptr(),
        wu.contiguous().data_ptr(), wd.contiguous().data_ptr(), out.data_ptr(), T, D, F, E, k,
        workspace.data_ptr(), workspace.numel(), _stream(x)))
    return out


def moe_layer_host(x_host: torch.Tensor, wr: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor,
                   wd: torch.Tensor, k: int, out_host: torch.Tensor | None = None,
                   chunk_tokens: int = 0, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The MoE layer on tokens in (pinned) host memory: chunks go up, through
    the layer and back on copy streams overlapped with the kernels.  Returns
    out_host after enqueueing; synchronise the current stream before reading."""
    if x_host.is_cuda or (out_host is not None and out_host.is_cuda):
        raise ValueError("moe_layer_host takes host tensors for x and out")
    _dev(wr, wg, wu, wd)
    _bf16(x_host, wr, wg, wu, wd)
    T, D = x_host.shape
    E, _, F = wg.shape
    need = lib().remora_b200_moe_layer_host_workspace_bytes(T, D, F, E, k, chunk_tokens)
    if need == 0:
        raise ValueError("moe_layer_host: unsupported sizes")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=wg.device)
    if out_host is None:
        out_host = torch.empty((T, D), dtype=torch.bfloat16, pin_memory=True)
    _check(lib().remora_b200_moe_layer_host_bf16(
        x_host.contiguous().data_ptr(), wr.contiguous().data_ptr(), wg.contiguous().data_ptr(),
        wu.contiguous().data_ptr(), wd.contiguous().data_ptr(), out_host.data_ptr(), T, D, F, E,
        k, chunk_tokens, workspace.data_ptr(), workspace.numel(), _stream(wg)))
    return out_host


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _i64s(vals):
    return (ctypes.c_int64 * len(vals))(*vals)


def moe_hetero_layer(x: torch.Tensor, wr: torch.Tensor, wg: list, wu: list, wd: list, k: int,
                     out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None) -> torch.Tensor:
    """MoE layer whose experts have their own FFN widths: wg[e], wu[e] bf16
    [D, F_e], wd[e] bf16 [F_e, D] (heterogeneous_moe_layer.mlir)."""
    _dev(x, wr, *wg, *wu, *wd)
    _bf16(x, wr, *wg, *wu, *wd)
    T, D = x.shape
    E = len(wg)
    if not (len(wu) == len(wd) == E == wr.shape[1]):
        raise ValueError("one gate, up and down weight per expert")
    F = [int(w.shape[1]) for w in wg]
    wg, wu, wd = ([w.contiguous() for w in ws] for ws in (wg, wu, wd))
    need = int(lib().remora_b200_moe_hetero_workspace_bytes(T, D, _i64s(F), E, k))
    if need == 0:
        raise ValueError("moe_hetero_layer: sizes rejected")
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    out = torch.empty((T, D), dtype=torch.bfloat16, device=x.device) if out is None else out
    _check(lib().remora_b200_moe_hetero_layer_bf16(
        x.contiguous().data_ptr(), wr.contiguous().data_ptr(), _ptrs(wg), _ptrs(wu), _ptrs(wd),
        _i64s(F), out.data_ptr(), T, D, E, k, workspace.data_ptr(), workspace.numel(),
        _stream(x)))
    return out


def grouped_gemm_swiglu_var(xs, wg: list, wu: list, offsets, ldh: int | None = None):
    """h[r, :F_e] = silu(xs[r] . wg[e]) * (xs[r] . wu[e]); h [rows, ldh]."""
    _dev(xs, offsets, *wg, *wu)
    _i32(offsets)
    rows, D = xs.shape
    F = [int(w.shape[1]) for w in wg]
    ldh = ldh or max(F)
    h = torch.zeros((rows, ldh), dtype=torch.bfloat16, device=xs.device)
    _check(lib().remora_b200_grouped_gemm_swiglu_var_bf16(
        xs.contiguous().data_ptr(), _ptrs([w.contiguous() for w in wg]),
        _ptrs([w.contiguous() for w in wu]), h.data_ptr(), ldh, offsets.data_ptr(), rows, D,
        _i64s(F), len(wg), _stream(xs)))
    return h


def grouped_gemm_var(h, wd: list, offsets):
    """y[r, :] = h[r, :F_e] . wd[e] for the rows of expert e (wd[e] [F_e, D])."""
    _dev(h, offsets, *wd)
    _i32(offsets)
    rows, ldh = h.shape
    F = [int(w.shape[0]) for w in wd]
    D = int(wd[0].shape[1])
    y = torch.empty((rows, D), dtype=torch.bfloat16, device=h.device)
    _check(lib().remora_b200_grouped_gemm_var_bf16(
        h.contiguous().data_ptr(), ldh, _ptrs([w.contiguous() for w in wd]), y.data_ptr(),
        offsets.data_ptr(), rows, _i64s(F), D, len(wd), _stream(h)))
    return y


def synchronize_and_check(device=None) -> None:
    """Synchronises the device and raises if a kernel reported an error
    (bad expert id, timed-out device wait)."""
    torch.cuda.synchronize(device)
    _check(lib().remora_b200_device_status())


# ---------------------------------------------------------- seeded inputs
def fill_normal(t: torch.Tensor, key: int, mean: float = 0.0, sigma: float = 1.0):
    _dev(t)
    dt = {torch.float32: 0, torch.bfloat16: 1}[t.dtype]
    _check(lib().remora_b200_fill_normal(t.data_ptr(), t.numel(), dt, key, mean, sigma,
                                         _stream(t)))
    return t


def fill_uniform(t: torch.Tensor, key: int, lo: float = -1.0, hi: float = 1.0):
    _dev(t)
    dt = {torch.float32: 0, torch.bfloat16: 1}[t.dtype]
    _check(lib().remora_b200_fill_uniform(t.data_ptr(), t.numel(), dt, key, lo, hi, _stream(t)))
    return t


_G = 0x9E3779B97F4A7C15
_MASK = (1 << 64) - 1


def _mix64(z: int) -> int:
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
    return z ^ (z >> 31)


def stream_key(stream: int, seed: int = 42) -> int:
    """Key of tensor stream `stream` under base seed `seed` (generator key schedule)."""
    return _mix64((seed * _G + stream) & _MASK)
