"""CPU oracle for the remora_b200 library -- TEST INFRASTRUCTURE ONLY.

This package is the checker: tests/, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg import it.  The product library
(``remora_b200``) never imports it and has no CPU fallback.

It wraps ``oracle/oracle.c`` (a C restatement of remora's CPU/LLVM loop
nests, built by ``oracle/Makefile`` into ``oracle/_build/liboracle.so``) with
numpy-facing functions, and carries a numpy restatement of the seeded input
generator so that inputs can be produced without the C library too.

bf16 arrays are numpy ``uint16`` bit patterns throughout.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

BASE_SEED = 42

# Tensor stream ids of the seeded generator, one per named input.
STREAMS = {
    "scores": 1, "bias": 2, "x": 3,
    "gemm_a": 10, "gemm_b": 11,
    "attn_q": 20, "attn_k": 21, "attn_v": 22,
    "moe_x": 30, "moe_router": 31, "moe_wg": 32, "moe_wu": 33, "moe_wd": 34,
}


def build() -> str:
    """Compile oracle.c with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I64, U64, I, F, D = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64,
                                ctypes.c_int, ctypes.c_float, ctypes.c_double)
        sig = {
            "orc_stream_key": ([U64, U64], U64),
            "orc_fill_uniform_f32": ([U64, I64, D, D, P], None),
            "orc_fill_normal_f32": ([U64, I64, D, D, P], None),
            "orc_f32_to_bf16_array": ([P, P, I64], None),
            "orc_bf16_to_f32_array": ([P, P, I64], None),
            "orc_num_threads": ([], I),
            "orc_set_num_threads": ([I], None),
            "orc_relu_bias_f32": ([P, P, P, I64, I64], None),
            "orc_scale_add_exp_f32": ([P, P, P, I64, F], None),
            "orc_gemm_f32": ([P, P, P, I64, I64, I64, I64, I64, I64, I], None),
            "orc_gemm_bf16_rows": ([P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I], None),
            "orc_gemm_bf16_samples": ([P, P, I64, I64, I64, I, P, P, I64, P], None),
            "orc_attention_rows_bf16": ([P, P, P, I64, I64, I64, I, D, P, I64, P], None),
            "orc_router_topk_bf16": ([P, P, I64, I64, I, I, P, P, P], None),
            "orc_router_topk_f32": ([P, P, I64, I64, I, I, P, P, P], None),
            "orc_dispatch": ([P, I64, I, I, P, P, P, P], I),
            "orc_expert_ffn_bf16": ([P, I64, P, P, P, I64, I64, P, P, P], None),
            "orc_combine_bf16": ([P, P, P, I64, I, I64, P], None),
            "orc_moe_f32": ([P, P, P, P, P, I64, I64, I64, I, I, P], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


# ---------------------------------------------------------------------------
# Seeded generator (numpy restatement; identical bits to orc_fill_*)
# ---------------------------------------------------------------------------
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_G = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def stream_key(stream: int | str, seed: int = BASE_SEED) -> int:
    if isinstance(stream, str):
        stream = STREAMS[stream]
    with np.errstate(over="ignore"):
        v = np.array([seed], dtype=np.uint64) * _G + np.uint64(stream)
    return int(_mix64(v)[0])


def _unit(key: int, ctr: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        b = _mix64(np.uint64(key) + (ctr + np.uint64(1)) * _G)
    return ((b >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal_np(key: int, n: int, mean: float = 0.0, sigma: float = 1.0) -> np.ndarray:
    i = np.arange(n, dtype=np.uint64)
    u1 = _unit(key, np.uint64(2) * i)
    u2 = _unit(key, np.uint64(2) * i + np.uint64(1))
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(6.283185307179586476925286766559 * u2)
    return (mean + sigma * z).astype(np.float32)


def uniform_np(key: int, n: int, lo: float, hi: float) -> np.ndarray:
    u = _unit(key, np.arange(n, dtype=np.uint64))
    return (lo + (hi - lo) * u).astype(np.float32)


def normal(stream, shape, sigma: float = 1.0, seed: int = BASE_SEED) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    lib().orc_fill_normal_f32(stream_key(stream, seed), n, 0.0, sigma, _p(out))
    return out.reshape(shape)


def uniform(stream, shape, lo: float = -1.0, hi: float = 1.0, seed: int = BASE_SEED) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    lib().orc_fill_uniform_f32(stream_key(stream, seed), n, lo, hi, _p(out))
    return out.reshape(shape)


def to_bf16(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().orc_f32_to_bf16_array(_p(a), _p(out), a.size)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.float32)
    lib().orc_bf16_to_f32_array(_p(a), _p(out), a.size)
    return out


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())


# ---------------------------------------------------------------------------
# Op restatements (thin wrappers over oracle.c)
# ---------------------------------------------------------------------------
def relu_bias(x: np.ndarray, bias: np.ndarray) -> np.ndarray:
    """E0: maximumf(x + bias[d], 0) over the last dim."""
    x = np.ascontiguousarray(x, np.float32)
    bias = np.ascontiguousarray(bias, np.float32)
    d = bias.shape[0]
    out = np.empty_like(x)
    lib().orc_relu_bias_f32(_p(x), _p(bias), _p(out), x.size // d, d)
    return out


def scale_add_exp(s: np.ndarray, b: np.ndarray, scale: float) -> np.ndarray:
    """E1: exp(s * scale + b)."""
    s = np.ascontiguousarray(s, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.empty_like(s)
    lib().orc_scale_add_exp_f32(_p(s), _p(b), _p(out), s.size, float(scale))
    return out


def gemm_f32(a: np.ndarray, b: np.ndarray, b_kn: bool = True) -> np.ndarray:
    """G0: f32 dot_general, fill 0 then increasing-k mulf/addf."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    M, K = a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    c = np.empty((M, N), np.float32)
    lib().orc_gemm_f32(_p(a), _p(b), _p(c), M, N, K, K, b.shape[1], N, int(b_kn))
    return c


def gemm_bf16_rows(a: np.ndarray, b: np.ndarray, r0: int, r1: int, b_kn: bool = True):
    """G1 rows [r0, r1): returns (fp32 accumulators, bf16 stored values)."""
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    M, K = a.shape
    N = b.shape[1] if b_kn else b.shape[0]
    cf = np.empty((r1 - r0, N), np.float32)
    cb = np.empty((r1 - r0, N), np.uint16)
    lib().orc_gemm_bf16_rows(_p(a), _p(b), _p(cf), _p(cb), r0, r1, N, K, K, b.shape[1], N,
                             int(b_kn))
    return cf, cb


def gemm_bf16_samples(a: np.ndarray, b: np.ndarray, ii: np.ndarray, jj: np.ndarray,
                      b_kn: bool = True) -> np.ndarray:
    a = np.ascontiguousarray(a, np.uint16)
    b = np.ascontiguousarray(b, np.uint16)
    ii = np.ascontiguousarray(ii, np.int64)
    jj = np.ascontiguousarray(jj, np.int64)
    out = np.empty(ii.shape[0], np.float32)
    K = a.shape[1]
    lib().orc_gemm_bf16_samples(_p(a), _p(b), K, K, b.shape[1], int(b_kn), _p(ii), _p(jj),
                                ii.shape[0], _p(out))
    return out


def attention_rows(q: np.ndarray, k: np.ndarray, v: np.ndarray, rows: np.ndarray,
                   causal: bool = True, scale: float | None = None) -> np.ndarray:
    """A1 for one (batch, head): q, k, v bf16 [S, Dh]; fp64 softmax."""
    q = np.ascontiguousarray(q, np.uint16)
    k = np.ascontiguousarray(k, np.uint16)
    v = np.ascontiguousarray(v, np.uint16)
    S, Dh = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(Dh)
    rows = np.ascontiguousarray(rows, np.int64)
    out = np.empty((rows.shape[0], Dh), np.float32)
    lib().orc_attention_rows_bf16(_p(q), _p(k), _p(v), S, Dh, Dh, int(causal), float(scale),
                                  _p(rows), rows.shape[0], _p(out))
    return out


def router_topk(x: np.ndarray, wr: np.ndarray, k: int, return_logits: bool = False):
    """M1: logits (increasing-d fp32), top-k indices, softmax weights."""
    T, D = x.shape
    if wr.ndim != 2 or wr.shape[0] != D or not 0 < k <= wr.shape[1]:
        raise ValueError(f"router_topk: x {x.shape}, wr {wr.shape}, k {k} do not match")
    E = wr.shape[1]
    idx = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    lg = np.empty((T, E), np.float32) if return_logits else None
    if x.dtype == np.uint16:
        x = np.ascontiguousarray(x)
        wr = np.ascontiguousarray(wr, np.uint16)
        lib().orc_router_topk_bf16(_p(x), _p(wr), T, D, E, k, _p(idx), _p(w), _p(lg))
    else:
        x = np.ascontiguousarray(x, np.float32)
        wr = np.ascontiguousarray(wr, np.float32)
        lib().orc_router_topk_f32(_p(x), _p(wr), T, D, E, k, _p(idx), _p(w), _p(lg))
    return (idx, w, lg) if return_logits else (idx, w)


def dispatch(idx: np.ndarray, E: int):
    """M2: counts[E], offsets[E+1], perm[T*k], inv[T*k] (stable by expert)."""
    idx = np.ascontiguousarray(idx, np.int32)
    T, k = idx.shape
    counts = np.empty(E, np.int32)
    offsets = np.empty(E + 1, np.int32)
    perm = np.empty(T * k, np.int32)
    inv = np.empty(T * k, np.int32)
    rc = lib().orc_dispatch(_p(idx), T, k, E, _p(counts), _p(offsets), _p(perm), _p(inv))
    if rc != 0:
        raise ValueError("expert index out of range")
    return counts, offsets, perm, inv


def expert_ffn(x: np.ndarray, wg: np.ndarray, wu: np.ndarray, wd: np.ndarray):
    """M3 for one expert on rows x bf16 [n, D]: returns (h bf16, y bf16, y f32)."""
    x = np.ascontiguousarray(x, np.uint16)
    n, D = x.shape
    F = wg.shape[1]
    h = np.empty((n, F), np.uint16)
    y = np.empty((n, D), np.uint16)
    yf = np.empty((n, D), np.float32)
    lib().orc_expert_ffn_bf16(_p(x), n, _p(np.ascontiguousarray(wg)), _p(np.ascontiguousarray(wu)),
                              _p(np.ascontiguousarray(wd)), D, F, _p(h), _p(y), _p(yf))
    return h, y, yf


def combine(y: np.ndarray, inv: np.ndarray, w: np.ndarray) -> np.ndarray:
    """M4: out[t] = sum_j w[t,j] * y[inv[t,j]] in slot order, bf16 store."""
    T, k = w.shape
    D = y.shape[1]
    out = np.empty((T, D), np.uint16)
    lib().orc_combine_bf16(_p(np.ascontiguousarray(y, np.uint16)),
                           _p(np.ascontiguousarray(inv, np.int32)),
                           _p(np.ascontiguousarray(w, np.float32)), T, k, D, _p(out))
    return out


def moe_f32(tokens, router, wg, wu, wd, k: int) -> np.ndarray:
    """M5 in f32 (export_mixtral_layer.py:175-208 loop structure)."""
    T, D = tokens.shape
    E, _, F = wg.shape
    out = np.empty((T, D), np.float32)
    c = lambda a: np.ascontiguousarray(a, np.float32)
    lib().orc_moe_f32(_p(c(tokens)), _p(c(router)), _p(c(wg)), _p(c(wu)), _p(c(wd)),
                      T, D, F, E, k, _p(out))
    return out


def moe_layer_bf16(x, wr, wg, wu, wd, k: int, tokens: np.ndarray | None = None):
    """The full bf16 MoE layer for the tokens listed (all if None).

    Routing and dispatch run over every token (the permutation depends on
    all of them); the expert FFN and combine run only for the listed tokens.
    Returns (idx, w, counts, offsets, perm, inv, out_rows bf16 [len(tokens), D]).
    """
    T, D = x.shape
    E = wr.shape[1]
    idx, w = router_topk(x, wr, k)
    counts, offsets, perm, inv = dispatch(idx, E)
    if tokens is None:
        tokens = np.arange(T)
    tokens = np.asarray(tokens, np.int64)
    out = np.empty((tokens.shape[0], D), np.uint16)
    ysel = np.empty((tokens.shape[0] * k, D), np.uint16)
    for j in range(k):
        ex = idx[tokens, j]
        for e in np.unique(ex):
            sel = np.nonzero(ex == e)[0]
            _, y, _ = expert_ffn(x[tokens[sel]], wg[e], wu[e], wd[e])
            ysel[sel * k + j] = y
    inv_local = np.arange(tokens.shape[0] * k, dtype=np.int32).reshape(-1, k)
    out[:] = combine(ysel, inv_local, w[tokens])
    return idx, w, counts, offsets, perm, inv, out


def moe_hetero_layer_bf16(x, wr, wg: list, wu: list, wd: list, k: int,
                          tokens: np.ndarray | None = None):
    """The heterogeneous MoE layer (heterogeneous_moe_layer.mlir:66-212):
    expert e has its own weights wg[e], wu[e] [D, F_e] and wd[e] [F_e, D].
    Routing and dispatch over every token; expert FFN and combine for the
    listed tokens (all if None).  Returns (idx, w, out_rows bf16)."""
    T, D = x.shape
    idx, w = router_topk(x, wr, k)
    if tokens is None:
        tokens = np.arange(T)
    tokens = np.asarray(tokens, np.int64)
    ysel = np.empty((tokens.shape[0] * k, D), np.uint16)
    for e in np.unique(idx[tokens]):
        sel_t, sel_j = np.nonzero(idx[tokens] == e)
        _, y, _ = expert_ffn(x[tokens[sel_t]], wg[e], wu[e], wd[e])
        ysel[sel_t * k + sel_j] = y
    inv_local = np.arange(tokens.shape[0] * k, dtype=np.int32).reshape(-1, k)
    return idx, w, combine(ysel, inv_local, w[tokens])
