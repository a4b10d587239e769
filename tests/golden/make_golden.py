"""Generates the committed golden fixtures in tests/golden/.

1. moe_mini_seed42.npz -- the reference's own MoE correctness check
   (scripts/export/export_mixtral_layer.py:154-235): T=4, D=16, F=32, E=8,
   top-2; inputs drawn from np.random.default_rng(42).standard_normal in the
   script's order (tokens, router, w_gate, w_up, w_down, :162-168), output of
   its explicit expert-loop numpy reference (`numpy_moe_reference`,
   :175-208), restated below.  The script compares JAX to that numpy output
   at atol 1e-4 (:230); JAX is not installed here, so the oracle is pinned to
   the numpy reference at the same tolerance.

2. known_answers.npz -- the reference harness's known answers:
   elementwise x=1, bias=-0.5 -> 0.5 (compiler/gpu_tests.cpp:53-56, :88-91;
   compiler/cpu_tests.cpp:26-58) and projection x=1, w=1/768 -> the fp32
   value of 768 separately rounded additions of fl(1/768)
   (compiler/cpu_tests.cpp:65-97 prints it as "expected 1.0").

3. oracle_small.npz -- small seeded cases produced by the C oracle (router
   top-k, dispatch permutation, bf16 GEMM, attention rows, expert FFN,
   combine) as a regression anchor for the oracle itself.

Run from the repository root: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))


def numpy_silu(x):
    return x / (1.0 + np.exp(-x))


def numpy_moe_reference(tokens, router_w, w_gate, w_up, w_down, top_k=2):
    """Explicit expert loop (restates export_mixtral_layer.py:175-208)."""
    T = tokens.shape[0]
    E = w_gate.shape[0]
    logits = tokens @ router_w
    idx = np.argsort(-logits, axis=-1)[:, :top_k]
    raw = logits[np.arange(T)[:, None], idx]
    raw = raw - raw.max(axis=-1, keepdims=True)
    ex = np.exp(raw)
    w = ex / ex.sum(axis=-1, keepdims=True)
    out = np.zeros_like(tokens)
    for j in range(top_k):
        ej = idx[:, j]
        wj = w[:, j]
        for e in range(E):
            mask = ej == e
            if not mask.any():
                continue
            x = tokens[mask]
            h = numpy_silu(x @ w_gate[e]) * (x @ w_up[e])
            out[mask] += wj[mask, None] * (h @ w_down[e])
    return out, idx.astype(np.int32), w.astype(np.float32)


def moe_mini():
    T, D, F, E = 4, 16, 32, 8
    rng = np.random.default_rng(42)
    tokens = rng.standard_normal((T, D)).astype(np.float32)
    router = rng.standard_normal((D, E)).astype(np.float32)
    w_gate = rng.standard_normal((E, D, F)).astype(np.float32)
    w_up = rng.standard_normal((E, D, F)).astype(np.float32)
    w_down = rng.standard_normal((E, F, D)).astype(np.float32)
    out, idx, w = numpy_moe_reference(tokens, router, w_gate, w_up, w_down)
    np.savez_compressed(os.path.join(HERE, "moe_mini_seed42.npz"), tokens=tokens, router=router,
                        w_gate=w_gate, w_up=w_up, w_down=w_down, out=out, idx=idx, w=w)


def known_answers():
    acc = np.float32(0.0)
    p = np.float32(1.0) * np.float32(1.0 / 768.0)
    for _ in range(768):
        acc = np.float32(acc + p)
    np.savez_compressed(os.path.join(HERE, "known_answers.npz"),
                        elementwise=np.float32(0.5), projection=np.float32(acc))


def oracle_small():
    import oracle as O

    T, D, E, k, F = 96, 64, 8, 2, 48
    x = O.to_bf16(O.normal("moe_x", (T, D)))
    wr = O.to_bf16(O.normal("moe_router", (D, E), sigma=0.02))
    wg = O.to_bf16(O.normal("moe_wg", (E, D, F), sigma=0.02))
    wu = O.to_bf16(O.normal("moe_wu", (E, D, F), sigma=0.02))
    wd = O.to_bf16(O.normal("moe_wd", (E, F, D), sigma=0.02))
    idx, w, lg = O.router_topk(x, wr, k, return_logits=True)
    counts, offsets, perm, inv = O.dispatch(idx, E)
    _, _, _, _, _, _, moe_out = O.moe_layer_bf16(x, wr, wg, wu, wd, k)

    a = O.to_bf16(O.uniform("gemm_a", (40, 72)))
    b = O.to_bf16(O.uniform("gemm_b", (72, 56)))
    gf, gb = O.gemm_bf16_rows(a, b, 0, 40)

    S, Dh = 80, 64
    q = O.to_bf16(O.normal("attn_q", (S, Dh)))
    kk = O.to_bf16(O.normal("attn_k", (S, Dh)))
    v = O.to_bf16(O.normal("attn_v", (S, Dh)))
    rows = np.arange(S)
    att = O.attention_rows(q, kk, v, rows, causal=True)

    np.savez_compressed(os.path.join(HERE, "oracle_small.npz"), moe_x=x, moe_wr=wr, moe_wg=wg,
                        moe_wu=wu, moe_wd=wd, idx=idx, w=w, logits=lg, counts=counts,
                        offsets=offsets, perm=perm, inv=inv, moe_out=moe_out, gemm_a=a,
                        gemm_b=b, gemm_f32=gf, gemm_bf16=gb, attn_q=q, attn_k=kk, attn_v=v,
                        attn_out=att)


if __name__ == "__main__":
    moe_mini()
    known_answers()
    oracle_small()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)), "bytes")
