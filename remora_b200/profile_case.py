"""Runs one kernel of the library on seeded inputs, for profiling and timing.

    python -m remora_b200.profile_case <case> [--reps N] [--warmup W] [shape options]

Cases: router, dispatch, gather, scatter, combine, swiglu, down, attention, gemm, layer, hetero.
Each run fills its inputs with the seeded generator, launches the kernel
`warmup` times, then `reps` times between CUDA events on the current
stream, and prints one line: case, shape, time per launch, and the
algorithmic work rate (FLOP/s or bytes/s, as the kernel's roofline counts
it).  Under ncu, select the kernel with -k and skip the warm-up launches
with -s.
"""
from __future__ import annotations

import argparse

import torch

import remora_b200 as rb


def _bf16(shape, key, sigma=1.0):
    t = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    return rb.fill_normal(t, rb.stream_key(key), 0.0, sigma)


def _routing(T, D, E, k):
    x = _bf16((T, D), 30)
    wr = _bf16((D, E), 31, 0.02)
    idx, w = rb.moe_router_topk(x, wr, k)
    return x, wr, idx, w


def build_case(a):
    """Returns (launch function, description, work per launch, work unit)."""
    T, D, F, E, k = a.T, a.D, a.F, a.E, a.k
    if a.case == "router":
        x, wr, idx, w = _routing(T, D, E, k)
        return (lambda: rb.moe_router_topk(x, wr, k, idx=idx, w=w),
                f"router T={T} D={D} E={E} k={k}", 2.0 * T * D * E, "FLOP")
    if a.case == "dispatch":
        _, _, idx, _ = _routing(T, D, E, k)
        return (lambda: rb.moe_dispatch(idx, E), f"dispatch T={T} k={k} E={E}",
                4.0 * T * k * 3, "B")  # idx read twice, perm and inv written
    if a.case == "gather":
        x, _, idx, _ = _routing(T, D, E, k)
        _, _, perm, _ = rb.moe_dispatch(idx, E)
        xs = torch.empty(T * k, D, dtype=torch.bfloat16, device="cuda")
        L = rb.lib()

        def run():
            rb._check(L.remora_b200_moe_gather(x.data_ptr(), perm.data_ptr(), T * k, k, D,
                                               xs.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream))
        return run, f"gather rows={T * k} D={D}", 2.0 * T * k * D * 2, "B"
    if a.case == "scatter":
        x, _, idx, _ = _routing(T, D, E, k)
        _, _, _, inv = rb.moe_dispatch(idx, E)
        xs = torch.empty(T * k, D, dtype=torch.bfloat16, device="cuda")
        L = rb.lib()

        def run():
            rb._check(L.remora_b200_moe_scatter(x.data_ptr(), inv.data_ptr(), T, k, D,
                                                xs.data_ptr(),
                                                torch.cuda.current_stream().cuda_stream))
        return run, f"scatter T={T} k={k} D={D}", (1.0 + k) * T * D * 2, "B"
    if a.case == "combine":
        _, _, idx, w = _routing(T, D, E, k)
        _, _, _, inv = rb.moe_dispatch(idx, E)
        y = _bf16((T * k, D), 40)
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: rb.moe_combine(y, inv, w, out=out), f"combine T={T} k={k} D={D}",
                (k + 1.0) * T * D * 2, "B")
    if a.case in ("swiglu", "down"):
        x, _, idx, _ = _routing(T, D, E, k)
        _, offsets, perm, _ = rb.moe_dispatch(idx, E)
        xs = rb.moe_gather(x, perm, k)
        if a.case == "swiglu":
            wg, wu = _bf16((E, D, F), 32, 0.02), _bf16((E, D, F), 33, 0.02)
            h = torch.empty(T * k, F, dtype=torch.bfloat16, device="cuda")
            return (lambda: rb.grouped_gemm_swiglu(xs, wg, wu, offsets, out=h),
                    f"grouped SwiGLU rows={T * k} D={D} F={F} E={E}", 4.0 * T * k * D * F, "FLOP")
        h = _bf16((T * k, F), 41, 0.05)
        wd = _bf16((E, F, D), 34, 0.02)
        y = torch.empty(T * k, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: rb.grouped_gemm(h, wd, offsets, out=y),
                f"grouped down rows={T * k} F={F} D={D} E={E}", 2.0 * T * k * D * F, "FLOP")
    if a.case == "attention":
        q, kk, v = (_bf16((a.B, a.H, a.S, 128), 20 + i) for i in range(3))
        o = torch.empty_like(q)
        return (lambda: rb.attention(q, kk, v, causal=True, out=o),
                f"causal attention [{a.B},{a.H},{a.S},128]", 2.0 * a.B * a.H * a.S * a.S * 128,
                "FLOP")
    if a.case == "gemm":
        n = a.n
        A, B = _bf16((n, n), 10), _bf16((n, n), 11)
        C = torch.empty(n, n, dtype=torch.bfloat16, device="cuda")
        return lambda: rb.gemm(A, B, out=C), f"gemm {n}^3", 2.0 * n ** 3, "FLOP"
    if a.case == "layer":
        x, wr, _, _ = _routing(T, D, E, k)
        wg, wu, wd = (_bf16(s, 32 + i, 0.02) for i, s in enumerate(((E, D, F), (E, D, F),
                                                                    (E, F, D))))
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        ws = torch.empty(rb.moe_workspace_bytes(T, D, F, E, k), dtype=torch.uint8, device="cuda")
        return (lambda: rb.moe_layer(x, wr, wg, wu, wd, k, out=out, workspace=ws),
                f"MoE layer T={T} D={D} F={F} E={E} k={k}", 6.0 * T * k * D * F, "FLOP")
    if a.case == "hetero":
        # heterogeneous_moe_layer.mlir: 8 experts of F 14336 x2, 8192 x2, 4096 x2, 2048 x2
        Fs = [14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048]
        x, wr, _, _ = _routing(T, D, len(Fs), k)
        wg = [_bf16((D, f), 32 + 10 * e, 0.02) for e, f in enumerate(Fs)]
        wu = [_bf16((D, f), 33 + 10 * e, 0.02) for e, f in enumerate(Fs)]
        wd = [_bf16((f, D), 34 + 10 * e, 0.02) for e, f in enumerate(Fs)]
        out = torch.empty(T, D, dtype=torch.bfloat16, device="cuda")
        return (lambda: rb.moe_hetero_layer(x, wr, wg, wu, wd, k, out=out),
                f"heterogeneous MoE layer T={T} D={D} F={Fs} top-{k}",
                6.0 * T * k * D * sum(Fs) / len(Fs), "FLOP")
    raise SystemExit(f"unknown case {a.case}")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--T", type=int, default=8192)
    ap.add_argument("--D", type=int, default=2048)
    ap.add_argument("--F", type=int, default=1536)
    ap.add_argument("--E", type=int, default=64)
    ap.add_argument("--k", type=int, default=8)
    ap.add_argument("--B", type=int, default=4)
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--S", type=int, default=4096)
    ap.add_argument("--n", type=int, default=8192)
    a = ap.parse_args(argv)
    from remora_b200 import build

    build.build()
    run, what, work, unit = build_case(a)
    for _ in range(a.warmup):
        run()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    s = torch.cuda.current_stream()
    ev[0].record(s)
    for _ in range(a.reps):
        run()
    ev[1].record(s)
    rb.synchronize_and_check()
    ms = ev[0].elapsed_time(ev[1]) / a.reps
    scale, u = (1e12, "TFLOP/s") if unit == "FLOP" else (1e9, "GB/s")
    print(f"{a.case}: {what}: {ms * 1e3:.1f} us per launch, {work / (ms * 1e-3) / scale:.1f} {u}",
          flush=True)
    return ms


if __name__ == "__main__":
    main()
