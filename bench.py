"""Benchmark of the remora_b200 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemm|elementwise]

Default workload (the headline config): stablehlo.dot_general GEMM, bf16
A [8192,8192] x B [8192,8192] -> bf16, fp32 accumulate, U(-1,1) seeded
inputs.  Under torchrun with N > 1 GPUs the workload is the batched form
[8,4096,4096] x [8,4096,4096] with the batch split across ranks (no
collective; the same 1.0995e12 FLOP per step in total, strong scaling).
One step = one GEMM over the whole job's batch.  Rank 0 prints one JSON line.

--impl reference times the reference's CPU path for the same metric: the C
restatement of remora's convert-linalg-to-loops loop nest (oracle/), on all
host threads, over a bounded row sample of the same GEMM per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE layer tokens/s; GEMM/attn TFLOP/s as % B200 peak; elementwise HBM GB/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant
# kernel, from the ncu captures summarised in profiles/ (None = not captured).
NCU_TRAFFIC_BYTES = {
    "gemm_8192": 1140578560,  # profiles/gemm_bf16_8192_dram.md
    "gemm_batched": None,
    "elementwise": None,
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting"}

    def __init__(self, device_index: int, period_s: float = 0.02):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.ok = False
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as e:  # reading clocks is best effort; report it
            self.err = repr(e)

    def _run(self):
        nv = self.nv
        get_r = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = get_r(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self.ok and self._thread is None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __enter__(self):
        return self.start()

    def __exit__(self, *a):
        if self._thread:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "note": "NVML unavailable: " + getattr(self, "err", "")}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------- distributed
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        if args.impl == "ours":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks(v: float, world: int) -> list:
    """Every rank's value (rank order), gathered over the process group."""
    if world == 1:
        return [v]
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(o.item()) for o in out]


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ------------------------------------------------------------- CPU timing
_CPU_INPUTS: dict = {}


def cpu_gemm_rows_rate(rows_per_call: int, budget_s: float, threads: int):
    """Times the oracle's bf16 GEMM loop nest on rows of the 8192^3 problem.

    Returns (TFLOP/s, rows timed, seconds).  The rows are the first rows of
    the same seeded A, the full seeded B.
    """
    import oracle

    oracle.set_threads(threads)
    K = N = 8192
    key = ("gemm", rows_per_call)
    if key not in _CPU_INPUTS:
        _CPU_INPUTS.clear()
        b = oracle.to_bf16(oracle.uniform("gemm_b", (K, N)))
        a_rows = oracle.to_bf16(oracle.uniform("gemm_a", (rows_per_call * 4, K)))
        _CPU_INPUTS[key] = (a_rows, b)
    a_rows, b = _CPU_INPUTS[key]
    done, t0 = 0, time.perf_counter()
    while True:
        r0 = (done % (rows_per_call * 4))
        oracle.gemm_bf16_rows(a_rows, b, r0, r0 + rows_per_call)
        done += rows_per_call
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return 2.0 * done * N * K / el / 1e12, done, el


def cpu_baseline_gemm(budget_s: float = 12.0):
    import oracle

    threads = os.cpu_count() or 1
    rate, rows, el = cpu_gemm_rows_rate(max(threads, 1), budget_s, threads)
    return {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} output rows of the 8192^3 bf16 GEMM (oracle/oracle.c "
                      f"orc_gemm_bf16_rows, gcc -O2 -fopenmp, {threads} threads), {el:.1f} s"}


def cpu_baseline_moe(cfg: str, sample_rows: int = 0):
    """Oracle MoE layer on the host: routing and dispatch of every token, then
    the SwiGLU expert FFN on a sample of routed rows (all through one
    expert's weights -- the work per row is the same for every expert) and
    the combine; tokens/s extrapolated to the whole batch."""
    import oracle

    c = MOE_CONFIGS[cfg]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    rows = sample_rows or 2 * threads
    x = oracle.to_bf16(oracle.normal("moe_x", (T, D)))
    wr = oracle.to_bf16(oracle.normal("moe_router", (D, E), sigma=0.02))
    wg = oracle.to_bf16(oracle.normal("moe_wg", (D, F), sigma=0.02))
    wu = oracle.to_bf16(oracle.normal("moe_wu", (D, F), sigma=0.02))
    wd = oracle.to_bf16(oracle.normal("moe_wd", (F, D), sigma=0.02))
    t0 = time.perf_counter()
    idx, w = oracle.router_topk(x, wr, k)
    _, _, perm, inv = oracle.dispatch(idx, E)
    t_route = time.perf_counter() - t0
    t0 = time.perf_counter()
    _, y, _ = oracle.expert_ffn(x[perm[:rows] // k], wg, wu, wd)
    t_rows = time.perf_counter() - t0
    ntok = max(1, rows // k)
    t0 = time.perf_counter()
    oracle.combine(y[: ntok * k], np.arange(ntok * k, dtype=np.int32).reshape(-1, k), w[:ntok])
    t_comb = time.perf_counter() - t0
    total = t_route + t_rows * (T * k) / rows + t_comb * T / ntok
    return {"value": T / total, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"router+dispatch of all {T} tokens ({t_route:.2f} s), SwiGLU FFN of "
                      f"{rows} routed rows ({t_rows:.2f} s), combine of {ntok} tokens; "
                      f"extrapolated to {T * k} rows; oracle/oracle.c, {threads} threads"}


# -------------------------------------------------------------------- GEMM
def bench_gemm(args, world, rank, local):
    import torch

    import remora_b200 as rb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if args.size:
        batch_local, M, N, K = 1, args.size, args.size, args.size
        workload = f"dot_general bf16 [{M},{K}]x[{K},{N}] (profiling case)"
        cfg_key = "gemm_size"
    elif world == 1:
        batch_local, M, N, K = 1, 8192, 8192, 8192
        workload = "dot_general bf16 [8192,8192]x[8192,8192]->[8192,8192], fp32 accumulate"
        cfg_key = "gemm_8192"
    else:
        if 8 % world:
            raise SystemExit("batched GEMM shards a batch of 8: --gpus must divide 8")
        batch_local, M, N, K = 8 // world, 4096, 4096, 4096
        workload = (f"dot_general bf16 batched [8,4096,4096]x[8,4096,4096], batch sharded "
                    f"{batch_local} per rank over {world} GPUs")
        cfg_key = "gemm_batched"
    flop_step = 2.0 * batch_local * M * N * K * world  # the whole job's work per step
    A = torch.empty(batch_local, M, K, dtype=torch.bfloat16, device=dev)
    B = torch.empty(batch_local, K, N, dtype=torch.bfloat16, device=dev)
    C = torch.empty(batch_local, M, N, dtype=torch.bfloat16, device=dev)
    # each rank fills its own batch slice of the job's seeded tensors
    rb.fill_uniform(A, rb.stream_key(10 + 100 * rank))
    rb.fill_uniform(B, rb.stream_key(11 + 100 * rank))
    a2, b2, c2 = (A[0], B[0], C[0]) if batch_local == 1 else (A, B, C)
    stream = torch.cuda.current_stream(dev)

    def step():
        rb.gemm(a2, b2, out=c2)

    for _ in range(args.warmup):
        step()
    clk = ClockSampler(local).start()  # NVML set-up before the barrier that aligns the ranks
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms_local, world)
    value = flop_step / (ms * 1e-3) / 1e12

    # end to end through the public API: pinned host inputs in, result out
    Ah = torch.empty(A.shape, dtype=A.dtype, pin_memory=True)
    Bh = torch.empty(B.shape, dtype=B.dtype, pin_memory=True)
    Ch = torch.empty(C.shape, dtype=C.dtype, pin_memory=True)
    Ah.copy_(A)
    Bh.copy_(B)
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        A.copy_(Ah, non_blocking=True)
        B.copy_(Bh, non_blocking=True)
        rb.gemm(a2, b2, out=c2)
        Ch.copy_(C, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    ev0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(ev0.elapsed_time(ev1) / e2e_steps, world)
    h2d = (A.numel() + B.numel()) * 2 * world
    d2h = C.numel() * 2 * world

    peaks, src = load_peaks()
    achieved = 2.0 * batch_local * M * N * K / (ms_local * 1e-3) / 1e12
    traffic = NCU_TRAFFIC_BYTES.get(cfg_key)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded U(-1,1) bf16)",
        "config": {"workload": workload, "M": M, "N": N, "K": K, "batch": 8 if world > 1 else 1,
                   "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                   "l2": f"inputs {(A.numel() + B.numel()) * 2 / 2**20:.0f} MiB per GPU "
                         "> 126 MB L2 (no flush)"},
        "roofline": {"bound": "tensor", "achieved": achieved,
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"],
                     "peak_sustained": peaks.get("bf16_tflops_sustained"),
                     "peak_source": src, "traffic": traffic,
                     "kernel": "rb::gemm::k_gemm_bf16<true>"},
        "e2e": {"value": flop_step / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    return line


# --------------------------------------------------------------------- MoE
MOE_CONFIGS = {
    "4": dict(T=8192, D=4096, F=14336, E=8, k=2),
    "5": dict(T=65536, D=2048, F=1536, E=64, k=8),
}


def _cuda_time(fn, reps, dev):
    import torch

    s = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(reps):
        fn()
    b.record(s)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def bench_moe(args, world, rank, local):
    """The MoE layer (router, dispatch, SwiGLU expert GEMMs, combine) on one
    GPU per rank; tokens/s = T / layer time."""
    import torch

    import remora_b200 as rb

    c = MOE_CONFIGS[args.moe_config]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    wg = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wu = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wd = torch.empty(E, F, D, dtype=torch.bfloat16, device=dev)
    for t, stream_id, sig in ((x, 30, 1.0), (wr, 31, 0.02), (wg, 32, 0.02), (wu, 33, 0.02),
                              (wd, 34, 0.02)):
        rb.fill_normal(t, rb.stream_key(stream_id + 100 * rank), 0.0, sig)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(rb.moe_workspace_bytes(T, D, F, E, k), dtype=torch.uint8, device=dev)

    def step():
        rb.moe_layer(x, wr, wg, wu, wd, k, out=out, workspace=ws)

    for _ in range(args.warmup):
        step()
    clk = ClockSampler(local).start()  # NVML set-up before the barrier that aligns the ranks
    rb.synchronize_and_check(dev)
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    rb.synchronize_and_check(dev)

    # per-kernel times of the expert GEMMs on the same routing (roofline)
    idx, w = rb.moe_router_topk(x, wr, k)
    counts, offsets, perm, inv = rb.moe_dispatch(idx, E)
    xs = rb.moe_gather(x, perm, k)
    h = rb.grouped_gemm_swiglu(xs, wg, wu, offsets)
    y = rb.grouped_gemm(h, wd, offsets)
    reps = 5
    t_up = _cuda_time(lambda: rb.grouped_gemm_swiglu(xs, wg, wu, offsets, out=h), reps, dev)
    t_down = _cuda_time(lambda: rb.grouped_gemm(h, wd, offsets, out=y), reps, dev)
    t_router = _cuda_time(lambda: rb.moe_router_topk(x, wr, k, idx=idx, w=w), reps, dev)
    rows = T * k
    flop_up = 2.0 * rows * D * F * 2
    flop_down = 2.0 * rows * F * D
    peaks, src = load_peaks()
    up_tf = flop_up / (t_up * 1e-3) / 1e12

    # end to end: tokens in from pinned host memory, layer output back
    xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    oh = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    xh.copy_(x)

    def e2e_step():
        x.copy_(xh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)

    for _ in range(2):
        e2e_step()
    e2e_ms = max_over_ranks(_cuda_time(e2e_step, max(3, min(args.steps, 10)), dev), world)
    tokens = T * world
    return {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, bf16)",
        "config": {"workload": f"MoE layer config {args.moe_config}: T={T} D={D} F={F} E={E} "
                               f"top-{k}, SwiGLU experts", "parallelism":
                   f"independent layer per rank x{world}" if world > 1 else "single GPU",
                   "expert_flop_per_step": (flop_up + flop_down) * world,
                   "expert_tflops": (flop_up + flop_down) / (ms * 1e-3) / 1e12,
                   "kernel_ms": {"grouped_swiglu": t_up, "grouped_down": t_down,
                                 "router_topk": t_router},
                   "l2": "weights and activations > 126 MB L2 (no flush)"},
        "roofline": {"bound": "tensor", "achieved": up_tf, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": up_tf / peaks["bf16_tflops"],
                     "peak_sustained": peaks.get("bf16_tflops_sustained"), "peak_source": src,
                     "traffic": NCU_TRAFFIC_BYTES.get("moe_swiglu_" + args.moe_config),
                     "kernel": "rb::moe::k_grouped_gemm<true>",
                     "down_tflops": flop_down / (t_down * 1e-3) / 1e12},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": x.numel() * 2 * world,
                "d2h_bytes_per_step": out.numel() * 2 * world, "ms_per_step": e2e_ms},
        "gpu_launches": 8 * args.steps, "clocks": clk.summary(),
    }


def bench_moe_ep(args, world, rank, local):
    """Expert-parallel MoE, config 5: 65536 tokens split over the ranks,
    64 experts split over the ranks (8 per GPU at 8 GPUs), token dispatch
    and combine by NCCL all-to-all.  One GPU runs the single-GPU layer."""
    import torch

    import remora_b200 as rb
    from remora_b200.ep import moe_ep_forward

    c = MOE_CONFIGS["5"]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    if T % world or E % world:
        raise SystemExit(f"config 5 does not split over {world} ranks")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    tl, Epr = T // world, E // world
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    rb.fill_normal(x, rb.stream_key(30), 0.0, 1.0)
    rb.fill_normal(wr, rb.stream_key(31), 0.0, 0.02)
    x = x[rank * tl:(rank + 1) * tl].contiguous()
    ws = []
    for sid, shape in ((32, (E, D, F)), (33, (E, D, F)), (34, (E, F, D))):
        full = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        rb.fill_normal(full, rb.stream_key(sid), 0.0, 0.02)
        ws.append(full if world == 1 else full[rank * Epr:(rank + 1) * Epr].contiguous())
        del full
    wg, wu, wd = ws
    out = torch.empty(tl, D, dtype=torch.bfloat16, device=dev)
    lws = (torch.empty(rb.moe_workspace_bytes(T, D, F, E, k), dtype=torch.uint8, device=dev)
           if world == 1 else None)

    pep = None
    if world > 1 and args.ep_mode in ("p2p", "p2p-split"):
        from remora_b200.ep_p2p import PeerEP

        pep = PeerEP(tl, D, F, E, k, device=dev, fused=args.ep_mode == "p2p")

    def step():
        if world == 1:
            rb.moe_layer(x, wr, wg, wu, wd, k, out=out, workspace=lws)
        elif pep is not None:
            pep.forward(x, wr, wg, wu, wd, out=out)
        else:
            out.copy_(moe_ep_forward(x, wr, wg, wu, wd, k, E, chunks=args.ep_chunks or None))

    for _ in range(args.warmup):
        step()
    clk = ClockSampler(local).start()  # NVML set-up before the barrier that aligns the ranks
    rb.synchronize_and_check(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    rank_ms = all_ranks(ms_local, world)
    ms = max(rank_ms)
    xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    oh = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    xh.copy_(x)

    def e2e_step():
        x.copy_(xh, non_blocking=True)
        step()
        oh.copy_(out, non_blocking=True)

    e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(_cuda_time(e2e_step, max(3, min(args.steps, 10)), dev), world)
    flop = 6.0 * D * F * T * k
    peaks, src = load_peaks()
    per_gpu_tf = flop / world / (ms * 1e-3) / 1e12
    return {
        "metric": METRIC, "value": T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, bf16)",
        "config": {"workload": f"expert-parallel MoE config 5: T={T} D={D} F={F} E={E} top-{k}, "
                               f"{Epr} experts and {tl} tokens per GPU",
                   "parallelism": (f"EP{world} ({EP_MODES[args.ep_mode]})"
                                   if world > 1 else "single GPU"),
                   "ep_chunks": args.ep_chunks or "default",
                   "expert_flop_per_step": flop,
                   "rank_ms": [round(v, 4) for v in rank_ms]},
        "roofline": {"bound": "tensor", "achieved": per_gpu_tf, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": per_gpu_tf / peaks["bf16_tflops"],
                     "peak_source": src, "traffic": None,
                     "kernel": "whole layer per GPU (expert FLOP / layer time)"},
        "e2e": {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": x.numel() * 2 * world,
                "d2h_bytes_per_step": out.numel() * 2 * world, "ms_per_step": e2e_ms},
        "gpu_launches": (EP_LAUNCHES[args.ep_mode] if world > 1 else 8) * args.steps,
        "clocks": clk.summary(),
    }


# kernels of one EP layer: router 1, dispatch 3, then (fused) meta, experts (copy + SwiGLU +
# down), barrier, combine; (split) scatter, barrier, segments, SwiGLU, down, barrier, combine
EP_LAUNCHES = {"p2p": 8, "p2p-split": 11, "nccl": 9}
EP_MODES = {"p2p": "NVLink peer memory: row copy, SwiGLU and down tiles in one cooperative "
                   "kernel, down epilogues store to the source ranks",
            "p2p-split": "NVLink peer memory: scatter kernel, barrier, GEMMs",
            "nccl": "NCCL all-to-all"}


def bench_attention(args, world, rank, local):
    """Causal softmax attention, Q, K, V bf16 [4, 32, 4096, 128]; the 128
    (batch, head) pairs are split over the ranks (no collective)."""
    import torch

    import remora_b200 as rb

    B, H, S, Dh = 4, 32, 4096, 128
    if (B * H) % world:
        raise SystemExit(f"{B * H} (batch, head) pairs do not split over {world} ranks")
    bh = B * H // world
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    q, k, v = (torch.empty(1, bh, S, Dh, dtype=torch.bfloat16, device=dev) for _ in range(3))
    for t, sid in ((q, 20), (k, 21), (v, 22)):
        rb.fill_normal(t, rb.stream_key(sid + 100 * rank))
    o = torch.empty_like(q)

    def step():
        rb.attention(q, k, v, causal=True, out=o)

    for _ in range(args.warmup):
        step()
    clk = ClockSampler(local).start()  # NVML set-up before the barrier that aligns the ranks
    torch.cuda.synchronize(dev)
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    ms_local = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms_local, world)
    flop = 4.0 * B * H * S * S * Dh / 2.0
    qh, kh, vh, oh = (torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (q, k, v, o))
    qh.copy_(q), kh.copy_(k), vh.copy_(v)

    def e2e_step():
        q.copy_(qh, non_blocking=True)
        k.copy_(kh, non_blocking=True)
        v.copy_(vh, non_blocking=True)
        step()
        oh.copy_(o, non_blocking=True)

    e2e_step()
    barrier(world)
    e2e_ms = max_over_ranks(_cuda_time(e2e_step, max(3, min(args.steps, 10)), dev), world)
    peaks, src = load_peaks()
    achieved = flop / world / (ms_local * 1e-3) / 1e12
    return {
        "metric": METRIC, "value": flop / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16)",
        "config": {"workload": f"causal attention bf16 [{B},{H},{S},{Dh}], {bh} (batch, head) "
                               f"pairs per GPU", "flop_convention": "4*B*H*S^2*Dh/2 (causal half)",
                   "parallelism": f"batch x heads sharded x{world}" if world > 1 else "single GPU",
                   "l2": "q, k, v 402 MB > 126 MB L2 (no flush)"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                     "peak_source": src, "traffic": None, "kernel": "rb::attn::k_attention_fwd"},
        "e2e": {"value": flop / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": 3 * q.numel() * 2 * world,
                "d2h_bytes_per_step": o.numel() * 2 * world, "ms_per_step": e2e_ms},
        "gpu_launches": args.steps, "clocks": clk.summary(),
    }


# ------------------------------------------------------------- elementwise
def bench_elementwise(args, world, rank, local):
    """scale -> add -> exp chain: the named [1,8,128,128] shape (latency
    bound, L2 resident) and a 2^28-element sweep where HBM BW is judged."""
    import torch

    import remora_b200 as rb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = 1 << 28
    s = torch.empty(n, device=dev)
    b = torch.empty(n, device=dev)
    o = torch.empty(n, device=dev)
    rb.fill_normal(s, rb.stream_key(1))
    rb.fill_normal(b, rb.stream_key(2))
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        rb.scale_add_exp(s, b, 0.125, out=o)
    clk = ClockSampler(local).start()  # NVML set-up before the barrier that aligns the ranks
    torch.cuda.synchronize(dev)
    barrier(world)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clk:
        ev0.record(stream)
        for _ in range(args.steps):
            rb.scale_add_exp(s, b, 0.125, out=o)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, world)
    bytes_step = 12.0 * n * world
    gbs = bytes_step / (ms * 1e-3) / 1e9
    small = rb.run_test("elementwise_chain", device=local, iters=200, warmup=20)
    peaks, src = load_peaks()
    return {
        "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) f32)",
        "config": {"workload": "exp(s*0.125+b) f32, 2^28 elements (3 GiB per step)",
                   "named_shape_us_per_call": small["ms_per_iter"] * 1e3,
                   "l2": "inputs 2 GiB > 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": gbs / world / peaks["hbm_gbs"],
                     "peak_source": src, "traffic": NCU_TRAFFIC_BYTES.get("elementwise")},
        "gpu_launches": args.steps, "clocks": clk.summary(),
    }


# --------------------------------------------------------- reference arm
def reference_arm(args, world, rank):
    """The reference's CPU path (its loop nest, restated in oracle/) on all
    host threads, on a bounded row sample of the same GEMM per step."""
    if rank != 0:
        return None
    import oracle

    threads = os.cpu_count() or 1
    # calibrate: rows per step so that the whole run stays within ~2 minutes
    rate, rows, el = cpu_gemm_rows_rate(threads, 2.0, threads)
    sec_per_row = el / rows
    per_step = max(1, int(min(threads * 4, 100.0 / (args.steps + args.warmup) / sec_per_row)))
    for _ in range(args.warmup):
        cpu_gemm_rows_rate(per_step, 0.0, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_gemm_rows_rate(per_step, 0.0, threads)
    el = time.perf_counter() - t0
    v = 2.0 * per_step * 8192 * 8192 * args.steps / el / 1e12
    sample = (f"{per_step} output rows of the 8192^3 bf16 GEMM per step "
              f"(oracle/oracle.c loop nest, {threads} threads)")
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded U(-1,1) bf16)",
        "config": {"workload": "dot_general bf16 [8192,8192]x[8192,8192]->[8192,8192], fp32 "
                               "accumulate (row sample per step)"},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gemm", "elementwise", "moe", "moe_ep", "attention"],
                    default="gemm")
    ap.add_argument("--moe-config", choices=sorted(MOE_CONFIGS), default="4")
    ap.add_argument("--ep-mode", choices=["p2p", "p2p-split", "nccl"], default="p2p",
                    help="moe_ep: token exchange by the library's peer-memory kernels or NCCL")
    ap.add_argument("--ep-chunks", type=int, default=0,
                    help="moe_ep: token pieces per layer for comm/compute overlap (0 = default)")
    ap.add_argument("--size", type=int, default=0,
                    help="gemm: run an MxNxK = size^3 case instead of the configuration")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    if args.impl == "reference":
        line = reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    from remora_b200 import build

    build.build()  # no-op when the in-tree library is current
    fn = {"gemm": bench_gemm, "elementwise": bench_elementwise, "moe": bench_moe,
          "moe_ep": bench_moe_ep, "attention": bench_attention}[args.workload]
    line = fn(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if args.workload == "gemm":
            line["cpu_baseline"] = cpu_baseline_gemm()
        elif args.workload == "moe":
            line["cpu_baseline"] = cpu_baseline_moe(args.moe_config)
        else:
            line["cpu_baseline"] = None
    elif rank == 0:
        line["cpu_baseline"] = None
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
