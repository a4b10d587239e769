"""Benchmark of the remora_b200 hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload moe_ep|moe|gemm|attention|elementwise]

Default workload: the expert-parallel MoE layer, 65536 tokens x d_model 2048
bf16, router [2048,64] with top-8 gating, 64 SwiGLU experts of ffn dim 1536,
metric tokens/s.  With N = 1 one GPU runs the whole layer
(remora_b200_moe_layer_bf16); under torchrun with N > 1 the tokens and the
experts are split over the ranks (65536/N tokens and 64/N experts per GPU)
and the token exchange runs over NVLink peer memory inside the library's
expert kernel (remora_b200/ep_p2p.py).  The job's total work is fixed, so
the scaling is strong.  Rank 0 prints one JSON line.

Other workloads: `moe` (one GPU per rank runs a whole layer: --moe-config 4
= 8192 x 4096, 8 experts of F 14336, top-2; 5 = the default shape), `gemm`
(dot_general bf16 8192^3; batch-sharded [8,4096,4096]^2 at N > 1),
`attention` (causal [4,32,4096,128], (batch, head) pairs sharded) and
`elementwise` (exp(s*0.125+b) f32 over 2^28 elements).

--impl reference times the reference's CPU path for the same workload and
metric: the C restatement of remora's loop nests (oracle/) on all host
threads, one bounded sample of the workload per step.  `cpu_baseline` in the
GPU arm's line is the same restatement timed single-threaded (the reference
CPU path is scalar and single-threaded) and on all host threads.
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
# NVLS (NVLink SHARP) binds NVLink multicast memory; nothing here needs it.
os.environ.setdefault("NCCL_NVLS_ENABLE", "0")

METRIC = "MoE layer tokens/s; GEMM/attn TFLOP/s as % B200 peak; elementwise HBM GB/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant
# kernel, from the ncu captures summarised in profiles/ (None = not captured).
NCU_TRAFFIC_BYTES = {
    "gemm_8192": 1140578560,  # profiles/gemm_bf16_8192_dram.md
    "gemm_batched": None,
    "elementwise": None,
    "moe_swiglu_5": 4612174000,  # profiles/grouped_gemm_swiglu_65536x2048_e64_dram.md
    "moe_swiglu_4": None,
    # one-rank capture of the merged expert kernel at the per-rank shape of the 8-GPU
    # layer (65536 rows): profiles/moe_ep_experts_p1_8x65536_full.md
    "moe_ep_experts": 1321200000,
    # [2,16,4096,128] capture of the persistent kernel (156.1 MB) scaled by 4 to the
    # [4,32,4096,128] launch: profiles/attention_causal_2x16x4096_full.md
    "attention": 624541696,
}

MOE_CONFIGS = {
    "4": dict(T=8192, D=4096, F=14336, E=8, k=2),
    "5": dict(T=65536, D=2048, F=1536, E=64, k=8),
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

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
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
# The reference CPU path (remora's ExecutionEngine over convert-linalg-to-loops
# scalar loops, compiler/cpu.cpp:25-92) cannot be built offline; its loop
# nests are restated in oracle/oracle.c, which is timed here on bounded
# samples of each workload.  Each sampler returns (units done, seconds) for
# one call of `chunk` units; rates are units per second.
_CPU_CACHE: dict = {}


def _oracle(threads: int):
    import oracle

    oracle.set_threads(threads)
    return oracle


def _gemm_sampler(threads):
    """Output rows of the 8192^3 bf16 GEMM (the oracle's increasing-k fp32
    loop nest); unit = FLOP (2*N*K per row)."""
    orc = _oracle(threads)
    if "gemm" not in _CPU_CACHE:
        b = orc.to_bf16(orc.uniform("gemm_b", (8192, 8192)))
        a = orc.to_bf16(orc.uniform("gemm_a", (256, 8192)))  # first rows of A
        _CPU_CACHE["gemm"] = (a, b)
    a, b = _CPU_CACHE["gemm"]
    state = {"r": 0}

    def run(chunk):
        r0 = state["r"] % (a.shape[0] - chunk + 1)
        orc.gemm_bf16_rows(a, b, r0, r0 + chunk)
        state["r"] += chunk
        return 2.0 * chunk * 8192 * 8192

    return run, "output rows of the 8192^3 bf16 GEMM (oracle/oracle.c orc_gemm_bf16_rows)"


def _moe_sampler(threads, cfg):
    """Whole tokens of the MoE layer: router + top-k over all experts,
    dispatch, the SwiGLU expert FFN of each routed row, combine (the oracle's
    loop nests).  Every routed row runs through the first expert's weights:
    the work per row is the same for every expert, and this keeps the sample
    from generating all expert weights.  unit = tokens."""
    orc = _oracle(threads)
    c = MOE_CONFIGS[cfg]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    key = ("moe", cfg)
    if key not in _CPU_CACHE:
        pool = 256
        x = orc.to_bf16(orc.normal("moe_x", (pool, D)))  # the first token rows of x
        wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.02))
        wg = orc.to_bf16(orc.normal("moe_wg", (D, F), sigma=0.02))
        wu = orc.to_bf16(orc.normal("moe_wu", (D, F), sigma=0.02))
        wd = orc.to_bf16(orc.normal("moe_wd", (F, D), sigma=0.02))
        _CPU_CACHE[key] = (x, wr, wg, wu, wd)
    x, wr, wg, wu, wd = _CPU_CACHE[key]
    state = {"t": 0}

    def run(chunk):
        t0 = state["t"] % (x.shape[0] - chunk + 1)
        xs = x[t0:t0 + chunk]
        idx, w = orc.router_topk(xs, wr, k)
        _, _, perm, inv = orc.dispatch(idx, E)
        _, y, _ = orc.expert_ffn(np.ascontiguousarray(xs[perm // k]), wg, wu, wd)
        orc.combine(y, inv, w)
        state["t"] += chunk
        return float(chunk)

    return run, (f"whole tokens of the MoE layer T={T} D={D} F={F} E={E} top-{k} (router, "
                 f"dispatch, SwiGLU FFN of every routed row, combine; oracle/oracle.c)")


def _attention_sampler(threads):
    """Query rows of one (batch, head) of causal [4,32,4096,128] attention
    (the oracle's fp64 softmax restatement), rows drawn uniformly so the
    average causal work matches the whole problem; unit = FLOP
    (4*(row+1)*128 per row)."""
    orc = _oracle(threads)
    S, Dh = 4096, 128
    if "attn" not in _CPU_CACHE:
        _CPU_CACHE["attn"] = tuple(orc.to_bf16(orc.normal(n, (S, Dh)))
                                   for n in ("attn_q", "attn_k", "attn_v"))
    q, k, v = _CPU_CACHE["attn"]
    rng = np.random.default_rng(7)

    def run(chunk):
        rows = rng.integers(0, S, chunk)
        orc.attention_rows(q, k, v, rows, causal=True)
        return float(np.sum(4.0 * (rows + 1) * Dh))

    return run, "query rows of causal attention [4,32,4096,128] (oracle/oracle.c, fp64 softmax)"


def _elementwise_sampler(threads):
    """exp(s*0.125 + b) over f32 elements (the oracle's loop); unit = bytes
    (12 per element: two reads, one write)."""
    orc = _oracle(threads)
    n = 1 << 22
    if "ew" not in _CPU_CACHE:
        _CPU_CACHE["ew"] = (orc.normal("scores", (n,)), orc.normal("bias", (n,)))
    s, b = _CPU_CACHE["ew"]

    def run(chunk):
        m = min(chunk, n)
        orc.scale_add_exp(s[:m], b[:m], 0.125)
        return 12.0 * m

    return run, "f32 elements of exp(s*0.125+b) (oracle/oracle.c)"


CPU_UNITS = {"gemm": ("TFLOP/s", 1e12), "attention": ("TFLOP/s", 1e12), "moe": ("tokens/s", 1.0),
             "moe_ep": ("tokens/s", 1.0), "elementwise": ("GB/s", 1e9)}


def cpu_sampler(workload: str, threads: int, moe_cfg: str = "5"):
    if workload == "gemm":
        return _gemm_sampler(threads)
    if workload in ("moe", "moe_ep"):
        return _moe_sampler(threads, "5" if workload == "moe_ep" else moe_cfg)
    if workload == "attention":
        return _attention_sampler(threads)
    return _elementwise_sampler(threads)


def _chunk(workload: str, threads: int) -> int:
    """Units per sampler call: enough parallel work for `threads` threads."""
    tokens = 1 if threads == 1 else -(-threads // 4)  # k >= 2 routed rows per token
    return {"gemm": threads, "moe": tokens, "moe_ep": tokens, "attention": 4 * threads,
            "elementwise": 1 << 22}[workload]


def cpu_rate(workload: str, threads: int, budget_s: float, moe_cfg: str = "5"):
    """(rate in the workload's unit, units done, seconds, sample text)."""
    run, what = cpu_sampler(workload, threads, moe_cfg)
    chunk = _chunk(workload, threads)
    run(chunk)  # warm-up (page-in, thread pool)
    done, t0 = 0.0, time.perf_counter()
    calls = 0
    while True:
        done += run(chunk)
        calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    unit, scale = CPU_UNITS[workload]
    return done / el / scale, calls * chunk, el, what


def cpu_baseline(workload: str, moe_cfg: str = "5", budget_s: float = 8.0):
    """The oracle restatement timed on this host: all threads (the line's
    value) and one thread (the reference CPU path is single-threaded)."""
    threads = os.cpu_count() or 1
    unit = CPU_UNITS[workload][0]
    v1, n1, e1, what = cpu_rate(workload, 1, budget_s, moe_cfg)
    vn, nn, en, _ = cpu_rate(workload, threads, budget_s, moe_cfg)
    return {"value": vn, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{nn} {what} on {threads} threads (gcc -O2 -fopenmp), {en:.1f} s",
            "single_thread": {"value": v1, "unit": unit, "cores": 1,
                              "sample": f"{n1} {what} on 1 thread, {e1:.1f} s"}}


# ------------------------------------------------------------ workloads
def workload_config(args, world: int) -> dict:
    """The workload's identity, the same in both arms' JSON lines."""
    w = args.workload
    if w == "moe_ep":
        c = MOE_CONFIGS["5"]
        T, E = c["T"], c["E"]
        par = ("single GPU" if world == 1 else
               f"expert-parallel x{world}: {T // world} tokens and {E // world} experts per GPU, "
               f"{EP_MODES[args.ep_mode]}")
        return {"workload": f"MoE layer: {T} tokens x d_model {c['D']} bf16, router "
                            f"[{c['D']},{E}] top-{c['k']}, {E} SwiGLU experts of ffn dim {c['F']}",
                **c, "parallelism": par,
                "l2": "per-step working set (tokens, expert weights, dispatched rows) > 126 MB "
                      "L2 (no flush)"}
    if w == "moe":
        c = MOE_CONFIGS[args.moe_config]
        return {"workload": f"MoE layer config {args.moe_config}: T={c['T']} D={c['D']} "
                            f"F={c['F']} E={c['E']} top-{c['k']}, SwiGLU experts", **c,
                "parallelism": f"one whole layer per GPU x{world}" if world > 1 else "single GPU",
                "l2": "weights and activations > 126 MB L2 (no flush)"}
    if w == "gemm":
        if args.size:
            n = args.size
            return {"workload": f"dot_general bf16 [{n},{n}]x[{n},{n}] (profiling case)",
                    "M": n, "N": n, "K": n, "batch": 1, "parallelism": "single GPU"}
        if world == 1:
            return {"workload": "dot_general bf16 [8192,8192]x[8192,8192]->[8192,8192], fp32 "
                                "accumulate", "M": 8192, "N": 8192, "K": 8192, "batch": 1,
                    "parallelism": "single GPU",
                    "l2": "inputs 256 MiB > 126 MB L2 (no flush)"}
        return {"workload": "dot_general bf16 batched [8,4096,4096]x[8,4096,4096], fp32 "
                            "accumulate", "M": 4096, "N": 4096, "K": 4096, "batch": 8,
                "parallelism": f"batch-sharded x{world} ({8 // world} per GPU)",
                "l2": "inputs > 126 MB L2 per GPU (no flush)"}
    if w == "attention":
        return {"workload": "causal softmax attention bf16 [4,32,4096,128], fp32 softmax "
                            "statistics", "B": 4, "H": 32, "S": 4096, "Dh": 128, "causal": True,
                "flop_convention": "4*B*H*S^2*Dh/2 (causal half)",
                "parallelism": (f"(batch, head) pairs sharded x{world}" if world > 1
                                else "single GPU"),
                "l2": "q, k, v 402 MB > 126 MB L2 (no flush)"}
    return {"workload": "exp(s*0.125+b) f32, 2^28 elements (3 GiB per step)", "n": 1 << 28,
            "parallelism": f"one chain per GPU x{world}" if world > 1 else "single GPU",
            "l2": "inputs 2 GiB > 126 MB L2 (no flush)"}


def _timed(step, args, world, dev, local):
    """W warm-up steps, then K steps between barriers and device syncs,
    CUDA events on the launching stream, SM clocks sampled meanwhile.
    Returns (this rank's ms per step, clock summary)."""
    import torch

    import remora_b200 as rb

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
    torch.cuda.synchronize(dev)
    rb.synchronize_and_check(dev)
    return ev0.elapsed_time(ev1) / args.steps, clk.summary()


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


def _e2e(step, ins, outs, args, world, dev):
    """The same step end to end through the public API: every step copies
    its inputs in from pinned host memory and its result back.  `ins` and
    `outs` are device tensors; returns (max-over-ranks ms, h2d, d2h bytes
    for the whole job)."""
    import torch

    hin = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ins]
    hout = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs]
    for h, t in zip(hin, ins):
        h.copy_(t)

    def e2e_step():
        for h, t in zip(hin, ins):
            t.copy_(h, non_blocking=True)
        step()
        for h, t in zip(hout, outs):
            h.copy_(t, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(_cuda_time(e2e_step, max(3, min(args.steps, 10)), dev), world)
    h2d = sum(t.numel() * t.element_size() for t in ins) * world
    d2h = sum(t.numel() * t.element_size() for t in outs) * world
    return ms, h2d, d2h


def _e2e_moe_host(rb, x, wr, wg, wu, wd, k, args, dev):
    """The one-GPU layer end to end through remora_b200_moe_layer_host_bf16:
    tokens in pinned host memory go up and the output comes back in chunks
    (the library's default: 16384 tokens, quarter- and half-size at both
    ends), overlapped with the layer's kernels.  Returns (ms, h2d, d2h bytes
    per step)."""
    import torch

    T, D = x.shape
    E, _, F = wg.shape
    x_host = x.cpu().pin_memory()
    out_host = torch.empty((T, D), dtype=torch.bfloat16, pin_memory=True)
    ws = torch.empty(rb.lib().remora_b200_moe_layer_host_workspace_bytes(T, D, F, E, k, 0),
                     dtype=torch.uint8, device=dev)

    def e2e_step():
        rb.moe_layer_host(x_host, wr, wg, wu, wd, k, out_host=out_host, workspace=ws)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    ms = _cuda_time(e2e_step, max(3, min(args.steps, 10)), dev)
    nbytes = T * D * 2
    return ms, nbytes, nbytes


def _line(args, world, value, unit, ms, scaling, dtype, data, roofline, e2e, launches, clocks,
          detail):
    return {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": dtype,
            "data": data, "config": workload_config(args, world), "roofline": roofline,
            "e2e": e2e, "gpu_launches": launches, "clocks": clocks, "detail": detail}


def _tensor_roofline(achieved, peaks, src, kernel, traffic=None, **extra):
    return {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
            "peak_sustained": peaks.get("bf16_tflops_sustained"), "peak_source": src,
            "traffic": traffic, "kernel": kernel, **extra}


def _moe_tensors(rb, c, dev, rank, world, sliced):
    """x [T, D] and the expert weights from the seeded generator; with
    `sliced`, this rank's T/world tokens and E/world experts."""
    import torch

    T, D, F, E = c["T"], c["D"], c["F"], c["E"]
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    rb.fill_normal(x, rb.stream_key(30), 0.0, 1.0)
    rb.fill_normal(wr, rb.stream_key(31), 0.0, 0.02)
    if sliced:
        tl = T // world
        x = x[rank * tl:(rank + 1) * tl].contiguous()
    ws = []
    Epr = E // world if sliced else E
    for sid, shape in ((32, (E, D, F)), (33, (E, D, F)), (34, (E, F, D))):
        full = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        rb.fill_normal(full, rb.stream_key(sid), 0.0, 0.02)
        ws.append(full[rank * Epr:(rank + 1) * Epr].contiguous() if sliced else full)
        del full
    torch.cuda.synchronize(dev)
    return x, wr, ws


def bench_moe_ep(args, world, rank, local):
    """The 65536-token, 64-expert MoE layer: one GPU runs it whole; N > 1
    GPUs split tokens and experts and exchange rows over NVLink."""
    import torch

    import remora_b200 as rb

    c = MOE_CONFIGS["5"]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    if T % world or E % world:
        raise SystemExit(f"the layer does not split over {world} ranks")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    tl = T // world
    x, wr, (wg, wu, wd) = _moe_tensors(rb, c, dev, rank, world, sliced=world > 1)
    out = torch.empty(tl, D, dtype=torch.bfloat16, device=dev)
    peaks, src = load_peaks()
    pep = None
    if world == 1:
        ws = torch.empty(rb.moe_workspace_bytes(T, D, F, E, k), dtype=torch.uint8, device=dev)

        def step():
            rb.moe_layer(x, wr, wg, wu, wd, k, out=out, workspace=ws)
    elif args.ep_mode == "nccl":
        from remora_b200.ep_nccl import NcclEP

        pep = NcclEP(tl, D, F, E, k, device=dev)

        def step():
            pep.forward(x, wr, wg, wu, wd, out=out)
    else:
        from remora_b200.ep_p2p import PeerEP

        pep = PeerEP(tl, D, F, E, k, device=dev, fused=args.ep_mode == "p2p")

        def step():
            pep.forward(x, wr, wg, wu, wd, out=out)

    ms_local, clocks = _timed(step, args, world, dev, local)
    rank_ms = all_ranks(ms_local, world)
    ms = max(rank_ms)
    if world == 1:
        e2e_ms, h2d, d2h = _e2e_moe_host(rb, x, wr, wg, wu, wd, k, args, dev)
    else:
        e2e_ms, h2d, d2h = _e2e(step, [x], [out], args, world, dev)

    # dominant kernel, timed by itself with CUDA events after the timed region
    if world == 1:
        idx, w = rb.moe_router_topk(x, wr, k)
        counts, offsets, perm, inv = rb.moe_dispatch(idx, E)
        xs = rb.moe_gather(x, perm, k)
        h = rb.grouped_gemm_swiglu(xs, wg, wu, offsets)
        y = rb.grouped_gemm(h, wd, offsets)
        t_up = _cuda_time(lambda: rb.grouped_gemm_swiglu(xs, wg, wu, offsets, out=h), 5, dev)
        t_down = _cuda_time(lambda: rb.grouped_gemm(h, wd, offsets, out=y), 5, dev)
        t_router = _cuda_time(lambda: rb.moe_router_topk(x, wr, k, idx=idx, w=w), 5, dev)
        rows = T * k
        up_tf = 4.0 * rows * D * F / (t_up * 1e-3) / 1e12
        roof = _tensor_roofline(up_tf, peaks, src, "rb::moe::k_grouped_gemm<true> (SwiGLU)",
                                NCU_TRAFFIC_BYTES.get("moe_swiglu_5"),
                                kernel_ms=t_up,
                                down_tflops=2.0 * rows * F * D / (t_down * 1e-3) / 1e12)
        detail = {"kernel_ms": {"grouped_swiglu": t_up, "grouped_down": t_down,
                                "router_topk": t_router},
                  "expert_tflops_layer": 6.0 * D * F * rows / (ms * 1e-3) / 1e12}
        launches = 8  # router, dispatch count/scan/scatter, row copy, SwiGLU, down, combine
    else:
        pep.profile = True
        phases = []
        for _ in range(5):
            step()
            phases.append(dict(pep.phase_ms))
        pep.profile = False
        rows_here = pep.rows_received()
        ph = {n: statistics.median(p[n] for p in phases) for n in phases[0]}
        t_exp = ph["experts"]
        exp_tf = 6.0 * D * F * rows_here / (t_exp * 1e-3) / 1e12
        roof = _tensor_roofline(exp_tf, peaks, src, pep.dominant_kernel,
                                NCU_TRAFFIC_BYTES.get("moe_ep_experts"), kernel_ms=t_exp,
                                rows=rows_here)
        detail = {"rank_ms": [round(v, 4) for v in rank_ms],
                  "phase_ms_rank0": {n: round(v, 4) for n, v in ph.items()},
                  "expert_tflops_per_gpu_layer": 6.0 * D * F * T * k / world / (ms * 1e-3) / 1e12}
        launches = pep.launches_per_layer
    line = _line(args, world, T / (ms * 1e-3), "tokens/s", ms, "strong", "bf16",
                 "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, bf16)", roof,
                 {"value": T / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                  "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                 launches * args.steps, clocks, detail)
    if pep is not None:
        pep.close()
    return line


def bench_moe(args, world, rank, local):
    """One whole MoE layer per GPU (config 4 or 5); tokens/s = T / layer time
    (summed over the ranks' independent layers)."""
    import torch

    import remora_b200 as rb

    c = MOE_CONFIGS[args.moe_config]
    T, D, F, E, k = c["T"], c["D"], c["F"], c["E"], c["k"]
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    x, wr, (wg, wu, wd) = _moe_tensors(rb, c, dev, rank, world, sliced=False)
    out = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(rb.moe_workspace_bytes(T, D, F, E, k), dtype=torch.uint8, device=dev)

    def step():
        rb.moe_layer(x, wr, wg, wu, wd, k, out=out, workspace=ws)

    ms_local, clocks = _timed(step, args, world, dev, local)
    ms = max_over_ranks(ms_local, world)
    e2e_ms, h2d, d2h = _e2e_moe_host(rb, x, wr, wg, wu, wd, k, args, dev)
    barrier(world)
    e2e_ms = max_over_ranks(e2e_ms, world)
    h2d, d2h = h2d * world, d2h * world
    idx, w = rb.moe_router_topk(x, wr, k)
    counts, offsets, perm, inv = rb.moe_dispatch(idx, E)
    xs = rb.moe_gather(x, perm, k)
    h = rb.grouped_gemm_swiglu(xs, wg, wu, offsets)
    y = rb.grouped_gemm(h, wd, offsets)
    t_up = _cuda_time(lambda: rb.grouped_gemm_swiglu(xs, wg, wu, offsets, out=h), 5, dev)
    t_down = _cuda_time(lambda: rb.grouped_gemm(h, wd, offsets, out=y), 5, dev)
    t_router = _cuda_time(lambda: rb.moe_router_topk(x, wr, k, idx=idx, w=w), 5, dev)
    rows = T * k
    peaks, src = load_peaks()
    up_tf = 4.0 * rows * D * F / (t_up * 1e-3) / 1e12
    roof = _tensor_roofline(up_tf, peaks, src, "rb::moe::k_grouped_gemm<true> (SwiGLU)",
                            NCU_TRAFFIC_BYTES.get("moe_swiglu_" + args.moe_config),
                            kernel_ms=t_up,
                            down_tflops=2.0 * rows * F * D / (t_down * 1e-3) / 1e12)
    tokens = T * world
    return _line(args, world, tokens / (ms * 1e-3), "tokens/s", ms, "weak", "bf16",
                 "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, bf16)", roof,
                 {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                 8 * args.steps, clocks,
                 {"kernel_ms": {"grouped_swiglu": t_up, "grouped_down": t_down,
                                "router_topk": t_router},
                  "expert_tflops_layer": 6.0 * D * F * rows / (ms * 1e-3) / 1e12})


def bench_gemm(args, world, rank, local):
    import torch

    import remora_b200 as rb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = workload_config(args, world)
    if args.size or world == 1:
        batch_local, M, N, K = 1, cfg["M"], cfg["N"], cfg["K"]
        key = "gemm_size" if args.size else "gemm_8192"
    else:
        if 8 % world:
            raise SystemExit("batched GEMM shards a batch of 8: --gpus must divide 8")
        batch_local, M, N, K = 8 // world, 4096, 4096, 4096
        key = "gemm_batched"
    A = torch.empty(batch_local, M, K, dtype=torch.bfloat16, device=dev)
    B = torch.empty(batch_local, K, N, dtype=torch.bfloat16, device=dev)
    C = torch.empty(batch_local, M, N, dtype=torch.bfloat16, device=dev)
    # each rank fills its own batch slice of the job's seeded tensors
    rb.fill_uniform(A, rb.stream_key(10 + 100 * rank))
    rb.fill_uniform(B, rb.stream_key(11 + 100 * rank))
    a2, b2, c2 = (A[0], B[0], C[0]) if batch_local == 1 else (A, B, C)

    def step():
        rb.gemm(a2, b2, out=c2)

    ms_local, clocks = _timed(step, args, world, dev, local)
    ms = max_over_ranks(ms_local, world)
    e2e_ms, h2d, d2h = _e2e(step, [A, B], [C], args, world, dev)
    flop_local = 2.0 * batch_local * M * N * K
    peaks, src = load_peaks()
    achieved = flop_local / (ms_local * 1e-3) / 1e12
    roof = _tensor_roofline(achieved, peaks, src, "rb::gemm::k_gemm_bf16",
                            NCU_TRAFFIC_BYTES.get(key), kernel_ms=ms_local)
    return _line(args, world, flop_local * world / (ms * 1e-3) / 1e12, "TFLOP/s", ms,
                 "strong", "bf16", "synthetic (seeded U(-1,1) bf16)", roof,
                 {"value": flop_local * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                 args.steps, clocks, {})


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

    ms_local, clocks = _timed(step, args, world, dev, local)
    ms = max_over_ranks(ms_local, world)
    e2e_ms, h2d, d2h = _e2e(step, [q, k, v], [o], args, world, dev)
    flop = 4.0 * B * H * S * S * Dh / 2.0
    peaks, src = load_peaks()
    achieved = flop / world / (ms_local * 1e-3) / 1e12
    roof = _tensor_roofline(achieved, peaks, src, "rb::attnp::k_attention_persist",
                            NCU_TRAFFIC_BYTES.get("attention"), kernel_ms=ms_local)
    return _line(args, world, flop / (ms * 1e-3) / 1e12, "TFLOP/s", ms, "strong", "bf16",
                 "synthetic (seeded N(0,1) bf16)", roof,
                 {"value": flop / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                 args.steps, clocks, {})


def bench_elementwise(args, world, rank, local):
    """scale -> add -> exp chain over 2^28 f32 elements (HBM bound), with the
    named [1,8,128,128] shape's time per call (latency bound) beside it."""
    import torch

    import remora_b200 as rb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = 1 << 28
    s = torch.empty(n, device=dev)
    b = torch.empty(n, device=dev)
    o = torch.empty(n, device=dev)
    rb.fill_normal(s, rb.stream_key(1 + 100 * rank))
    rb.fill_normal(b, rb.stream_key(2 + 100 * rank))

    def step():
        rb.scale_add_exp(s, b, 0.125, out=o)

    ms_local, clocks = _timed(step, args, world, dev, local)
    ms = max_over_ranks(ms_local, world)
    e2e_ms, h2d, d2h = _e2e(step, [s, b], [o], args, world, dev)
    bytes_step = 12.0 * n * world
    small = rb.run_test("elementwise_chain", device=local, iters=200, warmup=20)
    peaks, src = load_peaks()
    gbs_local = 12.0 * n / (ms_local * 1e-3) / 1e9
    roof = {"bound": "hbm", "achieved": gbs_local, "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": gbs_local / peaks["hbm_gbs"], "peak_source": src,
            "traffic": NCU_TRAFFIC_BYTES.get("elementwise"), "kernel": "rb::k_scale_add_exp_v4",
            "kernel_ms": ms_local}
    return _line(args, world, bytes_step / (ms * 1e-3) / 1e9, "GB/s", ms, "weak", "f32",
                 "synthetic (seeded N(0,1) f32)", roof,
                 {"value": bytes_step / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                  "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
                 args.steps, clocks, {"named_shape_us_per_call": small["ms_per_iter"] * 1e3})


# kernels of one layer: single GPU: router 1, dispatch 3, gather, SwiGLU, down, combine;
# expert-parallel over peer memory: router 1, dispatch 3, then (fused) meta, experts
# (copy + SwiGLU + down), barrier, combine; (split) scatter, barrier, segments, SwiGLU,
# down, barrier, combine
EP_MODES = {"p2p": "token exchange over NVLink peer memory inside the expert kernel",
            "p2p-split": "token exchange over NVLink peer memory (scatter kernel, barrier, "
                         "grouped GEMMs)",
            "nccl": "token exchange by NCCL all-to-all-v through the library's C ABI"}


# --------------------------------------------------------- reference arm
def reference_arm(args, world, rank):
    """The reference's CPU path (its loop nests, restated in oracle/) on all
    host threads, one bounded sample of the same workload per step; rank 0
    only."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    run, what = cpu_sampler(args.workload, threads, args.moe_config)
    chunk = _chunk(args.workload, threads)
    t0 = time.perf_counter()
    run(chunk)  # calibration call
    per_call = max(time.perf_counter() - t0, 1e-6)
    calls = max(1, int(90.0 / (args.steps + args.warmup) / per_call))
    for _ in range(args.warmup):
        for _ in range(calls):
            run(chunk)
    done, t0 = 0.0, time.perf_counter()
    for _ in range(args.steps):
        for _ in range(calls):
            done += run(chunk)
    el = time.perf_counter() - t0
    unit, scale = CPU_UNITS[args.workload]
    v = done / el / scale
    sample = f"{calls * chunk} {what} per step on {threads} threads (gcc -O2 -fopenmp)"
    return {
        "impl": "reference", "metric": METRIC, "value": v, "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": {"moe_ep": "strong", "gemm": "strong", "attention": "strong"}.get(
            args.workload, "weak"),
        "vs_baseline": None, "dtype": "f32" if args.workload == "elementwise" else "bf16",
        "data": "synthetic (seeded inputs, the GPU arm's generator)",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["moe_ep", "moe", "gemm", "attention", "elementwise"],
                    default="moe_ep")
    ap.add_argument("--moe-config", choices=sorted(MOE_CONFIGS), default="4",
                    help="moe: which layer each GPU runs")
    ap.add_argument("--ep-mode", choices=sorted(EP_MODES), default="p2p",
                    help="moe_ep at N > 1: how the token exchange runs")
    ap.add_argument("--size", type=int, default=0,
                    help="gemm: run an MxNxK = size^3 case instead of the configuration")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # no process group: rank 0 alone runs the CPU path, the other ranks exit
        world = int(os.environ.get("WORLD_SIZE", "1"))
        line = reference_arm(args, world, int(os.environ.get("RANK", "0")))
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args)
    from remora_b200 import build

    build.build()  # no-op when the in-tree library is current
    fn = {"gemm": bench_gemm, "elementwise": bench_elementwise, "moe": bench_moe,
          "moe_ep": bench_moe_ep, "attention": bench_attention}[args.workload]
    line = fn(args, world, rank, local)
    if rank == 0:
        line["cpu_baseline"] = (cpu_baseline(args.workload, args.moe_config)
                                if world == 1 and not args.no_cpu_baseline else None)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
