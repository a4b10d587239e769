"""Expert-parallel MoE on 2+ GPUs (NCCL all-to-all, and the peer-memory
paths with the scatter fused into the SwiGLU GEMM or run as its own
kernel): the EP layer must equal the single-GPU layer bit for bit (each
row's expert output depends only on the row and its expert).  The
peer-memory paths run three consecutive layers on two different inputs,
so rows left over from the previous layer cannot pass for this layer's.
Skipped when fewer than 2 GPUs are visible.

No rank is ever killed: every device wait in the layer is bounded (2 s, then
an error status), and the process group's 60 s timeout ends a collective
whose peer is gone, so each rank leaves by itself between layers.  NVLS
(NVLink SHARP, which binds multicast memory) is off in NCCL, and the
peer-memory buffers are plain cudaMalloc memory shared through CUDA IPC."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, cfg, outdir, mode="nccl"):
    sys.path.insert(0, ROOT)
    import remora_b200 as rb
    from remora_b200.ep import moe_ep_forward

    T, D, F, E, k = cfg
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    # every rank builds the same full tensors from the seeded generator
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    wg = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wu = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wd = torch.empty(E, F, D, dtype=torch.bfloat16, device=dev)
    for t, s, sig in ((x, 30, 1.0), (wr, 31, 0.02), (wg, 32, 0.02), (wu, 33, 0.02),
                      (wd, 34, 0.02)):
        rb.fill_normal(t, rb.stream_key(s), 0.0, sig)
    x2 = torch.empty_like(x)
    rb.fill_normal(x2, rb.stream_key(35), 0.0, 1.0)
    tl, Epr = T // world, E // world
    sl = slice(rank * tl, (rank + 1) * tl)
    xl, x2l = x[sl].contiguous(), x2[sl].contiguous()
    wl = [w_[rank * Epr:(rank + 1) * Epr].contiguous() for w_ in (wg, wu, wd)]
    ref = rb.moe_layer(x, wr, wg, wu, wd, k)[sl]
    ref2 = rb.moe_layer(x2, wr, wg, wu, wd, k)[sl]
    same = True
    if mode == "nccl":
        outs = [moe_ep_forward(xl, wr, *wl, k, E)]
        refs = [ref]
    elif mode == "nccl-capi":
        from remora_b200.ep_nccl import NcclEP

        ep = NcclEP(tl, D, F, E, k, blocking=False)
        outs = [ep.forward(xi, wr, *wl).clone() for xi in (xl, x2l, xl)]
        refs = [ref, ref2, ref]
    else:
        from remora_b200.ep_p2p import PeerEP

        ep = PeerEP(tl, D, F, E, k, fused=mode == "p2p")
        outs = [ep.forward(xi, wr, *wl).clone() for xi in (xl, x2l, xl)]  # consecutive layers
        refs = [ref, ref2, ref]
    rb.synchronize_and_check(dev)
    for out, r in zip(outs, refs):
        same = same and torch.equal(out.view(torch.int16), r.view(torch.int16))
    if mode != "nccl":
        ep.close()
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write("same" if same else "differ")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "nccl-capi", "p2p", "p2p-split"])
@pytest.mark.parametrize("cfg", [(4096, 512, 256, 16, 4), (8192, 2048, 1536, 64, 8)])
def test_ep_matches_single_gpu_layer(rb, tmp_path, cfg, mode):
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    while cfg[3] % world or cfg[0] % world:
        world //= 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, str(tmp_path), mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(600)  # bounded device waits and the process-group timeout end a stuck rank
    assert not any(p.is_alive() for p in procs), "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        assert (tmp_path / f"r{r}.txt").read_text() == "same", f"rank {r}"


def test_peer_ep_one_rank_matches_single_gpu_layer(rb):
    """The peer-memory layer (fused cooperative expert kernel, and the split
    form) on ONE GPU, where every routed row goes to the rank's own region:
    three consecutive layers bit-identical to the single-GPU layer.  Runs in
    a child process (its own process group); it finishes by itself."""
    import subprocess

    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get(
        "CUDA_VISIBLE_DEVICES", "0").split(",")[0])
    r = subprocess.run([sys.executable, "-m", "remora_b200.ep_p2p", str(_free_port())], cwd=ROOT,
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.count("same as single-GPU layer: True") == 2, r.stdout


def _timeout_worker(rank, world, port, outdir):
    """Rank 1 never enters the layer; rank 0's bounded host wait must end the
    call with REMORA_B200_ERR_TIMEOUT (communicator aborted) instead of
    hanging.  Rank 1 leaves between steps: it has nothing in flight."""
    sys.path.insert(0, ROOT)
    import remora_b200 as rb
    from remora_b200.ep_nccl import NcclEP

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    T, D, F, E, k = 1024, 256, 256, 8, 2
    ep = NcclEP(T, D, F, E, k, blocking=False, timeout_ms=3000, device=dev)
    x = torch.zeros(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.zeros(D, E, dtype=torch.bfloat16, device=dev)
    wl = [torch.zeros(s, dtype=torch.bfloat16, device=dev)
          for s in ((E // world, D, F), (E // world, D, F), (E // world, F, D))]
    status = "not run"
    if rank == 0:
        try:
            ep.forward(x, wr, *wl)
            status = "returned"
        except rb.RemoraError as e:
            status = f"code {e.code}"
    dist.barrier()  # rank 1 waits here on the host, with nothing on its GPU
    if ep.comm:  # rank 0's was aborted by the failed call
        rb.lib().remora_b200_nccl_comm_abort(ep.comm)
    torch.cuda.synchronize(dev)
    with open(os.path.join(outdir, f"t{rank}.txt"), "w") as f:
        f.write(status)
    dist.destroy_process_group()


def test_ep_nccl_missing_rank_times_out(rb, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 or more GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    assert not any(p.is_alive() for p in procs), "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert (tmp_path / "t0.txt").read_text() == f"code {rb.ERR_TIMEOUT}"
