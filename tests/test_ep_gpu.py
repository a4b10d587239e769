"""Expert-parallel MoE on 2+ GPUs (NCCL all-to-all, and the peer-memory
paths with the scatter fused into the SwiGLU GEMM or run as its own
kernel): the EP layer must equal the single-GPU layer bit for bit (each
row's expert output depends only on the row and its expert).  The
peer-memory paths run three consecutive layers on two different inputs,
so rows left over from the previous layer cannot pass for this layer's.
Skipped when fewer than 2 GPUs are visible."""
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
    else:
        from remora_b200.ep_p2p import PeerEP

        ep = PeerEP(tl, D, F, E, k, fused=mode == "p2p")
        outs = [ep.forward(xi, wr, *wl).clone() for xi in (xl, x2l, xl)]  # consecutive layers
        refs = [ref, ref2, ref]
    rb.synchronize_and_check(dev)
    for out, r in zip(outs, refs):
        same = same and torch.equal(out.view(torch.int16), r.view(torch.int16))
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write("same" if same else "differ")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "p2p", "p2p-split"])
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
        p.join(240)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
        p.join()
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs)
    for r in range(world):
        assert (tmp_path / f"r{r}.txt").read_text() == "same", f"rank {r}"
