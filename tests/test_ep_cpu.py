"""Expert-parallel MoE exchange on CPU ranks (gloo, world size 2).

The local compute is the oracle's (no GPU); what is tested is the
bookkeeping of remora_b200.ep: counts exchange, row splits, the
(source rank, local expert) segments and the reverse exchange.  The
2-rank result must equal the single-process oracle layer bit for bit.
A second test kills one rank before the exchange: the other must get an
error from the process group within its timeout, not hang."""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

T, D, F, E, K = 96, 32, 64, 4, 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _np16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _t16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


class OracleOps:
    """CPU restatements standing in for the CUDA kernels."""

    def __init__(self, orc):
        self.o = orc

    def router(self, x, wr, k):
        idx, w = self.o.router_topk(_np16(x), _np16(wr), k)
        return torch.from_numpy(idx), torch.from_numpy(w)

    def dispatch(self, idx, E):
        return tuple(torch.from_numpy(a) for a in self.o.dispatch(idx.numpy(), E))

    def gather(self, x, perm, k):
        return x[perm.long() // k].contiguous()

    def experts(self, xr, wg, wu, wd, seg_offsets, seg_expert):
        xs = _np16(xr)
        y = np.zeros((xs.shape[0], wd.shape[2]), np.uint16)
        offs, ex = seg_offsets.numpy(), seg_expert.numpy()
        for q in range(ex.shape[0]):
            a, b = offs[q], offs[q + 1]
            if a < b:
                e = ex[q]
                _, yy, _ = self.o.expert_ffn(xs[a:b], _np16(wg[e]), _np16(wu[e]), _np16(wd[e]))
                y[a:b] = yy
        return _t16(y)

    def combine(self, y, inv, w):
        return _t16(self.o.combine(_np16(y), inv.numpy(), w.numpy()))


def _inputs(orc):
    x = orc.to_bf16(orc.normal("moe_x", (T, D)))
    wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.3))
    wg = orc.to_bf16(orc.normal("moe_wg", (E, D, F), sigma=0.1))
    wu = orc.to_bf16(orc.normal("moe_wu", (E, D, F), sigma=0.1))
    wd = orc.to_bf16(orc.normal("moe_wd", (E, F, D), sigma=0.1))
    return x, wr, wg, wu, wd


def _worker(rank, world, port, mode, outdir):
    sys.path.insert(0, ROOT)
    import oracle as orc
    from remora_b200.ep import moe_ep_forward

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=15))
    x, wr, wg, wu, wd = _inputs(orc)
    Epr = E // world
    tl = T // world
    if mode == "die" and rank == 1:
        os._exit(3)  # leaves between steps, before any collective of the layer
    status = "ok"
    try:
        out = moe_ep_forward(_t16(x[rank * tl:(rank + 1) * tl]), _t16(wr),
                             _t16(wg[rank * Epr:(rank + 1) * Epr]),
                             _t16(wu[rank * Epr:(rank + 1) * Epr]),
                             _t16(wd[rank * Epr:(rank + 1) * Epr]), K, E, ops=OracleOps(orc))
        np.save(os.path.join(outdir, f"out{rank}.npy"), _np16(out))
    except Exception as e:  # the failure mode under test
        status = "error: " + type(e).__name__
    with open(os.path.join(outdir, f"status{rank}.txt"), "w") as f:
        f.write(status)
    if mode != "die":
        dist.destroy_process_group()


def _run(mode, tmp_path, world=2):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
            pytest.fail("a rank did not finish within 90 s")
    return procs


def test_ep_two_ranks_match_single_process_oracle(tmp_path, orc):
    procs = _run("ok", tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    x, wr, wg, wu, wd = _inputs(orc)
    *_, ref = orc.moe_layer_bf16(x, wr, wg, wu, wd, K)
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(2)])
    assert np.array_equal(got, ref)


def test_ep_rank_loss_raises_not_hangs(tmp_path):
    procs = _run("die", tmp_path)
    assert procs[1].exitcode == 3
    status = (tmp_path / "status0.txt").read_text()
    assert status.startswith("error"), status
