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


def _capi_worker(rank, world, port, outdir):
    """The exchange bookkeeping of remora_b200_moe_ep_nccl_bf16 on CPU ranks:
    the split sizes come from the library's host function
    remora_b200_moe_ep_splits (no GPU involved), the segments follow the
    device kernel's rule (sources in rank order, local experts in order),
    the rows travel by gloo all-gathers and the local compute is the
    oracle's."""
    sys.path.insert(0, ROOT)
    import ctypes

    import oracle as orc
    import remora_b200 as rb

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    x, wr, wg, wu, wd = _inputs(orc)
    Epr, tl = E // world, T // world
    xl = x[rank * tl:(rank + 1) * tl]
    idx, w = orc.router_topk(xl, wr, K)
    counts, offsets, perm, inv = orc.dispatch(idx, E)
    xs = xl[perm // K]
    allc = [torch.empty(E, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(allc, torch.from_numpy(counts))
    recv_counts = np.stack([c.numpy()[rank * Epr:(rank + 1) * Epr] for c in allc]).astype(np.int32)
    so, sr, ro, rr = (np.zeros(world, np.int64) for _ in range(4))
    p64 = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = rb.lib().remora_b200_moe_ep_splits(p64(offsets), p64(np.ascontiguousarray(recv_counts)),
                                            world, E, p64(so), p64(sr), p64(ro), p64(rr))
    assert rc == 0, rb.last_error()
    sent = [None] * world
    dist.all_gather_object(sent, (xs, so, sr))
    xr = np.concatenate([sx[sso[rank]:sso[rank] + ssr[rank]] for sx, sso, ssr in sent])
    assert [ssr[rank] for _, _, ssr in sent] == list(rr) and xr.shape[0] == rr.sum()
    # segments as k_nccl_segments builds them
    flat = recv_counts.reshape(-1)
    seg_off = np.concatenate([[0], np.cumsum(flat)])
    yr = np.zeros((xr.shape[0], D), np.uint16)
    for q in range(flat.shape[0]):
        a, b, e = seg_off[q], seg_off[q + 1], rank * Epr + q % Epr
        if a < b:
            _, yy, _ = orc.expert_ffn(xr[a:b], wg[e], wu[e], wd[e])
            yr[a:b] = yy
    back = [None] * world
    dist.all_gather_object(back, (yr, ro, rr))
    y = np.zeros_like(xs)
    for q, (qy, qro, qrr) in enumerate(back):
        assert qrr[rank] == sr[q]
        y[so[q]:so[q] + sr[q]] = qy[qro[rank]:qro[rank] + qrr[rank]]
    np.save(os.path.join(outdir, f"out{rank}.npy"), orc.combine(y, inv, w))
    dist.destroy_process_group()


def test_ep_capi_splits_two_ranks_match_single_process_oracle(tmp_path, orc):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_capi_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert not any(p.is_alive() for p in procs), "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs)
    x, wr, wg, wu, wd = _inputs(orc)
    *_, ref = orc.moe_layer_bf16(x, wr, wg, wu, wd, K)
    got = np.concatenate([np.load(tmp_path / f"out{r}.npy") for r in range(2)])
    assert np.array_equal(got, ref)


def test_ep_splits_rejects_bad_input():
    import ctypes

    import remora_b200 as rb

    off = np.array([0, 5, 9, 7, 7], np.int32)  # decreases between the two ranks' blocks
    rc_ = np.zeros(4, np.int32)
    out = [np.zeros(2, np.int64) for _ in range(4)]
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = rb.lib().remora_b200_moe_ep_splits(p(off), p(rc_), 2, 4, *(p(o) for o in out))
    assert rc == rb.ERR_INVALID
    rc = rb.lib().remora_b200_moe_ep_splits(p(off), p(rc_), 3, 4, *(p(o) for o in out))
    assert rc == rb.ERR_INVALID  # 4 experts do not split over 3 ranks
