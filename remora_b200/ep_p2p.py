"""Expert-parallel MoE layer with the token exchange done by the library's
own kernels over NVLink peer memory (no NCCL in the layer, no host round
trip for split sizes).

Buffers every rank can address come from torch symmetric memory, allocated
once per ``PeerEP`` (sized for the worst case: one rank may route all of
its T_local*k rows to one peer).  One layer on rank r (``fused=True``, the
default):

  router + top-k, dispatch over all E experts              (kernels)
  meta: counts -> every peer, barrier, segment table        (kernel, bounded)
  experts: one cooperative kernel; its copy warps put row p into region r
  of rank (expert // Epr)'s recv and raise that rank's ready flag of the
  expert when its rows are stored, while its tcgen05 pipeline runs SwiGLU
  tiles over the received segments (sources in arrival order, each
  segment waiting, bounded, for its flag) and down tiles whose epilogues
  store each output row into its source rank's y            (kernel, NVLink)
  barrier                                                   (kernel, bounded)
  combine of y in slot order                                (kernel)

``fused=False`` runs the exchange and the GEMMs one after the other
(scatter, barrier, segments, SwiGLU GEMM, down GEMM).  The barriers also
order consecutive layers: a rank writes a peer's recv / meta / y only after
every rank has finished reading them.  Results are bit-identical to the
single-GPU layer (each row's expert output depends only on that row and its
expert's weights).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerEP:
    def __init__(self, T_local: int, D: int, F: int, E: int, k: int, group=None, device=None,
                 fused: bool = True):
        import torch.distributed._symmetric_memory as symm_mem

        import remora_b200 as rb

        self.rb = rb
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.P or self.P > 8:
            raise ValueError(f"{E} experts over {self.P} ranks (at most 8) do not split")
        self.T, self.D, self.F, self.E, self.k = T_local, D, F, E, k
        self.Epr = E // self.P
        self.cap = T_local * k
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        P, cap = self.P, self.cap
        self.fused = fused
        self.off_flags = 0
        self.off_ready = _align(P * 4)
        self.off_meta = self.off_ready + _align(E * 4)
        self.off_recv = self.off_meta + _align(P * (self.Epr + 1) * 4)
        self.off_y = self.off_recv + _align(P * cap * D * 2)
        total = self.off_y + _align(cap * D * 2)
        self.buf = symm_mem.empty(total, dtype=torch.uint8, device=self.device)
        self.buf.zero_()
        torch.cuda.synchronize(self.device)
        gname = group.group_name if group is not None else dist.group.WORLD.group_name
        if hasattr(symm_mem, "enable_symm_mem_for_group"):
            try:
                symm_mem.enable_symm_mem_for_group(gname)
            except Exception:
                pass
        self.hdl = symm_mem.rendezvous(self.buf, gname)
        base = list(self.hdl.buffer_ptrs)
        arr = lambda off: (ctypes.c_uint64 * P)(*[b + off for b in base])
        self.flag_ptrs, self.meta_ptrs = arr(self.off_flags), arr(self.off_meta)
        self.ready_ptrs = arr(self.off_ready)
        self.recv_ptrs, self.y_ptrs = arr(self.off_recv), arr(self.off_y)
        view = lambda off, n, dt: self.buf[off:off + n * torch.tensor([], dtype=dt).element_size()].view(dt)
        self.flags = view(self.off_flags, P, torch.int32)
        self.ready = view(self.off_ready, E, torch.int32)
        self.done = torch.zeros(E, dtype=torch.int32, device=self.device)
        self.mt_done = torch.zeros(P * self.cap // 128 + E + 1, dtype=torch.int32,
                                   device=self.device)
        self.meta = view(self.off_meta, P * (self.Epr + 1), torch.int32)
        self.recv = view(self.off_recv, P * cap * D, torch.bfloat16).view(P * cap, D)
        self.y = view(self.off_y, cap * D, torch.bfloat16).view(cap, D)
        self.h = torch.empty(P * cap, F, dtype=torch.bfloat16, device=self.device)
        self.seg = torch.empty(5 * P * self.Epr, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.layer = 0
        self.profile = False   # when True, forward() records per-phase CUDA events
        self.phase_ms = {}
        dist.barrier(group)

    def _barrier(self, stream):
        self.epoch += 1
        self.rb._check(self.rb.lib().remora_b200_moe_ep_barrier(
            self.flags.data_ptr(), self.flag_ptrs, self.P, self.rank, self.epoch, stream))

    def forward(self, x, wr, wg_local, wu_local, wd_local, out=None):
        """x [T_local, D]; wr [D, E]; this rank's experts wg/wu [Epr, D, F],
        wd [Epr, F, D].  Returns out [T_local, D] bf16 (written into `out`
        when given)."""
        rb, L = self.rb, self.rb.lib()
        if x.shape != (self.T, self.D) or wg_local.shape[0] != self.Epr:
            raise ValueError("shapes differ from the ones this PeerEP was built for")
        cs = torch.cuda.current_stream(self.device)
        stream = cs.cuda_stream
        marks = []

        def mark(name):
            if self.profile:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(cs)
                marks.append((name, ev))

        mark("start")
        idx, w = rb.moe_router_topk(x, wr, self.k)
        counts, offsets, perm, inv = rb.moe_dispatch(idx, self.E)
        mark("route+dispatch")
        if self.fused:
            return self._forward_fused(x, w, offsets, perm, inv, wg_local, wu_local, wd_local,
                                       cs, mark, marks, out)
        rb._check(L.remora_b200_moe_ep_scatter_bf16(
            x.data_ptr(), perm.data_ptr(), offsets.data_ptr(), self.cap, self.k, self.D, self.E,
            self.P, self.rank, self.cap, self.recv_ptrs, self.meta_ptrs, stream))
        mark("scatter")
        self._barrier(stream)
        mark("barrier1")
        rb._check(L.remora_b200_moe_ep_segments(self.meta.data_ptr(), self.P, self.Epr, self.cap,
                                                self.seg.data_ptr(), stream))
        rb._check(L.remora_b200_moe_ep_experts_bf16(
            self.recv.data_ptr(), wg_local.contiguous().data_ptr(),
            wu_local.contiguous().data_ptr(), wd_local.contiguous().data_ptr(),
            self.h.data_ptr(), self.seg.data_ptr(), self.P, self.Epr, self.cap, self.D, self.F,
            self.y_ptrs, stream))
        mark("experts")
        self._barrier(stream)
        mark("barrier2")
        out = rb.moe_combine(self.y, inv, w, out=out)
        mark("combine")
        if self.profile:
            marks[-1][1].synchronize()
            self.phase_ms = {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(marks, marks[1:])}
        return out

    def _forward_fused(self, x, w, offsets, perm, inv, wg_local, wu_local, wd_local, cs, mark,
                       marks, out):
        rb, L = self.rb, self.rb.lib()
        stream = cs.cuda_stream
        self.epoch += 1
        rb._check(L.remora_b200_moe_ep_meta(
            offsets.data_ptr(), self.P, self.E, self.rank, self.cap, self.meta_ptrs,
            self.meta.data_ptr(), self.flags.data_ptr(), self.flag_ptrs, self.epoch,
            self.done.data_ptr(), self.seg.data_ptr(), stream))
        mark("meta")
        self.layer += 1
        rb._check(L.remora_b200_moe_ep_experts_fused_bf16(
            x.data_ptr(), perm.data_ptr(), offsets.data_ptr(), self.cap, self.k, self.D,
            self.F, self.E, self.P, self.rank, self.cap, self.recv_ptrs, self.ready_ptrs,
            self.ready.data_ptr(), self.done.data_ptr(), self.layer, self.recv.data_ptr(),
            wg_local.contiguous().data_ptr(), wu_local.contiguous().data_ptr(),
            wd_local.contiguous().data_ptr(), self.h.data_ptr(), self.seg.data_ptr(),
            self.mt_done.data_ptr(), self.y_ptrs, stream))
        mark("experts")
        self._barrier(stream)
        mark("barrier2")
        out = rb.moe_combine(self.y, inv, w, out=out)
        mark("combine")
        if self.profile:
            marks[-1][1].synchronize()
            self.phase_ms = {b[0]: a[1].elapsed_time(b[1]) for a, b in zip(marks, marks[1:])}
        return out


def _self_check(T=8192, D=2048, F=1536, E=8, k=8):
    """One-rank run of the peer-memory layer (every row copied into the
    rank's own region): four layers, a bit-for-bit comparison with the
    single-GPU layer, then one layer with per-phase CUDA-event times.
    ``python -m remora_b200.ep_p2p`` on one GPU."""
    import datetime
    import os

    import remora_b200 as rb

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    ws = [torch.empty(s, dtype=torch.bfloat16, device=dev) for s in ((E, D, F), (E, D, F), (E, F, D))]
    rb.fill_normal(x, rb.stream_key(30))
    rb.fill_normal(wr, rb.stream_key(31), 0.0, 0.02)
    for i, w in enumerate(ws):
        rb.fill_normal(w, rb.stream_key(32 + i), 0.0, 0.02)
    ep = PeerEP(T, D, F, E, k, device=dev)
    ref = rb.moe_layer(x, wr, *ws, k)
    for _ in range(4):
        out = ep.forward(x, wr, *ws)
    rb.synchronize_and_check(dev)
    same = bool(torch.equal(out.view(torch.int16), ref.view(torch.int16)))
    print("same as single-GPU layer:", same)
    ep.profile = True
    ep.forward(x, wr, *ws)
    print({name: round(ms, 3) for name, ms in ep.phase_ms.items()})
    dist.barrier()
    dist.destroy_process_group()
    if not same:
        raise SystemExit(1)


if __name__ == "__main__":
    _self_check()
