"""Expert-parallel MoE layer with the token exchange done by the library's
own kernels over NVLink peer memory (no NCCL in the layer, no host round
trip for split sizes).

Buffers every rank can address are plain ``cudaMalloc`` memory shared
through CUDA IPC (``remora_b200_peer_alloc`` / ``remora_b200_peer_open``,
handles exchanged over the process group), allocated once per ``PeerEP``
and sized for the worst case: one rank may route all of its T_local*k rows
to one peer.  No NVLink multicast object is created or bound, so a rank
that exits leaves its peers nothing worse than an unmapped range.  One
layer on rank r (``fused=True``, the default):

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


class _DeviceRange:
    """A raw device range as a torch tensor view (``__cuda_array_interface__``);
    the memory stays owned by the PeerEP that allocated it."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerEP:
    def __init__(self, T_local: int, D: int, F: int, E: int, k: int, group=None, device=None,
                 fused: bool = True):
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
        L = rb.lib()
        with torch.cuda.device(self.device):
            own = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(64)
            rb._check(L.remora_b200_peer_alloc(total, ctypes.byref(own), handle))  # zeroed
            self._own = own.value
            self._opened = []
            handles = [None] * self.P
            dist.all_gather_object(handles, handle.raw, group=group)
            base = []
            for r, hraw in enumerate(handles):
                if r == self.rank:
                    base.append(self._own)
                    continue
                p = ctypes.c_void_p()
                rb._check(L.remora_b200_peer_open(ctypes.create_string_buffer(hraw, 64),
                                                  ctypes.byref(p)))
                self._opened.append(p.value)
                base.append(p.value)
        self.buf = torch.as_tensor(_DeviceRange(self._own, total), device=self.device)
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

    def close(self):
        """Releases the peer buffers: every rank finishes its work, unmaps its
        peers' buffers, and only then frees its own (two barriers)."""
        if self._own is None:
            return
        L = self.rb.lib()
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self.rb._check(L.remora_b200_peer_close(p))
        self._opened = []
        dist.barrier(self.group)
        self.flags = self.ready = self.meta = self.recv = self.y = self.buf = None
        with torch.cuda.device(self.device):
            self.rb._check(L.remora_b200_peer_free(self._own))
        self._own = None

    @property
    def dominant_kernel(self) -> str:
        return ("rb::moe::k_ep_experts (row copy + SwiGLU + down, cooperative)" if self.fused
                else "rb::moe::k_grouped_gemm (SwiGLU + down over received segments)")

    @property
    def launches_per_layer(self) -> int:
        """The library's kernels in one forward(): router 1, dispatch 3, then
        meta, experts, barrier, combine (fused) or scatter, barrier,
        segments, SwiGLU, down, barrier, combine (split)."""
        return 8 if self.fused else 11

    def rows_received(self) -> int:
        """Rows this rank's experts processed in the last layer (synchronises)."""
        torch.cuda.synchronize(self.device)
        m = self.meta.view(self.P, self.Epr + 1)[:, :self.Epr]
        return int(m.sum().item())

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


def _self_check(T=8192, D=2048, F=1536, E=8, k=8, port=29533):
    """One-rank run of the peer-memory layer (every row goes to the rank's
    own region): for the fused and the split form, three consecutive layers
    on two different inputs, each compared bit for bit with the single-GPU
    layer, then one layer with per-phase CUDA-event times.  The default
    shape is one rank's share of the 65536-token, 64-expert configuration
    on 8 GPUs (8192 tokens, 8 experts).  ``python -m remora_b200.ep_p2p`` on
    one GPU; exits 1 on a mismatch."""
    import datetime
    import os

    import remora_b200 as rb

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(port))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    dist.init_process_group("gloo", rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60))
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    x2 = torch.empty_like(x)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    ws = [torch.empty(s, dtype=torch.bfloat16, device=dev) for s in ((E, D, F), (E, D, F), (E, F, D))]
    rb.fill_normal(x, rb.stream_key(30))
    rb.fill_normal(x2, rb.stream_key(35))
    rb.fill_normal(wr, rb.stream_key(31), 0.0, 0.02)
    for i, w in enumerate(ws):
        rb.fill_normal(w, rb.stream_key(32 + i), 0.0, 0.02)
    refs = [rb.moe_layer(xi, wr, *ws, k) for xi in (x, x2)]
    ok = True
    for fused in (True, False):
        ep = PeerEP(T, D, F, E, k, device=dev, fused=fused)
        outs = [ep.forward(xi, wr, *ws).clone() for xi in (x, x2, x)]
        rb.synchronize_and_check(dev)
        same = all(torch.equal(o.view(torch.int16), r.view(torch.int16))
                   for o, r in zip(outs, (refs[0], refs[1], refs[0])))
        ep.profile = True
        ep.forward(x, wr, *ws)
        print(f"{'fused' if fused else 'split'}: same as single-GPU layer: {same};",
              {name: round(ms, 3) for name, ms in ep.phase_ms.items()}, flush=True)
        ep.close()
        ok = ok and same
    dist.destroy_process_group()
    if not ok:
        raise SystemExit(1)


if __name__ == "__main__":
    import sys

    _self_check(port=int(sys.argv[1]) if len(sys.argv) > 1 else 29533)
