"""Expert-parallel MoE layer through the library's NCCL entry point,
``remora_b200_moe_ep_nccl_bf16`` (one process per GPU).

The layer runs entirely inside the C ABI on a communicator the library
creates with ``remora_b200_nccl_comm_init`` (rank 0's unique id is shared
over the torch process group); torch only supplies device memory, the
stream and the id exchange.  A C or C++ caller (remora's ``launchOnGpu``,
compiler/gpu_tests.cpp:101-125) makes the same calls with its own
communicator.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


class NcclEP:
    def __init__(self, T_local: int, D: int, F: int, E: int, k: int, group=None, device=None,
                 blocking: bool = False, timeout_ms: int = 60000):
        import remora_b200 as rb

        self.rb = rb
        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if E % self.P:
            raise ValueError(f"{E} experts do not split over {self.P} ranks")
        self.T, self.D, self.F, self.E, self.k = T_local, D, F, E, k
        self.Epr = E // self.P
        self.timeout_ms = timeout_ms
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        L = rb.lib()
        uid = ctypes.create_string_buffer(128)
        if self.rank == 0:
            rb._check(L.remora_b200_nccl_unique_id(uid))
        box = [uid.raw]
        dist.broadcast_object_list(box, src=0, group=group)
        self.comm = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            rb._check(L.remora_b200_nccl_comm_init(
                ctypes.byref(self.comm), self.P, ctypes.create_string_buffer(box[0], 128),
                self.rank, int(blocking), timeout_ms))
        nws = L.remora_b200_moe_ep_nccl_workspace_bytes(T_local, D, F, E, k, self.P)
        if nws == 0:
            raise ValueError("moe_ep_nccl: sizes rejected")
        self.ws = torch.empty(nws, dtype=torch.uint8, device=self.device)
        self.profile = False
        self.phase_ms = {}

    # the layer is timed as one call (its NCCL exchange and the grouped GEMMs)
    dominant_kernel = "whole layer (remora_b200_moe_ep_nccl_bf16 call)"
    # router 1, dispatch 3, gather, segments, SwiGLU, down, combine (+ NCCL's own kernels)
    launches_per_layer = 9

    def forward(self, x, wr, wg_local, wu_local, wd_local, out=None):
        """x [T_local, D]; wr [D, E]; this rank's experts wg/wu [E/P, D, F],
        wd [E/P, F, D].  Returns out [T_local, D] bf16."""
        rb = self.rb
        if x.shape != (self.T, self.D) or wg_local.shape[0] != self.Epr:
            raise ValueError("shapes differ from the ones this NcclEP was built for")
        out = torch.empty_like(x) if out is None else out
        cs = torch.cuda.current_stream(self.device)
        if self.profile:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
            ev[0].record(cs)
        if not self.comm:
            raise RuntimeError("the communicator was aborted by an earlier failure")
        rc = rb.lib().remora_b200_moe_ep_nccl_bf16(
            x.data_ptr(), wr.contiguous().data_ptr(), wg_local.contiguous().data_ptr(),
            wu_local.contiguous().data_ptr(), wd_local.contiguous().data_ptr(), out.data_ptr(),
            self.T, self.D, self.F, self.E, self.k, self.comm, self.timeout_ms,
            self.ws.data_ptr(), self.ws.numel(), cs.cuda_stream)
        if rc in (rb.ERR_NCCL, rb.ERR_TIMEOUT):
            self.comm = ctypes.c_void_p()  # the library aborted (and freed) it
        rb._check(rc)
        if self.profile:
            ev[1].record(cs)
            ev[1].synchronize()
            self.phase_ms = {"experts": ev[0].elapsed_time(ev[1])}
        return out

    def rows_received(self) -> int:
        # every row is processed once; on average a rank receives T*k rows
        return self.T * self.k

    def close(self):
        if self.comm:
            torch.cuda.synchronize(self.device)
            with torch.cuda.device(self.device):
                self.rb._check(self.rb.lib().remora_b200_nccl_comm_destroy(self.comm,
                                                                           self.timeout_ms))
            self.comm = ctypes.c_void_p()
