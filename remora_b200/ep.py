"""Expert-parallel MoE layer over torch.distributed (NCCL on B200, one
process per GPU).

Tokens are sharded across ranks (T/P per rank) and experts too (E/P per
rank, expert e on rank e // (E/P)).  One layer on rank r:

  1. router + top-k on the local tokens              (remora_b200 kernel)
  2. dispatch by global expert id, gather the rows    (kernels): the rows
     for rank q are then one contiguous block, ordered by q's local experts
  3. all-to-all of the per-expert row counts          (collective)
  4. all-to-all-v of the rows                         (collective)
  5. the SwiGLU and down expert GEMMs over the received rows, grouped by
     (source rank, local expert) segments             (kernels)
  6. all-to-all-v of the expert outputs back          (collective)
  7. weighted combine in slot order                   (kernel)

Every row's expert output depends only on that row and its expert's
weights, so the result is bit-identical to the single-GPU layer
(mixtral_moe_layer.mlir:8-68 semantics, remora_b200_moe_layer_bf16).

The local compute goes through an ``ops`` object (``GpuOps`` here: the
CUDA library; tests substitute CPU restatements to check the exchange
bookkeeping on gloo ranks).  The row counts are read on the host once per
layer: NCCL's all-to-all-v takes host split sizes.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GpuOps:
    """Local compute through libremora_b200."""

    def __init__(self):
        import remora_b200 as rb

        self.rb = rb

    def router(self, x, wr, k):
        return self.rb.moe_router_topk(x, wr, k)

    def dispatch(self, idx, E):
        return self.rb.moe_dispatch(idx, E)

    def gather(self, x, perm, k):
        return self.rb.moe_gather(x, perm, k)

    def experts(self, xr, wg, wu, wd, seg_offsets, seg_expert):
        h = self.rb.grouped_gemm_swiglu_segments(xr, wg, wu, seg_offsets, seg_expert)
        return self.rb.grouped_gemm_segments(h, wd, seg_offsets, seg_expert)

    def combine(self, y, inv, w):
        return self.rb.moe_combine(y, inv, w)


def segments(recv_counts: torch.Tensor, P: int, Epr: int):
    """Row segments of the received block: (source rank, local expert) in
    that order; returns (seg_offsets [P*Epr+1], seg_expert [P*Epr])."""
    c = recv_counts.view(P * Epr).to(torch.int64)
    offs = torch.zeros(P * Epr + 1, dtype=torch.int64, device=c.device)
    offs[1:] = torch.cumsum(c, 0)
    exp = torch.arange(Epr, dtype=torch.int32, device=c.device).repeat(P)
    return offs.to(torch.int32), exp


def moe_ep_forward(x, wr, wg_local, wu_local, wd_local, k: int, E: int, group=None, ops=None,
                   chunks: int | None = None):
    """One expert-parallel MoE layer on this rank.

    x [T_local, D] (this rank's tokens), wr [D, E] (replicated),
    wg_local / wu_local [E/P, D, F], wd_local [E/P, F, D] (this rank's
    experts).  Returns out [T_local, D] bf16.

    With ``chunks`` > 1 the local tokens are processed in pieces: all
    pieces' counts travel in one all-to-all (one host read), then piece
    c+1's rows are exchanged while piece c's expert GEMMs run, and piece c's
    outputs travel back while piece c+1 computes.  Measured on 8 B200s
    (config 5) one piece is faster: NCCL's kernels and the persistent expert
    GEMM then compete for SMs, so the default is 1.
    """
    ops = ops or GpuOps()
    P = dist.get_world_size(group)
    if E % P:
        raise ValueError(f"{E} experts do not split over {P} ranks")
    Epr = E // P
    if wg_local.shape[0] != Epr:
        raise ValueError(f"rank holds {wg_local.shape[0]} experts, expected {Epr}")
    T, D = x.shape
    C = chunks or 1
    C = max(1, min(C, T)) if T else 1
    pieces = torch.tensor_split(torch.arange(T), C) if T else [torch.arange(0)]

    # 1-2. local routing, dispatch by global expert, gather, per piece
    loc = []
    for pc in pieces:
        xt = x[int(pc[0]):int(pc[-1]) + 1] if pc.numel() else x[:0]
        idx, w = ops.router(xt, wr, k)
        counts, offsets, perm, inv = ops.dispatch(idx, E)
        loc.append((ops.gather(xt, perm, k), counts, inv, w))

    # 3. every piece's counts in one all-to-all: send [P][C][Epr], recv [P(src)][C][Epr]
    send_c = torch.stack([l[1] for l in loc]).view(C, P, Epr).transpose(0, 1).contiguous()
    recv_c = torch.empty_like(send_c)
    dist.all_to_all_single(recv_c, send_c, group=group)
    send_rows = send_c.sum(2).t().tolist()        # [C][P]: rows this rank sends
    recv_rows = recv_c.sum(2).t().tolist()        # [C][P]: rows this rank receives

    def rows_exchange(c):
        xs = loc[c][0]
        xr = torch.empty((sum(recv_rows[c]), D), dtype=xs.dtype, device=xs.device)
        work = dist.all_to_all_single(xr, xs, output_split_sizes=recv_rows[c],
                                      input_split_sizes=send_rows[c], group=group, async_op=True)
        return xr, work

    # 4-6. pipeline: rows of c+1 in flight while the experts of c run
    pending = rows_exchange(0)
    backs = []
    for c in range(C):
        xr, work = pending
        work.wait()
        if c + 1 < C:
            pending = rows_exchange(c + 1)
        seg_offsets, seg_expert = segments(recv_c[:, c, :].contiguous(), P, Epr)
        if xr.shape[0]:
            yr = ops.experts(xr, wg_local, wu_local, wd_local, seg_offsets, seg_expert)
        else:
            yr = torch.empty((0, D), dtype=xr.dtype, device=xr.device)
        y = torch.empty_like(loc[c][0])
        wb = dist.all_to_all_single(y, yr, output_split_sizes=send_rows[c],
                                    input_split_sizes=recv_rows[c], group=group, async_op=True)
        backs.append((y, wb, yr))

    # 7. combine each piece in slot order
    outs = []
    for c in range(C):
        y, wb, _ = backs[c]
        wb.wait()
        outs.append(ops.combine(y, loc[c][2], loc[c][3]))
    return torch.cat(outs) if C > 1 else outs[0]
