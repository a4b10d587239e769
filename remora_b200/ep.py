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
bookkeeping on gloo ranks).  The row counts are read on the host: NCCL's
all-to-all-v takes host split sizes, so a layer has two small
device-to-host reads.
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


def moe_ep_forward(x, wr, wg_local, wu_local, wd_local, k: int, E: int, group=None, ops=None):
    """One expert-parallel MoE layer on this rank.

    x [T_local, D] (this rank's tokens), wr [D, E] (replicated),
    wg_local / wu_local [E/P, D, F], wd_local [E/P, F, D] (this rank's
    experts).  Returns out [T_local, D] bf16.
    """
    ops = ops or GpuOps()
    P = dist.get_world_size(group)
    if E % P:
        raise ValueError(f"{E} experts do not split over {P} ranks")
    Epr = E // P
    if wg_local.shape[0] != Epr:
        raise ValueError(f"rank holds {wg_local.shape[0]} experts, expected {Epr}")
    T, D = x.shape
    idx, w = ops.router(x, wr, k)
    counts, offsets, perm, inv = ops.dispatch(idx, E)
    xs = ops.gather(x, perm, k)

    # 3. counts: rank r sends counts[q*Epr:(q+1)*Epr] to rank q
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    send_splits = counts.view(P, Epr).sum(1).tolist()
    recv_rows = recv_counts.view(P, Epr).sum(1)
    recv_splits = recv_rows.tolist()

    # 4. rows
    xr = torch.empty((sum(recv_splits), D), dtype=xs.dtype, device=xs.device)
    dist.all_to_all_single(xr, xs, output_split_sizes=recv_splits,
                           input_split_sizes=send_splits, group=group)

    # 5. local experts over (source, local expert) segments
    seg_offsets, seg_expert = segments(recv_counts, P, Epr)
    if xr.shape[0]:
        yr = ops.experts(xr, wg_local, wu_local, wd_local, seg_offsets, seg_expert)
    else:
        yr = torch.empty((0, D), dtype=xs.dtype, device=xs.device)

    # 6. outputs back to the token owners, in the order they were sent
    y = torch.empty_like(xs)
    dist.all_to_all_single(y, yr, output_split_sizes=send_splits,
                           input_split_sizes=recv_splits, group=group)

    # 7. combine
    return ops.combine(y, inv, w)
