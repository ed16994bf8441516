"""Expert parallelism for the MoE layer.

Upstream has no expert parallelism (every expert runs on every token in one
process, model.rs:561-565).  Here each of ``ep`` ranks holds E/ep experts:

1. every (token, slot) pair is sorted by global expert id, which orders it by
   destination rank and then by local expert;
2. per-destination counts are exchanged, then the token rows (and local expert
   ids) are exchanged with an all-to-all;
3. each rank runs its local experts on the rows it received with the grouped
   tcgen05 GEMM (:class:`~oxidizr_b200.ops.moe_kernels.GroupedExperts`, one
   expert per row);
4. the expert outputs travel back with the reverse all-to-all and are
   combined with the routing weights (fused with the residual add).

The all-to-all here is NCCL's (``torch.distributed.nn`` keeps it
differentiable); its split sizes are read on the host once per layer.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _a2a(x: torch.Tensor, out_splits, in_splits, group):
    from torch.distributed.nn.functional import all_to_all_single
    out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
    return all_to_all_single(out, x, out_splits, in_splits, group=group)


def ep_moe(moe, x: torch.Tensor, topi: torch.Tensor, topw: torch.Tensor) -> torch.Tensor:
    """Routed-expert output (without residual / shared experts) for tokens x [T, H]."""
    group = moe.ep_group
    W, El = moe.ep_size, moe.E_local
    T, H = x.shape
    k = topi.shape[1]
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    tok = order // k
    dest = flat.index_select(0, order) // El
    send_counts = torch.bincount(dest, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    s_split = send_counts.tolist()
    r_split = recv_counts.tolist()
    x_send = x.index_select(0, tok)
    local_ids = (flat.index_select(0, order) % El).to(torch.int64)
    ids_recv = torch.empty(sum(r_split), dtype=torch.int64, device=x.device)
    dist.all_to_all_single(ids_recv, local_ids, r_split, s_split, group=group)
    x_recv = _a2a(x_send, r_split, s_split, group)
    R = x_recv.shape[0]
    if R > 0:
        from ..models.moe import _grouped_ok
        if _grouped_ok(x_recv, moe.w_gu):
            from ..ops.moe_kernels import GroupedExperts
            ones = torch.ones(R, 1, dtype=torch.float32, device=x.device)
            y_recv = GroupedExperts.apply(x_recv, ids_recv[:, None], ones, moe.w_gu, moe.w_down, None)
        else:
            from ..ops import api
            y_recv = torch.zeros_like(x_recv)
            for e in range(El):
                sel = (ids_recv == e).nonzero().squeeze(1)
                if sel.numel():
                    y_recv = y_recv.index_copy(0, sel, api.swiglu_mlp(x_recv.index_select(0, sel), moe.w_gu[e],
                                                                      moe.w_down[e]))
    else:
        # keep the expert weights in the graph so every rank reaches the same collectives
        y_recv = x_recv + 0.0 * (moe.w_gu.sum() + moe.w_down.sum()).to(x_recv.dtype)
    y_send = _a2a(y_recv, s_split, r_split, group)
    w_sorted = topw.reshape(-1).index_select(0, order).to(y_send.dtype)
    return torch.zeros_like(x).index_add(0, tok, y_send * w_sorted[:, None])
