"""Expert-sharded CVMM over torch.distributed (all-to-all token dispatch).

Each rank holds the weights of E_local = E / world experts: rank r owns the
global experts [r * E_local, (r + 1) * E_local). A CVMM call with routing
`sel` (global expert ids) then runs in three steps:

1. dispatch: the routes are ordered by owning rank (stable, so route order is
   kept within a rank), the per-rank route counts are exchanged, and each
   route's input row and local expert id go to the owning rank with one
   all-to-all;
2. local compute: the owner runs CVMM (the sm_100a kernels) on the received
   rows against its own experts, every received row being one single-route
   token;
3. combine: the outputs return with the reverse all-to-all, are put back in
   route order and, with route weights, summed per token as the reference's
   weighted combine does (cvmm.py:1543-1545).

The all-to-alls are differentiable (torch.distributed.nn), so the backward
sends route-output gradients to the expert owners and input gradients back;
every rank's expert-weight gradient stays local (no weight all-reduce). The
route counts travel to the host to size the exchange, so a call synchronises
the host once. The reference has no multi-GPU code; this is the expert-sharded
mode of the benchmark contract, next to the token-sharded one in
cvmm_codex_b200.dist.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist
from torch.distributed.nn import functional as dfn


def expert_range(n_experts: int, rank: int, world: int) -> tuple[int, int]:
    """Global expert ids [lo, hi) owned by `rank`; n_experts must divide evenly."""
    if n_experts % world != 0:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    per = n_experts // world
    return rank * per, (rank + 1) * per


def _local_cvmm(x_rows: torch.Tensor, local_ids: torch.Tensor, keys_local: torch.Tensor) -> torch.Tensor:
    """CVMM of received rows, one route each, against this rank's experts."""
    from . import cvmm, cvmm_prepare_sel2
    if x_rows.shape[0] == 0:
        return x_rows.new_zeros((0, keys_local.shape[-1]))
    sel = local_ids.view(-1, 1)
    return cvmm(x_rows, cvmm_prepare_sel2(sel), keys_local).view(-1, keys_local.shape[-1])


def ep_cvmm(x: torch.Tensor, sel: torch.Tensor, keys_local: torch.Tensor, n_experts: int,
            weights: Optional[torch.Tensor] = None, group=None,
            local_fn: Optional[Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]] = None
            ) -> torch.Tensor:
    """Expert-sharded equivalent of cvmm(x, cvmm_prepare_sel2(sel, weights), keys).

    x: [..., d_in] token rows (token-shaped input); sel: [..., k] global expert
    ids; keys_local: [E_local, d_in, d_out], this rank's slice of the expert
    weights; weights: optional [..., k] route weights (weighted combine).
    Returns [..., k, d_out], or [..., d_out] with weights. `local_fn` replaces
    the local CVMM (used to test the exchange on CPU ranks)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = expert_range(n_experts, rank, world)
    if keys_local.shape[0] != hi - lo:
        raise ValueError(f"keys_local holds {keys_local.shape[0]} experts, rank {rank} owns {hi - lo}")
    local_fn = local_fn or _local_cvmm
    k = sel.shape[-1]
    lead = sel.shape[:-1]
    d_out = keys_local.shape[-1]
    flat = sel.reshape(-1).to(torch.int64)
    n_routes = flat.numel()
    per = n_experts // world
    owner = torch.div(flat, per, rounding_mode="floor")
    order = torch.sort(owner, stable=True).indices                 # routes grouped by owning rank
    send_counts = torch.bincount(owner, minlength=world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    send_sizes = send_counts.tolist()
    recv_sizes = recv_counts.tolist()
    n_recv = sum(recv_sizes)

    x_rows = x.reshape(-1, x.shape[-1]).index_select(0, torch.div(order, k, rounding_mode="floor"))
    ids_send = (flat.index_select(0, order) - owner.index_select(0, order) * per).to(torch.int32)
    ids_recv = torch.empty(n_recv, dtype=torch.int32, device=flat.device)
    dist.all_to_all_single(ids_recv, ids_send, recv_sizes, send_sizes, group=group)
    x_recv = dfn.all_to_all_single(x_rows.new_empty((n_recv, x_rows.shape[-1])), x_rows, recv_sizes, send_sizes,
                                   group=group)

    y_recv = local_fn(x_recv, ids_recv, keys_local)               # [n_recv, d_out]

    y_sorted = dfn.all_to_all_single(y_recv.new_empty((n_routes, d_out)), y_recv, send_sizes, recv_sizes,
                                     group=group)
    inv = torch.empty_like(order)
    inv[order] = torch.arange(n_routes, device=order.device)
    y = y_sorted.index_select(0, inv).view(*lead, k, d_out)      # back in route order
    if weights is None:
        return y
    # the reference's weighted combine: weights cast to the route dtype, summed
    # in fp32 for 16-bit routes
    acc = torch.float32 if y.dtype in (torch.bfloat16, torch.float16) else y.dtype
    wr = weights.to(y.dtype).to(acc)
    return torch.einsum("...k,...kn->...n", wr, y.to(acc)).to(y.dtype)
