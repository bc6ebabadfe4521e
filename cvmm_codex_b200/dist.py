"""Token-sharded data parallelism for CVMM over torch.distributed.

Every rank owns a contiguous slice of the tokens; selector preparation,
forward, grad-input and sel-weight gradients are local. The only exchange is
the sum of the fp32 expert-weight gradients over ranks, one all-reduce
(NCCL over NVLink on B200 boxes, gloo on CPU). The reference library has no
multi-GPU code; this is the partitioning the benchmark contract asks for.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def token_slice(n_tokens: int, rank: int, world: int) -> slice:
    """Contiguous, balanced token range of `rank` (sizes differ by at most one)."""
    base, extra = divmod(n_tokens, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def allreduce_expert_grads(keys: torch.Tensor, group=None, async_op: bool = False):
    """Sums keys.grad over the ranks of `group` in place (the weight-gradient
    exchange of token sharding). Returns the work handle when async_op."""
    if keys.grad is None:
        raise RuntimeError("allreduce_expert_grads: keys.grad is None (run backward first)")
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return None
    return dist.all_reduce(keys.grad, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
