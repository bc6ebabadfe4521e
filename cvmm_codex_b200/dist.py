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


class OverlappedGradReduce:
    """All-reduce of the expert-weight gradient overlapped with grad-x.

    CVMM.backward computes grad-W before grad-x (the sorted-grad GEMM, then
    the route-grad GEMM and the k-sum). While installed (a context manager),
    this object is CVMM's backward hook: it records an event on the compute
    stream as soon as grad-W is written, and the NCCL all-reduce of that
    gradient runs on a side stream that waits on the event, so the exchange
    crosses NVLink while the grad-x kernels run; the compute stream then waits
    for the reduction before anything after the backward reads the gradient.

    Two modes:
    * eager backward (no stream capture): the reduction is issued from the
      hook when the backward is about to return, after the grad-x kernels were
      queued, and the compute stream waits on it before the backward returns;
    * CUDA-graph replay: the hook's event is recorded as an external event
      node inside the captured graph and no collective is captured; after each
      replay, `launch(grad)` queues the side-stream all-reduce behind that node
      and makes the compute stream wait for it.
    The gradient is summed in place and in the same order as a plain
    all-reduce after the backward, so results are identical.

    From grad-W to the end of the backward the persistent GEMMs are capped at
    the device's SMs minus `reserve_sms` (default 16, env CVMM_B200_NCCL_SMS)
    through cvmm_set_sm_limit: they hold nearly all of an SM's shared memory,
    so without free SMs the all-reduce's kernels would only start after them.
    """

    def __init__(self, group=None, reserve_sms=None):
        import os
        self.group = group
        # SMs left free for the collective while grad-x runs: the persistent
        # GEMMs otherwise hold every SM and NCCL's kernels only start after them.
        self.reserve = int(os.environ.get("CVMM_B200_NCCL_SMS", "16")) if reserve_sms is None else int(reserve_sms)
        self._prev_limit = None
        self.side = torch.cuda.Stream()
        self.ready = torch.cuda.Event(external=True)
        self._grad = None
        self._prev = None

    def __enter__(self):
        from . import api
        self._prev = api.cvmm_backward_hook
        api.cvmm_backward_hook = self
        return self

    def __exit__(self, *exc):
        from . import api
        api.cvmm_backward_hook = self._prev
        return False

    # -- called by CVMM.backward on the compute stream
    def grad_keys_ready(self, grad_keys: torch.Tensor) -> None:
        self.ready.record()
        self._grad = None if torch.cuda.is_current_stream_capturing() else grad_keys
        if self.reserve > 0 and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            from . import _lib
            n = torch.cuda.get_device_properties(grad_keys.device).multi_processor_count
            self._prev_limit = _lib.load().cvmm_set_sm_limit(max(1, n - self.reserve))

    def backward_done(self) -> None:
        if self._prev_limit is not None:
            from . import _lib
            _lib.load().cvmm_set_sm_limit(self._prev_limit)
            self._prev_limit = None
        if self._grad is not None:
            grad, self._grad = self._grad, None
            self.launch(grad)

    # -- after a graph replay (or from the hook in eager mode)
    def launch(self, grad: torch.Tensor) -> None:
        """Side-stream all-reduce of `grad` after the recorded event; the
        current stream waits for it."""
        if not dist.is_initialized() or dist.get_world_size(self.group) == 1:
            return
        cur = torch.cuda.current_stream()
        self.side.wait_event(self.ready)
        with torch.cuda.stream(self.side):
            dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=self.group)
        cur.wait_stream(self.side)
