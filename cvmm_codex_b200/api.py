"""Drop-in replacement of the reference module ``cvmm.py`` (RobertCsordas/cvmm_codex).

Same public names, signatures, dataclass fields, dtypes and autograd behaviour:

* ``CVMMSel``                                  -- cvmm.py:12-21
* ``cvmm_prepare_sel(sel, n_experts)``         -- cvmm.py:24-27
* ``cvmm_prepare_sel2(sel, w=None, route_input=False)`` -- cvmm.py:1786-1803
* ``cvmm(x, sel, keys)``                       -- cvmm.py:1759-1783
* ``CVMM`` (torch.autograd.Function)           -- cvmm.py:1521-1755
* torch op ``cvmm_b200::cvmm_triton`` with the schema of ``mylib::cvmm_triton``
  (cvmm.py:808-867, fake impl as at cvmm.py:1436-1450)

Underneath, every operation runs in libcvmm_sm100.so (hand-written sm_100a
CUDA: device radix sort for the selector, tcgen05 tensor-core gather-GEMMs
for bf16/fp16 arithmetic, an exact-fp32 FFMA engine for fp32 arithmetic).
There is no Triton, no CPU path and no fallback: tensors must be on a CUDA
device and the library must be built.

The reference's backward chooses between six kernel paths with a VRAM probe
and OOM fallbacks (cvmm.py:1552-1755). Here the same gradients come from one
schedule per case (see ``CVMM.backward``) that needs no VRAM probe, so the
module-level tuning flags below are kept only so that code which sets them
keeps working; they do not change the computation.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Optional, Union

import torch

from ._torch_ops import calls as ops  # every device call: a registered torch custom op under torch.compile


@dataclass
class CVMMSel:
    """Prepared routing (reference cvmm.py:12-21).

    raw_sel:  int32, the routing in its original [..., k] shape.
    sel:      int32, expert ids in expert-sorted (stable) order, same shape.
    sel_index: int64 [n_routes], input row of each sorted route (token id for
              token-shaped input, route id for route-shaped input).
    out_index: int64 [n_routes] route id of each sorted route, or None for
              route-shaped input.
    reduction_weight: optional [..., k] weights of the weighted sum over k.
    """
    raw_sel: torch.Tensor
    sel: torch.Tensor
    sel_index: torch.Tensor
    out_index: Optional[torch.Tensor] = None
    reduction_weight: Optional[torch.Tensor] = None

    def clone(self) -> "CVMMSel":
        # Shallow, like the reference: the tensors are shared.
        return CVMMSel(self.raw_sel, self.sel, self.sel_index, self.out_index, self.reduction_weight)


def cvmm_prepare_sel(sel: torch.Tensor, n_experts: int) -> CVMMSel:
    """Route-indexed selector (reference cvmm.py:24-27): sel_index = sorted route ids."""
    raw, ssel, sel_index, _ = ops.sel_prepare(sel, sel.shape[-1] if sel.dim() else 1, True)
    return CVMMSel(raw.view_as(sel), ssel.view_as(sel), sel_index, None)


def cvmm_prepare_sel2(sel: Union[torch.Tensor, CVMMSel], w: Optional[torch.Tensor] = None,
                      route_input: bool = False) -> CVMMSel:
    """Prepare (or re-wrap) a selector (reference cvmm.py:1786-1803).

    A CVMMSel argument is re-wrapped without device work; with route_input the
    route ids become the input index (reference cvmm.py:1788-1792)."""
    if isinstance(sel, CVMMSel):
        if route_input:
            route_index = sel.out_index if sel.out_index is not None else sel.sel_index
            return CVMMSel(sel.raw_sel, sel.sel, route_index, None, w)
        return CVMMSel(sel.raw_sel, sel.sel, sel.sel_index, sel.out_index, w)

    n_per_batch = sel.shape[-1]
    raw, ssel, sel_index, out_index = ops.sel_prepare(sel, n_per_batch, route_input)
    if route_input:
        return CVMMSel(raw.view_as(sel), ssel.view_as(sel), sel_index, None, w)
    return CVMMSel(raw.view_as(sel), ssel.view_as(sel), sel_index, out_index, w)


def get_dtype():
    """Operation dtype: the autocast dtype when autocast is on, else float32 (cvmm.py:30-33)."""
    if not torch.is_autocast_enabled("cuda"):
        return torch.float32
    return torch.get_autocast_dtype("cuda")


def dtype_to_type_id(dtype: torch.dtype):
    """Reference dtype ids (cvmm.py:36-44); also the C ABI's float dtype codes."""
    if dtype == torch.float32:
        return 0
    elif dtype == torch.float16:
        return 1
    elif dtype == torch.bfloat16:
        return 2
    raise ValueError("Unknown dtype")


# Module attributes of the reference (cvmm.py:47-64) that callers and tests set.
# They are accepted for compatibility; the sm_100a implementation has a single
# schedule per case and no Triton autotuning, so they do not alter results.
cvmm_triton_call = None
cvmm_expert_offsets_call = None
cvmm_use_lowmem_grouped_backward = os.environ.get("CVMM_DISABLE_LOWMEM_GROUPED_BACKWARD", "0").lower() not in ("1", "true", "yes", "on")
cvmm_use_triton_expert_offsets = os.environ.get("CVMM_DISABLE_TRITON_EXPERT_OFFSETS", "0").lower() not in ("1", "true", "yes", "on")
cvmm_fast_single_expert_indexed_forward = os.environ.get("CVMM_FAST_SINGLE_EXPERT_INDEXED_FORWARD", "auto").lower()
cvmm_lowmem_min_top_k = int(os.environ.get("CVMM_LOWMEM_MIN_TOP_K", "32"))
cvmm_lowmem_chunk_size = int(os.environ.get("CVMM_LOWMEM_CHUNK_SIZE", "0"))
cvmm_force_gather_x_grad_w = os.environ.get("CVMM_GATHER_X_GRAD_W", "0").lower() in ("1", "true", "yes", "on")
cvmm_gather_x_grad_w_max_top_k = int(os.environ.get("CVMM_GATHER_X_GRAD_W_MAX_TOP_K", "8"))
# sm_100a engine knob (no reference counterpart): copy the GEMM operands into
# the expert-padded sorted layout so the tensor-core kernels read dense tiles.
# Costs one extra [n_routes + 128 * n_experts, d_in] op-dtype copy of x kept
# for the backward.
cvmm_sorted_operands = os.environ.get("CVMM_B200_SORTED_OPERANDS", "1").lower() not in ("0", "false", "no", "off")
# sm_100a engine knob: the weighted grad-W reads a weight-scaled, expert-padded
# sorted copy of the token grads (True) instead of gathering and scaling the
# token grad rows inside the GEMM (False). Both give bit-identical results.
cvmm_weighted_grad_copy = os.environ.get("CVMM_B200_WEIGHTED_GRAD_COPY", "1").lower() not in ("0", "false", "no", "off")
# sm_100a engine knob: the unweighted forward writes the sorted padded copy of
# the x rows it gathers, for the grad-W's dense x tiles (True), or writes none
# and the grad-W gathers x rows itself (False). Same results either way.
cvmm_forward_x_copy = os.environ.get("CVMM_B200_FORWARD_X_COPY", "1").lower() not in ("0", "false", "no", "off")
# sm_100a engine knob: the unweighted forward makes the sorted x copy in a separate
# copy pass (warp-per-row gathers) and then reads it as dense tiles (True), instead
# of writing it from its own cp.async gathers (False). Same results either way.
cvmm_forward_sort_first = os.environ.get("CVMM_B200_FORWARD_SORT_FIRST", "0").lower() in ("1", "true", "yes", "on")
# sm_100a engine knob: the keys cast loads the weights while the selector sort
# queued before it still runs and writes after it (True), or starts after it (False).
cvmm_cast_ahead = os.environ.get("CVMM_B200_CAST_AHEAD", "1").lower() not in ("0", "false", "no", "off")
# sm_100a engine knob: in the bf16_params mode (bf16 x and keys, no autocast)
# the unweighted backward runs on the bf16 tensor cores with the fp32 grad
# split into two bf16 parts (True) instead of the fp32 SIMT GEMMs (False).
cvmm_split_fp32_grad = os.environ.get("CVMM_B200_SPLIT_FP32_GRAD", "1").lower() not in ("0", "false", "no", "off")
# Data-parallel hook (None, or an object with grad_keys_ready(grad_keys) and
# backward_done()): CVMM.backward calls grad_keys_ready on the compute stream
# as soon as the fp32 expert-weight gradient is written, before the grad-x
# work, and backward_done just before it returns, so a caller can reduce the
# weight gradient across ranks while grad-x runs (dist.OverlappedGradReduce).
cvmm_backward_hook = None
# sm_100a engine knob: the weighted backward makes ONE unscaled expert-padded
# sorted copy of the token grads that both grad-W (weights applied in shared
# memory) and grad-x read as dense tiles (True), instead of the per-GEMM
# variants selected by cvmm_weighted_grad_copy. Same results (the sel-weight
# grad up to its fp32 summation order). Off by default: at ff_down_1024 it made
# grad-x faster (74 -> 59 us) but the in-shared-memory scaling slowed grad-W
# (62 -> 108 us).
cvmm_weighted_shared_grad_copy = os.environ.get("CVMM_B200_WEIGHTED_SHARED_GRAD", "0").lower() in ("1", "true", "yes", "on")
# Opt-in host check of the device status word after every CVMM forward and
# backward (synchronises the stream): raises RuntimeError when a kernel gave up
# on a bounded wait or met an out-of-range expert id.
cvmm_check_device_status = os.environ.get("CVMM_B200_CHECK_STATUS", "0").lower() in ("1", "true", "yes", "on")


def create_kernels():
    """Binds the op entry points (reference cvmm.py:95-1465). Idempotent."""
    global cvmm_triton_call, cvmm_expert_offsets_call
    if cvmm_triton_call is not None:
        return
    from . import _torch_ops  # registers cvmm_b200::* ops
    cvmm_triton_call = torch.ops.cvmm_b200.cvmm_triton
    cvmm_expert_offsets_call = ops.expert_offsets


def _cvmm_expert_offsets(sorted_experts: torch.Tensor, n_experts: int) -> torch.Tensor:
    """Inclusive end offset per expert (reference cvmm.py:68-78).

    With ``cvmm_expert_offsets_call`` bound (after create_kernels) this is the
    device binary-search kernel. Setting it to None selects the reference's
    own torch formulation (unique_consecutive + cumsum), which the reference's
    test uses as the expected value (test_cvmm_correctness.py:73-86); the CVMM
    forward/backward never take that branch."""
    if cvmm_use_triton_expert_offsets and cvmm_expert_offsets_call is not None and sorted_experts.is_cuda:
        return cvmm_expert_offsets_call(sorted_experts, n_experts)
    unique_experts, counts = torch.unique_consecutive(sorted_experts, return_counts=True)
    if unique_experts.numel() == n_experts:
        return counts.cumsum(0)
    expert_counts = torch.zeros((n_experts,), device=sorted_experts.device, dtype=counts.dtype)
    expert_counts[unique_experts.long()] = counts
    return expert_counts.cumsum(0)


def _lowmem_chunk_size(top_k: int) -> int:
    chunk = cvmm_lowmem_chunk_size
    if chunk <= 0:
        chunk = top_k
    return min(top_k, chunk)


def _operand(keys: torch.Tensor, op_dtype: torch.dtype) -> torch.Tensor:
    """Expert weights in the operation dtype for the tensor-core path.

    The reference casts each fp32 weight tile to bf16 inside the kernel
    (cvmm.py:202-204); the tcgen05 kernels read a bf16 copy made once per
    forward (RNE, the same rounding) and reused by the backward."""
    if op_dtype == torch.float32 or keys.dtype == op_dtype:
        return keys
    # No kernel of this library writes the keys: the cast may overlap the
    # selector kernels queued before it.
    return ops.cast(keys, op_dtype, ahead=cvmm_cast_ahead)


def _sortable(t: torch.Tensor, op_dtype: torch.dtype) -> bool:
    """Whether rows of `t` can be copied into the expert-padded sorted layout
    that the tensor-core kernels read as dense 16-byte-aligned TMA tiles."""
    return (cvmm_sorted_operands and op_dtype in (torch.bfloat16, torch.float16) and t.is_floating_point()
            and t.shape[-1] % 8 == 0)


def _routes_per_row(x: torch.Tensor, sel: torch.Tensor, out_index: Optional[torch.Tensor]) -> int:
    """Routes that share one row of x. 1 for the reference's two layouts
    (token-shaped x with out_index, route-shaped x without). A route-indexed
    selector sel [..., K] over x [..., H, d] with K = r * H (r > 1) means that
    the r consecutive routes of every row read that row: SwitchHead's output
    projection, whose 2 routes per head read the head's value row. The
    reference needs x repeated r times for this (x.repeat_interleave); here
    the kernels index row p // r instead (no reference counterpart)."""
    if out_index is not None or x.dim() < 2 or sel.dim() < 1:
        return 1
    rows = x.numel() // x.shape[-1]
    n = sel.numel()
    if rows == 0 or rows >= n or n % rows != 0 or tuple(x.shape[:-2]) != tuple(sel.shape[:-1]):
        return 1
    return n // rows


def _raise_on_device_status(where: str) -> None:
    """Reads and clears the library's device status word (synchronises) and
    raises if a kernel recorded a timeout or an out-of-range expert id."""
    from . import _lib
    code, site, aux = _lib.device_status(reset=True)
    if code != 0:
        what = {1: "a bounded wait ran out", 2: "an expert id outside [0, n_experts)"}.get(code, "error")
        raise RuntimeError(f"{where}: device status {code} ({what}; site {site}, value {aux})")


class CVMM(torch.autograd.Function):
    """Autograd function with the reference's signature (cvmm.py:1521-1755)."""

    warned = False

    @staticmethod
    def forward(ctx, x: torch.Tensor, raw_sel: torch.Tensor, sel_index: torch.Tensor,
                sel: torch.Tensor, keys: torch.Tensor, out_index: Optional[torch.Tensor] = None,
                reduction_weight: Optional[torch.Tensor] = None):
        op_dtype = get_dtype()
        n_experts = keys.shape[0]
        keys_op = _operand(keys, op_dtype)
        offsets = ops.expert_offsets(sel, n_experts)
        # Routes per x row: 1, except for a route-indexed selector over an x
        # whose rows are shared by consecutive routes (SwitchHead: the 2 routes
        # of a head read that head's value row; see _routes_per_row).
        rph = _routes_per_row(x, sel, out_index)
        x_index, oi = sel_index, out_index
        if rph > 1:
            x_index = torch.div(sel_index, rph, rounding_mode="floor")
            oi = sel_index  # outputs stay route-indexed
        xs = xpad = x_route_rows = None
        if _sortable(x, op_dtype) and reduction_weight is not None:
            # Expert-sorted, 128-row padded op-dtype copy of the route rows of x:
            # the forward and the grad-W read it as dense tiles (the reference's
            # grouped-x copy, cvmm.py:1123-1138).
            if out_index is None and rph == 1 and keys.shape[-1] % 8 == 0:
                # x rows are the routes: the copy also writes the route -> padded
                # row map the weighted combine reads.
                xs, xpad, x_route_rows = ops.sort_rows_padded(x, sel_index, 1, sel, offsets, n_experts,
                                                              dtype=op_dtype, route_rows=True)
            else:
                xs, xpad = ops.sort_rows_padded(x, sel_index, rph, sel, offsets, n_experts, dtype=op_dtype)
        a = x if xs is None else xs
        # fp32 op dtype (no autocast) over 16-bit x and keys (the reference's
        # bf16_params mode): every product of two 16-bit values is exact in
        # fp32, so the 16-bit tensor-core GEMM with fp32 accumulation and fp32
        # output computes the reference's fp32 dot (allow_tf32=False) up to the
        # order of the fp32 sums, instead of the SIMT fp32 GEMM.
        fwd_op, fwd_keys = op_dtype, keys_op
        if (op_dtype == torch.float32 and xs is None and x.dtype == keys.dtype
                and x.dtype in (torch.bfloat16, torch.float16)):
            fwd_op, fwd_keys = x.dtype, keys
        # The bf16_params backward (_split_bf16_backward) reads the same sorted
        # x copy as the autocast path.
        split_copy = (fwd_op == torch.bfloat16 and op_dtype == torch.float32 and cvmm_split_fp32_grad
                      and reduction_weight is None and _sortable(x, fwd_op) and cvmm_forward_x_copy)
        if (reduction_weight is None and cvmm_forward_sort_first and cvmm_forward_x_copy
                and _sortable(x, op_dtype) and fwd_op == op_dtype):
            # Copy pass first (warp-per-row gathers), then the forward over
            # dense A tiles of that copy; the backward reads the same copy.
            xs, xpad = ops.sort_rows_padded(x, sel_index, rph, sel, offsets, n_experts, dtype=op_dtype)
            res = ops.forward(xs, x_index, offsets, fwd_keys, oi, op_dtype, fwd_op, x_pad_start=xpad)
            res = res.view(*sel.shape, res.shape[-1])
        elif reduction_weight is None and ((_sortable(x, op_dtype) and cvmm_forward_x_copy) or split_copy):
            # The forward gathers x's rows anyway: it writes that sorted padded
            # copy for the grad-W as it goes, instead of a separate copy pass.
            # Its pad starts depend only on the offsets; the backward takes them
            # from the grad copy it makes anyway.
            res, xs = ops.forward(x, x_index, offsets, fwd_keys, oi, op_dtype, fwd_op, x_copy=True)
            res = res.view(*sel.shape, res.shape[-1])
        elif reduction_weight is not None:
            rows = out_pad = None
            if xs is not None and keys.shape[-1] % 8 == 0:
                # Route outputs stay in the padded sorted layout (dense TMA tile
                # stores); the weighted combine gathers them per token.
                out_pad = xpad
                rows = x_route_rows if x_route_rows is not None else ops.padded_route_rows(
                    out_index if out_index is not None else sel_index, sel, offsets, xpad)
            y = ops.forward(a, x_index, offsets, fwd_keys, oi, op_dtype, fwd_op, x_pad_start=xpad,
                            out_pad_start=out_pad)
            res = ops.weighted_combine(y, reduction_weight, op_dtype, y_rows=rows)
            res = res.view(*reduction_weight.shape[:-1], res.shape[-1])
        else:
            res = ops.forward(a, x_index, offsets, fwd_keys, oi, op_dtype, fwd_op, x_pad_start=xpad)
            res = res.view(*sel.shape, res.shape[-1])
        ctx.save_for_backward(x, keys_op, raw_sel, sel, sel_index, out_index, reduction_weight, offsets, xs, xpad)
        ctx.op_type = op_dtype
        ctx.keys_type = keys.dtype
        ctx.dtype = op_dtype
        ctx.rph = rph
        if cvmm_check_device_status:
            _raise_on_device_status("CVMM.forward")
        return res

    @staticmethod
    def backward(ctx, grad_output):
        return _cvmm_backward(ctx, ctx.saved_tensors, grad_output)


def _split_bf16_backward(ctx, x, keys_op, sel, sel_index, route, offsets, g, need_x, need_keys, n_routes, rph,
                         xs=None):
    """Unweighted backward of the bf16_params mode (bf16 x and keys, no
    autocast: fp32 op dtype, fp32 output grad) on the bf16 tensor cores.

    x and keys hold bf16 values; the fp32 grad is split as g = hi + lo with hi =
    bf16(g) and lo = bf16(g - hi) (g - hi is exact in fp32, lo keeps its next 8
    mantissa bits, a residual below 2^-16 |g|). Every product of two bf16
    values is exact in fp32, so grad-W = x^T [hi | lo] (one GEMM over 2 d_out
    columns, the halves summed in fp32) and grad-x = [hi | lo] [W | W]^T (one
    GEMM over 2 d_out of K) are the reference's fp32 results (cvmm.py:1141-1225,
    allow_tf32=False) up to fp32 summation order and that residual."""
    n_experts, _, d_out = keys_op.shape
    g2 = g.reshape(n_routes, d_out)
    hi = g2.to(torch.bfloat16)
    lo = (g2 - hi.float()).to(torch.bfloat16)
    gcat = torch.cat([hi, lo], dim=1)
    # One expert-padded sorted copy of [hi | lo] feeds both GEMMs dense TMA tiles.
    bf = torch.bfloat16
    gs, gpad = ops.sort_rows_padded(gcat, route, 1, sel, offsets, n_experts, dtype=bf)
    grad_x = grad_keys = None
    if need_keys:
        if xs is not None:  # the forward's sorted x copy: both operands dense
            gw = ops.backward_w(xs, None, 1, gs, None, 1, offsets, n_experts, bf, g_pad_start=gpad,
                                x_pad_start=gpad, n_routes=n_routes)
        else:
            gw = ops.backward_w(x, sel_index, rph, gs, None, 1, offsets, n_experts, bf, g_pad_start=gpad)
        grad_keys = (gw[..., :d_out] + gw[..., d_out:]).to(ctx.keys_type)
    if need_x:
        kh = keys_op.to(bf)
        kcat = torch.cat([kh, kh], dim=-1)
        x_rows = x.reshape(-1, x.shape[-1]).shape[0]
        if x_rows == n_routes:
            grad_x = ops.backward_x(gs, None, 1, route, offsets, kcat, x.dtype, bf, g_pad_start=gpad).view_as(x)
        else:
            gxs = ops.backward_x(gs, None, 1, None, offsets, kcat, x.dtype, bf, g_pad_start=gpad,
                                 out_pad_start=gpad, n_routes=n_routes)
            rows = ops.padded_route_rows(route, sel, offsets, gpad)
            grad_x = ops.sum_routes(gxs, n_routes // x_rows, x.dtype, src_rows=rows).view_as(x)
    if cvmm_backward_hook is not None:
        if grad_keys is not None:
            cvmm_backward_hook.grad_keys_ready(grad_keys)
        cvmm_backward_hook.backward_done()
    if cvmm_check_device_status:
        _raise_on_device_status("CVMM.backward")
    return grad_x, None, None, None, grad_keys, None, None


def _cvmm_backward(ctx, saved, grad_output):
    """CVMM.backward on the tensors saved by the forward (shared with CVMMGelu)."""
    x, keys_op, raw_sel, sel, sel_index, out_index, w, offsets, xs, xpad = saved
    need_x = ctx.needs_input_grad[0]
    need_keys = ctx.needs_input_grad[4]
    need_w = len(ctx.needs_input_grad) > 6 and ctx.needs_input_grad[6] and w is not None
    op = ctx.op_type
    rph = getattr(ctx, "rph", 1)
    n_experts = keys_op.shape[0]
    n_routes = sel.numel()
    top_k = raw_sel.shape[-1] if raw_sel.dim() > 0 else 1
    # Route id of every sorted position: where its output row lives.
    route = out_index if out_index is not None else sel_index
    g = grad_output
    if g.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        g = g.float()
    x_rows = x.reshape(-1, x.shape[-1]).shape[0]

    grad_x = grad_keys = grad_w = None
    if (w is None and op == torch.float32 and x.dtype == torch.bfloat16 and ctx.keys_type == torch.bfloat16
            and g.dtype == torch.float32 and cvmm_split_fp32_grad):
        return _split_bf16_backward(ctx, x, keys_op, sel, sel_index, route, offsets, g, need_x, need_keys,
                                    n_routes, rph, xs)
    if op == torch.float32:
        xs = xpad = None  # a 16-bit x copy only feeds the bf16 split path
    if w is None:
        g2 = g.reshape(n_routes, g.shape[-1])
        g_rows, g_idx, g_pad, g_route_rows = g2, route, None, None
        if _sortable(g2, op):
            # One expert-padded sorted copy of the route grads (the
            # reference's grouping copy, cvmm.py:1161) lets both GEMMs read
            # them as dense tensor-core tiles.
            if need_x and x_rows != n_routes and x.dtype == op and x.shape[-1] % 8 == 0:
                # The copy also writes the route -> padded row map the k-sum reads.
                g_rows, g_pad, g_route_rows = ops.sort_rows_padded(g2, route, 1, sel, offsets, n_experts, dtype=op,
                                                                   route_rows=True, pad_start=xpad)
            else:
                g_rows, g_pad = ops.sort_rows_padded(g2, route, 1, sel, offsets, n_experts, dtype=op, pad_start=xpad)
            g_idx = None
        if xs is not None and xpad is None:
            xpad = g_pad if g_pad is not None else ops.pad_starts(offsets, n_experts)
        if need_keys:
            # dW_e = sum_p x[sel_index[p]]^T g[route[p]]  (cvmm.py:1163-1198)
            if xs is not None:
                grad_keys = ops.backward_w(xs, None, 1, g_rows, g_idx, 1, offsets, n_experts, op,
                                           g_pad_start=g_pad, x_pad_start=xpad, n_routes=n_routes)
            else:
                grad_keys = ops.backward_w(x, sel_index, rph, g_rows, g_idx, 1, offsets, n_experts, op,
                                           g_pad_start=g_pad)
        if grad_keys is not None and cvmm_backward_hook is not None and ctx.keys_type == torch.float32:
            cvmm_backward_hook.grad_keys_ready(grad_keys)
        if need_x:
            # gx_route[route] = g[route] W_e^T, then summed over k (cvmm.py:1199-1223)
            if x_rows == n_routes:
                gxr = ops.backward_x(g_rows, g_idx, 1, route, offsets, keys_op, x.dtype, op, g_pad_start=g_pad)
                grad_x = gxr.view_as(x)
            elif g_pad is not None and x.dtype == op and x.shape[-1] % 8 == 0:
                # Route grads stay in the padded sorted layout (dense TMA
                # tile stores); the k-sum gathers them per token.
                gxs = ops.backward_x(g_rows, None, 1, None, offsets, keys_op, x.dtype, op, g_pad_start=g_pad,
                                     out_pad_start=g_pad, n_routes=n_routes)
                rows = g_route_rows if g_route_rows is not None else ops.padded_route_rows(route, sel, offsets, g_pad)
                grad_x = ops.sum_routes(gxs, n_routes // x_rows, x.dtype, src_rows=rows).view_as(x)
            else:
                gxr = ops.backward_x(g_rows, g_idx, 1, route, offsets, keys_op, x.dtype, op, g_pad_start=g_pad)
                grad_x = ops.sum_routes(gxr, n_routes // x_rows, x.dtype).view_as(x)
    else:
        k = w.shape[-1]
        gt = g.reshape(-1, g.shape[-1])  # token grads of the combined output
        gs = gpad = None
        if need_keys:
            # dW_e = sum_p x[sel_index[p]]^T (bf16(w_p) * g[route_p // k])  (cvmm.py:1341-1383)
            if xs is not None and _sortable(gt, op) and cvmm_weighted_shared_grad_copy:
                # One unscaled expert-padded sorted copy of the token grads feeds
                # both GEMMs as dense TMA boxes: grad-W applies op(op(g) op(w))
                # in shared memory (cvmm.py:591-599), grad-x reads it as A.
                gs, gpad = ops.sort_rows_padded(gt, route, k, sel, offsets, n_experts, dtype=op, pad_start=xpad)
                grad_keys = ops.backward_w(xs, None, 1, gs, None, 1, offsets, n_experts, op, w=w,
                                           w_index=route, g_pad_start=gpad, x_pad_start=xpad, n_routes=n_routes)
            elif xs is not None and _sortable(gt, op) and cvmm_weighted_grad_copy:
                # The weight product is applied (and rounded) in a sorted copy.
                # Same offsets as the forward's x copy: its pad starts are reused.
                gs, gpad = ops.sort_rows_padded(gt, route, k, sel, offsets, n_experts, dtype=op, scale=w,
                                                pad_start=xpad)
                grad_keys = ops.backward_w(xs, None, 1, gs, None, 1, offsets, n_experts, op,
                                           g_pad_start=gpad, x_pad_start=xpad, n_routes=n_routes)
                gs = None  # weight-scaled: not the operand grad-x needs
            elif xs is not None:
                # Token grad rows gathered straight from g (L2-resident) and
                # scaled by op(w) in shared memory (cvmm.py:591-599): no
                # R x d_out weighted copy is written.
                grad_keys = ops.backward_w(xs, None, 1, gt, route, k, offsets, n_experts, op,
                                           w=w, w_index=route, x_pad_start=xpad, n_routes=n_routes)
            else:
                grad_keys = ops.backward_w(x, sel_index, rph, gt, route, k, offsets, n_experts, op,
                                           w=w, w_index=route)
        if grad_keys is not None and cvmm_backward_hook is not None and ctx.keys_type == torch.float32:
            cvmm_backward_hook.grad_keys_ready(grad_keys)
        if need_x or need_w:
            if gs is not None:
                # grad-x / sel-weight grad from the same unscaled sorted copy
                # (dense A tiles instead of gathered token rows).
                ga, gia, gk, gpd = gs, None, 1, gpad
            else:
                ga, gia, gk, gpd = gt, route, k, None
            if out_index is None and rph > 1:
                # Route-indexed selector over shared x rows (SwitchHead heads):
                # the fused route grad-x + sel-weight grad reads x row p / rph,
                # then each row sums its rph route grads.
                gx, gsel = ops.backward_x(ga, gia, gk, route, offsets, keys_op, x.dtype, op, w=w, x=x,
                                          x_div=rph, g_pad_start=gpd, n_routes=n_routes)
                grad_x = ops.sum_routes(gx, rph, x.dtype).view_as(x) if need_x else None
                grad_w = gsel.view_as(w).to(w.dtype) if need_w else None
            elif out_index is None and tuple(x.shape[:-1]) == tuple(w.shape):
                # Route-shaped input: fused grad-x + sel-weight grad (cvmm.py:1386-1433)
                gx, gsel = ops.backward_x(ga, gia, gk, route, offsets, keys_op, x.dtype, op,
                                          w=w, x=x, g_pad_start=gpd, n_routes=n_routes)
                grad_x = gx.view_as(x) if need_x else None
                grad_w = gsel.view_as(w).to(w.dtype) if need_w else None
            else:
                # Token-shaped input: route grads, then weighted token sums (cvmm.py:1726-1750)
                rg = ops.backward_x(ga, gia, gk, route, offsets, keys_op, op, op, g_pad_start=gpd,
                                    n_routes=n_routes)
                gx, gsel = ops.weighted_token_backward(rg, w, x, need_x, need_w, x.dtype)
                grad_x = gx.view_as(x) if need_x else None
                grad_w = gsel.view_as(w).to(w.dtype) if need_w else None
    if grad_keys is not None and ctx.keys_type != torch.float32:
        grad_keys = grad_keys.to(ctx.keys_type)
    del top_k
    if cvmm_backward_hook is not None:
        if ctx.keys_type != torch.float32 and grad_keys is not None:
            cvmm_backward_hook.grad_keys_ready(grad_keys)  # after the cast: no overlap
        cvmm_backward_hook.backward_done()
    if cvmm_check_device_status:
        _raise_on_device_status("CVMM.backward")
    return grad_x, None, None, None, grad_keys, None, grad_w


class CVMMGelu(torch.autograd.Function):
    """gelu(cvmm(x, sel, keys)) with the activation fused into the forward
    GEMM's epilogue (unweighted selector; bf16/fp16 autocast): the forward
    writes h = gelu(z) and keeps z = the rounded GEMM output for the backward,
    which applies gelu'(z) to the incoming gradient and then runs CVMM's
    backward on it. The reference computes F.gelu(cvmm(...)) as two passes
    (benchmark_ffn_moe.py:93-94); the numerics are the same: z is rounded to
    the op dtype, the GELU is evaluated in fp32 on it and rounded."""

    @staticmethod
    def forward(ctx, x, raw_sel, sel_index, sel, keys, out_index):
        op_dtype = get_dtype()
        n_experts = keys.shape[0]
        keys_op = _operand(keys, op_dtype)
        offsets = ops.expert_offsets(sel, n_experts)
        want_copy = _sortable(x, op_dtype)
        h, z, xs = ops.forward_gelu(x, sel_index, offsets, keys_op, out_index, op_dtype, x_copy=want_copy)
        ctx.save_for_backward(x, keys_op, raw_sel, sel, sel_index, out_index, None, offsets, xs, None, z)
        ctx.op_type = op_dtype
        ctx.keys_type = keys.dtype
        ctx.dtype = op_dtype
        if cvmm_check_device_status:
            _raise_on_device_status("CVMMGelu.forward")
        return h.view(*sel.shape, h.shape[-1])

    @staticmethod
    def backward(ctx, grad_h):
        saved = ctx.saved_tensors
        z = saved[10]
        g = grad_h.reshape(z.shape)
        if g.dtype != z.dtype:
            g = g.to(z.dtype)
        dz = ops.gelu_backward(g, z).view(grad_h.shape)
        return _cvmm_backward(ctx, saved[:10], dz)[:6]


def cvmm_gelu(x: torch.Tensor, sel: Union[torch.Tensor, CVMMSel], keys: torch.Tensor) -> torch.Tensor:
    """F.gelu(cvmm(x, sel, keys)) with GELU fused into the GEMM epilogue (no
    reference counterpart as one call; the reference composes the two,
    benchmark_ffn_moe.py:93-94). Falls back to that composition, on the same
    device kernels plus torch's GELU, for fp32 arithmetic (no autocast) and
    for a weighted selector."""
    if not isinstance(sel, CVMMSel):
        sel = cvmm_prepare_sel(sel, keys.shape[0])
    op_dtype = get_dtype()
    if op_dtype == torch.float32 or sel.reduction_weight is not None:
        return torch.nn.functional.gelu(cvmm(x, sel, keys))
    if not torch.compiler.is_compiling():
        create_kernels()
    return CVMMGelu.apply(x, sel.raw_sel, sel.sel_index, sel.sel, keys, sel.out_index)


def router_topk(logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """(weights, sel) of the sigma-MoE router (benchmark_ffn_moe.py:89-92):
    softmax(float(logits)), top-k in descending order, weights renormalised
    to sum to one; one fused kernel. Differentiable w.r.t. the logits."""
    return _RouterTopK.apply(logits, int(top_k), bool(renormalize))


class _RouterTopK(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, top_k, renormalize):
        w, sel = ops.router_topk(logits, top_k, renormalize)
        ctx.save_for_backward(logits, sel, w)
        ctx.renormalize = renormalize
        ctx.mark_non_differentiable(sel)
        return w, sel

    @staticmethod
    def backward(ctx, grad_w, grad_sel):
        logits, sel, w = ctx.saved_tensors
        p = torch.softmax(logits.float(), dim=-1)
        gw = grad_w.float()
        if ctx.renormalize:
            # w = p_sel / s, s = sum(p_sel): d p_sel = (dw - sum(dw * w)) / s
            s = p.gather(-1, sel).sum(-1, keepdim=True).clamp_min(1e-20)
            gp_sel = (gw - (gw * w).sum(-1, keepdim=True)) / s
        else:
            gp_sel = gw
        gp = torch.zeros_like(p).scatter_(-1, sel, gp_sel)
        gl = p * (gp - (p * gp).sum(-1, keepdim=True))
        return gl.to(logits.dtype), None, None


known_shapes = set()


def cvmm(x: torch.Tensor, sel: Union[torch.Tensor, CVMMSel], keys: torch.Tensor):
    """x @ keys[sel] per route (reference cvmm.py:1759-1783)."""
    if not torch.compiler.is_compiling():
        # Module state and the stdout line of the reference (eager only: a
        # traced print would break the compiled graph).
        create_kernels()
        sh = (x.shape, keys.shape)
        if sh not in known_shapes:
            print("New shape:", sh)
            known_shapes.add(sh)
    if not isinstance(sel, CVMMSel):
        sel = cvmm_prepare_sel(sel, keys.shape[0])
    return CVMM.apply(x, sel.raw_sel, sel.sel_index, sel.sel, keys, sel.out_index, sel.reduction_weight)
