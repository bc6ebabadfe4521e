"""torch.library registration of every CVMM device operation.

Each operator of ``ops.py`` (one stream-ordered launch sequence of
libcvmm_sm100.so) is registered as a ``torch.library.custom_op`` in the
``cvmm_b200`` namespace with a fake (meta) implementation, so torch.compile
traces ``CVMM.forward`` / ``CVMM.backward`` and ``cvmm_prepare_sel2`` as
opaque operators instead of breaking the graph at the ctypes calls (the
reference registers its op the same way, cvmm.py:808-812, 1436-1450).

Optional outputs are returned as empty tensors (custom ops return tensors
only); ``api.py`` maps them back to None.

``cvmm_b200::cvmm_triton`` keeps the schema of the reference's
``mylib::cvmm_triton`` (cvmm.py:807-812):
    (Tensor x, Tensor sel_index, Tensor sel, Tensor keys, ScalarType out_dtype,
     Tensor out_index, ScalarType op_dtype) -> Tensor
with ``out_index`` a one-element tensor holding -1 when absent, and the same
fake implementation (cvmm.py:1442-1450).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops

PAD = ops.PAD_ROWS


# ------------------------------------------------------------------ selector
@torch.library.custom_op("cvmm_b200::sel_prepare", mutates_args=())
def sel_prepare(sel: torch.Tensor, top_k: int, route_input: bool) -> tuple[torch.Tensor, torch.Tensor,
                                                                          torch.Tensor, torch.Tensor]:
    raw, ssel, sel_index, out_index = ops.sel_prepare(sel, top_k, route_input)
    if out_index is None:
        out_index = torch.empty(0, dtype=torch.int64, device=sel.device)
    return raw, ssel, sel_index, out_index


@sel_prepare.register_fake
def _(sel, top_k, route_input):
    n = sel.numel()
    return (sel.new_empty((n,), dtype=torch.int32), sel.new_empty((n,), dtype=torch.int32),
            sel.new_empty((n,), dtype=torch.int64), sel.new_empty((0 if route_input else n,), dtype=torch.int64))


@torch.library.custom_op("cvmm_b200::expert_offsets", mutates_args=())
def expert_offsets(sorted_sel: torch.Tensor, n_experts: int) -> torch.Tensor:
    return ops.expert_offsets(sorted_sel, n_experts)


@expert_offsets.register_fake
def _(sorted_sel, n_experts):
    return sorted_sel.new_empty((n_experts,), dtype=torch.int64)


@torch.library.custom_op("cvmm_b200::pad_starts", mutates_args=())
def pad_starts(offsets: torch.Tensor, n_experts: int) -> torch.Tensor:
    return ops.pad_starts(offsets, n_experts)


@pad_starts.register_fake
def _(offsets, n_experts):
    return offsets.new_empty((n_experts,), dtype=torch.int32)


# ------------------------------------------------------------------ copies and small kernels
@torch.library.custom_op("cvmm_b200::cast", mutates_args=())
def cast(src: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return ops.cast(src, dtype)


@cast.register_fake
def _(src, dtype):
    return src.new_empty(src.shape, dtype=dtype)


@torch.library.custom_op("cvmm_b200::sort_rows_padded", mutates_args=())
def sort_rows_padded(src: torch.Tensor, index: torch.Tensor, div: int, sorted_sel: torch.Tensor,
                     offsets: torch.Tensor, n_experts: int, dtype: Optional[torch.dtype],
                     scale: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.sort_rows_padded(src, index, div, sorted_sel, offsets, n_experts, dtype=dtype, scale=scale)


@sort_rows_padded.register_fake
def _(src, index, div, sorted_sel, offsets, n_experts, dtype, scale):
    dt = src.dtype if dtype is None else dtype
    return (src.new_empty((index.numel() + n_experts * PAD, src.shape[-1]), dtype=dt),
            src.new_empty((n_experts,), dtype=torch.int32))


@torch.library.custom_op("cvmm_b200::sort_rows_padded_rows", mutates_args=())
def sort_rows_padded_rows(src: torch.Tensor, index: torch.Tensor, div: int, sorted_sel: torch.Tensor,
                          offsets: torch.Tensor, n_experts: int, dtype: Optional[torch.dtype],
                          scale: Optional[torch.Tensor]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return ops.sort_rows_padded(src, index, div, sorted_sel, offsets, n_experts, dtype=dtype, scale=scale,
                                route_rows=True)


@sort_rows_padded_rows.register_fake
def _(src, index, div, sorted_sel, offsets, n_experts, dtype, scale):
    dt = src.dtype if dtype is None else dtype
    return (src.new_empty((index.numel() + n_experts * PAD, src.shape[-1]), dtype=dt),
            src.new_empty((n_experts,), dtype=torch.int32),
            src.new_empty((index.numel(),), dtype=torch.int32))


@torch.library.custom_op("cvmm_b200::padded_route_rows", mutates_args=())
def padded_route_rows(route: torch.Tensor, sorted_sel: torch.Tensor, offsets: torch.Tensor,
                      pad_start: torch.Tensor) -> torch.Tensor:
    return ops.padded_route_rows(route, sorted_sel, offsets, pad_start)


@padded_route_rows.register_fake
def _(route, sorted_sel, offsets, pad_start):
    return route.new_empty((route.numel(),), dtype=torch.int32)


@torch.library.custom_op("cvmm_b200::weighted_combine", mutates_args=())
def weighted_combine(y: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype,
                     y_rows: Optional[torch.Tensor]) -> torch.Tensor:
    return ops.weighted_combine(y, w, out_dtype, y_rows=y_rows)


@weighted_combine.register_fake
def _(y, w, out_dtype, y_rows):
    return y.new_empty((w.numel() // w.shape[-1], y.shape[-1]), dtype=out_dtype)


@torch.library.custom_op("cvmm_b200::sum_routes", mutates_args=())
def sum_routes(src: torch.Tensor, top_k: int, out_dtype: torch.dtype,
               src_rows: Optional[torch.Tensor]) -> torch.Tensor:
    return ops.sum_routes(src, top_k, out_dtype, src_rows=src_rows)


@sum_routes.register_fake
def _(src, top_k, out_dtype, src_rows):
    d = src.shape[-1]
    rows = src.numel() // d if src_rows is None else src_rows.numel()
    return src.new_empty((rows // top_k, d), dtype=out_dtype)


@torch.library.custom_op("cvmm_b200::weighted_token_backward", mutates_args=())
def weighted_token_backward(route_grad: torch.Tensor, w: torch.Tensor, x: torch.Tensor, need_x: bool,
                            need_sel: bool, x_dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    gx, gsel = ops.weighted_token_backward(route_grad, w, x, need_x, need_sel, x_dtype)
    dev = route_grad.device
    return (gx if gx is not None else torch.empty(0, dtype=x_dtype, device=dev),
            gsel if gsel is not None else torch.empty(0, dtype=torch.float32, device=dev))


@weighted_token_backward.register_fake
def _(route_grad, w, x, need_x, need_sel, x_dtype):
    k = w.shape[-1]
    T = w.numel() // k
    d = route_grad.shape[-1]
    return (route_grad.new_empty((T, d) if need_x else (0,), dtype=x_dtype),
            route_grad.new_empty((T * k,) if need_sel else (0,), dtype=torch.float32))


# ------------------------------------------------------------------ GEMMs
@torch.library.custom_op("cvmm_b200::forward", mutates_args=())
def forward(x: torch.Tensor, sel_index: torch.Tensor, offsets: torch.Tensor, keys: torch.Tensor,
            out_index: Optional[torch.Tensor], out_dtype: torch.dtype, op_dtype: torch.dtype,
            x_pad_start: Optional[torch.Tensor], out_pad_start: Optional[torch.Tensor],
            x_copy: bool) -> tuple[torch.Tensor, torch.Tensor]:
    xs = None
    if x_copy:
        xs = torch.empty((sel_index.numel() + keys.shape[0] * PAD, x.shape[-1]), dtype=op_dtype, device=x.device)
    out = ops.forward(x, sel_index, offsets, keys, out_index, out_dtype, op_dtype, x_pad_start=x_pad_start,
                      out_pad_start=out_pad_start, x_copy=xs)
    return out, (xs if xs is not None else torch.empty(0, dtype=op_dtype, device=x.device))


@forward.register_fake
def _(x, sel_index, offsets, keys, out_index, out_dtype, op_dtype, x_pad_start, out_pad_start, x_copy):
    E, K, N = keys.shape
    R = sel_index.numel()
    rows = R + E * PAD if out_pad_start is not None else R
    xs = x.new_empty((R + E * PAD, K) if x_copy else (0,), dtype=op_dtype)
    return x.new_empty((rows, N), dtype=out_dtype), xs


@torch.library.custom_op("cvmm_b200::backward_x", mutates_args=())
def backward_x(g: torch.Tensor, g_index: Optional[torch.Tensor], g_div: int, out_index: Optional[torch.Tensor],
               offsets: torch.Tensor, keys: torch.Tensor, out_dtype: torch.dtype, op_dtype: torch.dtype,
               w: Optional[torch.Tensor], x: Optional[torch.Tensor], g_pad_start: Optional[torch.Tensor],
               out_pad_start: Optional[torch.Tensor], n_routes: int, x_div: int) -> tuple[torch.Tensor, torch.Tensor]:
    res = ops.backward_x(g, g_index, g_div, out_index, offsets, keys, out_dtype, op_dtype, w=w, x=x,
                         g_pad_start=g_pad_start, out_pad_start=out_pad_start, n_routes=n_routes, x_div=x_div)
    if w is None:
        return res, torch.empty(0, dtype=torch.float32, device=g.device)
    return res


@backward_x.register_fake
def _(g, g_index, g_div, out_index, offsets, keys, out_dtype, op_dtype, w, x, g_pad_start, out_pad_start,
      n_routes, x_div):
    E, K, N = keys.shape
    rows = n_routes + E * PAD if out_pad_start is not None else n_routes
    return (g.new_empty((rows, K), dtype=out_dtype),
            g.new_empty((n_routes if w is not None else 0,), dtype=torch.float32))


@torch.library.custom_op("cvmm_b200::backward_w", mutates_args=())
def backward_w(x: torch.Tensor, x_index: Optional[torch.Tensor], x_div: int, g: torch.Tensor,
               g_index: Optional[torch.Tensor], g_div: int, offsets: torch.Tensor, n_experts: int,
               op_dtype: torch.dtype, w: Optional[torch.Tensor], w_index: Optional[torch.Tensor],
               g_pad_start: Optional[torch.Tensor], x_pad_start: Optional[torch.Tensor],
               n_routes: int) -> torch.Tensor:
    return ops.backward_w(x, x_index, x_div, g, g_index, g_div, offsets, n_experts, op_dtype, w=w,
                          w_index=w_index, g_pad_start=g_pad_start, x_pad_start=x_pad_start, n_routes=n_routes)


@backward_w.register_fake
def _(x, x_index, x_div, g, g_index, g_div, offsets, n_experts, op_dtype, w, w_index, g_pad_start, x_pad_start,
      n_routes):
    return x.new_empty((n_experts, x.shape[-1], g.shape[-1]), dtype=torch.float32)


# ------------------------------------------------------------------ sigma-MoE layer pieces
@torch.library.custom_op("cvmm_b200::forward_gelu", mutates_args=())
def forward_gelu(x: torch.Tensor, sel_index: torch.Tensor, offsets: torch.Tensor, keys: torch.Tensor,
                 out_index: Optional[torch.Tensor], op_dtype: torch.dtype,
                 x_copy: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    xs = None
    if x_copy:
        xs = torch.empty((sel_index.numel() + keys.shape[0] * PAD, x.shape[-1]), dtype=op_dtype, device=x.device)
    h, z = ops.forward_gelu(x, sel_index, offsets, keys, out_index, op_dtype, x_copy=xs)
    return h, z, (xs if xs is not None else torch.empty(0, dtype=op_dtype, device=x.device))


@forward_gelu.register_fake
def _(x, sel_index, offsets, keys, out_index, op_dtype, x_copy):
    E, K, N = keys.shape
    R = sel_index.numel()
    return (x.new_empty((R, N), dtype=op_dtype), x.new_empty((R, N), dtype=op_dtype),
            x.new_empty((R + E * PAD, K) if x_copy else (0,), dtype=op_dtype))


@torch.library.custom_op("cvmm_b200::gelu_backward", mutates_args=())
def gelu_backward(grad: torch.Tensor, pre_act: torch.Tensor) -> torch.Tensor:
    return ops.gelu_backward(grad, pre_act)


@gelu_backward.register_fake
def _(grad, pre_act):
    return torch.empty_like(pre_act)


@torch.library.custom_op("cvmm_b200::router_topk", mutates_args=())
def router_topk(logits: torch.Tensor, top_k: int, renormalize: bool) -> tuple[torch.Tensor, torch.Tensor]:
    return ops.router_topk(logits, top_k, renormalize)


@router_topk.register_fake
def _(logits, top_k, renormalize):
    shape = (*logits.shape[:-1], top_k)
    return logits.new_empty(shape, dtype=torch.float32), logits.new_empty(shape, dtype=torch.int64)


# ------------------------------------------------------------------ the reference's op schema
@torch.library.custom_op("cvmm_b200::cvmm_triton", mutates_args=())
def cvmm_triton(x: torch.Tensor, sel_index: torch.Tensor, sel: torch.Tensor, keys: torch.Tensor,
                out_dtype: torch.dtype, out_index: torch.Tensor, op_dtype: torch.dtype) -> torch.Tensor:
    n_experts = keys.shape[0]
    offsets = ops.expert_offsets(sel, n_experts)
    oi = None if (out_index.numel() == 1 and int(out_index.reshape(-1)[0]) == -1) else out_index
    if op_dtype != torch.float32 and keys.dtype != op_dtype:
        keys = ops.cast(keys, op_dtype)
    out = ops.forward(x, sel_index, offsets, keys, oi, out_dtype, op_dtype)
    return out.view(*sel.shape, keys.shape[-1])


@cvmm_triton.register_fake
def _cvmm_triton_fake(x, sel_index, sel, keys, out_dtype, out_index, op_dtype):
    return x.new_empty((*sel.shape, keys.shape[-1]), dtype=out_dtype)


# ------------------------------------------------------------------ the calls CVMM makes
class _Calls:
    """The operations ``api.CVMM`` and the selector helpers call, with the
    signatures of ``ops.py``. Under torch.compile (tracing) every call goes
    through the registered custom op above, so the compiled graph holds the
    CVMM operators with their fake implementations and no graph break; in
    eager mode the same implementation runs without the dispatcher round
    trip. Both run the same native code on the same arguments."""

    PAD_ROWS = PAD

    @staticmethod
    def _tracing() -> bool:
        return torch.compiler.is_compiling()

    def sel_prepare(self, sel, top_k, route_input):
        if self._tracing():
            raw, ssel, si, oi = torch.ops.cvmm_b200.sel_prepare(sel, top_k, route_input)
            return raw, ssel, si, (None if route_input else oi)
        return ops.sel_prepare(sel, top_k, route_input)

    def expert_offsets(self, sorted_sel, n_experts):
        if self._tracing():
            return torch.ops.cvmm_b200.expert_offsets(sorted_sel, n_experts)
        return ops.expert_offsets(sorted_sel, n_experts)

    def pad_starts(self, offsets, n_experts):
        if self._tracing():
            return torch.ops.cvmm_b200.pad_starts(offsets, n_experts)
        return ops.pad_starts(offsets, n_experts)

    def cast(self, src, dtype, ahead=False):
        if self._tracing():
            return torch.ops.cvmm_b200.cast(src, dtype)
        return ops.cast(src, dtype, ahead=ahead)

    def sort_rows_padded(self, src, index, div, sorted_sel, offsets, n_experts, dtype=None, scale=None,
                         route_rows=False, pad_start=None):
        if self._tracing():
            # A custom op may not return its input, so traced graphs recompute
            # the pad starts instead of reusing pad_start.
            if route_rows:
                return torch.ops.cvmm_b200.sort_rows_padded_rows(src, index, div, sorted_sel, offsets, n_experts,
                                                                 dtype, scale)
            return torch.ops.cvmm_b200.sort_rows_padded(src, index, div, sorted_sel, offsets, n_experts, dtype, scale)
        return ops.sort_rows_padded(src, index, div, sorted_sel, offsets, n_experts, dtype=dtype, scale=scale,
                                    route_rows=route_rows, pad_start=pad_start)

    def padded_route_rows(self, route, sorted_sel, offsets, pad_start):
        if self._tracing():
            return torch.ops.cvmm_b200.padded_route_rows(route, sorted_sel, offsets, pad_start)
        return ops.padded_route_rows(route, sorted_sel, offsets, pad_start)

    def weighted_combine(self, y, w, out_dtype, y_rows=None):
        if self._tracing():
            return torch.ops.cvmm_b200.weighted_combine(y, w, out_dtype, y_rows)
        return ops.weighted_combine(y, w, out_dtype, y_rows=y_rows)

    def sum_routes(self, src, top_k, out_dtype, src_rows=None):
        if self._tracing():
            return torch.ops.cvmm_b200.sum_routes(src, top_k, out_dtype, src_rows)
        return ops.sum_routes(src, top_k, out_dtype, src_rows=src_rows)

    def weighted_token_backward(self, route_grad, w, x, need_x, need_sel, x_dtype):
        if self._tracing():
            gx, gsel = torch.ops.cvmm_b200.weighted_token_backward(route_grad, w, x, need_x, need_sel, x_dtype)
            return (gx if need_x else None), (gsel if need_sel else None)
        return ops.weighted_token_backward(route_grad, w, x, need_x, need_sel, x_dtype)

    def forward(self, x, sel_index, offsets, keys, out_index, out_dtype, op_dtype, x_pad_start=None,
                out_pad_start=None, x_copy=False):
        """Returns out, or (out, x_copy) when x_copy is requested."""
        if self._tracing():
            out, xs = torch.ops.cvmm_b200.forward(x, sel_index, offsets, keys, out_index, out_dtype, op_dtype,
                                                  x_pad_start, out_pad_start, bool(x_copy))
            return (out, xs) if x_copy else out
        xs = None
        if x_copy:
            xs = torch.empty((sel_index.numel() + keys.shape[0] * PAD, x.shape[-1]), dtype=op_dtype, device=x.device)
        out = ops.forward(x, sel_index, offsets, keys, out_index, out_dtype, op_dtype, x_pad_start=x_pad_start,
                          out_pad_start=out_pad_start, x_copy=xs)
        return (out, xs) if x_copy else out

    def backward_x(self, g, g_index, g_div, out_index, offsets, keys, out_dtype, op_dtype, w=None, x=None,
                   g_pad_start=None, out_pad_start=None, n_routes=None, x_div=1):
        if n_routes is None:
            n_routes = out_index.numel()
        if self._tracing():
            out, gsel = torch.ops.cvmm_b200.backward_x(g, g_index, g_div, out_index, offsets, keys, out_dtype,
                                                       op_dtype, w, x, g_pad_start, out_pad_start, int(n_routes),
                                                       int(x_div))
            return out if w is None else (out, gsel)
        return ops.backward_x(g, g_index, g_div, out_index, offsets, keys, out_dtype, op_dtype, w=w, x=x,
                              g_pad_start=g_pad_start, out_pad_start=out_pad_start, n_routes=n_routes, x_div=x_div)

    def backward_w(self, x, x_index, x_div, g, g_index, g_div, offsets, n_experts, op_dtype, w=None, w_index=None,
                   g_pad_start=None, x_pad_start=None, n_routes=None):
        if n_routes is None:
            n_routes = x_index.numel()
        if self._tracing():
            return torch.ops.cvmm_b200.backward_w(x, x_index, x_div, g, g_index, g_div, offsets, n_experts,
                                                  op_dtype, w, w_index, g_pad_start, x_pad_start, int(n_routes))
        return ops.backward_w(x, x_index, x_div, g, g_index, g_div, offsets, n_experts, op_dtype, w=w,
                              w_index=w_index, g_pad_start=g_pad_start, x_pad_start=x_pad_start, n_routes=n_routes)

    def forward_gelu(self, x, sel_index, offsets, keys, out_index, op_dtype, x_copy=False):
        """Returns (h, z, x_copy or None)."""
        if self._tracing():
            h, z, xs = torch.ops.cvmm_b200.forward_gelu(x, sel_index, offsets, keys, out_index, op_dtype,
                                                        bool(x_copy))
            return h, z, (xs if x_copy else None)
        xs = None
        if x_copy:
            xs = torch.empty((sel_index.numel() + keys.shape[0] * PAD, x.shape[-1]), dtype=op_dtype, device=x.device)
        h, z = ops.forward_gelu(x, sel_index, offsets, keys, out_index, op_dtype, x_copy=xs)
        return h, z, xs

    def gelu_backward(self, grad, pre_act):
        if self._tracing():
            return torch.ops.cvmm_b200.gelu_backward(grad, pre_act)
        return ops.gelu_backward(grad, pre_act)

    def router_topk(self, logits, top_k, renormalize=True):
        if self._tracing():
            return torch.ops.cvmm_b200.router_topk(logits, top_k, renormalize)
        return ops.router_topk(logits, top_k, renormalize)


calls = _Calls()
