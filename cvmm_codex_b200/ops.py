"""Host-side operators: allocate outputs and scratch through torch, call the C ABI.

Each function here is one stream-ordered launch sequence of libcvmm_sm100.so on
the tensors' CUDA device. They never synchronise the host. The same functions
are registered as torch custom ops (namespace ``cvmm_b200``) with fake
implementations so that torch.compile can trace through CVMM.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import check, dtype_code, ptr


# Kernels each native entry point launches (for launch accounting).
KERNELS_PER_CALL = {
    "cvmm_sel_prepare": 1, "cvmm_expert_offsets": 1, "cvmm_forward": 2, "cvmm_backward_x": 2,
    "cvmm_backward_w": 4, "cvmm_weighted_combine": 1, "cvmm_sum_routes": 1,
    "cvmm_weighted_token_backward": 1, "cvmm_cast": 1, "cvmm_sort_rows_padded": 2, "cvmm_sort_rows_padded_ex": 2, "cvmm_pad_starts": 1,
    "cvmm_forward_gelu": 1, "cvmm_gelu_backward": 1, "cvmm_router_topk": 1, "cvmm_padded_route_rows": 1,
}


class Recorder:
    """Optional per-call CUDA-event timing and launch counting of the native
    calls, used by the benchmark: events are recorded on the launching stream
    around every library call made while the recorder is active."""

    def __init__(self):
        self.events = {}
        self.launches = 0
        self.calls = 0
        self.steps = 0  # times the recorder was entered

    def __enter__(self):
        global _recorder
        self.steps += 1
        self._prev = _recorder
        _recorder = self
        return self

    def __exit__(self, *exc):
        global _recorder
        _recorder = self._prev
        return False

    def summary(self):
        """{name: (calls, total_ms)} after a synchronize."""
        out = {}
        for name, evs in self.events.items():
            out[name] = (len(evs), sum(a.elapsed_time(b) for a, b in evs))
        return out


_recorder = None


def _invoke(name, fn, *args, kernels=None):
    rec = _recorder
    if rec is None:
        return fn(*args)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    rc = fn(*args)
    b.record()
    rec.events.setdefault(name, []).append((a, b))
    rec.launches += KERNELS_PER_CALL.get(name, 1) if kernels is None else kernels
    rec.calls += 1
    return rc


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("cvmm_codex_b200 runs on CUDA tensors only (no CPU path)")


def _rows(t: torch.Tensor) -> torch.Tensor:
    """2-D row-major view [rows, cols] with unit column stride."""
    t2 = t.reshape(-1, t.shape[-1]) if t.dim() != 2 else t
    if t2.stride(-1) != 1 or (t2.shape[0] > 1 and t2.stride(0) < t2.shape[1]):
        t2 = t2.contiguous()
    return t2


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


class _Device:
    """Makes the tensor's device current for the duration of a native call."""

    def __init__(self, device: torch.device):
        self.device = device
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.device.index:
            self.prev = cur
            torch.cuda.set_device(self.device)
        return _lib.stream_of(self.device)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


# ------------------------------------------------------------------ selector prep
def sel_prepare(sel: torch.Tensor, top_k: int, route_input: bool):
    """Stable expert sort of routes (reference cvmm_prepare_sel2, cvmm.py:1786-1803).

    Returns (raw_sel int32, sorted_sel int32, sel_index int64, out_index int64
    or None), all flat [n_routes]."""
    _require_cuda(sel)
    lib = _lib.load()
    flat = sel.reshape(-1)
    if flat.dtype not in (torch.int64, torch.int32):
        flat = flat.to(torch.int64)
    flat = flat.contiguous()
    n = flat.numel()
    dev = flat.device
    raw = torch.empty(n, dtype=torch.int32, device=dev)
    ssel = torch.empty(n, dtype=torch.int32, device=dev)
    sel_index = torch.empty(n, dtype=torch.int64, device=dev)
    out_index = None if route_input else torch.empty(n, dtype=torch.int64, device=dev)
    ws = _ws(lib.cvmm_sel_prepare_workspace_size(n), dev)
    with _Device(dev) as stream:
        rc = _invoke("cvmm_sel_prepare", lib.cvmm_sel_prepare, ptr(flat), dtype_code(flat.dtype), n, int(top_k), int(route_input),
                                  ptr(raw), ptr(ssel), ptr(sel_index), ptr(out_index), ptr(ws),
                                  ws.numel(), stream)
    check(rc, "cvmm_sel_prepare")
    return raw, ssel, sel_index, out_index


def expert_offsets(sorted_sel: torch.Tensor, n_experts: int) -> torch.Tensor:
    """Inclusive end offsets per expert (reference _cvmm_expert_offsets, cvmm.py:68-78)."""
    _require_cuda(sorted_sel)
    lib = _lib.load()
    s = sorted_sel.reshape(-1)
    if s.dtype != torch.int32:
        s = s.to(torch.int32)
    s = s.contiguous()
    out = torch.empty(int(n_experts), dtype=torch.int64, device=s.device)
    with _Device(s.device) as stream:
        rc = _invoke("cvmm_expert_offsets", lib.cvmm_expert_offsets, ptr(s), s.numel(), int(n_experts), ptr(out), stream)
    check(rc, "cvmm_expert_offsets")
    return out


# ------------------------------------------------------------------ GEMMs
ROW_PLAN_EXPERTS = 1024  # kRowPlanExperts: tensor-core row GEMMs build their tile table in-kernel


def _row_gemm_launches(op_dtype: torch.dtype, n_experts: int) -> int:
    return 1 if op_dtype != torch.float32 and n_experts <= ROW_PLAN_EXPERTS else 2

def _gemm_ws(lib, n_routes, n_experts, dev, m_dim=0, n_dim=0, op_dtype=torch.bfloat16):
    return _ws(lib.cvmm_gemm_workspace_size(n_routes, n_experts, m_dim, n_dim, 0, 0,
                                            dtype_code(op_dtype), 0), dev)


def forward(x: torch.Tensor, sel_index: torch.Tensor, offsets: torch.Tensor, keys: torch.Tensor,
            out_index: Optional[torch.Tensor], out_dtype: torch.dtype,
            op_dtype: torch.dtype, x_pad_start: Optional[torch.Tensor] = None,
            out_pad_start: Optional[torch.Tensor] = None, x_copy: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Y[row_p] = x[sel_index[p]] @ keys[e_p] for every sorted route p; Y is [R, N]
    (reference cvmm_triton, cvmm.py:815-867). With x_pad_start, x is the
    expert-padded sorted layout from sort_rows_padded; with out_pad_start, Y is
    returned in that layout ([R + E*PAD_ROWS, N], read through padded_route_rows).
    With x_copy ([R + E*PAD_ROWS, K], op dtype), the forward also writes the
    expert-padded sorted copy of the x rows it gathers there."""
    _require_cuda(x, sel_index, offsets, keys, out_index)
    lib = _lib.load()
    x2 = _rows(x)
    n_routes = sel_index.numel()
    E, K, N = keys.shape
    if x2.shape[1] != K:
        raise ValueError(f"cvmm: x feature size {x2.shape[1]} != keys.shape[1] {K}")
    out_rows = n_routes + E * PAD_ROWS if out_pad_start is not None else n_routes
    out = torch.empty((out_rows, N), dtype=out_dtype, device=x.device)
    ws = _gemm_ws(lib, n_routes, E, x.device)
    with _Device(x.device) as stream:
        rc = _invoke("cvmm_forward", lib.cvmm_forward, ptr(x2), dtype_code(x2.dtype), x2.shape[0], x2.stride(0),
                              ptr(sel_index), ptr(out_index), ptr(offsets), n_routes,
                              ptr(keys), dtype_code(keys.dtype), E, K, N,
                              keys.stride(0), keys.stride(1), keys.stride(2),
                              ptr(out), dtype_code(out_dtype), out.stride(0), dtype_code(op_dtype),
                              ptr(x_pad_start), ptr(out_pad_start), ptr(x_copy), ptr(ws), ws.numel(), stream,
                              kernels=_row_gemm_launches(op_dtype, E))
    check(rc, "cvmm_forward")
    return out


def weighted_combine(y: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype,
                     y_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_j w[t, j] * y[row(t*k + j)] with w cast to y's dtype (cvmm.py:1543-1545);
    row(r) = y_rows[r] (padded sorted y) or r."""
    _require_cuda(y, w)
    lib = _lib.load()
    k = w.shape[-1]
    w2 = w.reshape(-1).contiguous()
    T = w2.numel() // k
    N = y.shape[-1]
    y2 = y.reshape(-1, N).contiguous()
    out = torch.empty((T, N), dtype=out_dtype, device=y.device)
    with _Device(y.device) as stream:
        rc = _invoke("cvmm_weighted_combine", lib.cvmm_weighted_combine, ptr(y2), dtype_code(y2.dtype), ptr(w2), dtype_code(w2.dtype),
                                       ptr(out), dtype_code(out_dtype), T, k, N, ptr(y_rows), stream)
    check(rc, "cvmm_weighted_combine")
    return out


def sum_routes(src: torch.Tensor, top_k: int, out_dtype: torch.dtype,
               src_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[t] = sum_j src[row(t*k + j)] (cvmm.py:1223); row(r) = src_rows[r] or r."""
    lib = _lib.load()
    d = src.shape[-1]
    s2 = src.reshape(-1, d).contiguous()
    T = (s2.shape[0] if src_rows is None else src_rows.numel()) // top_k
    out = torch.empty((T, d), dtype=out_dtype, device=src.device)
    with _Device(src.device) as stream:
        rc = _invoke("cvmm_sum_routes", lib.cvmm_sum_routes, ptr(s2), dtype_code(s2.dtype), ptr(out), dtype_code(out_dtype),
                                 T, int(top_k), d, ptr(src_rows), stream)
    check(rc, "cvmm_sum_routes")
    return out


def backward_x(g: torch.Tensor, g_index: Optional[torch.Tensor], g_div: int, out_index: torch.Tensor,
               offsets: torch.Tensor, keys: torch.Tensor, out_dtype: torch.dtype,
               op_dtype: torch.dtype, w: Optional[torch.Tensor] = None,
               x: Optional[torch.Tensor] = None, g_pad_start: Optional[torch.Tensor] = None,
               out_pad_start: Optional[torch.Tensor] = None, n_routes: Optional[int] = None, x_div: int = 1):
    """Route gradients a_p = g[g_index[p] // g_div] @ keys[e_p]^T stored at out_index[p].

    Plain (w is None): returns out [R, d_in]. Weighted route-shaped input (w and x
    given): returns (grad_x [R, d_in], grad_sel fp32 [R]) with the reference's
    fused rounding (cvmm.py:1073-1105). With g_pad_start, g is the expert-padded
    sorted layout from sort_rows_padded and g_index is unused; with out_pad_start
    the output is returned in that layout (out_index may be None, then pass n_routes)."""
    _require_cuda(g, g_index, out_index, offsets, keys, w, x)
    lib = _lib.load()
    g2 = _rows(g)
    n_routes = out_index.numel() if n_routes is None else int(n_routes)
    E, K, N = keys.shape
    out_rows = n_routes + E * PAD_ROWS if out_pad_start is not None else n_routes
    out = torch.empty((out_rows, K), dtype=out_dtype, device=g.device)
    mode = 0
    gsel = None
    x2 = None
    w2 = None
    if w is not None:
        mode = 1
        gsel = torch.zeros(n_routes, dtype=torch.float32, device=g.device)
        x2 = _rows(x)
        w2 = w.reshape(-1).contiguous()
    ws = _gemm_ws(lib, n_routes, E, g.device)
    with _Device(g.device) as stream:
        rc = _invoke("cvmm_backward_x", lib.cvmm_backward_x, ptr(g2), dtype_code(g2.dtype), g2.stride(0), ptr(g_index), int(g_div),
                                 ptr(out_index), ptr(offsets), n_routes, ptr(keys),
                                 dtype_code(keys.dtype), E, K, N, keys.stride(0), keys.stride(1),
                                 keys.stride(2), ptr(out), dtype_code(out_dtype), out.stride(0), mode,
                                 ptr(w2), dtype_code(w2.dtype) if w2 is not None else 0,
                                 ptr(x2), dtype_code(x2.dtype) if x2 is not None else 0,
                                 x2.stride(0) if x2 is not None else 0, int(x_div), ptr(gsel),
                                 dtype_code(op_dtype), ptr(g_pad_start), ptr(out_pad_start), ptr(ws), ws.numel(), stream,
                                 kernels=_row_gemm_launches(op_dtype, E))
    check(rc, "cvmm_backward_x")
    return out if mode == 0 else (out, gsel)


def backward_w(x: torch.Tensor, x_index: torch.Tensor, x_div: int, g: torch.Tensor,
               g_index: Optional[torch.Tensor], g_div: int, offsets: torch.Tensor, n_experts: int,
               op_dtype: torch.dtype, w: Optional[torch.Tensor] = None,
               w_index: Optional[torch.Tensor] = None,
               g_pad_start: Optional[torch.Tensor] = None,
               x_pad_start: Optional[torch.Tensor] = None,
               n_routes: Optional[int] = None) -> torch.Tensor:
    """fp32 grad_keys[e] = sum_{p in seg e} x[x_index[p]//x_div]^T (w-scaled) g[g_index[p]//g_div]
    (reference grouped grad-W kernels, cvmm.py:424-604). x_pad_start / g_pad_start:
    x / g is the expert-padded sorted layout (a padded g already carries the
    route weights); n_routes is required when x_index is None."""
    _require_cuda(x, x_index, g, g_index, offsets, w, w_index)
    lib = _lib.load()
    x2 = _rows(x)
    g2 = _rows(g)
    n_routes = x_index.numel() if n_routes is None else int(n_routes)
    M, N = x2.shape[1], g2.shape[1]
    out = torch.empty((int(n_experts), M, N), dtype=torch.float32, device=x.device)
    w2 = None if w is None else w.reshape(-1).contiguous()
    ws = _gemm_ws(lib, n_routes, int(n_experts), x.device, M, N, op_dtype)
    with _Device(x.device) as stream:
        rc = _invoke("cvmm_backward_w", lib.cvmm_backward_w, ptr(x2), dtype_code(x2.dtype), x2.stride(0), ptr(x_index), int(x_div),
                                 ptr(g2), dtype_code(g2.dtype), g2.stride(0), ptr(g_index), int(g_div),
                                 ptr(w2), dtype_code(w2.dtype) if w2 is not None else 0, ptr(w_index),
                                 ptr(offsets), n_routes, int(n_experts), M, N, ptr(out),
                                 dtype_code(op_dtype), ptr(x_pad_start), ptr(g_pad_start), ptr(ws), ws.numel(),
                                 stream, kernels=lib.cvmm_backward_w_launches(
                                     n_routes, int(n_experts), M, N, dtype_code(op_dtype),
                                     int(x_pad_start is not None and g_pad_start is not None), int(w2 is not None)))
    check(rc, "cvmm_backward_w")
    return out


PAD_ROWS = 128  # CVMM_PAD_ROWS


def pad_starts(offsets: torch.Tensor, n_experts: int) -> torch.Tensor:
    """pad_start int32 [E] of the expert-padded sorted layout for these offsets."""
    _require_cuda(offsets)
    lib = _lib.load()
    out = torch.empty(int(n_experts), dtype=torch.int32, device=offsets.device)
    with _Device(offsets.device) as stream:
        rc = _invoke("cvmm_pad_starts", lib.cvmm_pad_starts, ptr(offsets), int(n_experts), ptr(out), stream)
    check(rc, "cvmm_pad_starts")
    return out


def sort_rows_padded(src: torch.Tensor, index: torch.Tensor, div: int, sorted_sel: torch.Tensor,
                     offsets: torch.Tensor, n_experts: int, dtype: Optional[torch.dtype] = None,
                     scale: Optional[torch.Tensor] = None, route_rows: bool = False,
                     pad_start: Optional[torch.Tensor] = None):
    """Expert-padded sorted copy of route rows (the reference's grouping copy,
    cvmm.py:338-360), rounded to `dtype` (default: src's) and, with `scale`,
    multiplied by the op-rounded scale[index[p]] and rounded again (cvmm.py:591-599).
    Returns (dst [n_routes + n_experts*PAD_ROWS, cols], pad_start int32 [E]).
    pad_start: the pad starts of these offsets, already made (by pad_starts or an
    earlier copy over the same selector); they are read, not recomputed.
    route_rows: also return the int32 [n_routes] map padded_route_rows would
    make (route_rows[index[p]] = padded row of p), written by the same launch."""
    _require_cuda(src, index, sorted_sel, offsets, scale, pad_start)
    lib = _lib.load()
    s2 = _rows(src)
    n_routes = index.numel()
    cols = s2.shape[1]
    ss = sorted_sel.reshape(-1)
    if ss.dtype != torch.int32:
        ss = ss.to(torch.int32)
    dtype = s2.dtype if dtype is None else dtype
    sc = None if scale is None else scale.reshape(-1).contiguous()
    dst = torch.empty((n_routes + int(n_experts) * PAD_ROWS, cols), dtype=dtype, device=s2.device)
    ready = pad_start is not None
    if ready:
        if pad_start.dtype != torch.int32 or pad_start.numel() != int(n_experts) or not pad_start.is_contiguous():
            raise ValueError("sort_rows_padded: pad_start must be a contiguous int32 [n_experts] tensor")
        pstart = pad_start
    else:
        pstart = torch.empty(int(n_experts), dtype=torch.int32, device=s2.device)
    rows = torch.empty(n_routes, dtype=torch.int32, device=s2.device) if route_rows else None
    with _Device(s2.device) as stream:
        if ready or route_rows:
            rc = _invoke("cvmm_sort_rows_padded_ex", lib.cvmm_sort_rows_padded_ex, ptr(s2), dtype_code(s2.dtype),
                         s2.stride(0), ptr(index), int(div), ptr(sc), dtype_code(sc.dtype) if sc is not None else 0,
                         ptr(ss), ptr(offsets), n_routes, int(n_experts), cols, ptr(dst), dtype_code(dtype),
                         ptr(pstart), int(ready), ptr(rows), stream, kernels=1 if ready else 2)
            name = "cvmm_sort_rows_padded_ex"
        else:
            rc = _invoke("cvmm_sort_rows_padded", lib.cvmm_sort_rows_padded, ptr(s2), dtype_code(s2.dtype),
                         s2.stride(0), ptr(index), int(div), ptr(sc), dtype_code(sc.dtype) if sc is not None else 0,
                         ptr(ss), ptr(offsets), n_routes, int(n_experts), cols,
                         ptr(dst), dtype_code(dtype), ptr(pstart), stream)
            name = "cvmm_sort_rows_padded"
    check(rc, name)
    return (dst, pstart, rows) if route_rows else (dst, pstart)


def padded_route_rows(route: torch.Tensor, sorted_sel: torch.Tensor, offsets: torch.Tensor,
                      pad_start: torch.Tensor) -> torch.Tensor:
    """rows[route[p]] = pad_start[e] + p - seg_begin(e): where each route's row
    lives in the expert-padded sorted layout (int32 [n_routes])."""
    _require_cuda(route, sorted_sel, offsets, pad_start)
    lib = _lib.load()
    n = route.numel()
    ss = sorted_sel.reshape(-1)
    if ss.dtype != torch.int32:
        ss = ss.to(torch.int32)
    rows = torch.empty(n, dtype=torch.int32, device=route.device)
    with _Device(route.device) as stream:
        rc = _invoke("cvmm_padded_route_rows", lib.cvmm_padded_route_rows, ptr(route), ptr(ss), ptr(offsets),
                     ptr(pad_start), n, offsets.numel(), ptr(rows), stream)
    check(rc, "cvmm_padded_route_rows")
    return rows


def weighted_token_backward(route_grad: torch.Tensor, w: torch.Tensor, x: torch.Tensor,
                            need_x: bool, need_sel: bool, x_dtype: torch.dtype):
    """Token-input weighted backward tail (cvmm.py:1737-1746): returns
    (grad_x [T, d] or None, grad_sel fp32 [T*k] or None)."""
    lib = _lib.load()
    k = w.shape[-1]
    w2 = w.reshape(-1).contiguous()
    T = w2.numel() // k
    d = route_grad.shape[-1]
    rg = route_grad.reshape(-1, d).contiguous()
    x2 = _rows(x).contiguous()
    gx = torch.empty((T, d), dtype=x_dtype, device=rg.device) if need_x else None
    gsel = torch.empty(T * k, dtype=torch.float32, device=rg.device) if need_sel else None
    with _Device(rg.device) as stream:
        rc = _invoke("cvmm_weighted_token_backward", lib.cvmm_weighted_token_backward, ptr(rg), dtype_code(rg.dtype), ptr(w2), dtype_code(w2.dtype),
                                              ptr(x2), dtype_code(x2.dtype), ptr(gx),
                                              dtype_code(x_dtype), ptr(gsel), T, k, d, stream)
    check(rc, "cvmm_weighted_token_backward")
    return gx, gsel


def cast(src: torch.Tensor, dtype: torch.dtype, ahead: bool = False) -> torch.Tensor:
    """Round-to-nearest-even dtype conversion on the device (e.g. fp32 keys -> bf16).
    ahead: the cast's loads may overlap the previous kernel of this library on
    the stream (cvmm_cast_ahead); only for a src none of this library's kernels write."""
    _require_cuda(src)
    lib = _lib.load()
    s = src.contiguous()
    out = torch.empty(s.shape, dtype=dtype, device=s.device)
    fn = lib.cvmm_cast_ahead if ahead else lib.cvmm_cast
    with _Device(s.device) as stream:
        rc = _invoke("cvmm_cast", fn, ptr(s), dtype_code(s.dtype), ptr(out), dtype_code(dtype), s.numel(), stream)
    check(rc, "cvmm_cast")
    return out


# ------------------------------------------------------------------ sigma-MoE layer pieces
def forward_gelu(x: torch.Tensor, sel_index: torch.Tensor, offsets: torch.Tensor, keys: torch.Tensor,
                 out_index: Optional[torch.Tensor], op_dtype: torch.dtype, x_copy: Optional[torch.Tensor] = None):
    """Up projection with GELU fused into the epilogue: returns (h, z) [R, N]
    with z = op(x[sel_index[p]] @ keys[e_p]) and h = gelu(z) (F.gelu, erf form)
    at row out_index[p] (or sel_index[p]); x_copy as in forward()."""
    _require_cuda(x, sel_index, offsets, keys, out_index)
    lib = _lib.load()
    x2 = _rows(x)
    n_routes = sel_index.numel()
    E, K, N = keys.shape
    if x2.shape[1] != K:
        raise ValueError(f"cvmm: x feature size {x2.shape[1]} != keys.shape[1] {K}")
    h = torch.empty((n_routes, N), dtype=op_dtype, device=x.device)
    z = torch.empty((n_routes, N), dtype=op_dtype, device=x.device)
    ws = _gemm_ws(lib, n_routes, E, x.device)
    with _Device(x.device) as stream:
        rc = _invoke("cvmm_forward_gelu", lib.cvmm_forward_gelu, ptr(x2), dtype_code(x2.dtype), x2.shape[0],
                     x2.stride(0), ptr(sel_index), ptr(out_index), ptr(offsets), n_routes,
                     ptr(keys), dtype_code(keys.dtype), E, K, N, keys.stride(0), keys.stride(1), keys.stride(2),
                     ptr(h), ptr(z), dtype_code(op_dtype), h.stride(0), dtype_code(op_dtype), ptr(x_copy),
                     ptr(ws), ws.numel(), stream, kernels=_row_gemm_launches(op_dtype, E))
    check(rc, "cvmm_forward_gelu")
    return h, z


def gelu_backward(grad: torch.Tensor, pre_act: torch.Tensor) -> torch.Tensor:
    """grad * gelu'(pre_act), elementwise (16-bit tensors of one dtype)."""
    _require_cuda(grad, pre_act)
    lib = _lib.load()
    g = grad.contiguous()
    z = pre_act.contiguous()
    if g.dtype != z.dtype:
        g = g.to(z.dtype)
    out = torch.empty_like(z)
    with _Device(z.device) as stream:
        rc = _invoke("cvmm_gelu_backward", lib.cvmm_gelu_backward, ptr(g), ptr(z), ptr(out), dtype_code(z.dtype),
                     z.numel(), stream)
    check(rc, "cvmm_gelu_backward")
    return out


def router_topk(logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """(weights fp32 [..., k], sel int64 [..., k]): top-k of softmax(float(logits))
    in descending order, optionally renormalised to sum to one (the sigma-MoE
    router, benchmark_ffn_moe.py:89-92)."""
    _require_cuda(logits)
    lib = _lib.load()
    lg = logits.contiguous()
    E = lg.shape[-1]
    T = lg.numel() // E
    sel = torch.empty((*lg.shape[:-1], int(top_k)), dtype=torch.int64, device=lg.device)
    w = torch.empty((*lg.shape[:-1], int(top_k)), dtype=torch.float32, device=lg.device)
    with _Device(lg.device) as stream:
        rc = _invoke("cvmm_router_topk", lib.cvmm_router_topk, ptr(lg), dtype_code(lg.dtype), T, E, int(top_k),
                     int(bool(renormalize)), ptr(sel), ptr(w), stream)
    check(rc, "cvmm_router_topk")
    return w, sel
