"""Forward and backward on the GPU against the fp64 oracle and the reference's fixtures.

Tolerances:
  * against the oracle (exact math on op-dtype-rounded operands, float64):
    max-abs error relative to the largest magnitude <= 2e-2 for bf16/fp16
    arithmetic and <= 1e-3 for fp32 arithmetic (the contract's bounds), plus
    RMS error relative to the RMS <= 1e-2 / 1e-4;
  * against the reference's `_reference` outputs (fixtures): the reference's
    own per-tensor (atol, rtol) table (benchmark_correctness_original.py:47-66).
"""
import os

import numpy as np
import pytest
import torch

from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
from oracle import cvmm_oracle as O

pytestmark = pytest.mark.gpu
NUM = torch.load(os.path.join(os.path.dirname(__file__), "golden", "numerics.pt"))

REF_TOL = {  # (atol, rtol) per tensor, per dtype mode
    "float32": {"out": (2e-4, 2e-4), "x_grad": (5e-4, 5e-4), "keys_grad": (2e-3, 2e-3), "w_grad": (2e-3, 2e-3)},
    "bf16_amp": {"out": (1.5e-1, 6e-2), "x_grad": (2.5e-1, 8e-2), "keys_grad": (3.5e-1, 8e-2), "w_grad": (3.5e-1, 8e-2)},
    "bf16_params": {"out": (2.0e-1, 8e-2), "x_grad": (3.0e-1, 1e-1), "keys_grad": (3.5e-1, 1e-1), "w_grad": (3.5e-1, 1e-1)},
}
MAX_TOL = {"float32": 1e-3, "bfloat16": 2e-2, "float16": 2e-2}
RMS_TOL = {"float32": 1e-4, "bfloat16": 1e-2, "float16": 1e-2}


def run_case(x, keys, sel, w, grad, route_input, amp_dtype):
    x = x.cuda().requires_grad_(True)
    keys = keys.cuda().requires_grad_(True)
    sel = sel.cuda()
    wc = None if w is None else w.cuda().requires_grad_(True)
    sel2 = cvmm_prepare_sel2(sel, wc, route_input=route_input)
    if amp_dtype is not None:
        with torch.autocast(device_type="cuda", dtype=amp_dtype):
            out = cvmm(x, sel2, keys)
    else:
        out = cvmm(x, sel2, keys)
    out.backward(grad.cuda().to(out.dtype))
    return out, x.grad, keys.grad, None if wc is None else wc.grad


def _np(t):
    return None if t is None else t.detach().float().cpu().numpy().astype(np.float64)


def check_oracle(out, gx, gk, gw, x, keys, sel, w, grad, op):
    eo = O.forward(_np(x), sel.numpy(), _np(keys), _np(w), op=op)
    ex, ek, ew = O.backward(_np(x), sel.numpy(), _np(keys), _np(grad.to(out.dtype)), _np(w), op=op)
    pairs = [("out", out, eo), ("x_grad", gx, ex), ("keys_grad", gk, ek)]
    if w is not None:
        pairs.append(("w_grad", gw, ew))
    for name, a, e in pairs:
        a = _np(a)
        assert a.shape == e.shape, name
        assert O.rel_max_err(a, e) <= MAX_TOL[op], (name, O.rel_max_err(a, e))
        assert O.rel_rms_err(a, e) <= RMS_TOL[op], (name, O.rel_rms_err(a, e))


@pytest.mark.parametrize("key", sorted(NUM))
def test_reference_case_list(key):
    c = NUM[key]
    mode = c["mode"]
    amp = None if mode == "float32" else torch.bfloat16
    op = "float32" if mode == "float32" else "bfloat16"
    out, gx, gk, gw = run_case(c["x"], c["keys"], c["sel"], c["w"], c["grad"], c["route_input"], amp)
    # dtypes follow the reference: output in the op dtype, grads in the leaves' dtypes
    assert out.dtype == (torch.float32 if amp is None else torch.bfloat16)
    assert gx.dtype == c["x"].dtype and gk.dtype == c["keys"].dtype
    check_oracle(out, gx, gk, gw, c["x"], c["keys"], c["sel"], c["w"], c["grad"], op)
    tol = REF_TOL[mode]
    for name, a in (("out", out), ("x_grad", gx), ("keys_grad", gk), ("w_grad", gw)):
        if c[name] is None:
            continue
        at, rt = tol[name]
        torch.testing.assert_close(a.float().cpu(), c[name].float(), atol=at, rtol=rt)


@pytest.mark.parametrize("amp", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("weighted,route_input", [(False, False), (True, False), (True, True), (False, True)])
def test_aligned_tensor_core_shapes(amp, weighted, route_input):
    """Shapes whose rows meet the 16-byte cp.async fast path (d multiples of 8)."""
    g = torch.Generator().manual_seed(17 + weighted * 2 + route_input)
    T, k, E, d_in, d_out = 300, 4, 12, 192, 136
    x = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), generator=g).to(amp)
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    sel = torch.randint(0, E, (T, k), generator=g)
    w = torch.rand(T, k, generator=g) if weighted else None
    grad = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g)
    out, gx, gk, gw = run_case(x, keys, sel, w, grad, route_input, amp)
    check_oracle(out, gx, gk, gw, x, keys, sel, w, grad, "float16" if amp == torch.float16 else "bfloat16")


@pytest.mark.parametrize("d_in,d_out", [(64, 64), (128, 256), (256, 512), (72, 200), (1024, 128), (128, 1024)])
def test_tile_shapes(d_in, d_out):
    """Every N-tile variant (64/128/256), multi-tile N, K not a multiple of 64, ragged segments."""
    g = torch.Generator().manual_seed(d_in * 7 + d_out)
    T, k, E = 700, 3, 9
    x = torch.randn(T, d_in, generator=g).bfloat16()
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    sel = torch.randint(0, E, (T, k), generator=g)
    sel[:50] = 2  # one heavy expert: segments longer than several M tiles
    grad = torch.randn(T, k, d_out, generator=g)
    out, gx, gk, gw = run_case(x, keys, sel, None, grad, False, torch.bfloat16)
    check_oracle(out, gx, gk, gw, x, keys, sel, None, grad, "bfloat16")


def test_missing_experts_get_zero_grad():
    g = torch.Generator().manual_seed(3)
    T, k, E, d = 64, 2, 40, 32
    x = torch.randn(T, d, generator=g).bfloat16()
    keys = torch.randn(E, d, 24, generator=g)
    sel = torch.randint(0, 5, (T, k), generator=g) * 3  # experts 0,3,6,9,12 only
    grad = torch.randn(T, k, 24, generator=g)
    out, gx, gk, gw = run_case(x, keys, sel, None, grad, False, torch.bfloat16)
    used = set(sel.flatten().tolist())
    for e in range(E):
        if e not in used:
            assert torch.count_nonzero(gk[e]) == 0
    check_oracle(out, gx, gk, gw, x, keys, sel, None, grad, "bfloat16")


def test_top1_and_raw_selector():
    """A raw index tensor goes through cvmm_prepare_sel (route-indexed): x has one row per route."""
    g = torch.Generator().manual_seed(9)
    T, E, d, n = 333, 6, 40, 24
    x = torch.randn(T, d, generator=g).bfloat16().cuda().requires_grad_(True)
    keys = torch.randn(E, d, n, generator=g).cuda().requires_grad_(True)
    sel = torch.randint(0, E, (T,), generator=g).cuda()
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        out = cvmm(x, sel, keys)
    assert out.shape == (T, n)
    e = O.forward(_np(x), sel.cpu().numpy()[:, None], _np(keys), op="bfloat16").reshape(T, n)
    assert O.rel_max_err(_np(out), e) < 2e-2
    # Backward of the route-indexed selector path: grads of x and keys.
    grad = torch.randn(T, n, generator=g)
    out.backward(grad.cuda().to(out.dtype))
    gn = grad.to(out.dtype).float().double().numpy()[:, None, :]
    ex, ek, _ = O.backward(_np(x), sel.cpu().numpy()[:, None], _np(keys), gn, op="bfloat16")
    for a, e in ((x.grad, ex.reshape(T, d)), (keys.grad, ek)):
        assert O.rel_max_err(_np(a), e) < 2e-2
        assert O.rel_rms_err(_np(a), e) < 1e-2


def test_device_status_clean():
    from cvmm_codex_b200 import _lib
    code, where, aux = _lib.device_status(reset=True)
    assert code == 0, (code, where, aux)


@pytest.mark.parametrize("route_input,weighted,d_in,d_out", [
    (False, False, 256, 128), (True, True, 128, 256), (False, True, 64, 192), (True, False, 136, 72),
])
def test_sorted_operands_match_gathered_path_bitwise(route_input, weighted, d_in, d_out):
    """The expert-padded sorted copies change where operands are read from, not
    the arithmetic: results equal the row-gathered path bit for bit."""
    import cvmm_codex_b200.api as A
    g = torch.Generator().manual_seed(5)
    T, k, E = 700, 3, 9
    sel = torch.randint(0, E, (T, k), generator=g)
    sel[: T // 2, 0] = 2  # one expert with several tiles and split-K chunks
    x = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), generator=g).bfloat16()
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    w = torch.rand(T, k, generator=g) if weighted else None
    grad = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g)
    res = {}
    old = A.cvmm_sorted_operands
    try:
        for mode in (True, False):
            A.cvmm_sorted_operands = mode
            res[mode] = run_case(x, keys, sel, w, grad, route_input, torch.bfloat16)
    finally:
        A.cvmm_sorted_operands = old
    for i, (a, b) in enumerate(zip(res[True], res[False])):
        if a is None:
            assert b is None
            continue
        if i == 3:
            # The sel-weight grad is an fp32 sum of per-column-group partial dots
            # added with atomics; the dense path drains a tile with two epilogue
            # warp groups (two partials per row), the gathered path with one, so
            # only the fp32 summation order differs.
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6 * b.abs().max().item())
        else:
            assert torch.equal(a, b)


@pytest.mark.parametrize("route_input", [True, False])
def test_weighted_grad_gather_matches_scaled_copy_bitwise(route_input):
    """The weighted backward reads one unscaled sorted copy of the token grads
    in both GEMMs (weights applied in grad-W's shared memory), or a
    weight-scaled sorted copy in grad-W, or gathers and scales the token grad
    rows inside grad-W; all apply op(op(g) * op(w)) (cvmm.py:591-599) to the
    same operands in the same order, so every output is bit-identical."""
    import cvmm_codex_b200.api as A
    g = torch.Generator().manual_seed(8)
    T, k, E, d_in, d_out = 900, 4, 7, 64, 320
    sel = torch.randint(0, E, (T, k), generator=g)
    sel[: T // 2, 1] = 3  # one expert split into several chunks
    x = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), generator=g).bfloat16()
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    w = torch.rand(T, k, generator=g)
    grad = torch.randn(T, d_out, generator=g)
    res = {}
    old = (A.cvmm_weighted_shared_grad_copy, A.cvmm_weighted_grad_copy)
    try:
        # one unscaled copy shared by grad-W and grad-x; a weight-scaled copy
        # for grad-W; token grad rows gathered and scaled inside grad-W
        for mode in ((True, True), (False, True), (False, False)):
            A.cvmm_weighted_shared_grad_copy, A.cvmm_weighted_grad_copy = mode
            res[mode] = run_case(x, keys, sel, w, grad, route_input, torch.bfloat16)
    finally:
        A.cvmm_weighted_shared_grad_copy, A.cvmm_weighted_grad_copy = old
    for mode in ((False, True), (False, False)):
        for i, (a, b) in enumerate(zip(res[(True, True)], res[mode])):
            if i == 3:  # sel-weight grad: fp32 atomics of partial dots, order differs (see above)
                torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6 * b.abs().max().item())
            else:
                assert torch.equal(a, b), (mode, i)
    check_oracle(*res[(True, True)], x, keys, sel, w, grad, "bfloat16")


@pytest.mark.parametrize("n_experts,weighted", [(1024, False), (1100, False), (1024, True)])
def test_many_experts_tile_table_paths(n_experts, weighted):
    """Up to 1024 experts the tensor-core row GEMM derives its tile table from
    the offsets in the kernel; above that it reads the table build_tiles makes.
    Both, with most experts empty or holding a single route, against the oracle."""
    g = torch.Generator().manual_seed(17)
    T, k, d_in, d_out = 1500, 2, 64, 64
    x = torch.randn(T, d_in, generator=g)
    keys = torch.randn(n_experts, d_in, d_out, generator=g) / 8
    sel = torch.randint(0, n_experts, (T, k), generator=g)
    sel[:300, 0] = 7  # one expert with several 128-route tiles
    w = torch.rand(T, k, generator=g) if weighted else None
    grad = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g)
    out, gx, gk, gw = run_case(x.bfloat16(), keys, sel, w, grad, False, torch.bfloat16)
    check_oracle(out, gx, gk, gw, x.bfloat16(), keys, sel, w, grad, "bfloat16")


@pytest.mark.parametrize("weighted", [True, False])
def test_shared_head_rows_match_repeated_route_rows(weighted):
    """SwitchHead output projection: the 2 routes of each head read the head's
    value row. Passing the per-head rows [T, H, d] (the kernels index row
    route // 2) gives the same results as the reference's layout, the rows
    repeated per route with repeat_interleave [T, 2H, d]."""
    g = torch.Generator().manual_seed(21)
    T, H, rph, per, d, n = 400, 6, 2, 4, 64, 96
    E = H * per
    v = torch.randn(T, H, d, generator=g).bfloat16()
    keys = torch.randn(E, d, n, generator=g) / 8
    logits = torch.randn(T, H, per, generator=g)
    sel = (logits.topk(rph, dim=-1).indices + (torch.arange(H) * per).view(1, -1, 1)).reshape(T, H * rph)
    w = torch.rand(T, H * rph, generator=g) if weighted else None
    grad = torch.randn(*((T, n) if weighted else (T, H * rph, n)), generator=g)
    shared = run_case(v, keys, sel, w, grad, True, torch.bfloat16)
    vr = v.cuda().requires_grad_(True)
    rep = vr.repeat_interleave(rph, dim=1)
    kc = keys.cuda().requires_grad_(True)
    wc = None if w is None else w.cuda().requires_grad_(True)
    s2 = cvmm_prepare_sel2(sel.cuda(), wc, route_input=True)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        out = cvmm(rep, s2, kc)
    out.backward(grad.cuda().to(out.dtype))
    repeated = (out, vr.grad, kc.grad, None if wc is None else wc.grad)
    for name, a, b in zip(("out", "x_grad", "keys_grad", "w_grad"), shared, repeated):
        if a is None:
            assert b is None
            continue
        assert a.shape == b.shape, name
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-2, atol=1e-2 * b.float().abs().max().item())
        if name != "x_grad":
            assert torch.equal(a, b), name


@pytest.mark.parametrize("route_input,weighted", [(False, False), (True, True)])
def test_programmatic_launch_matches_plain_launch(route_input, weighted):
    """Programmatic dependent launch changes only when CTAs are scheduled: the
    outputs and gradients equal those of plain launches bit for bit (the
    sel-weight grad, an fp32 atomic sum, to rounding)."""
    from cvmm_codex_b200 import _lib
    lib = _lib.load()
    g = torch.Generator().manual_seed(31)
    T, k, E, d_in, d_out = 2000, 4, 16, 256, 512
    x = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), generator=g).bfloat16()
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    sel = torch.randint(0, E, (T, k), generator=g)
    w = torch.rand(T, k, generator=g) if weighted else None
    grad = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g)
    res = []
    prev = lib.cvmm_set_pdl(0)
    try:
        for pdl in (0, 1):
            lib.cvmm_set_pdl(pdl)
            res.append(run_case(x, keys, sel, w, grad, route_input, torch.bfloat16))
            torch.cuda.synchronize()
    finally:
        lib.cvmm_set_pdl(prev)
    (o0, gx0, gk0, gw0), (o1, gx1, gk1, gw1) = res
    for a, b in ((o0, o1), (gx0, gx1), (gk0, gk1)):
        assert torch.equal(a, b)
    if weighted:
        torch.testing.assert_close(gw0, gw1, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("route_input", [False, True])
def test_bf16_params_split_backward_matches_fp32_kernels(route_input, monkeypatch):
    """bf16 x and keys without autocast (the reference's bf16_params mode, fp32
    op dtype): the backward on the bf16 tensor cores with the fp32 grad split
    into two bf16 parts agrees with the fp32 SIMT kernels and with the fp64
    oracle (bf16 leaf grads: the bf16 bound)."""
    from cvmm_codex_b200 import api
    g = torch.Generator().manual_seed(41)
    T, k, E, d_in, d_out = 700, 4, 12, 256, 192
    x = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), generator=g).bfloat16()
    keys = (torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5).bfloat16()
    sel = torch.randint(0, E, (T, k), generator=g)
    grad = torch.randn(T, k, d_out, generator=g)
    res = {}
    for split in (True, False):
        monkeypatch.setattr(api, "cvmm_split_fp32_grad", split)
        res[split] = run_case(x, keys, sel, None, grad, route_input, None)
    for a, b in zip(res[True], res[False]):
        if a is None:
            continue
        assert a.dtype == b.dtype and a.shape == b.shape
        assert O.rel_max_err(_np(a), _np(b)) < 1e-2
    out, gx, gk, _ = res[True]
    assert out.dtype == torch.float32 and gx.dtype == torch.bfloat16 and gk.dtype == torch.bfloat16
    eo = O.forward(_np(x), sel.numpy(), _np(keys), None, op="float32")
    ex, ek, _ = O.backward(_np(x), sel.numpy(), _np(keys), _np(grad), None, op="float32")
    for name, a, e in (("out", out, eo), ("x_grad", gx, ex), ("keys_grad", gk, ek)):
        assert O.rel_max_err(_np(a), e) <= MAX_TOL["bfloat16"], name
        assert O.rel_rms_err(_np(a), e) <= RMS_TOL["bfloat16"], name


@pytest.mark.parametrize("n", [8, 1000, 4104, 64 * 1024 * 128, 148 * 8 * 256 * 4 * 8 + 24])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cast_ahead_matches_cast(n, dtype):
    """cvmm_cast_ahead (loads overlap the previous kernel, stores wait for it) gives
    cvmm_cast's result bit for bit, queued right behind a selector sort as in
    CVMM.forward; sizes cover the single pass, the grid-stride loop and the
    fallback for sizes that are not a multiple of 8."""
    from cvmm_codex_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(3)
    src = torch.randn(n, device="cuda", generator=g) * 3
    sel = torch.randint(0, 64, (16384, 4), device="cuda", generator=g)
    want = ops.cast(src, dtype)
    for _ in range(2):
        s = cvmm_prepare_sel2(sel)
        got = ops.cast(src, dtype, ahead=True)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert torch.equal(got, src.to(dtype))
        del s
