"""The reference's own correctness suite (test_cvmm_correctness.py), run against
this implementation through the drop-in module, with a plain PyTorch fp32
reference of the same op and the reference's tolerances."""
import pytest
import torch

import cvmm_codex_b200.api as cvmm_module
from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2

pytestmark = pytest.mark.gpu


def torch_fp32_reference(x, sel, keys, weights=None):
    """Per-route product in fp32 with autograd (same math as the reference's oracle)."""
    kw = keys.float()[sel]
    if x.shape[:-1] == sel.shape:
        y = torch.einsum("...kd,...kdn->...kn", x.float(), kw)
    else:
        y = torch.einsum("...d,...kdn->...kn", x.float(), kw)
    if weights is not None:
        y = torch.einsum("...k,...kn->...n", weights.float(), y)
    return y


def _check(weighted, route_input=False):
    torch.manual_seed(1234 + int(weighted) + 17 * int(route_input))
    b, t, d, out_d, n_experts, top_k = 3, 5, 16, 11, 7, 3
    x_shape = (b, t, top_k, d) if route_input else (b, t, d)
    x = torch.randn(*x_shape, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    keys = torch.randn(n_experts, d, out_d, device="cuda", dtype=torch.float32, requires_grad=True)
    sel = torch.randint(0, n_experts, (b, t, top_k), device="cuda")
    w = torch.randn(b, t, top_k, device="cuda", requires_grad=True) if weighted else None
    sel2 = cvmm_prepare_sel2(sel, w, route_input=route_input)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        actual = cvmm(x, sel2, keys)
    expected = torch_fp32_reference(x, sel, keys, w)
    rt, at = (5e-2, 1e-1) if route_input else (2e-2, 2e-2)
    torch.testing.assert_close(actual.float(), expected.float(), rtol=rt, atol=at)
    grad = torch.randn_like(actual.float())
    actual.backward(grad.to(actual.dtype))
    got = [x.grad.float(), keys.grad.float()] + ([w.grad.float()] if weighted else [])
    xr = x.detach().clone().requires_grad_(True)
    kr = keys.detach().clone().requires_grad_(True)
    wr = None if w is None else w.detach().clone().requires_grad_(True)
    torch_fp32_reference(xr, sel, kr, wr).backward(grad)
    want = [xr.grad.float(), kr.grad.float()] + ([wr.grad.float()] if weighted else [])
    rt, at = (6e-2, 1e-1) if route_input else (3e-2, 3e-2)
    for a, e in zip(got, want):
        torch.testing.assert_close(a, e, rtol=rt, atol=at)


def test_unweighted():
    _check(False)


def test_weighted():
    _check(True)


def test_weighted_route_input():
    _check(True, route_input=True)


def test_top32_lowmem_unweighted():
    torch.manual_seed(2026)
    b, t, d, out_d, n_experts, top_k = 2, 5, 32, 16, 64, 32
    x = torch.randn(b, t, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    keys = torch.randn(n_experts, d, out_d, device="cuda", requires_grad=True)
    sel = torch.randint(0, n_experts, (b, t, top_k), device="cuda")
    old = cvmm_module.cvmm_lowmem_chunk_size
    cvmm_module.cvmm_lowmem_chunk_size = 0
    try:
        sel2 = cvmm_prepare_sel2(sel)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            actual = cvmm(x, sel2, keys)
        torch.testing.assert_close(actual.float(), torch_fp32_reference(x, sel, keys).float(),
                                   rtol=5e-2, atol=1e-1)
        grad = torch.randn_like(actual.float())
        actual.backward(grad.to(actual.dtype))
        xr = x.detach().clone().requires_grad_(True)
        kr = keys.detach().clone().requires_grad_(True)
        torch_fp32_reference(xr, sel, kr).backward(grad)
        torch.testing.assert_close(x.grad.float(), xr.grad.float(), rtol=3e-1, atol=6e-1)
        torch.testing.assert_close(keys.grad.float(), kr.grad.float(), rtol=1e-1, atol=1e-1)
    finally:
        cvmm_module.cvmm_lowmem_chunk_size = old


def test_weighted_route_input_reused_selector():
    torch.manual_seed(1251)
    b, t, d, out_d, n_experts, top_k = 3, 5, 16, 11, 7, 3
    x = torch.randn(b, t, top_k, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    keys = torch.randn(n_experts, d, out_d, device="cuda", requires_grad=True)
    sel = torch.randint(0, n_experts, (b, t, top_k), device="cuda")
    w = torch.randn(b, t, top_k, device="cuda", requires_grad=True)
    reused = cvmm_prepare_sel2(cvmm_prepare_sel2(sel), w, route_input=True)
    fresh = cvmm_prepare_sel2(sel, w, route_input=True)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        a = cvmm(x, reused, keys)
        e = cvmm(x, fresh, keys)
    torch.testing.assert_close(a.float(), e.float(), rtol=0, atol=0)


def test_reference_op_schema():
    """cvmm_b200::cvmm_triton keeps mylib::cvmm_triton's schema and -1 out_index convention."""
    cvmm_module.create_kernels()
    torch.manual_seed(5)
    x = torch.randn(40, 24, device="cuda", dtype=torch.bfloat16)
    keys = torch.randn(5, 24, 16, device="cuda")
    sel = torch.randint(0, 5, (10, 4), device="cuda")
    s = cvmm_prepare_sel2(sel, route_input=True)
    out = torch.ops.cvmm_b200.cvmm_triton(x, s.sel_index, s.sel, keys, torch.bfloat16,
                                          torch.tensor(-1, device="cuda"), torch.bfloat16)
    assert out.shape == (10, 4, 16) and out.dtype == torch.bfloat16
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        ref = cvmm(x, s, keys)
    torch.testing.assert_close(out.float(), ref.float(), rtol=0, atol=0)
