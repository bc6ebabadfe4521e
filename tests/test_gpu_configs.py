"""Full-size benchmark configurations on the GPU.

At these sizes the fp64 CPU oracle is too slow, so each configuration is
checked (a) against a plain PyTorch fp32 per-expert reference of the same op on
the GPU (operands rounded to bf16 exactly as the kernels do, TF32 off), and
(b) through size-independent properties: exact linearity under power-of-two
scaling, and the grad-W checksum sum_e dW_e = X_routes^T G_routes.
"""
import pytest
import torch

from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
from cvmm_codex_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

CONFIGS = ["cpu_plumbing", "ff_up_1024", "ff_down_1024_weighted", "switch_o_2048_h32_weighted",
           "stress_up_4096_h512", "stress_down_4096_h512"]


def run(w, d, scale=1.0):
    x = (d["x"] * scale).requires_grad_(True)
    keys = d["keys"].clone().requires_grad_(True)
    wt = None if d["weights"] is None else d["weights"].clone().requires_grad_(True)
    sel2 = cvmm_prepare_sel2(d["sel"], wt, route_input=w.route_input)
    if w.amp:
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            out = cvmm(x, sel2, keys)
    else:
        out = cvmm(x, sel2, keys)
    out.backward(d["grad_out"])
    return out, x.grad, keys.grad, None if wt is None else wt.grad


def route_rows(w, t):
    return t.reshape(w.R, -1) if w.route_input else t.repeat_interleave(w.k, dim=0)


def torch_reference(w, d):
    """fp32 per-expert restatement on the GPU (the reference's math, cvmm.py:1524-1755)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    rnd = (lambda t: t.bfloat16().float()) if w.amp else (lambda t: t.float())
    xr = rnd(route_rows(w, d["x"]))
    kr = rnd(d["keys"])
    sel = d["sel"].reshape(-1)
    g = rnd(d["grad_out"].float())
    y = torch.empty(w.R, w.d_out, device="cuda")
    if w.weighted:
        wr = rnd(d["weights"].reshape(-1))
        gy = g.repeat_interleave(w.k, dim=0) * wr[:, None]
        gy_w = rnd(gy)
    else:
        gy = g.reshape(w.R, w.d_out)
        gy_w = gy
    gk = torch.zeros_like(kr)
    grows = torch.empty(w.R, w.d_in, device="cuda")
    for e in range(w.E):
        idx = (sel == e).nonzero().squeeze(1)
        if idx.numel() == 0:
            continue
        y[idx] = xr[idx] @ kr[e]
        gk[e] = xr[idx].T @ gy_w[idx]
        grows[idx] = gy[idx] @ kr[e].T
    if w.weighted:
        out = (rnd(y).view(w.T, w.k, -1) * wr.view(w.T, w.k, 1)).sum(1)
        gw = (g.repeat_interleave(w.k, dim=0) * y).sum(-1).view(w.T, w.k)
    else:
        out = y.view(w.T, w.k, -1)
        gw = None
    gx = grows.view(d["x"].shape) if w.route_input else grows.view(w.T, w.k, -1).sum(1)
    return out, gx, gk, gw


def rel(a, e):
    a = a.float()
    e = e.float()
    return ((a - e).abs().max() / e.abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("name", CONFIGS)
def test_config_against_torch_fp32(name):
    w = WORKLOADS[name]
    d = make_inputs(w, "cuda", seed=0)
    out, gx, gk, gw = run(w, d)
    eo, ex, ek, ew = torch_reference(w, d)
    tol = 2e-2 if w.amp else 1e-3
    assert out.shape == eo.shape and gx.shape == ex.shape and gk.shape == ek.shape
    assert rel(out, eo) < tol, rel(out, eo)
    assert rel(gx, ex) < tol, rel(gx, ex)
    assert rel(gk, ek) < tol, rel(gk, ek)
    if w.weighted:
        assert rel(gw, ew) < tol, rel(gw, ew)


@pytest.mark.parametrize("name", ["ff_up_1024", "ff_down_1024_weighted"])
def test_config_linearity_and_checksum(name):
    w = WORKLOADS[name]
    d = make_inputs(w, "cuda", seed=1)
    out1, gx1, gk1, _ = run(w, d)
    out2, gx2, gk2, _ = run(w, d, scale=2.0)
    # Power-of-two scaling is exact in bf16 and in fp32 accumulation.
    assert torch.equal(out2.float(), 2 * out1.float())
    assert torch.equal(gk2, 2 * gk1)
    assert torch.equal(gx2.float(), gx1.float())
    # Checksum: the expert gradients sum to the dense X^T G over all routes.
    xr = route_rows(w, d["x"]).float()
    if w.weighted:
        g = d["grad_out"].float().repeat_interleave(w.k, dim=0) * d["weights"].reshape(-1, 1).bfloat16().float()
    else:
        g = d["grad_out"].float().reshape(w.R, -1)
    torch.backends.cuda.matmul.allow_tf32 = False
    dense = xr.T @ g
    assert rel(gk1.sum(0), dense) < 2e-2
