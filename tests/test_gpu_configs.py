"""Full-size benchmark configurations on the GPU.

At these sizes the numpy fp64 oracle is too slow, so each configuration is
checked (a) against an FP64 evaluation of the same computation on the GPU:
torch float64 per-expert matmuls over operands rounded to the op dtype exactly
as the reference's kernels round them (cvmm.py:198-204, the weighted grad-W
product rounding of cvmm.py:591-599), the numerics model of
oracle/cvmm_oracle.py; every output and gradient must be within
max|a-e|/max|e| and RMS(a-e)/RMS(e) of 2e-2 (bf16 autocast) or 1e-3 (fp32);
and (b) through size-independent properties: exact linearity under
power-of-two scaling, and the grad-W checksum sum_e dW_e = X_routes^T G_routes.
"""
import pytest
import torch

from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
from cvmm_codex_b200.workloads import WORKLOADS, make_inputs

pytestmark = pytest.mark.gpu

CONFIGS = ["cpu_plumbing", "ff_up_1024", "ff_down_1024_weighted", "switch_o_2048_h32_weighted",
           "stress_up_4096_h512", "stress_down_4096_h512", "top32_up_1024", "bf16_params_ff_up_1024"]


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
    return w.route_rows(t)


def fp64_reference(w, d):
    """FP64 per-expert evaluation on the GPU of the reference's math
    (cvmm.py:1524-1755) with the reference's operand rounding."""
    rnd = (lambda t: t.bfloat16().double()) if (w.amp or w.bf16_params) else (lambda t: t.float().double())
    xr = rnd(route_rows(w, d["x"]))
    kr = rnd(d["keys"])
    sel = d["sel"].reshape(-1)
    g = rnd(d["grad_out"])
    y = torch.empty(w.R, w.d_out, device="cuda", dtype=torch.float64)
    if w.weighted:
        wr = rnd(d["weights"].reshape(-1))
        gy = g.repeat_interleave(w.k, dim=0) * wr[:, None]
        gy_w = rnd(gy)
    else:
        gy = g.reshape(w.R, w.d_out)
        gy_w = gy
    gk = torch.zeros_like(kr)
    grows = torch.empty(w.R, w.d_in, device="cuda", dtype=torch.float64)
    for e in range(w.E):
        idx = (sel == e).nonzero().squeeze(1)
        if idx.numel() == 0:
            continue
        y[idx] = xr[idx] @ kr[e]
        gk[e] = xr[idx].T @ gy_w[idx]
        grows[idx] = gy[idx] @ kr[e].T
    if w.weighted:
        out = (y.view(w.T, w.k, -1) * wr.view(w.T, w.k, 1)).sum(1)
        gw = (g.repeat_interleave(w.k, dim=0) * y).sum(-1).view(w.T, w.k)
    else:
        out = y.view(w.T, w.k, -1)
        gw = None
    if w.heads:
        gx = grows.view(w.T, w.heads, w.k // w.heads, -1).sum(2)
    else:
        gx = grows.view(d["x"].shape) if w.route_input else grows.view(w.T, w.k, -1).sum(1)
    return out, gx, gk, gw


def rel(a, e):
    a = a.double()
    e = e.double()
    return ((a - e).abs().max() / e.abs().max().clamp_min(1e-30)).item()


def rel_rms(a, e):
    a = a.double()
    e = e.double()
    return ((a - e).pow(2).mean().sqrt() / e.pow(2).mean().sqrt().clamp_min(1e-30)).item()


@pytest.mark.parametrize("name", CONFIGS)
def test_config_against_fp64(name):
    w = WORKLOADS[name]
    d = make_inputs(w, "cuda", seed=0)
    got = run(w, d)
    want = fp64_reference(w, d)
    tol = 2e-2 if (w.amp or w.bf16_params) else 1e-3  # BF16 2e-2, FP32 paths 1e-3
    names = ("out", "grad_x", "grad_keys", "grad_w")
    for nm, a, e in zip(names, got, want):
        if e is None:
            continue
        assert a.shape == e.shape, (nm, a.shape, e.shape)
        err_max, err_rms = rel(a, e), rel_rms(a, e)
        print(f"{name} {nm}: max {err_max:.3e} rms {err_rms:.3e}")
        assert err_max < tol, (nm, err_max)
        assert err_rms < tol, (nm, err_rms)
    del got, want
    torch.cuda.empty_cache()


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
