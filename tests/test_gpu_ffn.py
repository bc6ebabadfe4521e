"""The sigma-MoE FFN layer (reference benchmark_ffn_moe.py:83-100) on the
sm_100a kernels: fused router, one shared selector prep, GELU fused into the
up projection's epilogue. Checked against the reference's own composition
(torch softmax / topk / renormalisation, cvmm, F.gelu, weighted cvmm) and
against an fp64 evaluation of the layer."""
import pytest
import torch
import torch.nn.functional as F

from cvmm_codex_b200 import SigmaMoEFFN, cvmm, cvmm_gelu, cvmm_prepare_sel2, router_topk

pytestmark = pytest.mark.gpu


def rel(a, e):
    a, e = a.double(), e.double()
    return ((a - e).abs().max() / e.abs().max().clamp_min(1e-30)).item()


def rel_rms(a, e):
    a, e = a.double(), e.double()
    return ((a - e).pow(2).mean().sqrt() / e.pow(2).mean().sqrt().clamp_min(1e-30)).item()


def torch_router(logits, k):
    probs = torch.softmax(logits.float(), dim=-1)
    w, sel = probs.topk(k, dim=-1)
    return w / w.sum(dim=-1, keepdim=True).clamp_min(1e-20), sel


@pytest.mark.parametrize("E,k", [(64, 8), (512, 8), (128, 4), (1024, 32)])
def test_router_matches_torch_on_fp32_logits(E, k):
    g = torch.Generator(device="cuda").manual_seed(E + k)
    logits = torch.randn(3000, E, device="cuda", generator=g) * 2
    w, sel = router_topk(logits, k)
    wr, sr = torch_router(logits, k)
    assert torch.equal(sel, sr)  # distinct fp32 logits: no ties
    torch.testing.assert_close(w, wr, rtol=1e-5, atol=1e-7)


def test_router_bf16_logits_selects_the_top_probabilities():
    """bf16 logits tie often; the selected probabilities (in order) equal torch's."""
    g = torch.Generator(device="cuda").manual_seed(1)
    logits = torch.randn(4096, 512, device="cuda", generator=g).bfloat16()
    w, sel = router_topk(logits, 8)
    probs = torch.softmax(logits.float(), dim=-1)
    vr, _ = probs.topk(8, dim=-1)
    torch.testing.assert_close(probs.gather(-1, sel), vr, rtol=0, atol=0)
    torch.testing.assert_close(w, vr / vr.sum(-1, keepdim=True), rtol=1e-5, atol=1e-7)


def test_router_backward_matches_autograd_of_the_composition():
    g = torch.Generator(device="cuda").manual_seed(2)
    logits = (torch.randn(1000, 64, device="cuda", generator=g) * 2).requires_grad_(True)
    r = torch.randn(1000, 8, device="cuda", generator=g)
    w, sel = router_topk(logits, 8)
    (w * r).sum().backward()
    ours = logits.grad.clone()
    logits.grad = None
    probs = torch.softmax(logits.float(), dim=-1)
    pw = probs.gather(-1, sel)
    wr = pw / pw.sum(-1, keepdim=True).clamp_min(1e-20)
    (wr * r).sum().backward()
    torch.testing.assert_close(ours, logits.grad, rtol=1e-4, atol=1e-7)


def test_cvmm_gelu_matches_gelu_of_cvmm():
    """Fused epilogue GELU against F.gelu(cvmm(...)) (the reference's two passes)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    T, k, E, D, H = 1000, 4, 16, 256, 128
    x0 = torch.randn(T, D, device="cuda", generator=g).bfloat16()
    k0 = torch.randn(E, D, H, device="cuda", generator=g) / D ** 0.5
    sel = torch.randint(0, E, (T, k), device="cuda", generator=g)
    grad = torch.randn(T, k, H, device="cuda", generator=g).bfloat16()
    res = []
    for fused in (True, False):
        x = x0.clone().requires_grad_(True)
        keys = k0.clone().requires_grad_(True)
        s = cvmm_prepare_sel2(sel)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            h = cvmm_gelu(x, s, keys) if fused else F.gelu(cvmm(x, s, keys))
        h.backward(grad)
        res.append((h.detach(), x.grad, keys.grad))
    (h1, gx1, gk1), (h2, gx2, gk2) = res
    # Same rounded pre-activation, GELU in fp32, one rounding: equal up to the
    # last bit of the erf/exp evaluation order.
    assert (h1.float() - h2.float()).abs().max().item() <= 2 ** -7 * h2.float().abs().max().item()
    assert rel_rms(h1, h2) < 1e-3
    for a, b in ((gx1, gx2), (gk1, gk2)):
        assert rel(a, b) < 1e-2 and rel_rms(a, b) < 1e-3


def fp64_layer(x, gate, w_up, w_down, sel, weights):
    """fp64 evaluation of the layer's expert part for a given routing, with
    the op-dtype (bf16) rounding of the GEMM operands and of the stored
    intermediates (cvmm outputs, GELU output) the reference applies."""
    rnd = lambda t: t.bfloat16().double()  # noqa: E731
    T, D = x.shape
    k = sel.shape[-1]
    H = w_up.shape[-1]
    xr = rnd(x).repeat_interleave(k, 0)
    s = sel.reshape(-1)
    z = torch.empty(T * k, H, device=x.device, dtype=torch.float64)
    wu, wd = rnd(w_up), rnd(w_down)
    for e in range(w_up.shape[0]):
        idx = (s == e).nonzero().squeeze(1)
        if idx.numel():
            z[idx] = xr[idx] @ wu[e]
    h = rnd(F.gelu(rnd(z).float()).double())
    y = torch.empty(T * k, D, device=x.device, dtype=torch.float64)
    for e in range(w_down.shape[0]):
        idx = (s == e).nonzero().squeeze(1)
        if idx.numel():
            y[idx] = h[idx] @ wd[e]
    return (rnd(y).view(T, k, D) * rnd(weights).view(T, k, 1)).sum(1)


def test_sigma_moe_layer_forward_backward():
    """The whole layer: output against an fp64 evaluation for the routing the
    layer chose, and every gradient against the reference's composition
    (torch router, cvmm, F.gelu, weighted cvmm) run with autograd."""
    torch.manual_seed(0)
    T, D, H, E, k = 2048, 256, 128, 64, 8
    layer = SigmaMoEFFN(D, E, H, k, device="cuda")
    x = torch.randn(T, D, device="cuda").bfloat16().requires_grad_(True)
    grad = torch.randn(T, D, device="cuda").bfloat16()
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        out = layer(x)
        logits = x @ layer.gate
    out.backward(grad)
    ours = [x.grad.clone()] + [p.grad.clone() for p in (layer.gate, layer.w_up, layer.w_down)]
    w, sel = router_topk(logits.detach(), k)
    want = fp64_layer(x.detach(), layer.gate, layer.w_up, layer.w_down, sel, w)
    assert rel(out, want) < 2e-2 and rel_rms(out, want) < 1e-2

    # the reference's composition (benchmark_ffn_moe.py:88-98), same parameters
    x.grad = None
    for p in layer.parameters():
        p.grad = None
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        lg = x @ layer.gate
        # softmax + renormalisation in torch at the routing the layer chose
        # (bf16 logits tie often, and torch.topk may break a tie the other way)
        probs = torch.softmax(lg.float(), dim=-1)
        pw = probs.gather(-1, sel)
        wr = pw / pw.sum(dim=-1, keepdim=True).clamp_min(1e-20)
        su = cvmm_prepare_sel2(sel)
        hid = F.gelu(cvmm(x, su, layer.w_up))
        sd = cvmm_prepare_sel2(su, wr, route_input=True)
        ref = cvmm(hid.view(T, k, H), sd, layer.w_down)
    ref.backward(grad)
    theirs = [x.grad] + [p.grad for p in (layer.gate, layer.w_up, layer.w_down)]
    assert rel(out, ref) < 1e-2
    for name, a, b in zip(("x", "gate", "w_up", "w_down"), ours, theirs):
        assert rel(a, b) < 2e-2, (name, rel(a, b))
        assert rel_rms(a, b) < 1e-2, (name, rel_rms(a, b))
