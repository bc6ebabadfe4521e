"""torch.compile boundary (reference cvmm.py:808-812, 1436-1450).

Every device call of cvmm_prepare_sel2 / CVMM.forward / CVMM.backward is a
registered custom op with a fake implementation, so a model that calls the
drop-in API compiles with fullgraph=True (no graph break) and its outputs and
gradients equal the eager ones bit for bit (same kernels, same arguments).
"""
import pytest
import torch

from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2

pytestmark = pytest.mark.gpu


def _step(x, sel, keys, w, grad, route_input):
    s = cvmm_prepare_sel2(sel, w, route_input=route_input)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        out = cvmm(x, s, keys)
    return out


@pytest.mark.parametrize("weighted,route_input", [(False, False), (True, True), (True, False)])
def test_compile_fullgraph_matches_eager(weighted, route_input):
    torch._dynamo.reset()
    g = torch.Generator(device="cuda").manual_seed(4)
    T, k, E, d_in, d_out = 512, 4, 16, 128, 256
    x0 = torch.randn(*((T, k, d_in) if route_input else (T, d_in)), device="cuda", generator=g).bfloat16()
    k0 = torch.randn(E, d_in, d_out, device="cuda", generator=g) / d_in ** 0.5
    sel = torch.randint(0, E, (T, k), device="cuda", generator=g)
    w0 = torch.rand(T, k, device="cuda", generator=g) if weighted else None
    grad = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), device="cuda", generator=g).bfloat16()

    def run(fn):
        x = x0.clone().requires_grad_(True)
        keys = k0.clone().requires_grad_(True)
        w = None if w0 is None else w0.clone().requires_grad_(True)
        out = fn(x, sel, keys, w, grad, route_input)
        out.backward(grad)
        return out.detach(), x.grad, keys.grad, None if w is None else w.grad

    eager = run(_step)
    compiled = run(torch.compile(_step, fullgraph=True))
    for a, b in zip(eager, compiled):
        if a is None:
            assert b is None
            continue
        assert a.shape == b.shape and a.dtype == b.dtype
        assert torch.equal(a, b)


def test_custom_ops_pass_opcheck():
    """torch.library.opcheck: schema, fake implementation and dispatch of the
    selector and offsets ops agree with the real kernels."""
    sel = torch.randint(0, 8, (300, 2), device="cuda")
    torch.library.opcheck(torch.ops.cvmm_b200.sel_prepare.default, (sel, 2, False))
    raw, ssel, si, oi = torch.ops.cvmm_b200.sel_prepare(sel, 2, False)
    torch.library.opcheck(torch.ops.cvmm_b200.expert_offsets.default, (ssel, 8))
