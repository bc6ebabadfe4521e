"""The CPU oracle against fixtures generated from the reference itself (CPU, no GPU)."""
import os

import numpy as np
import pytest
import torch

from oracle import cvmm_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
SEL = torch.load(os.path.join(GOLDEN, "selector.pt"))
NUM = torch.load(os.path.join(GOLDEN, "numerics.pt"))


@pytest.mark.parametrize("name", sorted(SEL))
def test_selector_matches_reference(name):
    c = SEL[name]
    sel = c["sel"].numpy()
    k = sel.shape[-1]
    raw, ssel, sel_index, out_index = O.prepare_sel2(sel)
    # Values are bit-exact with the reference's cvmm_prepare_sel2.
    np.testing.assert_array_equal(raw, c["raw_sel"].flatten().numpy())
    np.testing.assert_array_equal(ssel, c["sorted_sel"].flatten().numpy())
    # The oracle's permutation is the stable one (torch.sort(stable=True)).
    np.testing.assert_array_equal(out_index, c["stable_index"].numpy())
    np.testing.assert_array_equal(sel_index, out_index // k)
    # The reference's own permutation (torch.sort default, ties unordered) is a
    # valid sort permutation with the same derived indices.
    ref_idx = c["tok_out_index"].numpy()
    assert sorted(ref_idx.tolist()) == list(range(ref_idx.size))
    np.testing.assert_array_equal(sel.reshape(-1)[ref_idx], ssel)
    np.testing.assert_array_equal(c["tok_sel_index"].numpy(), ref_idx // k)
    np.testing.assert_array_equal(sel.reshape(-1)[c["route_sel_index"].numpy()], ssel)
    np.testing.assert_array_equal(sel.reshape(-1)[c["prep_sel_index"].numpy()], ssel)
    # Expert offsets are exact.
    np.testing.assert_array_equal(O.expert_offsets(ssel, c["n_experts"]), c["offsets"].numpy())
    _, _, rsi, roi = O.prepare_sel2(sel, route_input=True)
    assert roi is None
    np.testing.assert_array_equal(rsi, c["stable_index"].numpy())


def _np(t):
    return None if t is None else t.float().numpy().astype(np.float64)


@pytest.mark.parametrize("key", sorted(NUM))
def test_numerics_match_reference(key):
    c = NUM[key]
    x, keys, sel, w, grad = _np(c["x"]), _np(c["keys"]), c["sel"].numpy(), _np(c["w"]), _np(c["grad"])
    # The reference's `_reference` evaluates in fp32 with unrounded operands.
    out = O.forward(x, sel, keys, w, op="float32")
    assert O.rel_max_err(out, _np(c["out"])) < 1e-5
    gx, gk, gw = O.backward(x, sel, keys, grad, w, op="float32")

    def tol(t):
        # autograd stores a gradient in its leaf's dtype: bf16 leaves carry one
        # bf16 rounding (relative 2^-9) on top of the fp32 math.
        return 1e-5 if t.dtype == torch.float32 else 5e-3

    assert O.rel_max_err(gx, _np(c["x_grad"])) < tol(c["x_grad"])
    # For bf16 keys `_reference` differentiates keys[sel] (an index on a bf16
    # tensor), whose backward accumulates the routes of one expert in bf16.
    k_tol = 1e-5 if c["keys_grad"].dtype == torch.float32 else 2e-2
    assert O.rel_max_err(gk, _np(c["keys_grad"])) < k_tol
    if w is not None:
        assert O.rel_max_err(gw, _np(c["w_grad"])) < tol(c["w_grad"])


def test_round_bf16_ties_to_even():
    # 1 + 2^-8 is halfway between two bf16 values; ties go to the even mantissa.
    v = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -2.5, 0.0], dtype=np.float32)
    r = O.round_bf16(v)
    np.testing.assert_array_equal(r, [1.0, 1.0 + 2 * 2.0 ** -7, -2.5, 0.0])
    t = torch.tensor(v).to(torch.bfloat16).double().numpy()
    np.testing.assert_array_equal(r, t)


def test_round_bf16_matches_torch_random():
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(100000) * 10.0 ** rng.integers(-6, 6, 100000)).astype(np.float32)
    np.testing.assert_array_equal(O.round_bf16(v), torch.tensor(v).to(torch.bfloat16).double().numpy())
