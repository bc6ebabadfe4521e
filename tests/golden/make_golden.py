"""Generates the golden fixtures in this folder from the reference itself.

Run with the path of a checkout of the reference (RobertCsordas/cvmm_codex)
as the argument (or in $CVMM_REFERENCE):

    python tests/golden/make_golden.py <path-to-reference-checkout>

It imports the reference module `cvmm.py` and its test oracle `_reference`
(test_cvmm_correctness.py:7-15) on CPU -- nothing here needs a GPU -- and
records:
  selector.pt : cvmm_prepare_sel2 / cvmm_prepare_sel outputs (cvmm.py:24-27,
                1786-1803) and the torch expert-offsets formula (cvmm.py:68-78)
                for seeded routings, including ties, missing experts, top-1,
                a single route and empty-expert cases;
  numerics.pt : the reference's correctness case list
                (benchmark_correctness_original.py:35-43) in its three dtype
                modes (:45, :85-94), inputs drawn with its payload recipe
                (:107-133), with `_reference` outputs and autograd gradients.
The fixtures are committed; the GPU box never reads the reference.
"""
import os
import sys

import torch

sys.dont_write_bytecode = True
REF = os.environ.get("CVMM_REFERENCE")  # checkout of the reference repository (required)
HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference():
    sys.path.insert(0, REF)
    import cvmm as ref_cvmm  # noqa: E402  (the reference module)
    import test_cvmm_correctness as ref_test  # noqa: E402
    return ref_cvmm, ref_test


SEL_CASES = [
    # (name, shape, n_experts, seed)
    ("single_route", (1, 1), 1, 0),
    ("top1", (13, 1), 7, 1),
    ("top3_small", (3, 5, 3), 7, 2),
    ("top8", (2, 16, 8), 16, 3),
    ("many_missing", (1, 5, 2), 32, 4),
    ("e1_r1000", (1000, 1), 1, 5),
    ("e64_r1000", (250, 4), 64, 6),
    ("e512_r1000", (125, 8), 512, 7),
    ("top32", (2, 5, 32), 64, 8),
    ("r4096_top2", (2048, 2), 8, 9),
    ("r16384_top4", (4096, 4), 64, 10),
    ("e3000_r4000", (1000, 4), 3000, 11),
]


def make_selector(ref_cvmm):
    out = {}
    for name, shape, n_experts, seed in SEL_CASES:
        g = torch.Generator().manual_seed(seed)
        sel = torch.randint(0, n_experts, shape, generator=g, dtype=torch.int64)
        tok = ref_cvmm.cvmm_prepare_sel2(sel)
        rte = ref_cvmm.cvmm_prepare_sel2(sel, route_input=True)
        ps = ref_cvmm.cvmm_prepare_sel(sel, n_experts)
        offs = ref_cvmm._cvmm_expert_offsets(tok.sel.flatten(), n_experts)
        out[name] = {
            "sel": sel, "n_experts": n_experts,
            "raw_sel": tok.raw_sel, "sorted_sel": tok.sel,
            "tok_sel_index": tok.sel_index, "tok_out_index": tok.out_index,
            "route_sel_index": rte.sel_index,
            "prep_sel_index": ps.sel_index,
            "offsets": offs,
            "stable_index": torch.sort(sel.flatten().to(torch.int32), stable=True).indices,
        }
    return out


CASES = [
    # name, B, T, N(d_in), E(d_out), K(top-k), N_E(experts), weighted, route_input
    ("top1_unweighted_masks", 2, 7, 17, 9, 1, 13, False, False),
    ("top3_unweighted", 3, 5, 19, 11, 3, 7, False, False),
    ("weighted_combine", 2, 9, 23, 13, 4, 11, True, False),
    ("weighted_route_input", 2, 8, 29, 17, 4, 9, True, True),
    ("larger_top8_unweighted", 2, 16, 64, 32, 8, 16, False, False),
    ("larger_top8_weighted_route_input", 2, 16, 32, 64, 8, 16, True, True),
    ("many_missing_experts", 1, 5, 15, 10, 2, 32, True, False),
]
MODES = ("float32", "bf16_amp", "bf16_params")


def _dtype_for(mode, name):
    if mode == "float32":
        return torch.float32
    if mode == "bf16_params":
        return torch.bfloat16
    return torch.bfloat16 if name == "x" else torch.float32


def _tensor(shape, dtype, gen, scale):
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * scale).to(dtype)


def make_numerics(ref_test):
    out = {}
    for seed_off, (name, B, T, N, E, K, NE, weighted, route_input) in enumerate(CASES):
        for mode in MODES:
            gen = torch.Generator().manual_seed(1000 + 17 * seed_off + MODES.index(mode))
            x_shape = (B, T, K, N) if route_input else (B, T, N)
            x = _tensor(x_shape, _dtype_for(mode, "x"), gen, 0.4)
            keys = _tensor((NE, N, E), _dtype_for(mode, "keys"), gen, 0.3)
            sel = torch.randint(0, NE, (B, T, K), generator=gen, dtype=torch.int64)
            out_shape = (B, T, E) if weighted else (B, T, K, E)
            grad = _tensor(out_shape, _dtype_for(mode, "x"), gen, 0.2)
            w = _tensor((B, T, K), _dtype_for(mode, "weights"), gen, 0.25) if weighted else None
            xr = x.clone().requires_grad_(True)
            kr = keys.clone().requires_grad_(True)
            wr = None if w is None else w.clone().requires_grad_(True)
            y = ref_test._reference(xr, sel, kr, wr)
            y.backward(grad.float())
            out[f"{name}/{mode}"] = {
                "mode": mode, "weighted": weighted, "route_input": route_input,
                "x": x, "keys": keys, "sel": sel, "w": w, "grad": grad,
                "out": y.detach(), "x_grad": xr.grad, "keys_grad": kr.grad,
                "w_grad": None if wr is None else wr.grad,
            }
    return out


if __name__ == "__main__":
    if len(sys.argv) > 1:
        REF = sys.argv[1]
    if not REF:
        sys.exit("usage: make_golden.py <path-to-reference-checkout> (or set CVMM_REFERENCE)")
    ref_cvmm, ref_test = _import_reference()
    torch.save(make_selector(ref_cvmm), os.path.join(HERE, "selector.pt"))
    torch.save(make_numerics(ref_test), os.path.join(HERE, "numerics.pt"))
    print("wrote", os.path.join(HERE, "selector.pt"), os.path.join(HERE, "numerics.pt"))
