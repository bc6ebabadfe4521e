"""Host-side logic of the drop-in module that needs no GPU."""
import numpy as np
import pytest
import torch

import cvmm_codex_b200.api as C
from oracle import cvmm_oracle as O


def test_public_api_names():
    for name in ("CVMMSel", "cvmm_prepare_sel", "cvmm_prepare_sel2", "cvmm", "CVMM", "get_dtype",
                 "dtype_to_type_id", "create_kernels", "_cvmm_expert_offsets",
                 "cvmm_expert_offsets_call", "cvmm_lowmem_chunk_size",
                 "cvmm_use_lowmem_grouped_backward", "cvmm_lowmem_min_top_k", "known_shapes"):
        assert hasattr(C, name), name
    assert [f for f in C.CVMMSel.__dataclass_fields__] == [
        "raw_sel", "sel", "sel_index", "out_index", "reduction_weight"]


def test_dtype_helpers():
    assert C.dtype_to_type_id(torch.float32) == 0
    assert C.dtype_to_type_id(torch.float16) == 1
    assert C.dtype_to_type_id(torch.bfloat16) == 2
    with pytest.raises(ValueError):
        C.dtype_to_type_id(torch.int8)
    assert C.get_dtype() == torch.float32


def _fake_sel(k=3):
    raw = torch.arange(12, dtype=torch.int32).view(4, k)
    s = C.CVMMSel(raw, raw.clone(), torch.arange(12) // k, torch.arange(12), None)
    return s


def test_clone_is_shallow():
    s = _fake_sel()
    c = s.clone()
    assert c.raw_sel is s.raw_sel and c.sel is s.sel and c.sel_index is s.sel_index
    assert c.out_index is s.out_index


def test_prepare_sel2_reuse_route_input():
    # cvmm.py:1788-1792: re-wrapping a token selector for route input uses the
    # route ids (out_index) as the input index and drops out_index.
    s = _fake_sel()
    w = torch.ones(4, 3)
    r = C.cvmm_prepare_sel2(s, w, route_input=True)
    assert r.sel_index is s.out_index and r.out_index is None and r.reduction_weight is w
    assert r.raw_sel is s.raw_sel and r.sel is s.sel
    t = C.cvmm_prepare_sel2(s, w)
    assert t.sel_index is s.sel_index and t.out_index is s.out_index and t.reduction_weight is w
    # A route selector has no out_index: its sel_index are the route ids already.
    rr = C.cvmm_prepare_sel2(C.CVMMSel(s.raw_sel, s.sel, s.out_index, None), None, route_input=True)
    assert rr.sel_index is s.out_index


def test_no_cpu_path():
    with pytest.raises(RuntimeError, match="CUDA"):
        C.cvmm_prepare_sel2(torch.zeros(4, 2, dtype=torch.int64))


def test_expert_offsets_reference_formula_matches_oracle():
    rng = np.random.default_rng(3)
    for E in (1, 7, 64, 512):
        for R in (1, 13, 1000):
            s = np.sort(rng.integers(0, E, R)).astype(np.int32)
            got = C._cvmm_expert_offsets(torch.from_numpy(s), E)
            np.testing.assert_array_equal(got.numpy(), O.expert_offsets(s, E))


def test_traced_call_layer_mirrors_ops_signatures():
    """Every call api.CVMM makes through the custom-op layer takes the same
    parameters as the ops.py function it forwards to (a keyword missing there
    only shows up on a GPU)."""
    import inspect

    from cvmm_codex_b200 import _torch_ops, ops
    for name, fn in vars(_torch_ops._Calls).items():
        if name.startswith("_") or not callable(fn) or not hasattr(ops, name):
            continue
        want = list(inspect.signature(getattr(ops, name)).parameters)
        got = [p for p in inspect.signature(fn).parameters if p != "self"]
        assert got == want, f"_Calls.{name}{got} != ops.{name}{want}"
