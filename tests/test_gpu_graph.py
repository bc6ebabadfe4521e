"""CUDA-graph replays of the full step on one GPU: the captured step (selector
prep, GEMMs, copies, reductions; programmatic dependent launches become
programmatic graph edges) gives the same outputs and gradients, bit for bit,
as the eager step, for the token-input and the weighted route-input layouts,
with programmatic launch on and off. The sel-weight gradient is an fp32
atomic sum and is compared to rounding."""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pdl", [1, 0])
@pytest.mark.parametrize("weighted", [False, True])
def test_graph_replay_matches_eager(weighted, pdl):
    import bench
    from cvmm_codex_b200 import _lib
    from cvmm_codex_b200.workloads import Workload, make_inputs
    lib = _lib.load()
    prev = lib.cvmm_set_pdl(pdl)
    # Inputs, eager step and capture all on one non-default stream: autograd's
    # leaf-gradient accumulation would otherwise order work against the legacy
    # stream the leaves were created on, which a capture does not allow.
    stream = torch.cuda.Stream()
    try:
        with torch.cuda.stream(stream):
            w = Workload("graph_test", 2048, 256, 384, 16, 4, weighted, weighted, True, "bias")
            d = make_inputs(w, "cuda", seed=5)
            step = bench.build_step(w, d, 1)
            out = step(d["sel"], d["grad_out"])
            torch.cuda.synchronize()
            eager = [out.detach().clone(), d["x"].grad.clone(), d["keys"].grad.clone()]
            if weighted:
                eager.append(d["weights"].grad.clone())
            g = bench.GraphedStep(step, d)
            for _ in range(3):
                out = g()
            torch.cuda.synchronize()
            graphed = [out.detach().clone(), d["x"].grad.clone(), d["keys"].grad.clone()]
            if weighted:
                graphed.append(d["weights"].grad.clone())
    finally:
        lib.cvmm_set_pdl(prev)
    for a, b in zip(eager[:3], graphed[:3]):
        assert a.shape == b.shape and a.dtype == b.dtype
        assert torch.equal(a, b)
    if weighted:
        torch.testing.assert_close(eager[3], graphed[3], rtol=1e-5, atol=1e-6)
