"""CPU baseline of the CVMM hot path -- TEST / BENCHMARK INFRASTRUCTURE ONLY.

The reference's pure-PyTorch formulation of one CVMM training step (selector
sort, forward, grad-x, grad-W, sel-weight grad), restated per expert in fp32
on the host cores: the same math as the reference's test oracle
(test_cvmm_correctness.py:7-15) and its per-expert gather/matmul structure
(cvmm.py:1141-1225, 1341-1433), without materialising keys[sel]. bench.py
times it as `cpu_baseline` and as the `--impl reference` arm; the product
never calls it.
"""
from __future__ import annotations

import torch


def make_sample(w, n_tokens: int, seed: int = 0):
    """Host fp32 inputs for `n_tokens` tokens of workload `w` (same recipe as the GPU run)."""
    from cvmm_codex_b200.workloads import make_inputs

    d = make_inputs(w, "cpu", seed=seed, token_slice=slice(0, n_tokens))
    return {k: (None if v is None else (v.float() if v.is_floating_point() else v)) for k, v in d.items()}


def step(w, d):
    """One fw+bw over the sample; returns (out, grad_x, grad_keys, grad_w)."""
    x, keys, sel, wt, g = d["x"], d["keys"], d["sel"], d["weights"], d["grad_out"]
    T = sel.shape[0]
    R = sel.numel()
    flat = sel.reshape(-1)
    order = torch.sort(flat.to(torch.int32), stable=True)
    idx = order.indices
    counts = torch.bincount(flat, minlength=w.E)
    rows = w.route_rows(x)
    y = torch.empty(R, w.d_out)
    gk = torch.zeros_like(keys)
    gr = torch.empty(R, w.d_in)
    if w.weighted:
        gy = g.repeat_interleave(w.k, dim=0) * wt.reshape(R, 1)
    else:
        gy = g.reshape(R, -1)
    start = 0
    for e in range(w.E):
        n = int(counts[e])
        if n == 0:
            continue
        r = idx[start:start + n]
        start += n
        xe = rows.index_select(0, r)
        ye = xe @ keys[e]
        ge = gy.index_select(0, r)
        y.index_copy_(0, r, ye)
        gk[e] = xe.T @ ge
        gr.index_copy_(0, r, ge @ keys[e].T)
    if w.weighted:
        out = (y.view(T, w.k, -1) * wt.view(T, w.k, 1)).sum(1)
        gw = (g.repeat_interleave(w.k, dim=0) * y).sum(-1).view(T, w.k)
    else:
        out, gw = y.view(T, w.k, -1), None
    if w.heads:
        gx = gr.view(T, w.heads, w.k // w.heads, -1).sum(2)
    else:
        gx = gr.view(x.shape) if w.route_input else gr.view(T, w.k, -1).sum(1)
    return out, gx, gk, gw
