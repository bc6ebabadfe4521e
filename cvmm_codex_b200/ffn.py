"""The sigma-MoE feed-forward layer on the sm_100a CVMM kernels.

The reference's caller of CVMM (benchmark_ffn_moe.py:83-100, the
feed-forward of sigma-MoE / MoEUT) is, under bf16 autocast:

    logits = x @ gate
    probs = softmax(float(logits)); weights, sel = probs.topk(k)
    weights = weights / weights.sum(-1).clamp_min(1e-20)
    sel_up = cvmm_prepare_sel2(sel)
    hidden = F.gelu(cvmm(x, sel_up, w_up))
    sel_down = cvmm_prepare_sel2(sel_up, weights, route_input=True)
    out = cvmm(hidden.view(..., k, H), sel_down, w_down)

Here the same layer runs with three fusions:
* the router (softmax, top-k, renormalisation) is one kernel
  (``api.router_topk``) instead of four torch passes over [T, E];
* one selector preparation serves both projections: the down projection
  re-wraps the up projection's sorted routes (cvmm.py:1788-1792), so the
  device sort runs once per layer;
* GELU is applied in the up projection's epilogue (``api.cvmm_gelu``), so the
  activation costs no pass of its own, and its backward is one vectorised
  elementwise kernel on the saved pre-activation.
The router matmul is a plain bf16 cuBLAS GEMM (x @ gate).
"""
from __future__ import annotations

import math

import torch

from .api import cvmm, cvmm_gelu, cvmm_prepare_sel2, router_topk


def sigma_moe_ffn(x: torch.Tensor, gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, k: int,
                  renormalize: bool = True) -> torch.Tensor:
    """The sigma-MoE FFN layer (benchmark_ffn_moe.py:87-98) on x [..., D]:
    gate [D, E], w_up [E, D, H], w_down [E, H, D]; returns [..., D]. Call it
    under torch.autocast(bfloat16) as the reference does."""
    logits = x @ gate
    weights, sel = router_topk(logits, k, renormalize)
    sel_up = cvmm_prepare_sel2(sel)
    hidden = cvmm_gelu(x, sel_up, w_up)
    sel_down = cvmm_prepare_sel2(sel_up, weights, route_input=True)
    return cvmm(hidden.view(*x.shape[:-1], k, w_up.shape[-1]), sel_down, w_down)


class SigmaMoEFFN(torch.nn.Module):
    """sigma-MoE feed-forward block: n_experts experts of width expert_size,
    top-k routing by a softmax router, GELU, weighted combine. Parameters
    are fp32 (autocast casts them per call), initialised N(0, 1/fan_in)."""

    def __init__(self, d_model: int, n_experts: int, expert_size: int, k: int, renormalize: bool = True,
                 device=None):
        super().__init__()
        self.k = int(k)
        self.renormalize = renormalize
        self.gate = torch.nn.Parameter(torch.randn(d_model, n_experts, device=device) / math.sqrt(d_model))
        self.w_up = torch.nn.Parameter(torch.randn(n_experts, d_model, expert_size, device=device)
                                       / math.sqrt(d_model))
        self.w_down = torch.nn.Parameter(torch.randn(n_experts, expert_size, d_model, device=device)
                                         / math.sqrt(expert_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return sigma_moe_ffn(x, self.gate, self.w_up, self.w_down, self.k, self.renormalize)
