"""Seeded synthetic CVMM workloads with the shapes of the benchmark configurations.

The reference measures on random tensors only (benchmark_moe_shapes.py:79-124);
there is no dataset. Each workload below follows one configuration of the
benchmark contract (T tokens, top-k routing over E experts, d_in -> d_out
expert matrices, weighted or not) and draws its tensors from a seeded torch
generator, in a fixed order: x, keys, router logits, bias / skew,
grad_out. Sel weights derive from the router logits.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    T: int              # tokens
    d_in: int           # keys.shape[1]
    d_out: int          # keys.shape[2]
    E: int              # experts
    k: int              # routes per token
    weighted: bool
    route_input: bool   # x is [T, k, d_in] (down projections)
    amp: bool           # bf16 autocast (False: fp32 throughout)
    skew: str = "bias"  # "none", "bias" (logit bias ~N(0, 0.5)), "zipf", "heads"
    heads: int = 0      # SwitchHead: experts grouped per head
    bf16_params: bool = False  # everything bf16 without autocast (the reference's bf16_params mode)

    @property
    def R(self) -> int:
        return self.T * self.k

    @property
    def x_rows(self) -> int:
        """Rows of x: tokens (token input), routes (route input), or token
        heads when the routes of one head share its value row (SwitchHead)."""
        if self.heads:
            return self.T * self.heads
        return self.R if self.route_input else self.T

    def route_rows(self, x):
        """x as one row per route (the layout the reference's API takes)."""
        if self.heads:
            return x.repeat_interleave(self.k // self.heads, dim=-2).reshape(self.R, -1)
        return x.reshape(self.R, -1) if self.route_input else x.repeat_interleave(self.k, dim=0)

    def flops(self) -> int:
        """fw + grad-x + grad-W multiply-adds x2 (the headline FLOP count)."""
        return 3 * 2 * self.R * self.d_in * self.d_out


WORKLOADS = {
    # CPU plumbing, fp32 throughout, top-2 of 8 experts, unweighted.
    "cpu_plumbing": Workload("cpu_plumbing", 2048, 256, 64, 8, 2, False, False, False, "none"),
    # sigma-MoE FFN up projection.
    "ff_up_1024": Workload("ff_up_1024", 16384, 1024, 128, 64, 4, False, False, True, "bias"),
    # sigma-MoE FFN down projection + weighted combine.
    "ff_down_1024_weighted": Workload("ff_down_1024_weighted", 16384, 128, 1024, 64, 4, True, True, True, "bias"),
    # SwitchHead output projection, 32 heads x 4 experts, top-2 per head.
    "switch_o_2048_h32_weighted": Workload("switch_o_2048_h32_weighted", 8192, 64, 2048, 128, 64, True, True, True,
                                           "heads", heads=32),
    # stress, d_model 4096, 128 experts of width 512, Zipf(1.1) skew.
    "stress_up_4096_h512": Workload("stress_up_4096_h512", 32768, 4096, 512, 128, 8, False, False, True, "zipf"),
    "stress_down_4096_h512": Workload("stress_down_4096_h512", 32768, 512, 4096, 128, 8, True, True, True, "zipf"),
    # Parity cases beyond the benchmark list: the reference's lowmem regime
    # (top-32 of 64 experts, cvmm.py:1228-1338) and its bf16_params mode
    # (x, keys and grads bf16, no autocast) at the ff_up shape.
    "top32_up_1024": Workload("top32_up_1024", 4096, 1024, 128, 64, 32, False, False, True, "bias"),
    "bf16_params_ff_up_1024": Workload("bf16_params_ff_up_1024", 16384, 1024, 128, 64, 4, False, False, False, "bias",
                                       bf16_params=True),
}


def make_inputs(w: Workload, device="cuda", seed: int = 0, token_slice: Optional[slice] = None):
    """Returns dict(x, keys, sel, weights, grad_out) for workload `w`.

    x, grad_out: bf16 under AMP (fp32 otherwise); keys fp32 ~N(0, 1/d_in);
    sel int64 [T, k]; weights fp32 [T, k] or None. With `token_slice` only those
    tokens' rows are returned (same values as the full draw's rows), which the
    multi-GPU token sharding uses."""
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    act = torch.bfloat16 if (w.amp or w.bf16_params) else torch.float32
    T = w.T
    x_shape = (T, w.k, w.d_in) if w.route_input else (T, w.d_in)
    if w.skew == "heads":
        # Per-head value rows [T, heads, d_head]; the 2 routes of a head read its
        # row (no repeat_interleave copy: the kernels index row route // 2).
        x = torch.randn(T, w.heads, w.d_in, generator=g, device=dev)
    else:
        x = torch.randn(*x_shape, generator=g, device=dev)
    keys = torch.randn(w.E, w.d_in, w.d_out, generator=g, device=dev) / math.sqrt(w.d_in)
    if w.skew == "heads":
        per = w.E // w.heads
        logits = torch.randn(T, w.heads, per, generator=g, device=dev)
        top = logits.topk(w.k // w.heads, dim=-1)
        base = (torch.arange(w.heads, device=dev) * per).view(1, -1, 1)
        sel = (top.indices + base).reshape(T, w.k)
        sel_logits = top.values.reshape(T, w.k)
    else:
        raw_logits = torch.randn(T, w.E, generator=g, device=dev)
        logits = raw_logits
        if w.skew == "bias":
            logits = logits + torch.randn(w.E, generator=g, device=dev) * math.sqrt(0.5)
        elif w.skew == "zipf":
            perm = torch.randperm(w.E, generator=g, device=dev)
            ranks = torch.empty(w.E, device=dev)
            ranks[perm] = torch.arange(1, w.E + 1, device=dev, dtype=torch.float32)
            p = ranks.pow(-1.1)
            logits = logits + (p / p.sum()).log()
        top = logits.topk(w.k, dim=-1)
        sel = top.indices
        sel_logits = top.values
    weights = None
    if w.weighted:
        if w.skew == "zipf":
            weights = torch.softmax(sel_logits, dim=-1)  # softmax over the selected logits
        elif w.skew == "heads":
            weights = torch.sigmoid(sel_logits)
        else:
            weights = torch.sigmoid(raw_logits.gather(1, sel))  # un-biased router logits
    out_shape = (T, w.d_out) if w.weighted else (T, w.k, w.d_out)
    grad_out = torch.randn(*out_shape, generator=g, device=dev)
    if token_slice is not None:
        x, sel, grad_out = x[token_slice], sel[token_slice], grad_out[token_slice]
        weights = None if weights is None else weights[token_slice]
    return {
        "x": x.to(act).contiguous(),
        "keys": (keys.bfloat16() if w.bf16_params else keys).contiguous(),
        "sel": sel.contiguous(),
        "weights": None if weights is None else weights.float().contiguous(),
        "grad_out": grad_out.to(act).contiguous(),
    }
