"""torch.library registration of the CVMM forward op.

``cvmm_b200::cvmm_triton`` keeps the schema of the reference's
``mylib::cvmm_triton`` (cvmm.py:807-812):
    (Tensor x, Tensor sel_index, Tensor sel, Tensor keys, ScalarType out_dtype,
     Tensor out_index, ScalarType op_dtype) -> Tensor
with ``out_index`` a one-element tensor holding -1 when absent, and the same
fake implementation for torch.compile (cvmm.py:1442-1450).
"""
from __future__ import annotations

import torch

from . import ops


@torch.library.custom_op("cvmm_b200::cvmm_triton", mutates_args=())
def cvmm_triton(x: torch.Tensor, sel_index: torch.Tensor, sel: torch.Tensor, keys: torch.Tensor,
                out_dtype: torch.dtype, out_index: torch.Tensor, op_dtype: torch.dtype) -> torch.Tensor:
    n_experts = keys.shape[0]
    offsets = ops.expert_offsets(sel, n_experts)
    oi = None if (out_index.numel() == 1 and int(out_index.reshape(-1)[0]) == -1) else out_index
    if op_dtype != torch.float32 and keys.dtype != op_dtype:
        keys = ops.cast(keys, op_dtype)
    out = ops.forward(x, sel_index, offsets, keys, oi, out_dtype, op_dtype)
    return out.view(*sel.shape, keys.shape[-1])


@cvmm_triton.register_fake
def _cvmm_triton_fake(x, sel_index, sel, keys, out_dtype, out_index, op_dtype):
    return x.new_empty((*sel.shape, keys.shape[-1]), dtype=out_dtype)


@torch.library.custom_op("cvmm_b200::expert_offsets", mutates_args=())
def expert_offsets(sorted_sel: torch.Tensor, n_experts: int) -> torch.Tensor:
    return ops.expert_offsets(sorted_sel, n_experts)


@expert_offsets.register_fake
def _expert_offsets_fake(sorted_sel, n_experts):
    return sorted_sel.new_empty((n_experts,), dtype=torch.int64)
