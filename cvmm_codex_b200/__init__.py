"""B200-native (sm_100a) CVMM: the top-k mixture-of-experts projection of
RobertCsordas/cvmm_codex behind the reference's own Python API.

    from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2, CVMMSel

The compute runs in libcvmm_sm100.so (hand-written CUDA for sm_100a, C ABI in
include/cvmm_sm100.h); see cvmm_codex_b200.api for the drop-in module.
"""
from .api import (CVMM, CVMMGelu, CVMMSel, create_kernels, cvmm, cvmm_gelu, cvmm_prepare_sel, cvmm_prepare_sel2,
                   dtype_to_type_id, get_dtype, router_topk)
from .ffn import SigmaMoEFFN, sigma_moe_ffn

__all__ = ["CVMM", "CVMMGelu", "CVMMSel", "create_kernels", "cvmm", "cvmm_gelu", "cvmm_prepare_sel",
           "cvmm_prepare_sel2", "dtype_to_type_id", "get_dtype", "router_topk", "SigmaMoEFFN", "sigma_moe_ffn"]
