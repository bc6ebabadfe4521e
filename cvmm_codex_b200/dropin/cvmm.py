"""`import cvmm` shim: put this folder first on sys.path and the reference's
scripts (`import cvmm`, `from cvmm import cvmm, cvmm_prepare_sel2`,
`cvmm_module.cvmm_expert_offsets_call = None`, ...) run unmodified on the
sm_100a implementation. The module object IS cvmm_codex_b200.api, so
attribute assignments reach the implementation."""
import importlib
import os
import sys

_root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _root not in sys.path:
    sys.path.append(_root)
sys.modules[__name__] = importlib.import_module("cvmm_codex_b200.api")
