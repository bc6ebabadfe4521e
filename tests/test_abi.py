"""The C-ABI library loads and exports every symbol the header declares (CPU only)."""
import ctypes
import os
import re

import pytest

from cvmm_codex_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "cvmm_sm100.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cvmm_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for must in ("cvmm_sel_prepare", "cvmm_expert_offsets", "cvmm_forward", "cvmm_backward_x",
                 "cvmm_backward_w", "cvmm_weighted_combine"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_lib.SIGNATURES) == set(declared_functions())
    assert lib.cvmm_abi_version() == 10


def test_workspace_queries_need_no_device():
    lib = _lib.load()
    assert lib.cvmm_sel_prepare_workspace_size(0) > 0
    assert lib.cvmm_sel_prepare_workspace_size(1 << 20) > lib.cvmm_sel_prepare_workspace_size(1024)
    assert lib.cvmm_gemm_workspace_size(65536, 64, 1024, 128, 2, 2, 2, 16384) >= 8 * (65536 // 64 + 64)


@pytest.mark.parametrize("call,code", [
    (lambda l: l.cvmm_forward(None, 7, 0, 0, None, None, None, 0, None, 0, 1, 1, 1, 0, 0, 0, None, 0, 1, 0, None, None, None, None, 0, None), -2),
    (lambda l: l.cvmm_forward(None, 2, 10, 4, None, None, None, 5, None, 0, 0, 4, 4, 0, 0, 0, None, 2, 4, 2, None, None, None, None, 0, None), -1),
    (lambda l: l.cvmm_sel_prepare(None, 0, 4, 1, 0, None, None, None, None, None, 0, None), -2),
    (lambda l: l.cvmm_sel_prepare(None, 4, 4, 0, 0, None, None, None, None, None, 0, None), -1),
    (lambda l: l.cvmm_backward_x(None, 2, 4, None, 1, None, None, 4, None, 2, 1, 4, 4, 0, 0, 0, None, 2, 4, 3, None, 0, None, 0, 0, 1, None, 2, None, None, None, 0, None), -1),
    (lambda l: l.cvmm_backward_w(None, 2, 4, None, 0, None, 2, 4, None, 1, None, 0, None, None, 4, 1, 4, 4, None, 2, None, None, None, 0, None), -1),
    (lambda l: l.cvmm_sort_rows_padded(None, 2, 4, None, 1, None, 0, None, None, 4, 2, 8, None, 2, None, None), -1),
    (lambda l: l.cvmm_sort_rows_padded_ex(None, 2, 4, None, 1, None, 0, None, None, 4, 2, 8, None, 2, None, 1, None, None), -1),
    # padded sorted x needs a 16-bit op dtype; a workspace is required
    (lambda l: l.cvmm_forward(16, 2, 4, 8, 16, None, 16, 4, 16, 2, 1, 8, 8, 64, 8, 1, 16, 2, 8, 0, 16, None, None, None, 0, None), -1),
    (lambda l: l.cvmm_backward_w(16, 2, 8, None, 1, 16, 2, 8, None, 1, 16, 0, 16, 16, 4, 1, 8, 8, 16, 2, 16, 16, None, 0, None), -4),
    # padded sorted outputs: only for 16-bit arithmetic, mode 0
    (lambda l: l.cvmm_forward(16, 0, 4, 8, 16, None, 16, 4, 16, 0, 1, 8, 8, 64, 8, 1, 16, 0, 8, 0, None, 16, None, None, 0, None), -1),
    (lambda l: l.cvmm_backward_x(16, 2, 8, None, 1, None, 16, 4, 16, 2, 1, 8, 8, 64, 8, 1, 16, 2, 8, 1, 16, 0, 16, 2, 8, 1, 16, 2, 16, 16, None, 0, None), -1),
    # mode 1 needs a positive x_div (routes per x row)
    (lambda l: l.cvmm_backward_x(16, 2, 8, 16, 1, 16, 16, 4, 16, 2, 1, 8, 8, 64, 8, 1, 16, 2, 8, 1, 16, 0, 16, 2, 8, 0, 16, 2, None, None, None, 0, None), -1),
    # the fused GELU forward needs 16-bit arithmetic; router top_k in [1, 32], gelu backward 16-bit
    (lambda l: l.cvmm_forward_gelu(16, 0, 4, 8, 16, None, 16, 4, 16, 0, 1, 8, 8, 64, 8, 1, 16, 16, 0, 8, 0, None, None, 0, None), -1),
    (lambda l: l.cvmm_router_topk(16, 0, 4, 8, 33, 1, 16, 16, None), -1),
    (lambda l: l.cvmm_router_topk(16, 3, 4, 8, 2, 1, 16, 16, None), -2),
    (lambda l: l.cvmm_gelu_backward(16, 16, 16, 0, 4, None), -2),
    (lambda l: l.cvmm_padded_route_rows(None, None, None, None, 4, 2, None, None), -1),
    (lambda l: l.cvmm_selftest_wait_timeout(0, None), -1),
    # x_copy needs 16-bit arithmetic and a row-indexed x
    (lambda l: l.cvmm_forward(16, 0, 4, 8, 16, None, 16, 4, 16, 0, 1, 8, 8, 64, 8, 1, 16, 0, 8, 0, None, None, 16, None, 0, None), -1),
    (lambda l: l.cvmm_pad_starts(None, 4, None, None), -1),
    (lambda l: l.cvmm_cast(None, 0, None, 9, 4, None), -2),
    (lambda l: l.cvmm_expert_offsets(None, 4, 0, None, None), -1),
])
def test_invalid_arguments_are_rejected_before_any_launch(call, code):
    lib = _lib.load()
    assert call(lib) == code
    assert len(lib.cvmm_last_error()) > 0


def test_check_maps_codes_to_exceptions():
    lib = _lib.load()
    assert lib.cvmm_cast(None, 0, None, 9, 4, None) == -2
    with pytest.raises(ValueError):
        _lib.check(-2, "cvmm_cast")
    with pytest.raises(RuntimeError):
        _lib.check(-3, "x")
    _lib.check(0, "ok")
