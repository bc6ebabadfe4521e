"""The allocation-free selector entry point, called through the C ABI.

cvmm_sel_prepare_noalloc serves callers that cannot allocate device memory on
the call path: it takes only inputs and outputs and uses a static scratch
array inside the library. This file is collected last so that a run stopping
at the first failure has already run every other test; it also passes alone
in a fresh process.
"""
import os
import sys

import numpy as np
import pytest
import torch

from cvmm_codex_b200 import _lib

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle import cvmm_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_ROUTES = 65536


def _outputs(n, route_input, device):
    return (torch.empty(n, dtype=torch.int32, device=device), torch.empty(n, dtype=torch.int32, device=device),
            torch.empty(n, dtype=torch.int64, device=device),
            None if route_input else torch.empty(n, dtype=torch.int64, device=device))


def _with_workspace(lib, sel, k, route_input):
    n = sel.numel()
    raw, ssel, si, oi = _outputs(n, route_input, sel.device)
    ws = torch.empty(lib.cvmm_sel_prepare_workspace_size(n), dtype=torch.uint8, device=sel.device)
    rc = lib.cvmm_sel_prepare(sel.data_ptr(), _lib.I64, n, k, int(route_input), raw.data_ptr(), ssel.data_ptr(),
                              si.data_ptr(), None if oi is None else oi.data_ptr(), ws.data_ptr(), ws.numel(),
                              _lib.stream_of(sel.device))
    _lib.check(rc, "cvmm_sel_prepare")
    return raw, ssel, si, oi


def _no_alloc(lib, sel, k, route_input):
    n = sel.numel()
    raw, ssel, si, oi = _outputs(n, route_input, sel.device)
    rc = lib.cvmm_sel_prepare_noalloc(sel.data_ptr(), _lib.I64, n, k, int(route_input), raw.data_ptr(),
                                      ssel.data_ptr(), si.data_ptr(), None if oi is None else oi.data_ptr(),
                                      _lib.stream_of(sel.device))
    _lib.check(rc, "cvmm_sel_prepare_noalloc")
    return raw, ssel, si, oi


@pytest.mark.parametrize("route_input", [False, True])
def test_no_alloc_matches_workspace_entry_point_twice(route_input):
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(123 + route_input)
    # Two calls in a row: the first fills the shared scratch with a large
    # input, the second (smaller, different key range) must not see stale data.
    cases = [(torch.randint(0, 64, (MAX_ROUTES // 4, 4), generator=g, device=dev), 4),
             (torch.randint(0, 3000, (1367, 3), generator=g, device=dev), 3)]
    for sel, k in cases:
        want = _with_workspace(lib, sel.reshape(-1).contiguous(), k, route_input)
        got = _no_alloc(lib, sel.reshape(-1).contiguous(), k, route_input)
        torch.cuda.synchronize()
        for a, b in zip(got, want):
            if b is None:
                assert a is None
            else:
                assert torch.equal(a, b)  # integer outputs: bit-exact
        # ... and both equal the oracle's stable sort (cvmm.py:1786-1803).
        for a, b in zip(got, O.prepare_sel2(sel.cpu().numpy(), route_input=route_input)):
            if b is None:
                assert a is None
            else:
                np.testing.assert_array_equal(a.cpu().numpy().astype(np.int64), b.astype(np.int64))


def test_no_alloc_rejects_oversize_input():
    lib = _lib.load()
    n = MAX_ROUTES + 1
    rc = lib.cvmm_sel_prepare_noalloc(None, _lib.I64, n, 1, 1, None, None, None, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"CVMM_NOALLOC_MAX_ROUTES" in lib.cvmm_last_error()
