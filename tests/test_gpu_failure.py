"""Failure detection on the GPU without a GPU fault.

Every persistent kernel bounds its waits; a wait that runs out records
CVMM_DEV_TIMEOUT in the device status word and the kernel unwinds. This
test makes such a wait run out on purpose (a barrier nothing arrives on, with
a 1 ms limit), then checks the status word and that the context still runs a
full forward and backward correctly afterwards."""
import numpy as np
import pytest
import torch

from cvmm_codex_b200 import _lib, cvmm, cvmm_prepare_sel2
from oracle import cvmm_oracle as O

pytestmark = pytest.mark.gpu

DEV_TIMEOUT = 1
SELFTEST_TAG = 99


def test_bounded_wait_times_out_and_reports():
    lib = _lib.load()
    _lib.device_status(reset=True)
    rc = lib.cvmm_selftest_wait_timeout(1_000_000, _lib.stream_of(torch.device("cuda", 0)))
    assert rc == 0
    code, where, _ = _lib.device_status(reset=True)
    assert (code, where) == (DEV_TIMEOUT, SELFTEST_TAG)
    assert _lib.device_status(reset=True)[0] == 0  # reset cleared it

    # The context is intact: a bf16 forward + backward still matches the oracle.
    g = torch.Generator().manual_seed(3)
    x = torch.randn(300, 64, generator=g).bfloat16()
    keys = torch.randn(5, 64, 32, generator=g) / 8
    sel = torch.randint(0, 5, (300, 2), generator=g)
    xc = x.cuda().requires_grad_(True)
    kc = keys.cuda().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = cvmm(xc, cvmm_prepare_sel2(sel.cuda()), kc)
    out.backward(torch.ones_like(out))
    want = O.forward(x.float().numpy(), sel.numpy(), keys.numpy(), op="bfloat16")
    assert O.rel_max_err(out.detach().float().cpu().numpy(), want) < 2e-2
    assert _lib.device_status(reset=True)[0] == 0


def test_selftest_rejects_out_of_range_limits():
    lib = _lib.load()
    assert lib.cvmm_selftest_wait_timeout(10, None) == -1
    assert lib.cvmm_selftest_wait_timeout(10**9, None) == -1
