"""Expert-sharded CVMM through the real kernels on one GPU (a 1-rank NCCL
group): the all-to-all dispatch, the local CVMM and the combine against the
plain cvmm with all experts and against the fp64 oracle. Tolerances as in
test_gpu_numerics: max-abs error relative to the largest magnitude <= 2e-2
(bf16 arithmetic)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist

from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
from cvmm_codex_b200.expert_parallel import ep_cvmm
from oracle import cvmm_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nccl_group():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    store = dist.TCPStore("127.0.0.1", port, 1, True)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", 0))
    yield
    dist.destroy_process_group()


def _np(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


@pytest.mark.parametrize("weighted", [False, True])
def test_expert_sharded_matches_cvmm_and_oracle(nccl_group, weighted):
    g = torch.Generator().manual_seed(31)
    T, k, E, d_in, d_out = 600, 3, 8, 128, 96
    x = torch.randn(T, d_in, generator=g).bfloat16()
    keys = torch.randn(E, d_in, d_out, generator=g) / d_in ** 0.5
    sel = torch.randint(0, E, (T, k), generator=g)
    w = torch.rand(T, k, generator=g) if weighted else None
    go = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g)

    res = {}
    for mode in ("ep", "full"):
        xc = x.cuda().requires_grad_(True)
        kc = keys.cuda().requires_grad_(True)
        wc = None if w is None else w.cuda()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if mode == "ep":
                out = ep_cvmm(xc, sel.cuda(), kc, E, weights=wc)
            else:
                out = cvmm(xc, cvmm_prepare_sel2(sel.cuda(), wc), kc)
        out.backward(go.cuda().to(out.dtype))
        res[mode] = (out, xc.grad, kc.grad)

    eo = O.forward(_np(x), sel.numpy(), keys.numpy(), None if w is None else w.numpy(), op="bfloat16")
    ex, ek, _ = O.backward(_np(x), sel.numpy(), keys.numpy(), _np(go.to(torch.bfloat16)),
                           None if w is None else w.numpy(), op="bfloat16")
    for name, a, b, e in zip(("out", "x_grad", "keys_grad"), res["ep"], res["full"], (eo, ex, ek)):
        assert O.rel_max_err(_np(a), e) <= 2e-2, (name, O.rel_max_err(_np(a), e))
        assert O.rel_max_err(_np(a), _np(b)) <= 2e-2, name
