"""Token sharding across 2 gloo ranks on CPU: per-rank grad-W of the rank's
tokens, summed by the all-reduce, equals the grad-W of the whole batch
(oracle math; no GPU)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cvmm_codex_b200.dist import allreduce_expert_grads, token_slice
from oracle import cvmm_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        T, k, E, d_in, d_out = 37, 3, 5, 16, 12
        x = torch.randn(T, d_in, generator=g, dtype=torch.float64)
        keys = torch.randn(E, d_in, d_out, generator=g, dtype=torch.float64)
        sel = torch.randint(0, E, (T, k), generator=g)
        grad = torch.randn(T, k, d_out, generator=g, dtype=torch.float64)
        sl = token_slice(T, rank, world)
        _, gk, _ = O.backward(x[sl].numpy(), sel[sl].numpy(), keys.numpy(), grad[sl].numpy(), op="float32")
        kp = torch.nn.Parameter(keys.clone())
        kp.grad = torch.from_numpy(gk)
        allreduce_expert_grads(kp)
        _, full, _ = O.backward(x.numpy(), sel.numpy(), keys.numpy(), grad.numpy(), op="float32")
        q.put((rank, float(np.max(np.abs(kp.grad.numpy() - full)))))
    finally:
        dist.destroy_process_group()


def test_token_slices_cover_tokens():
    for T in (1, 7, 16384):
        for world in (1, 2, 3, 8):
            parts = [token_slice(T, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == T
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))


def test_sharded_grad_w_allreduce_matches_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    errs = dict(q.get(timeout=10) for _ in range(2))
    assert max(errs.values()) < 1e-9
