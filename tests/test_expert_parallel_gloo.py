"""Expert-sharded CVMM across 2 gloo ranks on CPU: the all-to-all dispatch and
combine (with their backward) against the dense per-route computation with
all experts. The local expert compute is a torch stand-in here (the CUDA
kernels need a GPU); tests/test_gpu_expert_parallel.py runs the real one."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cvmm_codex_b200.expert_parallel import ep_cvmm, expert_range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _local(x_rows, ids, keys_local):
    return torch.bmm(x_rows.unsqueeze(1), keys_local[ids.long()]).squeeze(1)


def _dense(x, sel, keys, w):
    y = torch.einsum("tkd,tkdn->tkn", x.unsqueeze(1).expand(-1, sel.shape[1], -1), keys[sel])
    return y if w is None else torch.einsum("tk,tkn->tn", w, y)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        E, d_in, d_out, k = 6, 8, 5, 2
        keys = torch.randn(E, d_in, d_out, generator=torch.Generator().manual_seed(0), dtype=torch.float64)
        lo, hi = expert_range(E, rank, world)
        errs = []
        for weighted in (False, True):
            g = torch.Generator().manual_seed(10 + rank)
            T = 7 + 4 * rank  # uneven token counts per rank
            x = torch.randn(T, d_in, generator=g, dtype=torch.float64)
            sel = torch.randint(0, E, (T, k), generator=g)
            sel[0] = torch.tensor([0, E - 1])  # both ranks' experts appear
            w = torch.rand(T, k, generator=g, dtype=torch.float64) if weighted else None
            go = torch.randn(*((T, d_out) if weighted else (T, k, d_out)), generator=g, dtype=torch.float64)

            xe = x.clone().requires_grad_(True)
            kl = keys[lo:hi].clone().requires_grad_(True)
            out = ep_cvmm(xe, sel, kl, E, weights=w, local_fn=_local)
            out.backward(go)

            xd = x.clone().requires_grad_(True)
            kd = keys.clone().requires_grad_(True)
            ref = _dense(xd, sel, kd, w)
            ref.backward(go)
            kgrad = kd.grad.clone()
            dist.all_reduce(kgrad)  # expert e's gradient collects every rank's routes to e
            errs.append(max(float((out - ref).abs().max()), float((xe.grad - xd.grad).abs().max()),
                            float((kl.grad - kgrad[lo:hi]).abs().max())))
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


def test_expert_sharded_dispatch_and_backward_match_dense():
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
    assert max(errs.values()) < 1e-10, errs


def test_expert_range_splits_evenly():
    assert [expert_range(8, r, 4) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    try:
        expert_range(6, 0, 4)
    except ValueError:
        pass
    else:
        raise AssertionError("uneven split accepted")
