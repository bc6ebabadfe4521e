"""Token-sharded data parallelism on 2 GPUs (NCCL): the grad-W all-reduce
overlapped with grad-x gives the same gradients, bit for bit, as one
all-reduce after the backward, in eager steps and in CUDA-graph replays; and
the summed gradient equals the full batch's grad-W (within fp32 summation
order). Skipped on a box with fewer than 2 GPUs."""
import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import bench
        from cvmm_codex_b200.workloads import Workload, make_inputs
        w = Workload("dp_test", 2048, 256, 128, 16, 4, False, False, True, "bias")
        d = make_inputs(w, "cuda", seed=rank)
        res = {}
        for mode in ("serial", "overlap"):
            step = bench.build_step(w, d, world, overlap=(mode == "overlap"))
            step(d["sel"], d["grad_out"])
            torch.cuda.synchronize()
            res[mode] = d["keys"].grad.clone()
        g = bench.GraphedStep(bench.build_step(w, d, world, overlap=True), d)
        for _ in range(2):
            g()
        torch.cuda.synchronize()
        res["graph"] = d["keys"].grad.clone()
        # every rank's local grad-W, summed here = the full batch's grad-W
        step = bench.build_step(w, d, 1)
        step(d["sel"], d["grad_out"])
        local = d["keys"].grad.clone()
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        total = torch.stack(parts).sum(0)
        ok = (torch.equal(res["serial"], res["overlap"]) and torch.equal(res["serial"], res["graph"]))
        err = ((res["serial"] - total).abs().max() / total.abs().max()).item()
        q.put((rank, ok, err))
    finally:
        dist.destroy_process_group()


def test_overlapped_allreduce_matches_serial_on_2_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for _ in range(2):
        rank, ok, err = q.get(timeout=10)
        assert ok, f"rank {rank}: overlapped all-reduce differs from the serial one"
        assert err < 1e-5, (rank, err)
