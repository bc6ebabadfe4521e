"""CVMM fw+bw benchmark (B200, sm_100a).

One step = the whole CVMM hot path over one batch of the workload:
cvmm_prepare_sel2 (device radix sort) -> forward gather-GEMM (+ weighted
combine) -> backward (grad-W, grad-x, sel-weight grad); with N > 1 GPUs each
rank processes its own tokens (weak scaling) and the fp32 expert-weight
gradients are summed with an NCCL all-reduce inside the step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

Prints one JSON line (rank 0). The step is captured once as a CUDA graph and
replayed (`--eager` times Python-issued steps instead); every kernel of the
step runs on every replay. Timing: CUDA events on the compute stream around
each step, L2 flushed (256 MiB write) before every timed step and outside the
events, max over ranks. `e2e` repeats the step with the step's inputs copied
from pinned host memory into the step's input tensors and a scalar read back,
every step (host-to-device copies prefetched one step ahead on a copy stream). `roofline` covers the native call with the largest share of the
step, timed with CUDA events around its launches in eager steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "CVMM fw+bw ms/iter & TFLOP/s (% B200 BF16 TC peak), σ-MoE shapes, 1–8 GPU"
DEFAULT_WORKLOAD = "ff_up_1024"  # BASELINE configs[1]; its metric is quoted on ff_up_1024


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--workload", default=DEFAULT_WORKLOAD)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--eager", action="store_true", help="time eager steps instead of CUDA-graph replays")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--serial-allreduce", action="store_true",
                   help="N > 1: one grad-W all-reduce after the backward instead of overlapping it with grad-x")
    p.add_argument("--ep", action="store_true",
                   help="expert-sharded mode: each rank owns E/N experts, routes travel by all-to-all "
                        "(eager steps; e.g. --workload stress_up_4096_h512)")
    p.add_argument("--also", default="ff_down_1024_weighted,ffn_1024",
                   help="comma-separated extra workloads reported under 'also' (N=1 only)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            m = json.load(f)
        return {"hbm_gbs": m["hbm_gbs"], "bf16_tflops": m["bf16_tflops"],
                "bf16_tflops_sustained": m["bf16_tflops_sustained"], "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, active: bool = True, interval_ms: int = 20):
        # With several ranks on one box only one sampler runs (local rank 0):
        # one nvidia-smi poller per GPU would compete for the driver.
        self.index = index
        self.active = active
        self.interval_ms = interval_ms
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        if not self.active:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", str(self.interval_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, limit_s):
        t_end = time.perf_counter() + limit_s
        while self.proc is not None and not self.lines and time.perf_counter() < t_end:
            time.sleep(0.02)

    def mark(self):
        """Samples before this point (idle, warm-up) are left out of the summary."""
        self.start = len(self.lines)

    def since_mark(self):
        return len(self.lines) - getattr(self, "start", 0)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[getattr(self, "start", 0):]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ our arm
def build_step(w, d, world, overlap=True):
    """One step of the public API: cvmm_prepare_sel2 -> cvmm (autocast) ->
    backward. With N > 1 ranks the fp32 expert-weight gradient is summed over
    the ranks by NCCL: overlapped with grad-x (dist.OverlappedGradReduce, the
    default) or as one all-reduce after the backward (overlap=False)."""
    from contextlib import nullcontext

    from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
    from cvmm_codex_b200.dist import OverlappedGradReduce, allreduce_expert_grads

    x = d["x"].requires_grad_(True)
    keys = d["keys"].requires_grad_(True)
    wt = None if d["weights"] is None else d["weights"].requires_grad_(True)
    reducer = OverlappedGradReduce() if (world > 1 and overlap) else None

    def compute(sel, grad_out):
        x.grad = None
        keys.grad = None
        if wt is not None:
            wt.grad = None
        with (reducer if reducer is not None else nullcontext()):
            sel2 = cvmm_prepare_sel2(sel, wt, route_input=w.route_input)
            if w.amp:
                with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                    out = cvmm(x, sel2, keys)
            else:
                out = cvmm(x, sel2, keys)
            out.backward(grad_out)
        return out

    def exchange(graphed=False):
        """The weight-gradient exchange still to issue after `compute` (eager)
        or after a replay of its captured graph."""
        if world == 1:
            return
        if reducer is None:
            allreduce_expert_grads(keys)  # one NCCL all-reduce after the backward
        elif graphed:
            reducer.launch(keys.grad)  # side stream, behind the graph's grad-W event

    def step(sel, grad_out):
        out = compute(sel, grad_out)
        exchange()
        return out

    step.compute = compute
    step.exchange = exchange
    return step


class GraphedStep:
    """The step's computation captured once as a CUDA graph and replayed: every
    kernel of it (selector prep, GEMMs, copies, reductions) runs on each
    replay; only the host's per-launch work is gone. With N > 1 the NCCL
    all-reduce of grad-W is not captured: it is issued after each replay on a
    side stream that waits on an event node the graph records right after
    grad-W, so it overlaps the graph's grad-x kernels. Inputs are the captured
    tensors d["sel"], d["grad_out"], x, keys, weights, which the e2e loop
    overwrites in place before each replay."""

    def __init__(self, step, d):
        self.d = d
        self.exchange = step.exchange
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                step(d["sel"], d["grad_out"])
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step.compute(d["sel"], d["grad_out"])
        torch.cuda.synchronize()

    def __call__(self, sel=None, grad_out=None):
        self.graph.replay()
        self.exchange(graphed=True)
        return self.out


def time_steps(run, d, steps, flush, recorder=None):
    """Device time of `steps` steps (ms, summed), each bracketed by CUDA events
    on the current stream with the L2 flushed before it, outside the events.

    With a recorder (per-call events around every native call of eager
    steps), a spin kernel of about 10 ms is queued first, so that the host
    issues the whole step while the GPU is still busy: the per-call events
    then measure device time only, not the host's launch and tensor-map work
    between them."""
    times = []
    for _ in range(steps):
        flush.zero_()
        if recorder is not None:
            torch.cuda._sleep(20_000_000)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        if recorder is not None:
            with recorder:
                run(d["sel"], d["grad_out"])
        else:
            run(d["sel"], d["grad_out"])
        b.record()
        times.append((a, b))
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in times)


def time_e2e(run, d, steps, flush):
    """Public-API steps fed from host memory: every step's inputs (x, sel,
    grad_out and the weights) are copied from pinned host memory and a scalar
    result is read back. The host-to-device copies run on a copy stream into
    two staging buffers, one step ahead (as a prefetching data loader does), so
    step i+1's copy overlaps step i's compute; each step then moves its staged
    inputs into the step's input tensors on the device and runs. Timed as one
    region over all steps (the step's working set is far larger than L2)."""
    keys_in = [k for k, v in d.items() if k != "keys" and v is not None]
    host = {k: d[k].detach().cpu().pin_memory() for k in keys_in}
    stage = [{k: torch.empty_like(d[k], requires_grad=False) for k in keys_in} for _ in range(2)]
    res_h = torch.empty((), dtype=torch.float32).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    copy_s = torch.cuda.Stream()
    cur = torch.cuda.current_stream()
    loaded = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]

    def load(i):
        b = i % 2
        copy_s.wait_event(free[b])  # staging buffer b was consumed by step i - 2
        with torch.cuda.stream(copy_s):
            for k in keys_in:
                stage[b][k].copy_(host[k], non_blocking=True)
        loaded[b].record(copy_s)

    def one(i, prefetch=True):
        b = i % 2
        if prefetch and i + 1 < n_total:
            load(i + 1)
        cur.wait_event(loaded[b])
        with torch.no_grad():
            for k in keys_in:
                d[k].copy_(stage[b][k])
        free[b].record(cur)
        out = run(d["sel"], d["grad_out"])
        res_h.copy_(out.detach()[..., 0].float().sum(), non_blocking=True)

    n_total = steps + 2
    flush.zero_()
    torch.cuda.synchronize()
    load(0)
    one(0)  # warm the pinned buffers and the copy stream
    one(1, prefetch=False)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b_ev = torch.cuda.Event(enable_timing=True)
    a.record()
    load(2)  # every timed step's inputs cross PCIe inside the timed region
    for i in range(2, n_total):
        one(i)
    b_ev.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b_ev) / steps, h2d, 4


def run_ep(args, rank, world, local_rank):
    """Expert-sharded step: rank r owns experts [r E/N, (r+1) E/N) and its own
    T tokens; the routes go to their experts' owners and back by all-to-all
    (cvmm_codex_b200.expert_parallel). The route counts pass through the host,
    so the steps run eagerly (no CUDA graph)."""
    import torch.distributed as dist

    from cvmm_codex_b200.expert_parallel import ep_cvmm, expert_range
    from cvmm_codex_b200.workloads import WORKLOADS, make_inputs

    torch.cuda.set_device(local_rank)
    w = WORKLOADS[args.workload]
    if w.route_input:
        raise SystemExit("--ep takes token-shaped workloads (route rows are formed by the dispatch)")
    d = make_inputs(w, "cuda", seed=rank)
    keys_full = make_inputs(w, "cuda", seed=0)["keys"]  # the same weights on every rank
    lo, hi = expert_range(w.E, rank, world)
    kl = keys_full[lo:hi].clone().requires_grad_(True)
    x = d["x"].requires_grad_(True)
    wt = d["weights"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def step():
        x.grad = None
        kl.grad = None
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            out = ep_cvmm(x, d["sel"], kl, w.E, weights=wt)
        out.backward(d["grad_out"])
        return out

    with ClockSampler(local_rank, active=local_rank == 0, interval_ms=20 if world == 1 else 50) as clk:
        clk.wait_first(5.0)
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clk.mark()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            torch.cuda.synchronize()
            total += a.elapsed_time(b)
    t = torch.tensor([total], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item() / args.steps
    flops = w.flops() * world
    return {
        "metric": METRIC, "value": round(flops / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded; shapes of the BASELINE config, inputs generated on device)",
        "config": {"workload": w.name, "tokens_per_gpu": w.T, "d_in": w.d_in, "d_out": w.d_out, "experts": w.E,
                   "experts_per_gpu": hi - lo, "top_k": w.k, "weighted": w.weighted,
                   "parallelism": f"expert-sharded ep{world} (all-to-all dispatch)", "cuda_graph": False,
                   "l2": "flushed (256 MiB write) before every timed step"},
        "clocks": clk.summary(),
        "gpu_launches": None,
    }


def workload_config(w, world):
    """The workload keys of the JSON line, identical in both arms."""
    return {"workload": w.name, "tokens_per_gpu": w.T, "d_in": w.d_in, "d_out": w.d_out, "experts": w.E,
            "top_k": w.k, "weighted": w.weighted, "route_input": w.route_input, "global_tokens": w.T * world,
            "parallelism": f"token-sharded dp{world}", "flops_per_step_per_gpu": w.flops()}


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist

    from cvmm_codex_b200 import _lib, ops
    from cvmm_codex_b200.workloads import WORKLOADS, make_inputs

    torch.cuda.set_device(local_rank)
    pk = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def measure(name, with_e2e, with_roofline):
        w = WORKLOADS[name]
        d = make_inputs(w, "cuda", seed=rank)
        step = build_step(w, d, world, overlap=not args.serial_allreduce)
        rec = ops.Recorder()
        for _ in range(max(args.warmup, 3)):
            step(d["sel"], d["grad_out"])
        # Per-call device times and launch counts: eager steps with CUDA events
        # around every native call (the roofline's kernel durations).
        time_steps(step, d, max(3, min(args.steps, 10)), flush, rec)
        run, graphed = step, False
        if not args.eager:
            try:
                run, graphed = GraphedStep(step, d), True
            except Exception as exc:  # capture unsupported here: time the eager step
                print(f"CUDA graph capture failed ({exc!r}); timing eager steps", file=sys.stderr)
                torch.cuda.synchronize()
        with ClockSampler(local_rank, active=local_rank == 0, interval_ms=20 if world == 1 else 50) as clk:
            clk.wait_first(5.0)  # nvidia-smi takes a moment to print its first line
            for _ in range(max(args.warmup, 3)):
                run(d["sel"], d["grad_out"])
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            clk.mark()
            total_ms = time_steps(run, d, args.steps, flush)
            # A short timed region may end between two samples: keep the same
            # replays running (untimed) until the sampler (rank 0's) has seen
            # the load. With N > 1 every replay ends in an all-reduce, so rank 0
            # decides each round and broadcasts it: all ranks run the same
            # sequence of collectives.
            t_end = time.perf_counter() + 1.0
            while True:
                more = clk.since_mark() < 10 and time.perf_counter() < t_end
                if world > 1:
                    flag = torch.tensor([1 if more else 0], device="cuda")
                    dist.broadcast(flag, src=0)
                    more = bool(flag.item())
                if not more:
                    break
                for _ in range(20):
                    run(d["sel"], d["grad_out"])
                torch.cuda.synchronize()
        if world > 1:
            t = torch.tensor([total_ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            total_ms = t.item()
        torch.cuda.synchronize()
        ms = total_ms / args.steps
        flops = w.flops() * world
        res = {"w": w, "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "clocks": clk.summary(),
               "launches": rec.launches // max(rec.steps, 1), "per_call": rec.summary(), "graphed": graphed}
        if with_e2e:
            e_ms, bi, bo = time_e2e(run, d, max(3, args.steps // 5), flush)
            if world > 1:
                t = torch.tensor([e_ms], device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e_ms = t.item()
            res["e2e"] = {"value": round(flops / (e_ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
                          "ms_per_step": round(e_ms, 4), "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo}
        if with_roofline:
            res["roofline"], res["roofline_calls"] = roofline(w, res["per_call"], rec.steps, pk)
            res["step_roofline"] = step_roofline(w, ms, pk)
        # A bounded wait that ran out inside a kernel leaves partial outputs and
        # a code in the device status word: such a run has no valid number.
        code, where, aux = _lib.device_status(reset=True)
        if code != 0:
            raise RuntimeError(f"device status {code} (site {where}, aux {aux}) after the {name} steps: "
                               "a kernel gave up on a bounded wait; the measurement is invalid")
        return res

    main = measure(args.workload, not args.no_e2e, True)
    w = main["w"]
    line = {
        "metric": METRIC, "value": round(main["tflops"], 3), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main["ms"], 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if w.amp else "f32",
        "data": "synthetic (seeded; shapes of the BASELINE config, inputs generated on device)",
        "config": dict(workload_config(w, world),
                       grad_w_allreduce=None if world == 1 else ("after backward" if args.serial_allreduce
                                                                 else "overlapped with grad-x"),
                       l2="flushed (256 MiB write) before every timed step",
                       cuda_graph=main["graphed"],
                       pct_bf16_peak_sustained=round(100 * main["tflops"] / world / pk["bf16_tflops_sustained"], 2)),
        "clocks": main["clocks"],
        "gpu_launches": main["launches"] * args.steps,
        "roofline": main["roofline"],
        "step_roofline": main["step_roofline"],
        "roofline_calls": main["roofline_calls"],
        "device_status": 0,
    }
    if "e2e" in main:
        line["e2e"] = main["e2e"]
    if world == 1 and args.also:
        also = {}
        for name in [s for s in args.also.split(",") if s in WORKLOADS and s != args.workload]:
            r = measure(name, False, True)
            also[name] = {"value": round(r["tflops"], 3), "unit": "TFLOP/s", "ms_per_step": round(r["ms"], 4),
                          "pct_bf16_peak_sustained": round(100 * r["tflops"] / pk["bf16_tflops_sustained"], 2),
                          "roofline": r["roofline"], "step_roofline": r["step_roofline"]}
        for name in [s for s in args.also.split(",") if s in FFN_SHAPES]:
            also[name] = measure_ffn(FFN_SHAPES[name], args, flush, pk)
        line["also"] = also
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, budget_s=10.0)
    return line


def gemm_bytes(w):
    """Algorithmic HBM bytes of the three GEMMs of one fw+bw step, as the
    benchmark contract counts them: 16-bit activations and fp32 weights (16-bit
    weights in the bf16_params mode), every
    input read once and every output written once per GEMM (no padding, no
    intermediate copies). For ff_up_1024 each GEMM is 83.9 MB (x 33.5 + W 33.5
    + Y 16.8), 252 MB per step; ff_down_1024_weighted moves 269 MB (its grad-x
    also reads the route rows of x for the sel-weight grad)."""
    R, T, E, di, do = w.R, w.T, w.E, w.d_in, w.d_out
    act = 2 if (w.amp or w.bf16_params) else 4
    wts = E * di * do * (2 if w.bf16_params else 4)
    x_rows = w.x_rows                         # unique input rows
    g_rows = T if w.weighted else R           # unique grad rows
    fw = x_rows * di * act + wts + g_rows * do * act + (R * 4 if w.weighted else 0)
    gx = g_rows * do * act + wts + x_rows * di * act
    if w.weighted:
        gx += R * 4 + R * 4 + (w.x_rows * di * act if w.route_input else 0)  # w in, sel grad out, x for the dot
    gw = x_rows * di * act + g_rows * do * act + wts + (R * 4 if w.weighted else 0)
    return {"cvmm_forward": fw, "cvmm_backward_x": gx, "cvmm_backward_w": gw}


# ------------------------------------------------------------------ the sigma-MoE layer
# The reference's FFN benchmark shapes (benchmark_ffn_moe.py:26-38): B x T tokens,
# model width D, expert width H, top-K of E experts.
FFN_SHAPES = {
    "ffn_1024": dict(B=8, T=2048, D=1024, H=128, K=8, E=512),
    "ffn_2048": dict(B=4, T=2048, D=2048, H=128, K=8, E=512),
}


def measure_ffn(shape, args, flush, pk):
    """One sigma-MoE FFN layer step (router matmul, fused router top-k, one
    selector prep, up projection with fused GELU, weighted down projection,
    full backward) as a CUDA graph, against the same layer composed as the
    reference writes it (torch softmax/topk/renormalisation, F.gelu, two
    selector preps) on the same CVMM kernels. Seeded synthetic inputs; fp32
    parameters under bf16 autocast."""
    import math

    import torch.nn.functional as F

    from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2, sigma_moe_ffn

    B, T, D, H, K, E = (shape[k] for k in ("B", "T", "D", "H", "K", "E"))
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(B * T, D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    gate = (torch.randn(D, E, device="cuda", generator=g) / math.sqrt(D)).requires_grad_(True)
    w_up = (torch.randn(E, D, H, device="cuda", generator=g) / math.sqrt(D)).requires_grad_(True)
    w_down = (torch.randn(E, H, D, device="cuda", generator=g) / math.sqrt(H)).requires_grad_(True)
    grad = torch.randn(B * T, D, device="cuda", generator=g).bfloat16()
    params = (x, gate, w_up, w_down)

    def fused():
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            out = sigma_moe_ffn(x, gate, w_up, w_down, K)
        out.backward(grad)

    def composed():  # benchmark_ffn_moe.py:87-98
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            logits = x @ gate
            probs = torch.softmax(logits.float(), dim=-1)
            weights, sel = probs.topk(K, dim=-1)
            weights = weights / weights.sum(dim=-1, keepdim=True).clamp_min(1e-20)
            sel_up = cvmm_prepare_sel2(sel)
            hidden = F.gelu(cvmm(x, sel_up, w_up))
            sel_down = cvmm_prepare_sel2(sel_up, weights, route_input=True)
            out = cvmm(hidden.view(B * T, K, H), sel_down, w_down)
        out.backward(grad)

    def run(fn):
        def step():
            for p in params:
                p.grad = None
            fn()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(max(args.warmup, 3)):
            graph.replay()
        torch.cuda.synchronize()
        total = 0.0
        for _ in range(args.steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            b.synchronize()
            total += a.elapsed_time(b)
        del graph
        return total / args.steps

    ms = run(fused)
    ms_composed = run(composed)
    R = B * T * K
    flops_cvmm = 12.0 * R * D * H        # up + down, 3 GEMMs each
    flops_router = 6.0 * B * T * D * E   # x @ gate forward and its two backward GEMMs
    return {"value": round((flops_cvmm + flops_router) / (ms * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
            "ms_per_step": round(ms, 4), "ms_per_step_reference_composition": round(ms_composed, 4),
            "config": {"tokens": B * T, "d_model": D, "expert_width": H, "top_k": K, "experts": E,
                       "flops_cvmm": flops_cvmm, "flops_router": flops_router,
                       "what": "sigma-MoE FFN layer fw+bw: fused router top-k, one selector prep, "
                               "GELU in the up projection's epilogue"}}


def call_work(w, name):
    """(algorithmic bytes, flops, design bytes) of ONE call of native entry
    point `name` in a step of workload `w`.

    The three GEMM calls carry the contract's algorithmic bytes (gemm_bytes);
    every other call (selector prep, weight cast, sorted copies, k-sum,
    combine) moves bytes only because of this design's data layout, so its
    algorithmic bytes are 0 and its traffic is reported as design bytes (what
    it must read and write at the least in this design)."""
    R, T, E, di, do = w.R, w.T, w.E, w.d_in, w.d_out
    wts = E * di * do
    gemm = 2.0 * R * di * do
    alg = gemm_bytes(w)
    if name in alg:
        return float(alg[name]), gemm, float(alg[name])
    if name == "cvmm_sel_prepare":
        return 0.0, 0.0, float(R * 8 + R * (4 + 4 + 8 + (0 if w.route_input else 8)))
    if name == "cvmm_expert_offsets":
        return 0.0, 0.0, float(R * 4 + E * 8)
    if name == "cvmm_cast":
        return 0.0, 0.0, float(wts * (4 + 2))
    if name in ("cvmm_sort_rows_padded", "cvmm_sort_rows_padded_ex"):
        # weighted steps: the forward's x copy (plain call) and the grad copy
        # (_ex, pad starts reused); unweighted: the grad copy, with the route
        # row map (_ex) when the k-sum follows.
        x_copy = w.x_rows * di * 2 + R * di * 2
        g_copy = (T * do * 2 + R * 4 if w.weighted else R * do * 2) + R * do * 2
        if w.weighted:
            return 0.0, 0.0, float(x_copy if name == "cvmm_sort_rows_padded" else g_copy)
        return 0.0, 0.0, float(g_copy + (R * 4 if name == "cvmm_sort_rows_padded_ex" else 0))
    if name == "cvmm_pad_starts":
        return 0.0, 0.0, float(E * 12)
    if name == "cvmm_padded_route_rows":
        return 0.0, 0.0, float(R * 16)
    if name == "cvmm_sum_routes":
        return 0.0, 0.0, float(R * di * 2 + T * di * 2)
    if name == "cvmm_weighted_combine":
        return 0.0, 0.0, float(R * do * 2 + R * 4 + T * do * 2)
    return 0.0, 0.0, 0.0


def dram_traffic(workload, call):
    """DRAM bytes (read + write) per launch of the call's main kernel from the
    committed ncu capture summary, or None."""
    path = os.path.join(ROOT, "profiles", "dram_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)["workloads"][workload].get(call)
    except (OSError, KeyError, ValueError):
        return None


def roofline(w, per_call, steps, pk):
    """Per native call: bytes and FLOPs over its device time (CUDA events on
    the launching stream, host work kept off the clock). The GEMM calls use
    the contract's algorithmic bytes; the others their design bytes. The bound
    is whichever of HBM (measured copy bandwidth) and the tensor cores
    (measured sustained bf16) gives the longer ideal time. Returns the entry of
    the GEMM call with the largest share of the step and the whole table."""
    table = {}
    step_total = sum(v[1] for v in per_call.values())
    for name, (calls, total) in per_call.items():
        avg_ms = total / max(calls, 1)
        alg, flops, design = call_work(w, name)
        nbytes = alg if alg else design
        t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
        t_tc = flops / (pk["bf16_tflops_sustained"] * 1e12)
        if flops and t_tc >= t_hbm:
            ach, peak, unit, bound = flops / (avg_ms * 1e-3) / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s", "tensor"
        else:
            ach, peak, unit, bound = nbytes / (avg_ms * 1e-3) / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
        table[name] = {"bound": bound, "achieved": round(ach, 2), "peak": peak, "unit": unit,
                       "frac": round(ach / peak, 4), "avg_ms": round(avg_ms, 5),
                       "calls_per_step": calls // max(steps, 1),
                       "share": round(total / step_total, 3) if step_total else None,
                       "algorithmic_bytes": int(alg), "design_bytes": int(design), "flops": int(flops)}
    gemms = [k for k in per_call if k in gemm_bytes(w)] or list(per_call)
    name = max(gemms, key=lambda k: per_call[k][1])
    top = dict(table[name])
    top["kernel"] = name
    top["traffic"] = dram_traffic(w.name, name)
    top["peak_source"] = f"{pk['source']} ({'hbm copy' if top['bound'] == 'hbm' else 'bf16 sustained'})"
    return top, table


def step_roofline(w, ms, pk):
    """Whole step against the contract: algorithmic bytes of the three GEMMs
    over the step time, and the FLOPs over the step time."""
    nbytes = sum(gemm_bytes(w).values())
    flops = w.flops()
    t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
    t_tc = flops / (pk["bf16_tflops_sustained"] * 1e12)
    return {"algorithmic_bytes": int(nbytes), "flops": int(flops),
            "ideal_ms": round(max(t_hbm, t_tc) * 1e3, 4), "bound": "hbm" if t_hbm >= t_tc else "tensor",
            "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / pk["hbm_gbs"], 4),
            "tensor_frac": round(flops / (ms * 1e-3) / 1e12 / pk["bf16_tflops_sustained"], 4)}


# ------------------------------------------------------------------ CPU baseline / reference arm
def cpu_tokens(w, max_flops=1.2e11):
    """Tokens of the CPU sample: the whole configuration when its fw+bw is at
    most `max_flops` (ff_up_1024 and ff_down_1024_weighted: 51.5 GFLOP, about
    0.2-0.5 s per step on 16 host cores), else the leading tokens that make up
    that many FLOPs."""
    if w.flops() <= max_flops:
        return w.T
    return max(64, int(w.T * max_flops / w.flops()))


def time_cpu_reference(w, reps: int, warmup: int, budget_s: float):
    """The reference's pure-PyTorch per-expert step (fp32, all host cores) on
    `cpu_tokens(w)` tokens: `warmup` untimed steps, then at least `reps` timed
    steps (more while the budget lasts). Returns (min s/step, mean s/step,
    reps, n_tokens, threads). The minimum is the reported figure: the host is
    shared with the driver and its samplers, and the fastest repeat is the one
    least disturbed by them."""
    sys.path.insert(0, ROOT)
    from oracle import cpu_baseline as cb

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_tok = cpu_tokens(w)
    d = cb.make_sample(w, n_tok)
    for _ in range(max(warmup, 1)):
        cb.step(w, d)
    times = []
    t_start = time.perf_counter()
    while len(times) < reps or (time.perf_counter() - t_start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        cb.step(w, d)
        times.append(time.perf_counter() - t0)
    return min(times), sum(times) / len(times), len(times), n_tok, threads


def cpu_baseline(w, budget_s: float):
    """The reference's pure-PyTorch per-expert math on the host cores (fp32),
    minimum over at least 3 repeats, in TFLOP/s."""
    best, mean, reps, n_tok, threads = time_cpu_reference(w, 3, 1, budget_s)
    flops = 3 * 2 * n_tok * w.k * w.d_in * w.d_out
    return {"value": round(flops / best / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n_tok} of {w.T} tokens of {w.name}, fp32 torch-CPU per-expert fw+bw, "
                      f"min of {reps} reps: {best * 1e3:.1f} ms/rep (mean {mean * 1e3:.1f})"}


def run_reference(args, rank):
    """The reference arm: the reference's own CPU path of the step (its
    pure-PyTorch per-expert gather + matmul, the oracle port) on the host
    cores, rank 0 only. Each timed step is one fw+bw over the bench's
    configuration (the whole token set for ff_*_1024); ms_per_step is the
    minimum over the K steps, the same method as `cpu_baseline`."""
    from cvmm_codex_b200.workloads import WORKLOADS

    if rank != 0:
        return None
    w = WORKLOADS[args.workload]
    best, mean, reps, n_tok, threads = time_cpu_reference(w, max(args.steps, 3), min(args.warmup, 2), 0.0)
    flops = 3 * 2 * n_tok * w.k * w.d_in * w.d_out
    tf = flops / best / 1e12
    sample = (f"{n_tok} of {w.T} tokens of {w.name} per step (fp32 torch-CPU per-expert fw+bw, the reference's "
              f"math); min of {reps} steps, mean {mean * 1e3:.1f} ms")
    return {
        "metric": METRIC, "value": round(tf, 5), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": reps,
        "warmup": args.warmup, "ms_per_step": round(best * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, same recipe as our arm)",
        "config": dict(workload_config(w, args.gpus), tokens_timed=n_tok, host="CPU, all host cores"),
        "impl": "reference",
        "cpu_baseline": {"value": round(tf, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tf, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    # The drop-in module prints "New shape:" like the reference and NCCL prints
    # its banner from C++: both go to stderr (file-descriptor level) so stdout
    # carries only the one JSON line.
    import contextlib
    sys.stdout.flush()
    saved_fd = os.dup(1)
    os.dup2(2, 1)
    try:
        if world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        with contextlib.redirect_stdout(sys.stderr):
            line = (run_ep if args.ep else run_ours)(args, rank, world, local_rank)
    finally:
        sys.stdout.flush()
        os.dup2(saved_fd, 1)
        os.close(saved_fd)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
