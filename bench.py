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
    p.add_argument("--ep", action="store_true",
                   help="expert-sharded mode: each rank owns E/N experts, routes travel by all-to-all "
                        "(eager steps; e.g. --workload stress_up_4096_h512)")
    p.add_argument("--also", default="ff_down_1024_weighted",
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
def build_step(w, d, world):
    from cvmm_codex_b200 import cvmm, cvmm_prepare_sel2
    from cvmm_codex_b200.dist import allreduce_expert_grads

    x = d["x"].requires_grad_(True)
    keys = d["keys"].requires_grad_(True)
    wt = None if d["weights"] is None else d["weights"].requires_grad_(True)

    def compute(sel, grad_out):
        x.grad = None
        keys.grad = None
        if wt is not None:
            wt.grad = None
        sel2 = cvmm_prepare_sel2(sel, wt, route_input=w.route_input)
        if w.amp:
            with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
                out = cvmm(x, sel2, keys)
        else:
            out = cvmm(x, sel2, keys)
        out.backward(grad_out)
        return out

    def exchange():
        if world > 1:
            allreduce_expert_grads(keys)  # the token-sharding exchange (NCCL)

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
    all-reduce of grad-W follows each replay as an ordinary (eager) collective
    on the same stream; collectives are kept out of the graph. Inputs are the
    captured tensors d["sel"], d["grad_out"], x, keys, weights, which the e2e
    loop overwrites in place before each replay."""

    def __init__(self, step, d):
        self.d = d
        self.exchange = step.exchange
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                step.compute(d["sel"], d["grad_out"])
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = step.compute(d["sel"], d["grad_out"])
        torch.cuda.synchronize()

    def __call__(self, sel=None, grad_out=None):
        self.graph.replay()
        self.exchange()
        return self.out


def time_steps(run, d, steps, flush, recorder=None):
    """Device time of `steps` steps (ms, summed), each bracketed by CUDA events
    on the current stream with the L2 flushed before it, outside the events."""
    times = []
    for _ in range(steps):
        flush.zero_()
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


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist

    from cvmm_codex_b200 import ops
    from cvmm_codex_b200.workloads import WORKLOADS, make_inputs

    torch.cuda.set_device(local_rank)
    pk = peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def measure(name, with_e2e, with_roofline):
        w = WORKLOADS[name]
        d = make_inputs(w, "cuda", seed=rank)
        step = build_step(w, d, world)
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
        return res

    main = measure(args.workload, not args.no_e2e, True)
    w = main["w"]
    line = {
        "metric": METRIC, "value": round(main["tflops"], 3), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(main["ms"], 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if w.amp else "f32",
        "data": "synthetic (seeded; shapes of the BASELINE config, inputs generated on device)",
        "config": {"workload": w.name, "tokens_per_gpu": w.T, "d_in": w.d_in, "d_out": w.d_out,
                   "experts": w.E, "top_k": w.k, "weighted": w.weighted, "route_input": w.route_input,
                   "global_tokens": w.T * world, "parallelism": f"token-sharded dp{world}",
                   "l2": "flushed (256 MiB write) before every timed step",
                   "cuda_graph": main["graphed"],
                   "flops_per_step_per_gpu": w.flops(),
                   "pct_bf16_peak_sustained": round(100 * main["tflops"] / world / pk["bf16_tflops_sustained"], 2)},
        "clocks": main["clocks"],
        "gpu_launches": main["launches"] * args.steps,
        "roofline": main["roofline"],
        "roofline_calls": main["roofline_calls"],
    }
    if "e2e" in main:
        line["e2e"] = main["e2e"]
    if world == 1 and args.also:
        also = {}
        for name in [s for s in args.also.split(",") if s in WORKLOADS and s != args.workload]:
            r = measure(name, False, True)
            also[name] = {"value": round(r["tflops"], 3), "unit": "TFLOP/s", "ms_per_step": round(r["ms"], 4),
                          "pct_bf16_peak_sustained": round(100 * r["tflops"] / pk["bf16_tflops_sustained"], 2),
                          "roofline": r["roofline"]}
        line["also"] = also
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(w, budget_s=10.0)
    return line


def call_work(w, name):
    """Algorithmic (bytes, flops) of ONE call of native entry point `name` in a
    step of workload `w`: the bytes the call must move to and from HBM with
    16-bit activations (inputs read once, outputs written once, the padding of
    the sorted layout not counted) and its multiply-add FLOPs."""
    R, T, E, di, do = w.R, w.T, w.E, w.d_in, w.d_out
    wts = E * di * do
    gemm = 2.0 * R * di * do
    if name == "cvmm_sel_prepare":
        return R * 8 + R * (4 + 4 + 8 + (0 if w.route_input else 8)), 0.0
    if name == "cvmm_expert_offsets":
        return R * 4 + E * 8, 0.0
    if name == "cvmm_cast":
        return wts * (4 + 2), 0.0
    if name == "cvmm_sort_rows_padded":
        # weighted: the x copy and the weight-scaled grad copy (mean of the two
        # calls); unweighted: the grad copy (the forward writes the x copy)
        x_copy = (R if w.route_input else T) * di * 2 + R * di * 2
        g_copy = (T * do * 2 + R * 4 if w.weighted else R * do * 2) + R * do * 2
        return ((x_copy + g_copy) / 2 if w.weighted else g_copy), 0.0
    if name == "cvmm_pad_starts":
        return E * 8 + E * 4, 0.0
    if name == "cvmm_padded_route_rows":
        return R * 16, 0.0
    if name == "cvmm_forward":
        if w.weighted:  # sorted x in, padded route outputs out
            return R * di * 2 + wts * 2 + R * do * 2, gemm
        # gathered token rows in, route outputs and the sorted x copy out
        return (R if w.route_input else T) * di * 2 + wts * 2 + R * do * 2 + R * di * 2, gemm
    if name == "cvmm_backward_w":
        return R * di * 2 + R * do * 2 + wts * 4, gemm
    if name == "cvmm_backward_x":
        if w.weighted:  # token grads, route weights, route x for the sel-weight grad
            return T * do * 2 + R * 4 + R * di * 2 + wts * 2 + R * di * 2 + R * 4, gemm
        return R * do * 2 + wts * 2 + R * di * 2, gemm
    if name == "cvmm_sum_routes":
        return R * di * 2 + T * di * 2, 0.0
    if name == "cvmm_weighted_combine":
        return R * do * 2 + R * 4 + T * do * 2, 0.0
    return 0.0, 0.0


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
    """Per native call: algorithmic bytes and FLOPs over its CUDA-event time;
    the bound is whichever of HBM (measured copy bandwidth) and the tensor
    cores (measured sustained bf16) allows the shorter time. Returns the entry
    of the call with the largest share of the step and the whole table."""
    table = {}
    step_total = sum(v[1] for v in per_call.values())
    for name, (calls, total) in per_call.items():
        avg_ms = total / max(calls, 1)
        nbytes, flops = call_work(w, name)
        t_hbm = nbytes / (pk["hbm_gbs"] * 1e9)
        t_tc = flops / (pk["bf16_tflops_sustained"] * 1e12)
        if flops and t_tc >= t_hbm:
            ach, peak, unit, bound = flops / (avg_ms * 1e-3) / 1e12, pk["bf16_tflops_sustained"], "TFLOP/s", "tensor"
        else:
            ach, peak, unit, bound = nbytes / (avg_ms * 1e-3) / 1e9, pk["hbm_gbs"], "GB/s", "hbm"
        table[name] = {"bound": bound, "achieved": round(ach, 2), "peak": peak, "unit": unit,
                       "frac": round(ach / peak, 4), "avg_ms": round(avg_ms, 5), "calls_per_step": calls // max(steps, 1),
                       "share": round(total / step_total, 3) if step_total else None,
                       "algorithmic_bytes": int(nbytes), "flops": int(flops)}
    name = max(per_call, key=lambda k: per_call[k][1])
    top = dict(table[name])
    top["kernel"] = name
    top["traffic"] = dram_traffic(w.name, name)
    top["peak_source"] = f"{pk['source']} ({'hbm copy' if top['bound'] == 'hbm' else 'bf16 sustained'})"
    return top, table


# ------------------------------------------------------------------ CPU baseline / reference arm
def cpu_baseline(w, budget_s: float):
    """The reference's pure-PyTorch per-expert math on the host cores (fp32),
    timed on a bounded token sample and scaled to the metric (TFLOP/s)."""
    sys.path.insert(0, ROOT)
    from oracle import cpu_baseline as cb

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_tok = max(64, min(w.T, 2048))
    d = cb.make_sample(w, n_tok)
    cb.step(w, d)  # warm
    t0 = time.perf_counter()
    reps = 0
    while True:
        cb.step(w, d)
        reps += 1
        el = time.perf_counter() - t0
        if el > budget_s or reps >= 50:
            break
    per = el / reps
    flops = 3 * 2 * n_tok * w.k * w.d_in * w.d_out
    return {"value": round(flops / per / 1e12, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{n_tok} of {w.T} tokens of {w.name}, fp32 torch-CPU per-expert fw+bw, "
                      f"{reps} reps, {per * 1e3:.1f} ms/rep"}


def run_reference(args, rank):
    from cvmm_codex_b200.workloads import WORKLOADS

    if rank != 0:
        return None
    w = WORKLOADS[args.workload]
    sys.path.insert(0, ROOT)
    from oracle import cpu_baseline as cb

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    n_tok = max(64, min(w.T, 2048))
    d = cb.make_sample(w, n_tok)
    for _ in range(min(args.warmup, 3)):
        cb.step(w, d)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cb.step(w, d)
    per = (time.perf_counter() - t0) / args.steps
    flops_sample = 3 * 2 * n_tok * w.k * w.d_in * w.d_out
    tf = flops_sample / per / 1e12
    full_ms = per * 1e3 * (w.T / n_tok)
    sample = f"{n_tok} of {w.T} tokens of {w.name} per step (fp32 torch-CPU per-expert fw+bw, the reference's math)"
    return {
        "metric": METRIC, "value": round(tf, 5), "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(full_ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, same recipe as our arm)",
        "config": {"workload": w.name, "tokens_per_gpu": w.T, "d_in": w.d_in, "d_out": w.d_out, "experts": w.E,
                   "top_k": w.k, "parallelism": "host CPU"},
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
