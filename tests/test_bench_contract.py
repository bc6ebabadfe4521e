"""The benchmark's reporting contract, on CPU: the reference arm prints one
JSON line with the required keys, and the roofline arithmetic picks the call
with the largest share and bounds each call by HBM or the tensor cores."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from cvmm_codex_b200 import ops  # noqa: E402
from cvmm_codex_b200.workloads import WORKLOADS  # noqa: E402


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1", "--workload", "cpu_plumbing"],
                       capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["cpu_baseline"]["kind"] == "port"


def test_every_native_call_has_algorithmic_work():
    for w in WORKLOADS.values():
        for name in ops.KERNELS_PER_CALL:
            alg, flops, design = bench.call_work(w, name)
            assert alg >= 0 and flops >= 0 and design >= 0
            if name in ("cvmm_forward", "cvmm_backward_x", "cvmm_backward_w"):
                assert flops == 2.0 * w.R * w.d_in * w.d_out and alg > 0
            else:
                assert alg == 0 and flops == 0


def test_algorithmic_bytes_follow_the_contract():
    """ff_up_1024: every GEMM moves x 33.5 MB + W 33.5 MB (fp32) + Y 16.8 MB;
    ff_down_1024_weighted moves 269 MB per step."""
    up = bench.gemm_bytes(WORKLOADS["ff_up_1024"])
    for v in up.values():
        assert v == 16384 * 1024 * 2 + 64 * 1024 * 128 * 4 + 65536 * 128 * 2
    down = sum(bench.gemm_bytes(WORKLOADS["ff_down_1024_weighted"]).values())
    assert abs(down / 1e6 - 269) < 2


def test_roofline_picks_the_largest_gemm_and_bounds():
    w = WORKLOADS["ff_up_1024"]
    pk = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "source": "test"}
    per_call = {"cvmm_forward": (10, 0.5), "cvmm_backward_w": (10, 0.8), "cvmm_sum_routes": (10, 0.9),
                "cvmm_cast": (10, 0.1)}
    top, table = bench.roofline(w, per_call, 10, pk)
    assert top["kernel"] == "cvmm_backward_w"  # the largest GEMM, not the k-sum
    b, f, _ = bench.call_work(w, "cvmm_backward_w")
    # ff_up's GEMMs are HBM-bound: bytes / HBM peak exceeds FLOPs / tensor peak
    assert b / 6500e9 > f / 1400e12 and top["bound"] == "hbm"
    assert abs(top["achieved"] - b / 0.08e-3 / 1e9) < 0.01
    assert abs(top["frac"] - top["achieved"] / 6500.0) < 1e-4
    assert table["cvmm_cast"]["bound"] == "hbm" and abs(sum(t["share"] for t in table.values()) - 1) < 1e-2
    s = bench.step_roofline(w, 0.2, pk)
    assert abs(s["hbm_frac"] - 3 * b / 0.2e-3 / 1e9 / 6500.0) < 1e-3
