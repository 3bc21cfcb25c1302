"""The reference arm of bench.py (the reference's CPU path, the oracle, timed
on the host cores) runs without a GPU: for every workload it prints one JSON
line with the contract's keys, on the same metric and unit the GPU arm uses."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = [
    (["--workload", "fp4_decode"], "fp4_decode_GBps", "GB/s"),
    (["--workload", "fp8_roundtrip", "--src", "bf16", "--fmt", "e5m2"], "fp8_roundtrip_GBps", "GB/s"),
    (["--workload", "fp8_quantize"], "fp8_quantize_GBps", "GB/s"),
    (["--workload", "quantize_rows"], "quantize_rows_GBps", "GB/s"),
    (["--workload", "scaled_mm", "--size", "1024"], "scaled_mm_TFLOPS", "TFLOP/s"),
    (["--workload", "linear_fp8w", "--m", "16", "--shape", "0"], "linear_fp8w_GBps", "GB/s"),
    (["--workload", "scaled_mm_small_m", "--m", "1"], "scaled_mm_small_m_GBps", "GB/s"),
    (["--workload", "fp4_scaled_mm", "--size", "1024"], "fp4_scaled_mm_TFLOPS", "TFLOP/s"),
    (["--workload", "fp8_quantize_noalloc"], "fp8_quantize_noalloc_GBps", "GB/s"),
]


@pytest.mark.parametrize("args,metric,unit", CASES, ids=[c[0][1] for c in CASES])
def test_reference_arm_line(args, metric, unit):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd + args, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == metric and line["unit"] == unit
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    for k in ("n_gpus", "steps", "warmup", "higher_is_better", "scaling", "config", "ms_per_step"):
        assert k in line, k


def test_default_run_prints_the_suite_in_order():
    """With no --workload both arms print config 1 (f32, then bf16 source), config 3
    and the FP4 decode headline last; every reference line has ms_per_step."""
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [json.loads(l) for l in r.stdout.strip().splitlines() if l.startswith("{")]
    got = [(l["metric"], l["config"].get("src")) for l in lines]
    assert got == [("fp8_roundtrip_GBps", "f32"), ("fp8_roundtrip_GBps", "bf16"), ("scaled_mm_TFLOPS", None),
                   ("fp4_decode_GBps", None)], got
    assert lines[2]["config"]["M"] == 8192
    for l in lines:
        assert l["ms_per_step"] > 0 and l["config"]["parallelism"] == "single"


def test_row_split_configs_match_between_arms():
    """The GPU arm and the reference arm take their config dicts from the same
    describe(); at N > 1 the row-split workloads say rows/N and strong scaling,
    the others replicas."""
    sys.path.insert(0, ROOT)
    import argparse
    import bench
    args = argparse.Namespace(src="f32", fmt="e4m3", elems=0, size=8192, shape=0, m=0, layers=0, eager=False)
    for ws in (2, 8):
        ctx = bench.Ctx(rank=0, local=0, ws=ws, weak=False)
        for name in ("fp4_decode", "fp8_roundtrip", "scaled_mm", "scaled_mm_rowwise", "fp4_scaled_mm",
                     "quantize_rows"):
            d = bench.WORKLOADS[name].describe(args, ctx)
            assert d["config"]["parallelism"] == f"rows/{ws}" and ctx.scaling(d["splits"]) == "strong", name
            json.dumps(d)
        for name in ("scaled_mm_small_m", "linear_fp8w", "fp8_quantize", "fp4_quantize"):
            d = bench.WORKLOADS[name].describe(args, ctx)
            assert d["config"]["parallelism"] == f"replicas{ws}" and ctx.scaling(d["splits"]) == "weak", name
        weak = bench.Ctx(rank=0, local=0, ws=ws, weak=True)
        assert bench.WORKLOADS["fp4_decode"].describe(args, weak)["config"]["parallelism"] == f"replicas{ws}"
    # rows split by shard_rows: the 16384-row FP4 input over 8 ranks keeps 2048 rows each,
    # so the working set rotates through buffer sets to stay above L2
    d = bench.WORKLOADS["fp4_decode"].describe(args, bench.Ctx(0, 0, 8, False))
    assert "rotating" in d["config"]["l2"]
