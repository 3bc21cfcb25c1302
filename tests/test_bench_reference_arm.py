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
    for k in ("n_gpus", "steps", "warmup", "higher_is_better", "scaling", "config"):
        assert k in line, k
