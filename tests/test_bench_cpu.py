"""bench.py's reference arm on the CPU: the reference's CPU decode path
(transformers' Qwen3ForCausalLM, qwen3/reference.py's model) timed on a tiny
shape prints the one JSON line of the benchmark contract, with the same
metric, unit and workload keys as the GPU arm."""

import argparse
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--preset", "tiny", "--context", "32",
                        "--steps", "3", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    sys.path.insert(0, str(ROOT))
    import bench
    from xpu_playground_b200.qwen3_config import PRESETS
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "tok/s" and line["higher_is_better"] is True and line["value"] > 0
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 1
    assert abs(line["ms_per_step"] - 1000.0 / line["value"]) < 1e-2 * line["ms_per_step"]
    args = argparse.Namespace(preset="tiny", context=32, steps=3)
    expected = bench.decode_config(args, PRESETS["tiny"])
    assert {k: line["config"][k] for k in expected} == expected
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["sample"] and cpu["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_gemv_gemm_cpu_baselines_small():
    from oracle.cpu_baseline import gemm_cpu_baseline, gemv_cpu_baseline
    g = gemv_cpu_baseline(256, 512, min_seconds=0.05)
    assert g["unit"] == "GB/s" and g["value"] > 0 and g["kind"] == "port" and g["cores"] >= 1
    m = gemm_cpu_baseline(64, 96, 128, sample_rows=16, min_seconds=0.05)
    assert m["unit"] == "TFLOP/s" and m["value"] > 0 and "16 of 64 rows" in m["sample"]
