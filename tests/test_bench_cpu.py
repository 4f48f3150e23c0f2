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
    # the GPU arm prints exactly this config too (the driver compares them)
    assert line["config"] == bench.decode_config(args, PRESETS["tiny"])
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["sample"] and cpu["value"] == line["value"]
    assert set(cpu["fit"]["repeat_spread"]) == {"1", "2", "4", "8"}
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_gemv_gemm_cpu_baselines_small():
    from oracle.cpu_baseline import gemm_cpu_baseline, gemv_cpu_baseline
    g = gemv_cpu_baseline(256, 512, min_seconds=0.05)
    assert g["unit"] == "GB/s" and g["value"] > 0 and g["kind"] == "port" and g["cores"] >= 1
    m = gemm_cpu_baseline(64, 96, 128, sample_rows=16, min_seconds=0.05)
    assert m["unit"] == "TFLOP/s" and m["value"] > 0 and "16 of 64 rows" in m["sample"]


def test_fit_line_recovers_a_line_and_reports_residual():
    from oracle.cpu_baseline import fit_line
    fixed, per_layer, resid = fit_line({1: 3.0, 2: 5.0, 4: 9.0, 8: 17.0})
    assert abs(fixed - 1.0) < 1e-12 and abs(per_layer - 2.0) < 1e-12 and resid < 1e-12
    _, _, resid = fit_line({1: 3.0, 2: 5.0, 4: 9.0, 8: 20.0})
    assert resid > 0.05


def test_host_threads_is_a_positive_count():
    from oracle.cpu_baseline import host_threads
    assert 1 <= host_threads() <= (__import__("os").cpu_count() or 1)


def test_token_check_against_a_stored_run(tmp_path, monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    args = argparse.Namespace(preset="qwen3-8b", context=2048)
    ids = [5, 6, 7, 8]
    gold = tmp_path / "g.json"
    gold.write_text(json.dumps({"preset": "qwen3-8b", "context": 2048, "weight_seed": bench.WEIGHT_SEED,
                                "first_position": 2047, "prefill": bench.PREFILL_PATH, "n_gpus": 1,
                                "ids": [5, 6, 7, 8, 9, 10]}))
    monkeypatch.setattr(bench, "GOLDEN_TOKENS", gold)
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    info = bench.check_tokens(args, 2047, ids)
    assert info["golden"]["match"] and info["golden"]["compared"] == 4
    assert info["sha256"] == bench.token_digest(ids) != bench.token_digest([5, 6, 7, 9])
    assert not bench.check_tokens(args, 2047, [5, 6, 7, 9])["golden"]["match"]
    assert bench.check_tokens(args, 100, ids)["golden"] is None  # another run: not compared
    stale = json.loads(gold.read_text())
    stale["prefill"] = "token by token"
    gold.write_text(json.dumps(stale))
    assert bench.check_tokens(args, 2047, ids)["golden"] is None  # another prefill: not compared


def test_row_shards_cover_the_matrix_once():
    sys.path.insert(0, str(ROOT))
    import bench
    for m in (16384, 4096, 1000, 7):
        for world in (1, 2, 4, 8):
            spans = [bench.row_shard(m, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == m
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
