"""The benchmark programs' command-line contract, checked without a GPU:
usage text and exit codes, option validation with the reference's messages
(gemv.cpp:26-64, gemm.cpp:24-59, peak_mem_2d.cpp:61-99,
peak_compute_dpas.cpp:33-77), the peak_sycl dispatcher (peak_sycl.cpp:10-56)
and the run_* entries of libxpu_bench.so."""

import ctypes
import subprocess

import pytest

from xpu_playground_b200 import build

BIN = build.BIN_DIR


def run(*args):
    return subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=60)


@pytest.mark.parametrize("prog,flag", [("gemv", "--size"), ("gemm", "--size"), ("peak_mem_2d", "--size-mib"),
                                       ("peak_compute_dpas", "--rounds")])
def test_help_and_positive_integers(prog, flag):
    r = run(BIN / prog, "--help")
    assert r.returncode == 0 and "Usage:" in r.stdout
    for bad in ("0", "-3", "12x", ""):
        r = run(BIN / prog, flag, bad)
        assert r.returncode == 1
        assert r.stderr.strip() == f"Error: {flag} requires a positive integer"
    r = run(BIN / prog, flag)
    assert r.returncode == 1 and r.stderr.strip() == f"Error: {flag} requires a value"
    r = run(BIN / prog, "--bogus", "1")
    assert r.returncode == 1 and r.stderr.strip() == "Error: unknown option: --bogus"


@pytest.mark.parametrize("prog", ["gemv", "gemm"])
def test_type_option(prog):
    r = run(BIN / prog, "--type", "fp32")
    assert r.returncode == 1 and r.stderr.strip() == "Error: --type must be bf16 or fp16"


def test_peak_sycl_dispatch():
    r = run(BIN / "peak_sycl")
    assert r.returncode == 1 and "Error: missing benchmark mode" in r.stderr and "Usage:" in r.stdout
    r = run(BIN / "peak_sycl", "--help")
    assert r.returncode == 0 and " gemm [--size N" in r.stdout
    r = run(BIN / "peak_sycl", "flops")
    assert r.returncode == 1 and r.stderr.strip() == "Error: unknown benchmark mode: flops"
    # each mode runs the sibling program with the remaining arguments
    for mode, prog in (("mem", "peak_mem_2d"), ("compute", "peak_compute_dpas"), ("gemv", "gemv"),
                       ("gemm", "gemm")):
        r = run(BIN / "peak_sycl", mode, "--help")
        assert r.returncode == 0 and r.stdout.startswith(f"Usage: {BIN / prog}")


def test_bench_library_exports_run_entries():
    lib = ctypes.CDLL(str(build.BENCH_LIB))
    for name in ("run_gemv", "run_gemm", "run_peak_mem_2d", "run_peak_compute_dpas"):
        assert getattr(lib, name)
    # an option error returns 1 without touching a device
    argv = (ctypes.c_char_p * 3)(b"gemm", b"--size", b"0")
    lib.run_gemm.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]
    assert lib.run_gemm(3, argv) == 1


def test_qwen3_cli_arguments(tmp_path):
    """qwen3/main.cpp:15-67 option rules, checked before any GPU work."""
    q = BIN / "qwen3"
    r = run(q, "--help")
    assert r.returncode == 0 and r.stdout.startswith("Usage: qwen3 --model-dir DIR")
    r = run(q, "--model-dir", str(tmp_path), "--input-ids", "-")
    assert r.returncode == 1 and r.stderr.startswith("qwen3: --max-new-tokens is required")
    r = run(q, "--model-dir", str(tmp_path), "--input-ids", "-", "--max-new-tokens", "x")
    assert r.returncode == 1 and "invalid value for --max-new-tokens: x" in r.stderr
    r = run(q, "--model-dir", str(tmp_path), "--input-ids", "-", "--max-new-tokens", "4", "--max-seq-len", "50000")
    assert r.returncode == 1 and "--max-seq-len cannot exceed 40960" in r.stderr
    r = run(q, "--model-dir", str(tmp_path), "--input-ids", "-", "--max-new-tokens", "4")
    assert r.returncode == 1 and "config.json" in r.stderr  # no checkpoint there


def test_qwen3_cli_rejects_bad_token_ids(tmp_path):
    import json
    from tests._ckpt import config_dict
    from xpu_playground_b200.qwen3_config import PRESETS
    (tmp_path / "config.json").write_text(json.dumps(config_dict(PRESETS["tiny"])))
    ids = tmp_path / "ids.txt"
    for text, needle in (("1 2 4096", "outside [0, 4095]: 4096"), ("1 x", "invalid input token ID: x"),
                         ("", "at least one input token ID is required")):
        ids.write_text(text)
        r = run(BIN / "qwen3", "--model-dir", str(tmp_path), "--input-ids", str(ids), "--max-new-tokens", "2")
        assert r.returncode == 1 and needle in r.stderr, r.stderr
