"""The reference's Qwen3 kernel runtime API (qwen3/level_zero_runtime.hpp)
implemented on CUDA: its own dispatch test (qwen3/tests/test_gpu_dispatch.cpp,
compiled unchanged against that header by oracle/build.py) and our self-test
of the API's error behaviour, both run on the GPU."""

import subprocess

import pytest

from xpu_playground_b200 import build

pytestmark = pytest.mark.gpu
ROOT = build.ROOT


def test_runtime_selftest():
    r = subprocess.run([str(build.BIN_DIR / "runtime_selftest")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("runtime selftest: PASS on ")


def test_reference_dispatch_test_passes_on_cuda_runtime():
    binary = ROOT / "oracle" / "_ref" / "test_gpu_dispatch_cuda"
    if not binary.exists():
        pytest.skip("reference dispatch test not built (needs the reference tree at build time)")
    r = subprocess.run([str(binary)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "Qwen3 BMG Level Zero kernel dispatch: PASS on " in r.stdout
