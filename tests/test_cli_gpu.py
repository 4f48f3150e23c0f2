"""The benchmark programs on the GPU: each runs a small case end to end,
verifies itself (the reference's closed-form / 64-row / checksum checks) and
prints the reference's output lines; the calibrator kernels are also checked
against the oracle for every read unit."""

import re
import subprocess

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from xpu_playground_b200 import build, kernels

pytestmark = pytest.mark.gpu
BIN = build.BIN_DIR


def run(*args):
    r = subprocess.run([str(a) for a in args], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_gemm_program():
    out = run(BIN / "gemm", "--size", "1024", "--iterations", "3", "--warmups", "1")
    assert out.startswith("Device: ")
    assert "Type: BF16, shape: 1024x1024x1024\n" in out
    assert re.search(r"Median: \d+\.\d\d TFLOP/s\nBest:   \d+\.\d\d TFLOP/s\nVerification: PASS\n", out)
    out = run(BIN / "gemm", "--m", "300", "--n", "200", "--k", "100", "--type", "fp16", "--iterations", "2")
    assert "Type: FP16, shape: 300x200x100\n" in out and "Verification: PASS" in out
    out = run(BIN / "gemm", "--m", "33", "--n", "7", "--k", "5", "--iterations", "1")  # CUDA-core path
    assert "Verification: PASS" in out


def test_gemv_program():
    out = run(BIN / "gemv", "--size", "4096", "--iterations", "5")
    assert "Type: BF16, shape: 4096x4096\n" in out
    assert re.search(r"Median: [\d.]+ GFLOP/s, [\d.]+ GB/s\nBest:   [\d.]+ GFLOP/s, [\d.]+ GB/s\n"
                     r"Verification: PASS\n", out)
    out = run(BIN / "gemv", "--m", "37", "--k", "1000", "--type", "fp16", "--iterations", "2")
    assert "Type: FP16, shape: 37x1000\n" in out and "Verification: PASS" in out


def test_peak_programs_and_dispatcher():
    out = run(BIN / "peak_sycl", "mem", "--size-mib", "256", "--iterations", "3")
    assert "Surface: 256 MiB, 1024 x 65536 floats\n" in out and "Checksum: PASS" in out
    assert re.search(r"Median read bandwidth: [\d.]+ GB/s \([\d.]+% of 7700.0 GB/s\)", out)
    out = run(BIN / "peak_sycl", "compute", "--rounds", "256", "--iterations", "3")
    assert "MMA shape: 128x256x16 BF16, 1048576 FLOP/instruction" in out and "Checksum: PASS" in out
    out = run(BIN / "peak_sycl", "gemm", "--size", "512", "--iterations", "2")
    assert "Verification: PASS" in out


def test_peak_mem_read_every_unit_matches_oracle():
    height = 64 * 32 + 32  # 65 bands: more bands than one per SM is not needed for coverage
    surface = torch.empty(height * 1024, dtype=torch.float32, device="cuda")
    kernels.peak_mem_fill(surface)
    host = surface.cpu().numpy()
    assert np.array_equal(host, orc.peak_mem_surface(height * 1024))
    sink = kernels.peak_mem_read(surface)
    assert np.array_equal(sink.cpu().numpy(), orc.peak_mem_checksums(host))
    # a surface with more bands than CTAs: every band is visited once
    big = torch.empty(4096 * 32 * 1024, dtype=torch.float32, device="cuda")
    kernels.peak_mem_fill(big)
    got = kernels.peak_mem_read(big).cpu().numpy()
    assert np.array_equal(got, orc.peak_mem_checksums(big.cpu().numpy()))
    assert kernels.device_status() == 0


@pytest.mark.parametrize("ctas,rounds", [(1, 1), (148, 3), (300, 17)])
def test_peak_compute_checksum(ctas, rounds):
    sink = kernels.peak_compute(ctas, rounds)
    assert torch.all(sink == orc.peak_compute_checksum(rounds)).item()
    assert kernels.device_status() == 0
