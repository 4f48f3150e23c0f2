"""GEMV parity on the GPU: libxpu_cuda's xpu_gemv against the FP32 host
oracle (gemv.cpp:191-196 restated), 1e-2 relative Frobenius over all rows."""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import close, to_bits, to_device
from xpu_playground_b200 import kernels

pytestmark = pytest.mark.gpu

TOL = 1e-2  # relative Frobenius, the north-star GEMV/GEMM tolerance


def _dt(fp16):
    return torch.float16 if fp16 else torch.bfloat16


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("m,k", [(4096, 4096), (1, 8), (1, 1), (5, 1), (37, 1000), (1000, 37),
                                 (33, 4104), (8192, 2048), (300, 12288), (2, 16384)])
def test_gemv_seeded_uniform(fp16, m, k):
    A = orc.uniform16(m * k, seed=m * 7 + k, tag=1, fp16=fp16).reshape(m, k)
    x = orc.uniform16(k, seed=m * 7 + k, tag=2, fp16=fp16)
    y = kernels.gemv(to_device(A, _dt(fp16)), to_device(x, _dt(fp16)))
    ref = orc.gemv(A, x, fp16)
    got = orc.decode(to_bits(y), fp16)
    assert orc.rel_frobenius(got, ref) < TOL
    # each output is the FP32 sum rounded once: at most one 16-bit step away
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2 ** -7 + 1e-6)


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
def test_gemv_16384_square(fp16):
    """BASELINE configs[1] shape, seeded uniform[-1, 1]."""
    m = k = 16384
    A = orc.uniform16(m * k, seed=16384, tag=1, fp16=fp16).reshape(m, k)
    x = orc.uniform16(k, seed=16384, tag=2, fp16=fp16)
    y = kernels.gemv(to_device(A, _dt(fp16)), to_device(x, _dt(fp16)))
    assert orc.rel_frobenius(orc.decode(to_bits(y), fp16), orc.gemv(A, x, fp16)) < TOL


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
def test_gemv_reference_benchmark_inputs(fp16):
    """gemv.cpp:156-199: hash-generated inputs, the reference's max(1, 1%) check
    on every row (the reference checks the first 64)."""
    A, x = orc.gemv_bench_inputs(4096, 4096, fp16)
    y = kernels.gemv(to_device(A, _dt(fp16)), to_device(x, _dt(fp16)))
    ref = orc.gemv(A, x, fp16)
    got = orc.decode(to_bits(y), fp16)
    assert np.all(np.abs(got - ref) <= np.maximum(1.0, 0.01 * np.abs(ref)))


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 4096), (12288, 4096), (4096, 12288),
                                       (151936, 4096)])
def test_gemv_production_shapes_reference_patterns(rows, cols):
    """test_cpu_reference.cpp:58-83 patterns on every Qwen3-8B GEMV shape,
    checked for the rows the reference checks (0 and rows-1) and a sample."""
    dev = torch.device("cuda")
    r = torch.arange(rows, device=dev)[:, None]
    c = torch.arange(cols, device=dev)[None, :]
    A = ((((r + c) % 13) - 6).float() / 256.0).to(torch.bfloat16)
    x = ((torch.arange(cols, device=dev) % 17 - 8).float() / 128.0).to(torch.bfloat16)
    y = kernels.gemv(A, x)
    rows_checked = sorted({0, rows - 1, *range(1, rows, max(1, rows // 97))})
    ref = (A[rows_checked].double() @ x.double()).cpu().numpy()
    close(y[rows_checked].float().cpu().numpy(), ref)
    del A


def test_gemv_unaligned_views_take_the_scalar_path():
    m, k = 64, 96
    A = orc.uniform16(m * k + 1, seed=3, tag=1)
    x = orc.uniform16(k + 1, seed=3, tag=2)
    dA, dx = to_device(A), to_device(x)
    A1, x1 = dA[1:].view(m, k), dx[1:]  # 2-byte offsets: not 16-byte aligned
    y = kernels.gemv(A1, x1)
    ref = orc.gemv(A[1:].reshape(m, k), x[1:])
    assert orc.rel_frobenius(orc.bf16_to_float(to_bits(y)), ref) < TOL
