"""GEMM parity on the GPU: libxpu_cuda's xpu_gemm (tcgen05 tensor cores, and
the CUDA-core kernel for shapes TMA cannot describe) against the FP32 host
oracle, 1e-2 relative Frobenius, plus the reference's own closed-form check
(gemm.cpp:109-117: A = 0.5, B = 0.25 gives k * 0.125 in every element)."""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import to_bits, to_device
from xpu_playground_b200 import kernels

pytestmark = pytest.mark.gpu

TOL = 1e-2  # relative Frobenius, the north-star GEMV/GEMM tolerance


def _dt(fp16):
    return torch.float16 if fp16 else torch.bfloat16


def _check(got_bits, A, B, fp16, rows=None):
    """Compares (a row sample of) C with the oracle: the Frobenius gate, and
    per element one 16-bit rounding of the FP32 sum plus an FP32
    accumulation-order allowance that grows with k."""
    if rows is not None:
        A = A[rows]
        got_bits = got_bits[rows]
    ref = orc.gemm(A, B, fp16)
    got = orc.decode(got_bits, fp16).reshape(ref.shape)
    assert orc.rel_frobenius(got, ref) < TOL
    k = A.shape[1]
    bound = np.abs(ref) * 2.0 ** -7 + 1e-5 * k
    bad = np.argwhere(np.abs(got - ref) > bound)
    assert bad.size == 0, f"{len(bad)} elements off, first at {bad[0]}: {got[tuple(bad[0])]} vs {ref[tuple(bad[0])]}"
    assert kernels.device_status() == 0


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("m,n,k", [
    (128, 256, 64),      # exactly one tile, one K stage
    (256, 512, 1024),    # 2 x 2 tiles, 16 K stages (ring wraps 4 times)
    (129, 264, 72),      # ragged in every dimension (zero-filled edge tiles)
    (1, 8, 8),           # smallest tensor-core shape
    (7, 40, 4096),       # few rows, deep K
    (1000, 1000, 1000),  # 8 x 4 tiles with ragged edges
    (2048, 2048, 256),
])
def test_gemm_seeded_uniform(fp16, m, n, k):
    A = orc.uniform16(m * k, seed=m + 3 * n + 7 * k, tag=1, fp16=fp16).reshape(m, k)
    B = orc.uniform16(k * n, seed=m + 3 * n + 7 * k, tag=2, fp16=fp16).reshape(k, n)
    C = kernels.gemm(to_device(A, _dt(fp16)), to_device(B, _dt(fp16)))
    _check(to_bits(C), A, B, fp16)


@pytest.mark.parametrize("fp16,m,n,k", [(False, 4096, 4096, 4096), (True, 3072, 4096, 2048)],
                         ids=["bf16-4096cube", "fp16-3072x4096x2048"])
def test_gemm_benchmark_shapes_sampled(fp16, m, n, k):
    """The two benchmark shapes, seeded uniform[-1, 1]; the oracle checks a
    spread of 96 rows (every column) including the first and last tile rows."""
    A = orc.uniform16(m * k, seed=k, tag=1, fp16=fp16).reshape(m, k)
    B = orc.uniform16(k * n, seed=k, tag=2, fp16=fp16).reshape(k, n)
    C = kernels.gemm(to_device(A, _dt(fp16)), to_device(B, _dt(fp16)))
    rows = sorted({0, 1, 127, 128, m - 1, *range(5, m, m // 90)})
    _check(to_bits(C), A, B, fp16, rows)


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("m,n,k", [(4096, 4096, 4096), (3072, 4096, 2048), (100, 300, 50),
                                   (4000, 4000, 4000), (33, 7, 5)])
def test_gemm_reference_closed_form(fp16, m, n, k):
    """gemm.cpp:79-117: A filled with 0.5 and B with 0.25; every element of C
    must be exactly k * 0.125 (exact in FP32 and in the 16-bit output for
    these k). The reference pads to its tiles; here the shape is used as is."""
    dt = _dt(fp16)
    A = torch.full((m, k), 0.5, dtype=dt, device="cuda")
    B = torch.full((k, n), 0.25, dtype=dt, device="cuda")
    C = kernels.gemm(A, B)
    expected = torch.tensor(k * 0.125, dtype=dt)
    assert torch.all(C == expected.to(C.device)), "closed-form GEMM mismatch"
    assert kernels.device_status() == 0


def test_gemm_fallback_shapes_and_unaligned_views():
    """n or k not a multiple of 8, or a base that is not 16-byte aligned, take
    the CUDA-core kernel; results still match the oracle."""
    for m, n, k in [(37, 100, 1000), (64, 64, 60), (5, 3, 2)]:
        A = orc.uniform16(m * k, seed=n, tag=1).reshape(m, k)
        B = orc.uniform16(k * n, seed=n, tag=2).reshape(k, n)
        _check(to_bits(kernels.gemm(to_device(A), to_device(B))), A, B, False)
    m, n, k = 48, 64, 64
    A = orc.uniform16(m * k + 1, seed=9, tag=1)
    B = orc.uniform16(k * n, seed=9, tag=2).reshape(k, n)
    dA = to_device(A)[1:].view(m, k)  # 2-byte offset
    _check(to_bits(kernels.gemm(dA, to_device(B))), A[1:].reshape(m, k), B, False)


def test_gemm_rejects_bad_arguments():
    from xpu_playground_b200._lib import XpuError, call
    with pytest.raises(XpuError):
        call("xpu_gemm", 0, None, None, None, 1, 1, 1, None)
    a = torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(XpuError):
        call("xpu_gemm", 0, a.data_ptr(), a.data_ptr(), a.data_ptr(), 0, 8, 8, None)
    with pytest.raises(XpuError):
        call("xpu_gemm", 7, a.data_ptr(), a.data_ptr(), a.data_ptr(), 8, 8, 8, None)


@pytest.mark.parametrize("fp16", [False, True], ids=["bf16", "fp16"])
@pytest.mark.parametrize("m,n,k", [(256, 256, 128), (300, 512, 4096), (2048, 6144, 4096), (37, 24576, 1024),
                                   (5, 128, 264)])
def test_gemm_bt_against_fp32(fp16, m, n, k):
    """C = A . W^T with W stored [n, k] (xpu_gemm_bt, the dense prefill's
    projection): 1e-2 relative Frobenius of the FP32 product, every element
    within one 16-bit rounding plus the accumulation-order allowance."""
    dt = torch.float16 if fp16 else torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    A = torch.empty(m, k, device="cuda").uniform_(-1, 1, generator=g).to(dt)
    W = torch.empty(n, k, device="cuda").uniform_(-1, 1, generator=g).to(dt)
    C = kernels.gemm_bt(A, W)
    ref = A.float() @ W.float().t()
    got = C.float()
    assert (torch.linalg.norm(got - ref) / torch.linalg.norm(ref)).item() < 1e-2
    step = 2.0 ** -10 if fp16 else 2.0 ** -7
    assert torch.all((got - ref).abs() <= ref.abs() * step + 1e-5 * k + 1e-6).item()
    assert kernels.device_status() == 0
