"""Qwen3 operator ABI on the GPU (qwen3/kernels_entry.cpp:8-72 semantics).

Part 1 replays the known-answer tests of qwen3/tests/test_gpu_dispatch.cpp
through the C ABI; part 2 compares every operator with the oracle's
restatement of qwen3/kernels.hpp on seeded random inputs.
"""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import close, to_bits, to_device
from xpu_playground_b200 import kernels as K

pytestmark = pytest.mark.gpu
b = orc.bf16_bits
f = orc.bf16_to_float
ONE = int(b(np.float32([1.0]))[0])


def dev_empty(n, dtype=torch.bfloat16):
    return torch.empty(n, dtype=dtype, device="cuda")


# ------------------------------------------------- test_gpu_dispatch.cpp ----

def test_dispatch_embedding():
    table = b((np.arange(4096) % 29 - 14) / 16.0)
    out = dev_empty(4096)
    K.qwen_embedding(to_device(table), out, 0, 4096)
    assert np.array_equal(to_bits(out), table)


@pytest.mark.parametrize("width", [128, 4096])
def test_dispatch_rms_norm(width):
    x = b((np.arange(width) % 31 - 15) / 32.0)
    w = np.full(width, b(np.float32([0.75]))[0], np.uint16)
    out = dev_empty(width)
    K.qwen_rms_norm(to_device(x), to_device(w), out, width, 1e-6)
    xs = f(x).astype(np.float64)
    close(f(to_bits(out)), xs * 0.75 / math.sqrt((xs * xs).sum() / width + 1e-6))


def test_dispatch_gemv_32x32():
    vec = b((np.arange(32) % 7 - 3) / 8.0)
    mat = b((np.arange(32 * 32) % 11 - 5) / 16.0)
    out = dev_empty(32)
    K.qwen_gemv(to_device(mat), to_device(vec), out, 32, 32)
    close(f(to_bits(out)), f(mat).reshape(32, 32).astype(np.float64) @ f(vec))


def _kat_inputs(q_heads=32, kv_heads=8):
    q = b((np.arange(q_heads * 128) % 17 - 8) / 16.0)
    k = b((np.arange(kv_heads * 128) % 13 - 6) / 16.0)
    v = b((np.arange(kv_heads * 128) % 19 - 9) / 16.0)
    return q, k, v


def test_dispatch_qkv_rope_cache_and_attention():
    q, k, v = _kat_inputs()
    norm = to_device(np.full(128, ONE, np.uint16))
    cos = to_device(np.full(128, ONE, np.uint16))
    sin = to_device(np.zeros(128, np.uint16))
    dq, dk, dv = to_device(q), to_device(k), to_device(v)
    kc, vc = dev_empty(k.size), dev_empty(v.size)
    K.qwen_qkv_rope_cache(dq, dk, dv, norm, norm, cos, sin, kc, vc, 0, 1, 32, 8)
    assert np.array_equal(to_bits(vc), v)
    out = dev_empty(4096)
    ws = torch.empty(K.qwen_attention_workspace_size(32, 1), dtype=torch.uint8, device="cuda")
    K.qwen_attention(dq, kc, vc, out, 0, 32, 8, ws)
    got = f(to_bits(out))
    for h in range(32):
        close(got[h * 128:(h + 1) * 128], f(v[(h // 4) * 128:(h // 4 + 1) * 128]))


def test_dispatch_last_cache_slot():
    q, k, v = _kat_inputs()
    maximum = 40960
    cache_elems = maximum * 8 * 128
    kc = torch.zeros(cache_elems, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    cos = torch.zeros(maximum * 128, dtype=torch.bfloat16, device="cuda")
    sin = torch.zeros_like(cos)
    cos[-128:] = 1.0
    norm = to_device(np.full(128, ONE, np.uint16))
    K.qwen_qkv_rope_cache(to_device(q), to_device(k), to_device(v), norm, norm, cos, sin, kc, vc,
                          maximum - 1, maximum, 32, 8)
    assert np.array_equal(to_bits(vc[-v.size:]), v)
    assert not torch.any(vc[:-v.size] != 0)


def test_dispatch_add_silu_argmax():
    width = 12288
    i = np.arange(width)
    left, right = b((i % 11 - 5) / 8.0), b((i % 7 - 3) / 8.0)
    dl, dr = to_device(left), to_device(right)
    K.qwen_add(dl, dr, width)
    close(f(to_bits(dl)), f(left) + f(right))
    dl = to_device(left)
    K.qwen_silu_multiply(dl, dr, width)
    g = f(left).astype(np.float64)
    close(f(to_bits(dl)), g / (1 + np.exp(-g)) * f(right))
    logits = np.full(151936, b(np.float32([-1.0]))[0], np.uint16)
    logits[17] = logits[42] = b(np.float32([3.0]))[0]
    token = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.qwen_argmax(to_device(logits), token, 151936)
    assert int(token.item()) == 17
    logits[3] = b(np.float32([np.nan]))[0]
    K.qwen_argmax(to_device(logits), token, 151936)
    assert int(token.item()) & 0xFFFFFFFF == 0xFFFFFFFF


# ------------------------------------------- seeded inputs vs the oracle ----

def _bits_frac_equal(a, b_):
    return float(np.mean(a == b_))


@pytest.mark.parametrize("width", [1, 7, 1024, 4096, 5000])
def test_rms_norm_vs_oracle(width):
    x = orc.uniform16(width, 11, 1)
    w = orc.normal_bf16(width, 11, 2, 0.5)
    out = dev_empty(width)
    K.qwen_rms_norm(to_device(x), to_device(w), out, width, 1e-6)
    ref = orc.rms_norm(x, w)
    got = to_bits(out)
    close(f(got), f(ref), atol=1e-3, rtol=8e-3)
    assert _bits_frac_equal(got, ref) > 0.97


@pytest.mark.parametrize("q_heads,kv_heads,position", [(32, 8, 0), (32, 8, 77), (16, 8, 300),
                                                       (8, 8, 5), (8, 1, 130)])
def test_qkv_rope_cache_vs_oracle(q_heads, kv_heads, position):
    max_seq = position + 3
    q = orc.uniform16(q_heads * 128, 5, 1)
    k = orc.uniform16(kv_heads * 128, 5, 2)
    v = orc.uniform16(kv_heads * 128, 5, 3)
    qn = orc.normal_bf16(128, 5, 4, 0.3)
    kn = orc.normal_bf16(128, 5, 5, 0.3)
    cos, sin = orc.rope_tables(max_seq)
    kc = np.zeros(max_seq * kv_heads * 128, np.uint16)
    vc = np.zeros_like(kc)
    dq, dk, dkc, dvc = to_device(q), to_device(k), to_device(kc), to_device(vc)
    K.qwen_qkv_rope_cache(dq, dk, to_device(v), to_device(qn), to_device(kn), to_device(cos),
                          to_device(sin), dkc, dvc, position, max_seq, q_heads, kv_heads)
    orc.qkv_rope_cache(q, k, v, qn, kn, cos, sin, kc, vc, position, max_seq, q_heads, kv_heads)
    assert np.array_equal(to_bits(dvc), vc)
    for got, ref in ((to_bits(dq), q), (to_bits(dk), k), (to_bits(dkc), kc)):
        close(f(got), f(ref), atol=2e-2, rtol=1e-2)
        assert _bits_frac_equal(got, ref) > 0.97


@pytest.mark.parametrize("q_heads,kv_heads,position", [(32, 8, 0), (32, 8, 127), (32, 8, 128),
                                                       (32, 8, 2303), (16, 8, 1000), (8, 1, 40959),
                                                       (4, 2, 9)])
def test_attention_vs_oracle(q_heads, kv_heads, position):
    n = position + 1
    q = orc.uniform16(q_heads * 128, position, 1)
    kc = orc.uniform16(n * kv_heads * 128, position, 2)
    vc = orc.uniform16(n * kv_heads * 128, position, 3)
    out = dev_empty(q_heads * 128)
    ws = torch.empty(K.qwen_attention_workspace_size(q_heads, n), dtype=torch.uint8, device="cuda")
    K.qwen_attention(to_device(q), to_device(kc), to_device(vc), out, position, q_heads, kv_heads, ws)
    ref = orc.attention(q, kc, vc, position, q_heads, kv_heads)
    close(f(to_bits(out)), f(ref), atol=4e-3, rtol=1e-2)


@pytest.mark.parametrize("width", [1, 9, 3072, 12288, 12289])
def test_add_and_silu_vs_oracle(width):
    a = orc.uniform16(width, width, 1)
    c = orc.uniform16(width, width, 2)
    da = to_device(a)
    K.qwen_add(da, to_device(c), width)
    assert np.array_equal(to_bits(da), orc.add(a, c))  # one FP32 add, one rounding: exact
    da = to_device(a)
    K.qwen_silu_multiply(da, to_device(c), width)
    ref = orc.silu_multiply(a, c)
    close(f(to_bits(da)), f(ref), atol=1e-3, rtol=8e-3)
    assert _bits_frac_equal(to_bits(da), ref) > 0.99


@pytest.mark.parametrize("width", [1, 2, 1000, 151936])
def test_argmax_vs_oracle(width):
    vals = orc.uniform16(width, width, 9)
    token = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.qwen_argmax(to_device(vals), token, width)
    assert int(token.item()) == orc.argmax(vals)
    # ties: all equal -> index 0; ±Inf -> sentinel
    same = np.full(width, b(np.float32([0.5]))[0], np.uint16)
    K.qwen_argmax(to_device(same), token, width)
    assert int(token.item()) == 0
    same[-1] = b(np.float32([np.inf]))[0]
    K.qwen_argmax(to_device(same), token, width)
    assert int(token.item()) & 0xFFFFFFFF == 0xFFFFFFFF
