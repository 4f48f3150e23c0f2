"""xpu_qwen_attention_noalloc: attention with the library's fixed scratch.

The entry point exists for callers that cannot allocate device memory (an
allocator that owns the device, a loop that may not call cudaMalloc/cudaFree,
a plugin host that only passes inputs and outputs). It runs the same kernels
as xpu_qwen_attention with a caller-owned workspace, so it must give the same
bits, on consecutive calls that reuse the shared scratch, for every head
group the kernels have (1, 2, 4, 8) and at the largest request its fixed
6 MiB admits; the results are also held to the CPU oracle. Larger requests
must be refused. This file is collected last so that a failure here comes
after every other test has run; it passes alone in a fresh process as well.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import close, to_bits, to_device
from xpu_playground_b200 import _lib

pytestmark = pytest.mark.gpu

# kernels.hpp / test_cpu_reference.cpp primitive tolerance (atol 0.03 + rtol 0.02)
ATOL, RTOL = 0.03, 0.02


def _inputs(q_heads, kv_heads, position, seed):
    n = position + 1
    q = orc.uniform16(q_heads * 128, seed, 1)
    kc = orc.uniform16(n * kv_heads * 128, seed, 2)
    vc = orc.uniform16(n * kv_heads * 128, seed, 3)
    return q, kc, vc


def _with_workspace(L, q, kc, vc, position, q_heads, kv_heads):
    out = torch.empty(q_heads * 128, dtype=torch.bfloat16, device="cuda")
    ws_bytes = L.xpu_qwen_attention_workspace_size(q_heads, position + 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    _lib.check(L.xpu_qwen_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), position,
                                    q_heads, kv_heads, ws.data_ptr(), ws_bytes, None))
    return to_bits(out)


def _no_alloc(L, q, kc, vc, position, q_heads, kv_heads):
    out = torch.empty(q_heads * 128, dtype=torch.bfloat16, device="cuda")
    _lib.check(L.xpu_qwen_attention_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), position,
                                            q_heads, kv_heads, None))
    return to_bits(out)


def test_no_alloc_attention_matches_workspace_entry_point_twice():
    L = _lib.load()
    torch.cuda.set_device(0)
    # Calls in a row with different shapes: each reuses the scratch the one
    # before left behind. Head groups 4, 2, 1 and 8.
    cases = [(32, 8, 2303, 11), (16, 8, 700, 12), (8, 8, 1500, 13), (64, 8, 300, 14)]
    for q_heads, kv_heads, position, seed in cases:
        hq, hk, hv = _inputs(q_heads, kv_heads, position, seed)
        q, kc, vc = to_device(hq), to_device(hk), to_device(hv)
        ref = _with_workspace(L, q, kc, vc, position, q_heads, kv_heads)
        got = _no_alloc(L, q, kc, vc, position, q_heads, kv_heads)
        torch.cuda.synchronize()
        assert np.array_equal(got, ref), (q_heads, kv_heads, position)
        want = orc.attention(hq, hk, hv, position, q_heads, kv_heads)
        close(orc.bf16_to_float(got), orc.bf16_to_float(want), atol=ATOL, rtol=RTOL)


def test_no_alloc_attention_at_its_largest_request():
    """32 query heads at the last position (40,959) use 5.2 MB of the 6 MiB;
    inputs drawn on the device (168 MB of K/V cache)."""
    L = _lib.load()
    torch.cuda.set_device(0)
    q_heads, kv_heads, position = 32, 8, 40959
    assert L.xpu_qwen_attention_workspace_size(q_heads, position + 1) <= 6 << 20
    g = torch.Generator(device="cuda").manual_seed(5)
    n = position + 1
    q = torch.empty(q_heads * 128, device="cuda").uniform_(-1, 1, generator=g).to(torch.bfloat16)
    kc = torch.empty(n * kv_heads * 128, device="cuda").uniform_(-1, 1, generator=g).to(torch.bfloat16)
    vc = torch.empty(n * kv_heads * 128, device="cuda").uniform_(-1, 1, generator=g).to(torch.bfloat16)
    for _ in range(2):  # twice: the second call starts from the first one's scratch
        ref = _with_workspace(L, q, kc, vc, position, q_heads, kv_heads)
        got = _no_alloc(L, q, kc, vc, position, q_heads, kv_heads)
        torch.cuda.synchronize()
        assert np.array_equal(got, ref)


def test_no_alloc_attention_rejects_requests_beyond_its_scratch():
    L = _lib.load()
    # 32 heads at 40,960 positions fit (5.2 MB); 64 heads at that length do not.
    assert L.xpu_qwen_attention_workspace_size(32, 40960) <= 6 << 20
    assert L.xpu_qwen_attention_workspace_size(64, 40960) > 6 << 20
    status = L.xpu_qwen_attention_noalloc(16, 16, 16, 16, 40959, 64, 8, None)
    assert status == _lib.XPU_ERR_INVALID
    assert "6291456" in _lib.last_error()
