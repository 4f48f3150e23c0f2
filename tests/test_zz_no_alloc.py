"""xpu_qwen_attention_noalloc: attention with the library's fixed scratch.

The entry point exists for callers that cannot allocate device memory (an
allocator that owns the device, a loop that may not call cudaMalloc/cudaFree,
a plugin host that only passes inputs and outputs). It must give the same
output as xpu_qwen_attention with a caller-owned workspace, on consecutive
calls that reuse the shared scratch, and must refuse requests larger than its
fixed 6 MiB. This file is collected last so that a failure here comes after
every other test has run; it passes alone in a fresh process as well.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as orc
from tests._util import close, to_bits, to_device
from xpu_playground_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(q_heads, kv_heads, position, seed):
    n = position + 1
    q = orc.uniform16(q_heads * 128, seed, 1)
    kc = orc.uniform16(n * kv_heads * 128, seed, 2)
    vc = orc.uniform16(n * kv_heads * 128, seed, 3)
    return to_device(q), to_device(kc), to_device(vc)


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
    # Two calls in a row with different shapes: the second reuses the scratch
    # the first one left behind.
    cases = [(32, 8, 2303, 11), (16, 8, 700, 12)]
    for q_heads, kv_heads, position, seed in cases:
        q, kc, vc = _inputs(q_heads, kv_heads, position, seed)
        ref = _with_workspace(L, q, kc, vc, position, q_heads, kv_heads)
        got = _no_alloc(L, q, kc, vc, position, q_heads, kv_heads)
        torch.cuda.synchronize()
        close(orc.bf16_to_float(got), orc.bf16_to_float(ref), atol=4e-3, rtol=1e-2)


def test_no_alloc_attention_rejects_requests_beyond_its_scratch():
    L = _lib.load()
    # 32 heads at 40,960 positions fit (5.1 MB); 64 heads at that length do not.
    assert L.xpu_qwen_attention_workspace_size(32, 40960) <= 6 << 20
    assert L.xpu_qwen_attention_workspace_size(64, 40960) > 6 << 20
    status = L.xpu_qwen_attention_noalloc(16, 16, 16, 16, 40959, 64, 8, None)
    assert status == _lib.XPU_ERR_INVALID
    assert "6291456" in _lib.last_error()
