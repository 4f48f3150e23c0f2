"""Helpers shared by the tests: bf16 bit arrays <-> torch tensors."""

from __future__ import annotations

import numpy as np
import torch


def to_device(bits: np.ndarray, dtype=torch.bfloat16) -> torch.Tensor:
    """uint16 bit patterns -> a CUDA tensor of `dtype` with the same bits."""
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy())
    return t.view(dtype).cuda()


def to_bits(t: torch.Tensor) -> np.ndarray:
    """16-bit CUDA/CPU tensor -> uint16 bit patterns (numpy)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def close(actual: np.ndarray, expected: np.ndarray, atol=0.03, rtol=0.02) -> None:
    """The reference's primitive tolerance (qwen3/tests/test_cpu_reference.cpp:17-25,
    test_gpu_dispatch.cpp:19-26): |a - e| <= atol + rtol * |e|, all finite."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert np.all(np.isfinite(a)), "non-finite values"
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), f"{bad.sum()} mismatches, first at {np.argmax(bad)}: {a[bad][:4]} vs {e[bad][:4]}"
