"""torch-tensor wrappers over the C ABI (one function per entry point).

These pass device pointers and sizes straight through to libxpu_cuda; torch
only provides device memory and the current CUDA stream. Every tensor must be
a contiguous CUDA tensor; 16-bit tensors are passed by their bit patterns.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import XPU_BF16, XPU_FP16, call


def _ptr(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("libxpu_cuda entry points take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return XPU_BF16
    if t.dtype == torch.float16:
        return XPU_FP16
    raise ValueError(f"unsupported dtype {t.dtype}")


def gemv(matrix: torch.Tensor, vector: torch.Tensor, out: torch.Tensor | None = None,
         stream=None) -> torch.Tensor:
    m, k = matrix.shape
    if out is None:
        out = torch.empty(m, dtype=matrix.dtype, device=matrix.device)
    call("xpu_gemv", _dtype_code(matrix), _ptr(matrix), _ptr(vector), _ptr(out), m, k,
         _stream(stream))
    return out


def gemm_bt(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """C[m,n] = A[m,k] . W^T for W [n,k] (row-major, contiguous, bf16 or fp16)."""
    m, k = a.shape
    n, k2 = w.shape
    if k2 != k or a.dtype != w.dtype:
        raise ValueError("gemm_bt: A is [m,k] and W is [n,k] of the same dtype")
    if out is None:
        out = torch.empty(m, n, dtype=a.dtype, device=a.device)
    call("xpu_gemm_bt", _dtype_code(a), _ptr(a), _ptr(w), _ptr(out), m, n, k, _stream(stream))
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
         stream=None) -> torch.Tensor:
    """C[m,n] = A[m,k] . B[k,n] (row-major, contiguous, bf16 or fp16)."""
    m, k = a.shape
    k2, n = b.shape
    if k2 != k or a.dtype != b.dtype:
        raise ValueError("gemm: A is [m,k] and B is [k,n] of the same dtype")
    if out is None:
        out = torch.empty(m, n, dtype=a.dtype, device=a.device)
    call("xpu_gemm", _dtype_code(a), _ptr(a), _ptr(b), _ptr(out), m, n, k, _stream(stream))
    return out


def device_status() -> int:
    """Reads and clears the library's sticky device error word (synchronises)."""
    flags = ctypes.c_uint32(0)
    call("xpu_device_status", ctypes.byref(flags))
    return flags.value


def peak_mem_fill(surface: torch.Tensor, stream=None) -> None:
    """surface[i] = 1 + (hash(i) & 0xffff) / 65536 (float32 tensor)."""
    call("xpu_peak_mem_fill", _ptr(surface), surface.numel(), _stream(stream))


def peak_mem_read(surface: torch.Tensor, sink: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """One read of a [height, 1024] float32 surface; returns the per-unit
    checksums (one per 2 KiB unit: height * 2 of them)."""
    height = surface.numel() // 1024
    if sink is None:
        sink = torch.zeros(height * 2, dtype=torch.float32, device=surface.device)
    call("xpu_peak_mem_read", _ptr(surface), _ptr(sink), height, _stream(stream))
    return sink


def peak_compute(ctas: int, rounds: int, sink: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """ctas x rounds x 8 tensor-core MMAs; returns sink (1 + 32 rounds each)."""
    if sink is None:
        sink = torch.zeros(ctas, dtype=torch.float32, device="cuda")
    call("xpu_peak_compute", _ptr(sink), ctas, rounds, _stream(stream))
    return sink


def qwen_embedding(table, output, token: int, width: int, stream=None):
    call("xpu_qwen_embedding", _ptr(table), _ptr(output), token, width, _stream(stream))


def qwen_rms_norm(inp, weight, output, width: int, epsilon: float = 1e-6, stream=None):
    call("xpu_qwen_rms_norm", _ptr(inp), _ptr(weight), _ptr(output), width, epsilon, _stream(stream))


def qwen_gemv(matrix, vector, output, rows: int, columns: int, stream=None):
    call("xpu_qwen_gemv", _ptr(matrix), _ptr(vector), _ptr(output), rows, columns, _stream(stream))


def qwen_qkv_rope_cache(query, key, value, query_norm, key_norm, rope_cos, rope_sin, key_cache,
                        value_cache, position: int, maximum_sequence: int, query_heads: int,
                        key_value_heads: int, stream=None):
    call("xpu_qwen_qkv_rope_cache", _ptr(query), _ptr(key), _ptr(value), _ptr(query_norm),
         _ptr(key_norm), _ptr(rope_cos), _ptr(rope_sin), _ptr(key_cache), _ptr(value_cache),
         position, maximum_sequence, query_heads, key_value_heads, _stream(stream))


def qwen_attention_workspace_size(query_heads: int, maximum_positions: int) -> int:
    return int(_lib.load().xpu_qwen_attention_workspace_size(query_heads, maximum_positions))


def qwen_attention(query, key_cache, value_cache, output, position: int, query_heads: int,
                   key_value_heads: int, workspace: torch.Tensor, stream=None):
    call("xpu_qwen_attention", _ptr(query), _ptr(key_cache), _ptr(value_cache), _ptr(output),
         position, query_heads, key_value_heads, _ptr(workspace),
         workspace.numel() * workspace.element_size(), _stream(stream))


def qwen_add(left, right, width: int, stream=None):
    call("xpu_qwen_add", _ptr(left), _ptr(right), width, _stream(stream))


def qwen_silu_multiply(gate, up, width: int, stream=None):
    call("xpu_qwen_silu_multiply", _ptr(gate), _ptr(up), width, _stream(stream))


def qwen_argmax(values, token, width: int, stream=None):
    call("xpu_qwen_argmax", _ptr(values), _ptr(token), width, _stream(stream))
