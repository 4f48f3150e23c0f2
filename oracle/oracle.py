"""numpy/ctypes face of the CPU oracle (oracle/xpu_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, as the checker and the CPU
baseline. The product (libxpu_cuda.so and its host programs) never imports it.
Every function cites the reference code it restates in xpu_oracle.c.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB_PATH = HERE / "_build" / "liboracle.so"
_lib = None

u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
c_u32, c_u64, c_f32, c_int = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float, ctypes.c_int


class Qwen3Config(ctypes.Structure):
    _fields_ = [("hidden", c_u32), ("intermediate", c_u32), ("q_heads", c_u32),
                ("kv_heads", c_u32), ("layers", c_u32), ("vocab", c_u32), ("max_seq", c_u32),
                ("eps", c_f32)]


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            from . import build as _build  # noqa: F401  (package import when available)
            _build.build_oracle()
        L = ctypes.CDLL(str(_LIB_PATH))
        sig = {
            "orc_f32_to_bf16": (ctypes.c_uint16, [c_f32]),
            "orc_bf16_to_f32": (c_f32, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [c_f32]),
            "orc_f16_to_f32": (c_f32, [ctypes.c_uint16]),
            "orc_encode16": (None, [f32p, u16p, c_u64, c_int]),
            "orc_decode16": (None, [u16p, f32p, c_u64, c_int]),
            "orc_hash_u32": (c_u32, [c_u32]),
            "orc_gemv_bench_inputs": (None, [u16p, u16p, c_u32, c_u32, c_int]),
            "orc_peak_mem_value": (c_f32, [c_u64]),
            "orc_fill_uniform16": (None, [u16p, c_u64, c_u64, c_u64, c_int]),
            "orc_fill_normal_bf16": (None, [u16p, c_u64, c_u64, c_u64, c_f32]),
            "orc_gemv": (None, [u16p, u16p, f32p, c_u32, c_u32, c_int]),
            "orc_gemm": (None, [u16p, u16p, f32p, c_u32, c_u32, c_u32, c_int]),
            "orc_num_threads": (c_int, []),
            "orc_set_num_threads": (None, [c_int]),
            "orc_embedding": (None, [u16p, u16p, c_u32, c_u32]),
            "orc_rms_norm": (None, [u16p, u16p, u16p, c_u32, c_f32]),
            "orc_qkv_rope_cache": (None, [u16p, u16p, u16p, u16p, u16p, u16p, u16p, u16p, u16p,
                                          c_u32, c_u32, c_u32, c_u32]),
            "orc_attention": (None, [u16p, u16p, u16p, u16p, c_u32, c_u32, c_u32]),
            "orc_add": (None, [u16p, u16p, c_u32]),
            "orc_silu_multiply": (None, [u16p, u16p, c_u32]),
            "orc_argmax": (c_u32, [u16p, c_u32]),
            "orc_rope_tables": (None, [u16p, u16p, c_u32, c_f32]),
            "orc_qwen3_decode": (c_u32, [ctypes.POINTER(Qwen3Config), ctypes.c_void_p, u16p, u16p,
                                         u16p, u16p, c_u32, c_u32, ctypes.c_void_p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


# ------------------------------------------------------------- codecs ----

def bf16_bits(values) -> np.ndarray:
    """fp32 -> bf16 bit patterns, RNE (qwen3/model.cpp:497-502)."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    out = np.empty(v.size, np.uint16)
    lib().orc_encode16(v, out, v.size, 0)
    return out.reshape(np.shape(values))


def fp16_bits(values) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    out = np.empty(v.size, np.uint16)
    lib().orc_encode16(v, out, v.size, 1)
    return out.reshape(np.shape(values))


def decode(bits, fp16: bool = False) -> np.ndarray:
    b = np.ascontiguousarray(bits, dtype=np.uint16).ravel()
    out = np.empty(b.size, np.float32)
    lib().orc_decode16(b, out, b.size, int(fp16))
    return out.reshape(np.shape(bits))


def bf16_to_float(bits) -> np.ndarray:
    return decode(bits, False)


# ---------------------------------------------------------- generators ----

def uniform16(n: int, seed: int, tag: int = 0, fp16: bool = False) -> np.ndarray:
    out = np.empty(int(n), np.uint16)
    lib().orc_fill_uniform16(out, int(n), seed, tag, int(fp16))
    return out


def normal_bf16(n: int, seed: int, tag: int, std: float = 0.02) -> np.ndarray:
    out = np.empty(int(n), np.uint16)
    lib().orc_fill_normal_bf16(out, int(n), seed, tag, std)
    return out


def gemv_bench_inputs(m: int, k: int, fp16: bool = False):
    """The reference's hash-generated GEMV matrix and vector (gemv.cpp:156-167)."""
    A = np.empty(m * k, np.uint16)
    x = np.empty(k, np.uint16)
    lib().orc_gemv_bench_inputs(A, x, m, k, int(fp16))
    return A.reshape(m, k), x


# --------------------------------------------------------- GEMV / GEMM ----

def gemv(A: np.ndarray, x: np.ndarray, fp16: bool = False) -> np.ndarray:
    """FP32 host GEMV over 16-bit inputs (gemv.cpp:191-196)."""
    m, k = A.shape
    y = np.empty(m, np.float32)
    lib().orc_gemv(np.ascontiguousarray(A), np.ascontiguousarray(x), y, m, k, int(fp16))
    return y


def gemm(A: np.ndarray, B: np.ndarray, fp16: bool = False) -> np.ndarray:
    m, k = A.shape
    k2, n = B.shape
    assert k == k2
    C = np.empty((m, n), np.float32)
    lib().orc_gemm(np.ascontiguousarray(A), np.ascontiguousarray(B), C.reshape(-1), m, n, k, int(fp16))
    return C


def rel_frobenius(actual, expected) -> float:
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))


# ------------------------------------------------------- calibrators ----

def _hash_u32(i: np.ndarray) -> np.ndarray:
    b = i.astype(np.uint32)
    b ^= b >> np.uint32(16)
    b *= np.uint32(0x7FEB352D)
    b ^= b >> np.uint32(15)
    b *= np.uint32(0x846CA68B)
    b ^= b >> np.uint32(16)
    return b


def peak_mem_surface(elements: int) -> np.ndarray:
    """The read calibrator's fill, 1 + (hash(i) & 0xffff) / 65536
    (peak_mem_2d.cpp:36-47); index truncated to 32 bits like the reference."""
    idx = np.arange(elements, dtype=np.uint64).astype(np.uint32)
    return (np.float32(1.0) + (_hash_u32(idx) & np.uint32(0xFFFF)).astype(np.float32)
            * np.float32(1.0 / 65536.0)).astype(np.float32)


def peak_mem_checksums(surface: np.ndarray) -> np.ndarray:
    """Per read unit (16 columns x 32 rows of the 1024-wide surface), the FP32
    sum in load order of the elements at rows y, y+8, y+16, y+24 of column x
    (peak_mem_2d.cpp:49-59, peak_mem_2d_kernel.cpp:28-50)."""
    s = surface.reshape(-1, 32, 1024)          # band, row in band, column
    picks = s[:, 0::8, 0::16]                  # band, load, unit column
    out = np.zeros((s.shape[0], 64), np.float32)
    for load in range(4):
        out = (out + picks[:, load, :]).astype(np.float32)
    return out.reshape(-1)


def peak_compute_checksum(rounds: int) -> float:
    """Tensor calibrator sink value: accumulator offsets 0 + 1 plus 4 per
    MMA, 8 MMAs per round (the closed form of peak_compute_dpas.cpp:197-198
    for this kernel's two accumulators)."""
    return float(np.float32(1.0) + np.float32(8 * rounds * 4))


# ------------------------------------- Qwen3 operators (kernels.hpp) ----

def embedding(table, token, width):
    out = np.empty(width, np.uint16)
    lib().orc_embedding(np.ascontiguousarray(table).ravel(), out, token, width)
    return out


def rms_norm(x, w, eps=1e-6):
    out = np.empty_like(x)
    lib().orc_rms_norm(x, w, out, x.size, eps)
    return out


def qkv_rope_cache(q, k, v, qn, kn, cos_t, sin_t, kc, vc, position, max_seq, q_heads, kv_heads):
    """In place on q, k, kc, vc (kernels.hpp:71-154)."""
    lib().orc_qkv_rope_cache(q, k, v, qn, kn, cos_t, sin_t, kc, vc, position, max_seq, q_heads, kv_heads)


def attention(q, kc, vc, position, q_heads, kv_heads):
    out = np.empty(q_heads * 128, np.uint16)
    lib().orc_attention(q, kc, vc, out, position, q_heads, kv_heads)
    return out


def add(left, right):
    out = left.copy()
    lib().orc_add(out, right, out.size)
    return out


def silu_multiply(gate, up):
    out = gate.copy()
    lib().orc_silu_multiply(out, up, out.size)
    return out


def argmax(values) -> int:
    return int(lib().orc_argmax(np.ascontiguousarray(values, np.uint16), values.size))


def rope_tables(max_seq: int, theta: float = 1e6):
    c = np.empty(max_seq * 128, np.uint16)
    s = np.empty(max_seq * 128, np.uint16)
    lib().orc_rope_tables(c, s, max_seq, theta)
    return c, s


def set_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def num_threads() -> int:
    return int(lib().orc_num_threads())
