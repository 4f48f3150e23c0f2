"""ctypes binding of libxpu_cuda.so (the C ABI declared in include/xpu_cuda.h).

The library is loaded from this package's lib/ directory, where
``python -m xpu_playground_b200.build`` puts it. There is no fallback: if the
library is missing, importing a kernel wrapper raises ``XpuLibraryMissing``.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "lib" / "libxpu_cuda.so"
HEADER = PKG.parent / "include" / "xpu_cuda.h"

XPU_OK, XPU_ERR_INVALID, XPU_ERR_CUDA, XPU_ERR_UNSUPPORTED = 0, 1, 2, 3
XPU_ERR_TIMEOUT, XPU_ERR_NONFINITE, XPU_ERR_NO_MEMORY = 4, 5, 6
XPU_BF16, XPU_FP16 = 0, 1

STATUS_NAMES = {0: "XPU_OK", 1: "XPU_ERR_INVALID", 2: "XPU_ERR_CUDA", 3: "XPU_ERR_UNSUPPORTED",
                4: "XPU_ERR_TIMEOUT", 5: "XPU_ERR_NONFINITE", 6: "XPU_ERR_NO_MEMORY"}


class XpuLibraryMissing(ImportError):
    pass


class XpuError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


vp, sz = ctypes.c_void_p, ctypes.c_size_t
u32, u64, i32, f32, f64 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_float, ctypes.c_double

class Qwen3ShapeC(ctypes.Structure):
    """xpu_qwen3_shape."""
    _fields_ = [("hidden_size", u32), ("intermediate_size", u32), ("num_hidden_layers", u32),
                ("num_attention_heads", u32), ("num_key_value_heads", u32), ("vocab_size", u32),
                ("tie_word_embeddings", u32), ("rms_norm_eps", f32), ("rope_theta", f64)]


class Qwen3InfoC(ctypes.Structure):
    """xpu_qwen3_info_t."""
    _fields_ = [("weight_bytes", u64), ("kernels_per_step", u32), ("vocab_rows", u32),
                ("vocab_offset", u32), ("stream", vp)]

# name -> (restype, argtypes). Keep in step with include/xpu_cuda.h.
SIGNATURES: dict[str, tuple] = {
    "xpu_last_error": (ctypes.c_char_p, []),
    "xpu_abi_version": (i32, []),
    "xpu_gemv": (i32, [i32, vp, vp, vp, u32, u32, vp]),
    "xpu_gemm": (i32, [i32, vp, vp, vp, u32, u32, u32, vp]),
    "xpu_gemm_bt": (i32, [i32, vp, vp, vp, u32, u32, u32, vp]),
    "xpu_device_status": (i32, [ctypes.POINTER(u32)]),
    "xpu_peak_mem_fill": (i32, [vp, u64, vp]),
    "xpu_peak_mem_read": (i32, [vp, vp, u32, vp]),
    "xpu_peak_compute": (i32, [vp, u32, u32, vp]),
    "xpu_qwen_embedding": (i32, [vp, vp, u32, u32, vp]),
    "xpu_qwen_rms_norm": (i32, [vp, vp, vp, u32, f32, vp]),
    "xpu_qwen_gemv": (i32, [vp, vp, vp, u32, u32, vp]),
    "xpu_qwen_qkv_rope_cache": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, vp]),
    "xpu_qwen_attention_workspace_size": (sz, [u32, u32]),
    "xpu_qwen_attention": (i32, [vp, vp, vp, vp, u32, u32, u32, vp, sz, vp]),
    "xpu_qwen_attention_noalloc": (i32, [vp, vp, vp, vp, u32, u32, u32, vp]),
    "xpu_qwen_add": (i32, [vp, vp, u32, vp]),
    "xpu_qwen_silu_multiply": (i32, [vp, vp, u32, vp]),
    "xpu_qwen_argmax": (i32, [vp, vp, u32, vp]),
    "xpu_fill_uniform16": (i32, [i32, vp, u64, u64, u64, vp]),
    "xpu_fill_normal_bf16": (i32, [vp, u64, u64, u64, f32, vp]),
    "xpu_qwen3_create": (i32, [vp, u32, i32, u32, u32, vp]),
    "xpu_qwen3_destroy": (i32, [vp]),
    "xpu_qwen3_read_config": (i32, [ctypes.c_char_p, ctypes.POINTER(Qwen3ShapeC)]),
    "xpu_qwen3_validate_checkpoint": (i32, [ctypes.c_char_p, ctypes.POINTER(Qwen3ShapeC), ctypes.POINTER(u64)]),
    "xpu_qwen3_load_checkpoint": (i32, [vp, ctypes.c_char_p]),
    "xpu_qwen3_tp_handle": (i32, [vp, vp]),
    "xpu_qwen3_tp_connect": (i32, [vp, vp, u32]),
    "xpu_qwen3_init_synthetic": (i32, [vp, u64, f32]),
    "xpu_qwen3_set_tensor": (i32, [vp, ctypes.c_char_p, vp, u64]),
    "xpu_qwen3_decode": (i32, [vp, u32, u32, vp]),
    "xpu_qwen3_generate": (i32, [vp, vp, u32, u32, i32, vp, vp]),
    "xpu_qwen3_set_state": (i32, [vp, u32, u32, u32]),
    "xpu_qwen3_enqueue_steps": (i32, [vp, u32, vp]),
    "xpu_qwen3_get_state": (i32, [vp, vp, vp, vp]),
    "xpu_qwen3_synchronize": (i32, [vp]),
    "xpu_qwen3_set_mode": (i32, [vp, i32]),
    "xpu_qwen3_trace": (i32, [vp, vp, u32, vp]),
    "xpu_qwen3_token_log": (i32, [vp, u32, u32, vp]),
    "xpu_qwen3_logits": (i32, [vp, vp, u32]),
    "xpu_qwen3_info": (i32, [vp, vp]),
    "xpu_qwen3_bytes_per_token": (u64, [vp, u32]),
    "xpu_qwen3_create_batched": (i32, [vp, u32, i32, u32, vp]),
    "xpu_qwen3_create_batched_tp": (i32, [vp, u32, i32, u32, u32, u32, vp]),
    "xpu_qwen3_prefill": (i32, [vp, vp, u32, vp]),
    "xpu_qwen3_prefill_dense": (i32, [vp, vp, u32, vp]),
    "xpu_qwen3_batch_decode": (i32, [vp, u32, vp, vp, vp]),
    "xpu_qwen3_batch_generate": (i32, [vp, u32, vp, vp, u32, i32, vp, vp]),
    "xpu_qwen3_batch_set_state": (i32, [vp, u32, vp, vp]),
    "xpu_qwen3_batch_enqueue_steps": (i32, [vp, u32, vp]),
    "xpu_qwen3_batch_get_state": (i32, [vp, u32, vp, vp, vp]),
    "xpu_qwen3_batch_logits": (i32, [vp, u32, vp, u32]),
    "xpu_qwen3_batch_bytes_per_step": (u64, [vp, u32, u32]),
    "xpu_qwen3_batch_kernels_per_step": (u32, [vp]),
    "xpu_qwen3_batch_trace": (i32, [vp, vp, u32, vp]),
}


_lib = None


def load() -> ctypes.CDLL:
    """Load libxpu_cuda.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise XpuLibraryMissing(
            f"{LIB_PATH} is missing: build it with `python -m xpu_playground_b200.build` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _lib = lib
    return lib


def last_error() -> str:
    return load().xpu_last_error().decode()


def check(status: int) -> None:
    if status != XPU_OK:
        raise XpuError(status, last_error())


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise XpuError on failure."""
    check(getattr(load(), name)(*args))


def declared_functions(header: Path = HEADER) -> list[str]:
    """Names of the functions include/xpu_cuda.h declares."""
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(xpu_\w+|run_\w+)\s*\(", text)))
