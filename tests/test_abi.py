"""The C ABI surface without a GPU: the library loads, exports every function
include/xpu_cuda.h declares, and rejects bad arguments on the host with a
status code and a message (no device work is queued for those calls)."""

import ctypes
import subprocess

import pytest

from xpu_playground_b200 import _lib


def test_library_loads_and_reports_abi_version():
    lib = _lib.load()
    assert lib.xpu_abi_version() >= 1


def test_every_declared_function_is_exported():
    declared = _lib.declared_functions()
    assert "xpu_gemv" in declared and "xpu_qwen_attention" in declared
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [name for name in declared if name not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # and the Python binding knows every declared function's signature
    assert not [n for n in declared if n not in _lib.SIGNATURES]


def test_signatures_cover_only_declared_functions():
    declared = set(_lib.declared_functions())
    assert set(_lib.SIGNATURES) <= declared


@pytest.mark.parametrize("call", [
    lambda L: L.xpu_gemv(0, None, None, None, 4, 4, None),
    lambda L: L.xpu_gemv(7, 1, 1, 1, 4, 4, None),
    lambda L: L.xpu_gemv(0, 1, 1, 1, 0, 4, None),
    lambda L: L.xpu_qwen_rms_norm(None, None, None, 8, 1e-6, None),
    lambda L: L.xpu_qwen_qkv_rope_cache(*([1] * 9), 0, 1, 30, 8, None),
    lambda L: L.xpu_qwen_attention(1, 1, 1, 1, 10, 32, 8, 16, 8, None),
    lambda L: L.xpu_qwen_attention(1, 1, 1, 1, 0, 32, 8, None, 0, None),
    lambda L: L.xpu_qwen_argmax(None, None, 5, None),
])
def test_invalid_arguments_fail_on_host(call):
    L = _lib.load()
    status = call(L)
    assert status in (_lib.XPU_ERR_INVALID, _lib.XPU_ERR_UNSUPPORTED)
    assert _lib.last_error()


@pytest.mark.parametrize("call", [
    lambda L: L.xpu_qwen3_create_batched(None, 16, 0, 4, None),
    lambda L: L.xpu_qwen3_batch_decode(None, 1, 1, 1, 1),
    lambda L: L.xpu_qwen3_batch_generate(None, 1, 1, 1, 4, 0, 1, 1),
    lambda L: L.xpu_qwen3_batch_set_state(None, 1, 1, 1),
    lambda L: L.xpu_qwen3_batch_get_state(None, 1, None, None, None),
    lambda L: L.xpu_qwen3_batch_enqueue_steps(None, 1, None),
    lambda L: L.xpu_qwen3_batch_logits(None, 0, 1, 4),
    lambda L: L.xpu_qwen3_batch_trace(None, None, 0, None),
    lambda L: L.xpu_qwen3_prefill(None, 1, 4, 1),
])
def test_batched_entries_reject_null_engine(call):
    """The batched-decode and prefill entries check their handle and
    pointers on the host (no device is touched)."""
    L = _lib.load()
    assert call(L) == _lib.XPU_ERR_INVALID
    assert _lib.last_error()


def test_batched_byte_model_without_engine():
    L = _lib.load()
    assert L.xpu_qwen3_batch_bytes_per_step(None, 16, 2048) == 0
    assert L.xpu_qwen3_batch_kernels_per_step(None) == 0


def test_batched_tensor_parallel_create_checks_arguments():
    L = _lib.load()
    # null shape / output pointer: refused before any device work
    assert L.xpu_qwen3_create_batched_tp(None, 16, 0, 0, 2, 4, None) == _lib.XPU_ERR_INVALID


def test_attention_group_sizes():
    L = _lib.load()
    # 12 query heads over 8 kv heads is not a whole group -> invalid
    assert L.xpu_qwen_attention(16, 16, 16, 16, 0, 12, 8, 16, 1 << 20, None) == _lib.XPU_ERR_INVALID
    # group of 3 is rejected as unsupported before any launch
    assert L.xpu_qwen_attention(16, 16, 16, 16, 0, 24, 8, 16, 1 << 20, None) == _lib.XPU_ERR_UNSUPPORTED
    assert L.xpu_qwen_attention_workspace_size(32, 128) == 32 * 1 * 130 * 4
    assert L.xpu_qwen_attention_workspace_size(32, 129) == 32 * 2 * 130 * 4


def test_check_raises_with_message():
    with pytest.raises(_lib.XpuError, match="XPU_ERR_INVALID"):
        _lib.call("xpu_gemv", 0, None, None, None, 1, 1, None)


def test_runtime_library_exports_the_reference_class_api():
    """libxpu_qwen3_runtime.so defines qwen3::LevelZeroRuntime's members
    (qwen3/level_zero_runtime.hpp:19-32)."""
    import subprocess
    from xpu_playground_b200 import build
    out = subprocess.run(["nm", "-DC", "--defined-only", str(build.RUNTIME_LIB)], capture_output=True,
                         text=True, check=True).stdout
    for sym in ("qwen3::LevelZeroRuntime::LevelZeroRuntime(std::__cxx11::basic_string",
                "qwen3::LevelZeroRuntime::~LevelZeroRuntime()",
                "qwen3::LevelZeroRuntime::require_bmg_and_memory(unsigned long) const",
                "qwen3::LevelZeroRuntime::allocate_device(unsigned long, unsigned long)",
                "qwen3::LevelZeroRuntime::copy_to_device(void*, void const*, unsigned long)",
                "qwen3::LevelZeroRuntime::copy_from_device(void*, void const*, unsigned long)",
                "qwen3::LevelZeroRuntime::launch(std::__cxx11::basic_string"):
        assert sym in out, sym
