"""Build recipe for the CPU oracle (test infrastructure only).

* oracle/_build/liboracle.so  <- oracle/xpu_oracle.c (gcc -O2 -fopenmp -ffp-contract=off)
* oracle/_ref/ (only where the reference tree is present): the reference's own
  CPU C++ compiled from its sources in place, never copied:
    - test_cpu_reference  <- qwen3/tests/test_cpu_reference.cpp + qwen3/model.cpp
      (the reference's host-primitive test; prints "... PASS")
    - libref_model.so     <- qwen3/model.cpp + oracle/ref_model_shim.cpp
      (its bf16 codec and config/checkpoint validator behind a C shim)
    - test_gpu_dispatch_cuda <- qwen3/tests/test_gpu_dispatch.cpp + qwen3/model.cpp,
      unchanged, against the reference's own runtime header, with the CUDA
      implementation of that runtime (xpu_playground_b200/host/qwen3/
      level_zero_runtime_cuda.cpp, Level Zero handle types from host/ze_shim)
      and libxpu_cuda: the reference's kernel-dispatch test run on a B200.
  The GPU box has no reference tree; it uses the files built here.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
LIB = BUILD / "liboracle.so"
# The reference checkout: XPU_REFERENCE_TREE, else a directory named
# "reference" beside this repository (absent on GPU boxes: the prebuilt
# oracle/_ref files are used there).
REFERENCE = Path(os.environ.get("XPU_REFERENCE_TREE", str(HERE.parent.parent / "reference")))


def _stale(target: Path, sources: list[Path]) -> bool:
    return not target.exists() or any(s.stat().st_mtime > target.stat().st_mtime for s in sources)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout)
        raise RuntimeError("oracle build step failed")


def build_oracle() -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    src = HERE / "xpu_oracle.c"
    if _stale(LIB, [src, Path(__file__)]):
        _run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-std=c11",
              "-Wall", "-Wextra", str(src), "-o", str(LIB), "-lm"])
    return LIB


def build_reference() -> list[Path]:
    """Compile the reference's CPU C++ where its tree exists (this container)."""
    qwen3 = REFERENCE / "qwen3"
    if not (qwen3 / "model.cpp").exists():
        return []
    REF_OUT.mkdir(parents=True, exist_ok=True)
    outs = []
    test_bin = REF_OUT / "test_cpu_reference"
    srcs = [qwen3 / "tests" / "test_cpu_reference.cpp", qwen3 / "model.cpp"]
    if _stale(test_bin, srcs + [Path(__file__)]):
        _run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", *map(str, srcs),
              "-o", str(test_bin)])
    outs.append(test_bin)
    shim = HERE / "ref_model_shim.cpp"
    lib = REF_OUT / "libref_model.so"
    if _stale(lib, [shim, qwen3 / "model.cpp", Path(__file__)]):
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{qwen3}", str(shim),
              str(qwen3 / "model.cpp"), "-o", str(lib)])
    outs.append(lib)

    repo = HERE.parent
    pkg = repo / "xpu_playground_b200"
    runtime_src = pkg / "host" / "qwen3" / "level_zero_runtime_cuda.cpp"
    libdir = pkg / "lib"
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    dispatch = REF_OUT / "test_gpu_dispatch_cuda"
    srcs = [qwen3 / "tests" / "test_gpu_dispatch.cpp", qwen3 / "model.cpp", runtime_src]
    if (libdir / "libxpu_cuda.so").exists() and _stale(dispatch, srcs + [Path(__file__), libdir / "libxpu_cuda.so"]):
        _run(["g++", "-std=c++17", "-O2", f"-I{qwen3}", f"-I{pkg / 'host' / 'ze_shim'}", f"-I{repo / 'include'}",
              f"-I{cuda / 'include'}", *map(str, srcs), "-o", str(dispatch), f"-L{libdir}", "-lxpu_cuda",
              f"-L{cuda / 'lib64'}", "-lcudart_static", "-ldl", "-lpthread", "-lrt",
              f"-Wl,-rpath,{libdir}", "-Wl,-rpath,$ORIGIN/../../xpu_playground_b200/lib"])
    if dispatch.exists():
        outs.append(dispatch)
    return outs


def build_all() -> None:
    build_oracle()
    build_reference()


if __name__ == "__main__":
    build_all()
    print(LIB)
