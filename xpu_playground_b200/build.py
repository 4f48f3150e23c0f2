"""Build recipe for libxpu_cuda.so and the C++ host binaries (in-tree).

Everything is compiled for sm_100a only:
    nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3 ...
Objects go to xpu_playground_b200/_build/, the shared library to
xpu_playground_b200/lib/ and the CLI/test binaries to xpu_playground_b200/bin/.
A target is rebuilt when any source or header it may include is newer.

    python -m xpu_playground_b200.build          # build everything
    python -m xpu_playground_b200.build --clean  # remove the outputs first
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB_DIR = PKG / "lib"
BIN_DIR = PKG / "bin"
LIB = LIB_DIR / "libxpu_cuda.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
CXX_FLAGS = ["-O2", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fPIC", f"-I{INCLUDE}", f"-I{HOST}",
             f"-I{CUDA_HOME / 'include'}"]
CUDART_LINK = [f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
BENCH_LIB = LIB_DIR / "libxpu_bench.so"

# Benchmark programs (name -> source under host/): each source defines its
# extern "C" run_* entry (collected into libxpu_bench.so) and, built with
# -DXPU_STANDALONE_HOST, a main() of its own.
BENCH_PROGRAMS: dict[str, str] = {
    "gemv": "gemv.cpp",
    "gemm": "gemm.cpp",
    "peak_mem_2d": "peak_mem_2d.cpp",
    "peak_compute_dpas": "peak_compute_dpas.cpp",
}
# Other C++ host programs: name -> sources under host/ (all link libxpu_cuda.so;
# peak_sycl also links libxpu_bench.so, whose run_* entries it calls).
HOST_PROGRAMS: dict[str, list[str]] = {
    "peak_sycl": ["peak_sycl.cpp"],
    "qwen3": ["qwen3_cli.cpp"],
    "runtime_selftest": ["qwen3/runtime_selftest.cpp", "qwen3/level_zero_runtime_cuda.cpp"],
}
# The reference's Qwen3 kernel runtime API on CUDA (class qwen3::LevelZeroRuntime,
# declared in host/qwen3_api/level_zero_runtime.hpp).
RUNTIME_LIB = LIB_DIR / "libxpu_qwen3_runtime.so"
RUNTIME_SRC = HOST / "qwen3" / "level_zero_runtime_cuda.cpp"
QWEN3_API = HOST / "qwen3_api"


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")) +
                  list(HOST.glob("**/*.hpp")) + list(HOST.glob("**/*.h")))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + proc.stdout)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def build_library(jobs: int | None = None) -> Path:
    """Compile csrc/*.cu and csrc/*.cpp into lib/libxpu_cuda.so."""
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    objects, todo = [], []
    for src in sources:
        obj = BUILD / (src.name + ".o")
        objects.append(obj)
        if _stale(obj, [src, Path(__file__), *headers]):
            todo.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as pool:
        for fut in [pool.submit(_run, cmd) for cmd in todo]:
            fut.result()
    if todo or _stale(LIB, objects):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objects), "-ldl"])
    return LIB


def build_programs() -> list[Path]:
    """Link the benchmark programs, libxpu_bench.so and the other C++ host
    programs against libxpu_cuda.so."""
    BIN_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    rpath = "-Wl,-rpath,$ORIGIN/../lib"
    link = [f"-L{LIB_DIR}", "-lxpu_cuda", *CUDART_LINK]
    outputs = []
    bench_srcs = [HOST / f for f in BENCH_PROGRAMS.values()]
    if _stale(BENCH_LIB, [*bench_srcs, LIB, Path(__file__), *headers]):
        _run([CXX, *CXX_FLAGS, "-shared", *map(str, bench_srcs), "-o", str(BENCH_LIB), *link,
              "-Wl,-rpath,$ORIGIN"])
    outputs.append(BENCH_LIB)
    for name, src in BENCH_PROGRAMS.items():
        out = BIN_DIR / name
        outputs.append(out)
        if _stale(out, [HOST / src, LIB, Path(__file__), *headers]):
            _run([CXX, *CXX_FLAGS, "-DXPU_STANDALONE_HOST", str(HOST / src), "-o", str(out), *link, rpath])
    if _stale(RUNTIME_LIB, [RUNTIME_SRC, LIB, Path(__file__), *headers]):
        _run([CXX, *CXX_FLAGS, f"-I{QWEN3_API}", "-shared", str(RUNTIME_SRC), "-o", str(RUNTIME_LIB), *link,
              "-Wl,-rpath,$ORIGIN"])
    outputs.append(RUNTIME_LIB)
    for name, files in HOST_PROGRAMS.items():
        srcs = [HOST / f for f in files]
        out = BIN_DIR / name
        outputs.append(out)
        extra = ["-lxpu_bench"] if name == "peak_sycl" else []
        if _stale(out, [*srcs, LIB, BENCH_LIB, Path(__file__), *headers]):
            _run([CXX, *CXX_FLAGS, f"-I{QWEN3_API}", *map(str, srcs), "-o", str(out), f"-L{LIB_DIR}", *extra, *link,
                  rpath])
    return outputs


def build_all(jobs: int | None = None) -> None:
    build_library(jobs)
    build_programs()


def clean() -> None:
    for d in (BUILD, LIB_DIR, BIN_DIR):
        if d.exists():
            shutil.rmtree(d)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    args = ap.parse_args()
    if args.clean:
        clean()
    build_all(args.jobs)
    print(LIB)


if __name__ == "__main__":
    main()
