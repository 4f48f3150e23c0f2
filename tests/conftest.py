"""pytest configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs on a CPU-only machine: the oracle against the reference's
golden vectors, the host logic, and the C ABI surface (load + exported
symbols + host-side argument checks). `-m gpu` tests are the parity tests
proper: they call libxpu_cuda through its C ABI on a B200.
"""

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); calls libxpu_cuda kernels")


@pytest.fixture(scope="session", autouse=True)
def _built_artifacts():
    """Build the oracle (gcc) if it is missing; the CUDA library must exist
    already on a GPU box, and is built here when nvcc is present."""
    from oracle import build as oracle_build
    oracle_build.build_oracle()
    from xpu_playground_b200 import _lib, build as lib_build
    if not _lib.LIB_PATH.exists() and Path(lib_build.NVCC).exists():
        lib_build.build_all()
    yield
