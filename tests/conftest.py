import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "ggml-compiler_b200"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (runs through the CUDA library)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(scope="session")
def rtlib():
    """The product library, built in-tree if needed."""
    from ggml_compiler_b200 import build, runtime

    if not (PKG_ROOT / "ggml_compiler_b200" / "lib" / "libggml_compiler_rt.so").exists():
        build.build()
    return runtime.load_library()


@pytest.fixture(scope="session")
def gpu():
    """Skip unless a B200 is visible to the library (the -m gpu suite runs on one)."""
    from ggml_compiler_b200 import runtime

    if not runtime.has_backend("cuda"):
        pytest.fail("no B200 visible to libggml_compiler_rt (the gpu tests need one)")
    return True
