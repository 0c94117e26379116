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

    if not runtime.cuda_available():
        pytest.fail("no B200 visible to libggml_compiler_rt (the gpu tests need one)")
    return True


REFERENCE_PY = REPO / "baseline" / "_ref"  # the reference's Python package (installed without its CMake build)


@pytest.fixture(scope="session")
def reference_pkg(rtlib):
    """The reference's own Python front end (ggml_compiler), bound to this repository's library
    through $GGML_COMPILER_RT, as a user of the reference switches backends. It lives in
    baseline/_ref: `pip install --no-index --no-build-isolation --no-deps
    --config-settings=wheel.cmake=false --target baseline/_ref <reference checkout>` (the
    reference's own build backend with its CMake step, which needs the network, switched off)."""
    if not (REFERENCE_PY / "ggml_compiler" / "runtime" / "session.py").exists():
        pytest.skip("the reference's Python package is not installed in baseline/_ref")
    from ggml_compiler_b200 import runtime

    os.environ["GGML_COMPILER_RT"] = str(runtime.library_path())
    if str(REFERENCE_PY) not in sys.path:
        sys.path.append(str(REFERENCE_PY))
    import ggml_compiler
    import ggml_compiler.runtime.session as session

    assert Path(session.library_path()) == Path(runtime.library_path())
    return ggml_compiler
