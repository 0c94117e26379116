"""The reference's own Python bindings over this library, on the CPU: the reference's
ggml_compiler.runtime binds its whole signature table (session.py:81-116) against
libggml_compiler_rt.so, encodes weights through it byte-exact with gguf-py, reports no CPU backend,
and its Session surfaces this library's load errors as GgmlCompilerRuntimeError. The compute side
of the same drop-in runs in tests/test_gpu_reference_driver.py."""

import numpy as np
import pytest
from conftest import GOLDEN


def test_reference_binds_every_signature(reference_pkg):
    from ggml_compiler.runtime import session

    lib = session._load()  # raises AttributeError if any bound symbol were missing
    assert "sm_100a" in session.version()
    assert session.has_backend("cpu") is False
    assert lib.ggml_compiler_row_size(b"q4_0", 4096) == 2304


@pytest.mark.parametrize("typ", ["q4_0", "q8_0"])
def test_reference_quantize_is_gguf_py_exact(reference_pkg, typ):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T
    from ggml_compiler.runtime import session

    x = np.random.default_rng(7).standard_normal((64, 256), dtype=np.float32) * np.float32(0.02)
    x[3, :32] = 0.0  # an all-zero block
    want = quants.quantize(x, T.Q4_0 if typ == "q4_0" else T.Q8_0)
    assert session.quantize(x, typ).tobytes() == want.tobytes()


def test_reference_session_reports_library_errors(reference_pkg, tmp_path):
    from ggml_compiler.runtime import GgmlCompilerRuntimeError, Session

    with pytest.raises(GgmlCompilerRuntimeError, match="CPU backend is not available"):
        Session(GOLDEN / "ref_llama_q8_0.gguf", backend="cpu")
    with pytest.raises(GgmlCompilerRuntimeError, match="cannot read GGUF"):
        Session(tmp_path / "missing.gguf", backend="cuda")
