"""The C ABI surface on the CPU: the library loads, exports every function include/ggml_compiler_rt.h
declares (and every symbol the reference's Python bindings bind, session.py:81-116), reports no CPU
backend, and fails loudly with the reference's error conventions: malformed GGUFs and programs are
rejected with a message before any device is touched (host-side failure injection)."""

import ctypes
import json
import re
import struct

import numpy as np
import pytest
from conftest import GOLDEN, REPO

from ggml_compiler_b200 import runtime
from ggml_compiler_b200.gguf_write import TensorEntry, write_gguf

HEADER = REPO / "include" / "ggml_compiler_rt.h"
# ggml_compiler/runtime/session.py:81-116 of the reference
REFERENCE_BINDS = """version last_error default_options has_backend load quantize row_size free backend_name
n_inputs n_outputs input_info output_info set_input n_entries entry_name entry_n_inputs entry_n_outputs
entry_input_info entry_output_info run_entry reset metadata n_symbols symbol_info set_symbol
set_input_shape run get_output last_stats n_stages stage_stats""".split()


def declared(headers=(HEADER,)):
    text = "".join(h.read_text() for h in headers)
    return sorted(set(re.findall(r"GGML_COMPILER_API[^;]*?\b(ggml_compiler_[a-z0-9_]+)\s*\(", text, re.S)))


def test_every_declared_symbol_is_exported(rtlib):
    assert len(declared()) >= 40
    names = declared(sorted((REPO / "include").glob("*.h")))  # the reference's ABI and this backend's extensions
    for n in names:
        assert hasattr(rtlib, n), n
    for n in REFERENCE_BINDS:
        assert hasattr(rtlib, "ggml_compiler_" + n), n


def test_version_and_backends(rtlib):
    assert "sm_100a" in runtime.version()
    assert rtlib.ggml_compiler_has_backend(0) is False  # no CPU fallback in this backend
    o = rtlib.ggml_compiler_default_options()
    assert (o.backend, o.device, o.n_threads, o.allow_cpu_fallback) == (2, 0, 0, False)


def test_struct_layouts():
    # ctypes mirrors of ggml_compiler_rt.h:57-75 (identical to the reference's session.py:24-35)
    assert ctypes.sizeof(runtime.COptions) == 16
    assert ctypes.sizeof(runtime.CTensorInfo) == 8 + 4 + 4 + 64 + 8
    assert ctypes.sizeof(runtime.CStats) == 16


BACKENDS = {"cpu": 0, "cuda": 1, "auto": 2}


def _load_error(path, backend="auto"):
    """Loads through the C ABI with the given backend option; returns the error message."""
    lib = runtime.load_library()
    opts = lib.ggml_compiler_default_options()
    opts.backend = BACKENDS[backend]
    handle = lib.ggml_compiler_load(str(path).encode(), ctypes.byref(opts))
    if handle:
        lib.ggml_compiler_free(handle)
        pytest.fail(f"{path} loaded with backend {backend}")
    return lib.ggml_compiler_last_error().decode()


def test_cpu_backend_refused(tmp_path):
    assert "CPU backend is not available" in _load_error(GOLDEN / "ref_llama_q8_0.gguf", backend="cpu")


def test_missing_file(tmp_path):
    assert "cannot read GGUF" in _load_error(tmp_path / "nope.gguf")


def test_truncated_gguf(tmp_path):
    data = (GOLDEN / "ref_llama_q8_0.gguf").read_bytes()
    p = tmp_path / "cut.gguf"
    p.write_bytes(data[: len(data) // 2])
    assert "truncated GGUF" in _load_error(p)
    p.write_bytes(data[:100])
    assert "truncated GGUF" in _load_error(p)


def test_not_a_gguf(tmp_path):
    p = tmp_path / "x.gguf"
    p.write_bytes(b"NOPE" + b"\0" * 64)
    assert "is not a GGUF file" in _load_error(p)


def _tiny(tmp_path, program, name="t.gguf"):
    p = tmp_path / name
    write_gguf(p, program, [TensorEntry("w.0", "f32", (4, 4), np.zeros((4, 4), np.float32))])
    return p


def test_no_program_key(tmp_path):
    p = tmp_path / "np.gguf"
    with open(p, "wb") as f:
        f.write(b"GGUF" + struct.pack("<IQQ", 3, 0, 0))
    assert "has no ggml_compiler.program" in _load_error(p)


def test_corrupt_program(tmp_path):
    good = json.loads((GOLDEN / "ref_program_gqa2.json").read_text())["program"]
    assert "format_version 9 is not supported" in _load_error(_tiny(tmp_path, {**good, "format_version": 9}))
    bad = json.loads(json.dumps(good))
    bad["stages"][0]["nodes"][3]["ne"] = [1, 2]
    assert "'ne' must be an array of 4 dims" in _load_error(_tiny(tmp_path, bad, "b.gguf"))
    bad = json.loads(json.dumps(good))
    bad["values"][0]["ne"][0] = ["^", 2, 3]
    assert "unknown dim operator" in _load_error(_tiny(tmp_path, bad, "c.gguf"))
    bad = json.loads(json.dumps(good))
    bad["entries"][2]["driver"][0]["op"] = "while"
    assert "driver op 'while' is not supported" in _load_error(_tiny(tmp_path, bad, "d.gguf"))
    p = tmp_path / "e.gguf"
    write_gguf(p, {"format_version": 3}, [])
    assert "malformed program" in _load_error(p)


def test_no_device_is_a_clear_error(tmp_path):
    """On a machine without a B200, a well-formed program fails at the device check (never a crash,
    never a silent CPU run)."""
    if runtime.cuda_available():
        pytest.skip("a GPU is present")
    msg = _load_error(GOLDEN / "ref_llama_q8_0.gguf")
    assert "no CUDA device available" in msg or "not a B200" in msg


def test_load_with_builders_is_refused(rtlib):
    class Builder(ctypes.Structure):
        _fields_ = [("stage", ctypes.c_char_p), ("build", ctypes.c_void_p)]

    b = (Builder * 1)(Builder(b"decode", None))
    m = rtlib.ggml_compiler_load_with(str(GOLDEN / "ref_llama_q8_0.gguf").encode(), None, ctypes.cast(b, ctypes.c_void_p), 1)
    assert not m
    assert "cannot run them" in rtlib.ggml_compiler_last_error().decode()
