"""Q4_0 / Q8_0 encoding: the library's ggml_compiler_quantize and the CPU oracle are byte-exact with
gguf-py 0.19's encoders (the ones the reference pins; gguf/quants.py Q4_0 :220-252, Q8_0 :378-402),
on the golden vectors in tests/golden (made by tests/golden/make_quant_golden.py): edge-case rows and
SHA-256 digests at the full op-sweep shapes of BASELINE config 2. No GPU needed."""

import hashlib
import json

import numpy as np
import pytest
from conftest import GOLDEN

import oracle
from ggml_compiler_b200 import runtime


def weights(shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(0.02)


@pytest.mark.parametrize("typ", ["q4_0", "q8_0"])
def test_edge_cases_match_gguf_py(rtlib, typ):
    g = np.load(GOLDEN / "quant_small.npz")
    x = g["x"]
    got = runtime.encode(x, typ)
    assert got.tobytes() == g[typ].tobytes()
    assert oracle.quantize(x, typ).tobytes() == g[typ].tobytes()
    dec = oracle.dequantize(got, typ, x.shape[-1])
    np.testing.assert_array_equal(dec, g[f"{typ}_dec"].reshape(dec.shape))


@pytest.mark.parametrize("shape", [(4096, 4096), (14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("typ", ["q4_0", "q8_0"])
def test_sweep_digests(rtlib, shape, typ):
    golden = json.loads((GOLDEN / "quant_golden.json").read_text())[f"{shape[0]}x{shape[1]}"]
    w = weights(shape)
    assert hashlib.sha256(w.tobytes()).hexdigest() == golden["f32"]
    assert hashlib.sha256(runtime.encode(w, typ).tobytes()).hexdigest() == golden[typ]


def test_oracle_digest_one_shape():
    golden = json.loads((GOLDEN / "quant_golden.json").read_text())["4096x4096"]
    w = weights((4096, 4096))
    assert hashlib.sha256(oracle.quantize(w, "q4_0").tobytes()).hexdigest() == golden["q4_0"]
    assert hashlib.sha256(oracle.quantize(w, "q8_0").tobytes()).hexdigest() == golden["q8_0"]


def test_row_size(rtlib):
    assert runtime.encoded_row_bytes("q4_0", 4096) == 4096 // 32 * 18
    assert runtime.encoded_row_bytes("q8_0", 4096) == 4096 // 32 * 34
    assert runtime.encoded_row_bytes("f16", 10) == 20
    assert runtime.encoded_row_bytes("q4_K", 256) == 144
    assert runtime.encoded_row_bytes("nope", 32) == 0


def test_quantize_errors(rtlib):
    with pytest.raises(runtime.BackendError, match="multiple"):
        runtime.encode(np.zeros((2, 40), np.float32), "q8_0")
    with pytest.raises(runtime.BackendError, match="unknown tensor type"):
        runtime.encode(np.zeros((2, 32), np.float32), "q9_9")
    lib = runtime.load_library()
    x = np.zeros((2, 32), np.float32)
    out = np.zeros(10, np.uint8)
    assert lib.ggml_compiler_quantize(b"q8_0", x.ctypes.data, 2, 32, out.ctypes.data, out.nbytes) == 0
    assert "too small" in lib.ggml_compiler_last_error().decode()


def test_f16_bf16_encoding(rtlib):
    x = np.array([[0.1, -2.5, 65504.0, 1e-8, 70000.0, -0.0, 3.0e-5, 1.0]], np.float32)
    np.testing.assert_array_equal(runtime.encode(x, "f16").view(np.float16), x.astype(np.float16))
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    assert runtime.encode(x, "bf16").tobytes() == quants.quantize(x, T.BF16).tobytes()


def test_activation_quant_rule():
    """The oracle's activation Q8_0 rule (ggml's x86 CPU from_float): d = amax/127 in fp16,
    codes = nearest-even(x * 127/amax), so exact halves round to even."""
    x = np.zeros(32, np.float32)
    x[0] = 127.0
    x[1] = 2.5
    x[2] = -3.5
    x[3] = 0.5
    q, d = oracle.act_q8_0(x)
    assert q[0] == 127 and q[1] == 2 and q[2] == -4 and q[3] == 0
    assert d[0] == np.float16(1.0).view(np.uint16)
