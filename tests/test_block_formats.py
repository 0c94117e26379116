"""The other GGUF block formats the reference stores weights in (ggml_compiler/quant/types.py:6-19:
q4_1, q5_0, q5_1, iq4_nl, q4_k, q5_k, q6_k), host side, no GPU:

- the library's encoder (ggml_compiler_quantize) and the CPU oracle's are byte-exact with gguf-py
  0.19 for q4_1 / q5_0 / q5_1 (edge-case rows and the digest of a 4096 x 4096 matrix); gguf-py has no
  encoder for iq4_nl or the K-quants, and neither has this library (it computes with them);
- the oracle's decoding of every format equals gguf-py's bit for bit on seeded random blocks;
- the oracle's activation quantizers follow ggml's rules (Q8_1: the Q8_0 codes plus s = d * sum;
  Q8_K: iscale = -127 / max, codes capped at 127, sums of 16);
- the oracle's matmul for each format equals the f64 dot of the decoded weight with the decoded
  activation up to f32 rounding (the layout, the signs and the per-unit terms are right).
Golden vectors: tests/golden/block_formats.npz, made by tests/golden/make_block_golden.py."""

import hashlib

import numpy as np
import pytest
from conftest import GOLDEN

import oracle
from ggml_compiler_b200 import runtime

G = np.load(GOLDEN / "block_formats.npz")
ENCODED = ["q4_1", "q5_0", "q5_1"]
ALL = ENCODED + ["iq4_nl", "q4_k", "q5_k", "q6_k"]


@pytest.mark.parametrize("typ", ENCODED)
def test_encoders_match_gguf_py(rtlib, typ):
    x = G["x"]
    assert runtime.encode(x, typ).tobytes() == G[typ].tobytes()
    assert oracle.quantize(x, typ).tobytes() == G[typ].tobytes()
    np.testing.assert_array_equal(oracle.dequantize(G[typ], typ, x.shape[-1]), G[f"{typ}_dec"].reshape(x.shape))


@pytest.mark.parametrize("typ", ENCODED)
def test_encoder_digest_4096(rtlib, typ):
    w = np.random.default_rng(0).standard_normal((4096, 4096), dtype=np.float32) * np.float32(0.02)
    assert hashlib.sha256(runtime.encode(w, typ).tobytes()).hexdigest() == str(G[f"sha_{typ}_4096x4096"])


@pytest.mark.parametrize("typ", ["iq4_nl", "q4_K", "q5_K", "q6_K"])
def test_library_refuses_encoders_it_lacks(rtlib, typ):
    with pytest.raises(runtime.BackendError, match="computes with iq4_nl and the K-quants"):
        runtime.encode(np.zeros((1, 256), np.float32), typ)


@pytest.mark.parametrize("typ", ALL)
def test_oracle_decoding_matches_gguf_py(typ):
    raw, dec = G[f"raw_{typ}"], G[f"dec_{typ}"]
    got = oracle.dequantize(raw, typ, dec.shape[-1])
    np.testing.assert_array_equal(got.view(np.uint32), dec.view(np.uint32))


def test_row_sizes(rtlib):
    for typ, (blk, size) in {"q4_1": (32, 20), "q5_0": (32, 22), "q5_1": (32, 24), "iq4_nl": (32, 18),
                             "q4_k": (256, 144), "q5_k": (256, 176), "q6_k": (256, 210)}.items():
        assert oracle.lib().orc_row_size(oracle.TYPES[typ], 1024) == 1024 // blk * size
        assert runtime.encoded_row_bytes(typ.replace("_k", "_K"), 1024) == 1024 // blk * size


def q8_k_reference(x):
    """ggml quantize_row_q8_K_ref, in numpy (one super-block at a time)."""
    q = np.zeros(x.size, np.int8)
    d = np.zeros(x.size // 256, np.float32)
    bs = np.zeros(x.size // 16, np.int16)
    for b in range(x.size // 256):
        xb = x[b * 256:(b + 1) * 256]
        i = int(np.argmax(np.abs(xb)))  # first maximum
        mx = xb[i]
        if mx == 0:
            continue
        iscale = np.float32(-127.0) / mx
        v = np.minimum(np.rint(iscale * xb), 127).astype(np.int8)
        q[b * 256:(b + 1) * 256] = v
        bs[b * 16:(b + 1) * 16] = v.reshape(16, 16).astype(np.int32).sum(axis=1)
        d[b] = np.float32(1.0) / iscale
    return q, d, bs


def test_activation_quantizers():
    rng = np.random.default_rng(5)
    x = rng.standard_normal(1024).astype(np.float32)
    x[256:512] = 0.0  # an all-zero super-block
    x[600] = -x[512:768].__abs__().max() * 3  # a negative maximum
    x[800], x[801] = 5.0, -5.0  # a tie: the first one wins
    q, d, bs = oracle.act_q8_k(x)
    rq, rd, rbs = q8_k_reference(x)
    np.testing.assert_array_equal(q, rq)
    np.testing.assert_array_equal(d.view(np.uint32), rd.view(np.uint32))
    np.testing.assert_array_equal(bs, rbs)
    q1, d1, s1 = oracle.act_q8_1(x)
    q0, d0 = oracle.act_q8_0(x)
    np.testing.assert_array_equal(q1, q0)
    np.testing.assert_array_equal(d1, d0)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1)
    want = ((amax / np.float32(127)) * q0.reshape(-1, 32).astype(np.int32).sum(axis=1).astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(s1, want.view(np.uint16))


def decoded_activation(x, typ):
    if typ in ("q4_k", "q5_k", "q6_k"):
        q, d, _ = oracle.act_q8_k(x)
        return q.reshape(-1, 256).astype(np.float64) * d.astype(np.float64)[:, None]
    q, d = oracle.act_q8_0(x)
    return q.reshape(-1, 32).astype(np.float64) * d.view(np.float16).astype(np.float64)[:, None]


@pytest.mark.parametrize("typ", ALL)
def test_oracle_matmul_is_the_decoded_dot(typ):
    raw, dec = G[f"raw_{typ}"], G[f"dec_{typ}"]
    K = dec.shape[-1]
    x = np.random.default_rng(6).standard_normal((3, K)).astype(np.float32)
    y = oracle.mul_mat(raw, typ, K, x)
    for m in range(3):
        xd = decoded_activation(x[m], typ).reshape(-1)
        want = dec.astype(np.float64) @ xd
        scale = np.abs(dec.astype(np.float64)) @ np.abs(xd)
        assert np.all(np.abs(y[m] - want) <= 1e-5 * scale + 1e-30), typ


def test_oracle_expanded_formats_are_q8_0_matmuls():
    """q5_0 / iq4_nl multiply as Q8_0 rows with the same scale and the expanded codes."""
    for typ in ("q5_0", "iq4_nl"):
        raw, dec = G[f"raw_{typ}"], G[f"dec_{typ}"]
        K = dec.shape[-1]
        n = K // 32
        blocks = raw.reshape(raw.shape[0], n, -1)
        d = blocks[:, :, :2].copy().view(np.float16).astype(np.float32)
        codes = np.rint(dec.reshape(raw.shape[0], n, 32) / np.where(d == 0, 1, d)).astype(np.int8)
        q8 = np.concatenate([blocks[:, :, :2], codes.view(np.uint8)], axis=-1).reshape(raw.shape[0], -1)
        ok = (d != 0).all()
        x = np.random.default_rng(7).standard_normal((9, K)).astype(np.float32)
        if ok:
            np.testing.assert_array_equal(oracle.mul_mat(raw, typ, K, x), oracle.mul_mat(q8, "q8_0", K, x))


@pytest.mark.parametrize("typ", ["q4_k", "q6_k", "q4_1"])
def test_oracle_model_close_to_its_decoded_weights(tmp_path, typ):
    """A whole decoder in `typ` on the oracle against the same decoder with every block decoded to
    f32 (the oracle's decoding, pinned to gguf-py above): they differ only by the activation
    quantization ggml applies for the format (Q8_K / Q8_1), so the logits agree to a few percent of
    their range and the greedy token is the same."""
    import gguf

    from ggml_compiler_b200.llm import LlamaShape, build_llama_gguf, llama_weights
    from ggml_compiler_b200.programs import random_block_rows
    from oracle.interp import OracleGenerator, Program

    sh = LlamaShape(layers=2, d_model=256, heads=4, kv_heads=2, ffn=512, vocab=128, max_context=768,
                    max_prompt=64, weight_type=typ)

    def enc(w, t):
        if t in ENCODED:
            return runtime.encode(w, t)
        return random_block_rows(t, w.shape[0], w.shape[1], seed=w.shape[0] * 7 + w.shape[1])

    qpath = tmp_path / f"{typ}.gguf"
    build_llama_gguf(qpath, sh, seed=21, encoder=enc)
    hf_of = {g: hf for g, hf, _, _ in llama_weights(sh)}
    full = {}
    for t in gguf.GGUFReader(str(qpath)).tensors:
        shape = tuple(int(x) for x in reversed(t.shape))  # [rows, row length]
        data = np.asarray(t.data)
        if t.tensor_type.name.lower() == typ:
            full[hf_of[t.name]] = oracle.dequantize(data.reshape(shape[0], -1), typ, shape[-1]).reshape(shape)
        else:
            full[hf_of[t.name]] = np.asarray(data, np.float32).reshape(shape)
    fpath = tmp_path / "f32.gguf"
    build_llama_gguf(fpath, LlamaShape(**{**sh.__dict__, "weight_type": "f32"}), weights=full)
    prompt = [1, 7, 33, 90, 4, 12]
    a, b = OracleGenerator(Program(qpath)), OracleGenerator(Program(fpath))
    a.reset()
    b.reset()
    la, lb = a.feed(prompt), b.feed(prompt)
    rng = float(np.max(np.abs(lb)))
    # measured: 1.1 % (q4_k), 2.2 % (q6_k), 1.1 % (q4_1) of the logits' range
    assert float(np.max(np.abs(la - lb))) <= 0.04 * rng, (float(np.max(np.abs(la - lb))), rng)
    assert int(np.argmax(la)) == int(np.argmax(lb))


@pytest.mark.parametrize("typ", ENCODED)
def test_encoder_refusals(rtlib, typ):
    with pytest.raises(runtime.BackendError, match="multiple of"):
        runtime.encode(np.zeros((2, 48), np.float32), typ)  # 48 values: not whole 32-blocks
    # a row of one block at each edge of the code range round-trips through the oracle's decoding
    x = np.array([np.linspace(-1, 1, 32, dtype=np.float32)])
    raw = runtime.encode(x, typ)
    assert raw.shape == (1, oracle.lib().orc_row_size(oracle.TYPES[typ], 32))
    dec = oracle.dequantize(raw, typ, 32)
    assert np.max(np.abs(dec - x)) <= 2.0 / (15 if typ == "q4_1" else 31) + 1e-3
