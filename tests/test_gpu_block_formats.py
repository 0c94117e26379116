"""The other GGUF block formats on the B200 against the CPU oracle, bit for bit (the reference stores
weights in them, ggml_compiler/quant/types.py:6-19):

- mul_mat for every format at one, a few, 8, 9 and many activation rows, with GQA-style broadcast:
  q5_0 / iq4_nl through the Q8_0 kernels they are expanded for at load (fused GEMV, tensor-core
  GEMV and GEMM), q4_1 / q5_1 / q4_K / q5_K / q6_K through the block kernel in their GGUF layout;
- get_rows (an embedding table stored in each format) against the oracle's decoding;
- a whole decoder with q5_0 weights (the fused decode path) and one with q4_K projections, a q6_K
  output head and a q4_1 embedding table (the block kernel and get_rows inside a real step).
Blocks the library cannot encode (iq4_nl, K-quants) are seeded random bytes with finite scales."""

import numpy as np
import pytest

import oracle
from ggml_compiler_b200 import runtime
from ggml_compiler_b200.gguf_write import TensorEntry, write_gguf
from ggml_compiler_b200.llm import Decoder, LlamaShape, build_llama_gguf
from ggml_compiler_b200.programs import random_block_rows, single_node_program, write_mul_mat
from ggml_compiler_b200.runtime import Model
from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu
ENCODED = ("q4_1", "q5_0", "q5_1")
RAW_ONLY = ("iq4_nl", "q4_k", "q5_k", "q6_k")


def random_blocks(typ, rows, K, seed, scale=1e-3):
    return random_block_rows(typ, rows, K, seed, scale)


def weight_rows(typ, N, K, seed):
    if typ in ENCODED:
        w = np.random.default_rng(seed).standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
        return runtime.encode(w, typ)
    return random_blocks(typ, N, K, seed)


def run_mm(tmp_path, raw, typ, x, batch=1):
    p = tmp_path / f"mm_{typ}_{raw.shape[0]}_{x.shape[-2]}_{batch}.gguf"
    write_mul_mat(p, raw, typ, x.shape[-2], batch)
    with Model(p) as m:
        return m.entries["main"](x=x.reshape(batch, x.shape[-2], -1))["out.0"].reshape(batch, x.shape[-2], raw.shape[0])


CASES = [(256, 1024, 1), (300, 4096, 3), (64, 2048, 8), (100, 1024, 9), (128, 512, 33), (1000, 4096, 1),
         (14336, 4096, 1), (4096, 14336, 8)]  # the last two: BASELINE config 2's FFN shapes


@pytest.mark.parametrize("typ", ENCODED + RAW_ONLY)
@pytest.mark.parametrize("N,K,M", CASES)
def test_mul_mat_bit_exact(gpu, tmp_path, typ, N, K, M):
    raw = weight_rows(typ, N, K, seed=N + K)
    x = np.random.default_rng(M).standard_normal((M, K), dtype=np.float32)
    got = run_mm(tmp_path, raw, typ, x)[0]
    np.testing.assert_array_equal(got, oracle.mul_mat(raw, typ, K, x))


@pytest.mark.parametrize("typ", ["q4_1", "q4_k", "q6_k"])
def test_mul_mat_batched_and_edges(gpu, tmp_path, typ):
    """A batch of 3 activation matrices against one weight; an all-zero activation row (Q8_K scale 0)
    and rows with a huge and a tiny value."""
    K = 512
    raw = weight_rows(typ, 72, K, seed=9)
    x = np.random.default_rng(10).standard_normal((3, 4, K), dtype=np.float32)
    x[1, 2] = 0.0
    x[2, 0, :3] = [1e4, -1e-30, 3.0]
    got = run_mm(tmp_path, raw, typ, x, batch=3)
    for b in range(3):
        np.testing.assert_array_equal(got[b], oracle.mul_mat(raw, typ, K, x[b]))


@pytest.mark.parametrize("typ", ENCODED + RAW_ONLY)
def test_get_rows_bit_exact(gpu, tmp_path, typ):
    V, d = 50, 512
    raw = weight_rows(typ, V, d, seed=11)
    idx = np.array([0, 7, 49, 7, 23], np.int32)
    prog = single_node_program("get_rows", [("ids", "i32", [5, 1, 1, 1], [5])], ["w.0", "ids"], "f32",
                               [d, 5, 1, 1], [5, d])
    p = tmp_path / f"rows_{typ}.gguf"
    write_gguf(p, prog, [TensorEntry("w.0", typ, (d, V), raw)])
    with Model(p) as m:
        got = m.entries["main"](ids=idx)["out.0"].reshape(5, d)
    want = oracle.dequantize(raw[idx], typ, d)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def block_encoder(w, typ):
    """Encodes what the library can; seeded random blocks (scaled near N(0, 0.02) weights) otherwise."""
    if typ in ENCODED or typ in ("q4_0", "q8_0"):
        return runtime.encode(w, typ)
    return random_block_rows(typ, w.shape[0], w.shape[1], seed=w.shape[0] * 7 + w.shape[1])


def decode_vs_oracle(path, prompt, steps):
    with Model(path) as m:
        d = Decoder(m)
        d.restart()
        o = OracleGenerator(Program(path))
        o.reset()
        np.testing.assert_array_equal(d.prompt(prompt), o.feed(prompt))
        tok = 3
        for _ in range(steps):
            a, b = d.step(tok), o.feed([tok])
            np.testing.assert_array_equal(a, b)
            tok = int(np.argmax(a))


def test_decoder_q5_0_fused(gpu, tmp_path):
    sh = LlamaShape(layers=2, d_model=256, heads=4, kv_heads=2, ffn=512, vocab=128, max_context=768,
                    max_prompt=64, weight_type="q5_0")
    path = tmp_path / "q5_0.gguf"
    build_llama_gguf(path, sh, seed=12, encoder=block_encoder)
    decode_vs_oracle(path, [1, 5, 9, 33, 2, 7], 4)
    with Model(path) as m:  # the expanded weights run the fused decode kernels
        d = Decoder(m)
        d.restart()
        d.prompt([1, 2, 3])
        m.profile(True)
        d.step(4)
        ks = m.kernel_table()
        m.profile(False)
    assert ks["gemv_q8_0_qkv"]["launches"] == 2 and "mul_mat" not in ks


def test_decoder_k_quants(gpu, tmp_path, monkeypatch):
    """q4_K projections, a q6_K output head (its own matmul after the final norm) and a q4_1
    embedding table."""
    import ggml_compiler_b200.llm as llm

    sh = LlamaShape(layers=2, d_model=512, heads=4, kv_heads=2, ffn=768, vocab=256, max_context=768,
                    max_prompt=64, weight_type="q4_k", embed_type="q4_1")
    path = tmp_path / "k.gguf"
    orig = llm.llama_weights

    def weights_with_q6_k_head(s):
        out = orig(s)
        name, hf, shape, _ = out[-1]
        return out[:-1] + [(name, hf, shape, "q6_k")]

    monkeypatch.setattr(llm, "llama_weights", weights_with_q6_k_head)
    build_llama_gguf(path, sh, seed=13, encoder=block_encoder)
    decode_vs_oracle(path, [1, 5, 9, 33, 2, 7, 100, 200], 4)
