"""Prefill attention on the tensor cores (GGML_COMPILER_B200_PREFILL_ATTN=tc,
kernels/gc_flash_prefill_tc.cu): mma.sync f16 products with f32 accumulation in the tensor core's
own order and f16 probabilities, so it is compared with the CPU oracle within tolerance, not bit
for bit (the default prefill kernel is the bit-exact one):
- the flash_attn node alone at the prefill shapes (GQA 1-8, head sizes 64 and 128, causal masks
  with -65504 and -inf, a finite random mask, no mask, ragged chunks): max-abs error against the
  oracle below 5e-3 of max(1, max|out|);
- a whole prefill of the reference-compiled tiny Llama: logits within the north star's 1e-2 max-abs
  and greedy token equal to the oracle's, and the default kernel still bit-exact in the same process."""

import numpy as np
import pytest
from conftest import GOLDEN

from ggml_compiler_b200.gguf_write import write_gguf
from ggml_compiler_b200.llm import Decoder
from ggml_compiler_b200.programs import single_node_program
from ggml_compiler_b200.runtime import Model
from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu


def flash_case(tmp_path, D, H, HKV, NQ, NKV, mask):
    rng = np.random.default_rng(D + H + NQ)
    q = rng.standard_normal((1, H, NQ, D), dtype=np.float32)
    k = (rng.standard_normal((1, HKV, NKV, D), dtype=np.float32) * 0.5).astype(np.float16)
    v = rng.standard_normal((1, HKV, NKV, D), dtype=np.float32).astype(np.float16)
    ins = [("q", "f32", [D, NQ, H, 1], [1, H, NQ, D]), ("k", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D]),
           ("v", "f16", [D, NKV, HKV, 1], [1, HKV, NKV, D])]
    feed = {"q": q, "k": k, "v": v}
    if mask != "none":
        m = np.zeros((NQ, NKV), np.float32)
        if mask == "random":
            m = rng.standard_normal((NQ, NKV), dtype=np.float32) * 2
        else:
            hide = np.float32(-65504.0) if mask == "causal" else np.float32(-np.inf)
            for i in range(NQ):
                m[i, NKV - NQ + i + 1:] = hide
        ins.append(("mask", "f16", [NKV, NQ, 1, 1], [1, 1, NQ, NKV]))
        feed["mask"] = m.astype(np.float16)[None, None]
    prog = single_node_program("flash_attn", ins, [n for n, *_ in ins], "f32", [D, H, NQ, 1], [1, NQ, H, D],
                               {"scale": float(1.0 / np.sqrt(D))})
    path = tmp_path / f"fa_{D}_{H}_{HKV}_{NQ}_{NKV}_{mask}.gguf"
    write_gguf(path, prog, [])
    return path, feed


@pytest.mark.parametrize("D,H,HKV,NQ,NKV,mask", [
    (128, 32, 8, 300, 700, "causal"),
    (128, 8, 8, 16, 130, "none"),
    (64, 16, 2, 40, 260, "inf"),
    (64, 4, 4, 70, 64, "random"),
    (128, 32, 8, 1024, 1024, "causal"),
])
def test_flash_prefill_tc_within_tolerance(gpu, tmp_path, monkeypatch, D, H, HKV, NQ, NKV, mask):
    path, feed = flash_case(tmp_path, D, H, HKV, NQ, NKV, mask)
    monkeypatch.setenv("GGML_COMPILER_B200_PREFILL_ATTN", "tc")
    with Model(path) as m:
        got = m.entries["main"](**feed)["out.0"]
    want = Program(path).run("main", **feed)["out.0"]
    assert np.isfinite(got).all()
    err = float(np.max(np.abs(got.astype(np.float64) - want)))
    assert err <= 5e-3 * max(1.0, float(np.max(np.abs(want)))), err


def test_prefill_logits_within_north_star_tolerance(gpu, monkeypatch):
    gguf = GOLDEN / "ref_llama_q8_0.gguf"
    prompt = np.random.default_rng(8).integers(0, 128, 60).tolist()
    o = OracleGenerator(Program(gguf))
    o.reset()
    want = o.feed(prompt)
    monkeypatch.setenv("GGML_COMPILER_B200_PREFILL_ATTN", "tc")
    with Model(gguf) as m:
        d = Decoder(m)
        d.restart()
        got = d.prompt(prompt)
    assert float(np.max(np.abs(got.astype(np.float64) - want))) <= 1e-2
    assert int(np.argmax(got)) == int(np.argmax(want))
    monkeypatch.delenv("GGML_COMPILER_B200_PREFILL_ATTN")
    with Model(gguf) as m:  # a model loaded without the switch stays on the bit-exact kernel
        d = Decoder(m)
        d.restart()
        np.testing.assert_array_equal(d.prompt(prompt), want)
