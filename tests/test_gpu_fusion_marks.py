"""Emitter fusion marks on the B200 (csrc/gc_fuse.cpp): a program whose nodes carry `"fuse"` marks
(ggml_compiler_b200/fusion.py) runs the marked groups as fused kernels and nothing else; the same
program without marks is matched by the backend into the same launches; a group whose mark is
dropped runs as separate ops. The logits are the same bits in all three (the fused and separate
kernels share the arithmetic and its order)."""

import numpy as np
import pytest

import ggml_compiler_b200.llm as llm
from ggml_compiler_b200.fusion import mark_fusion_groups
from ggml_compiler_b200.llm import Decoder, LlamaShape, build_llama_gguf
from ggml_compiler_b200.runtime import Model

pytestmark = pytest.mark.gpu
SHAPE = LlamaShape(layers=2, d_model=256, heads=4, kv_heads=2, ffn=512, vocab=128, max_context=768,
                   max_prompt=64, weight_type="q4_0")


def decode_step(path):
    with Model(path) as m:
        d = Decoder(m)
        d.restart()
        d.prompt([1, 2, 3, 4, 5])
        m.profile(True)
        try:
            logits = d.step(6)
            ks = m.kernel_table()
        finally:
            m.profile(False)
    return logits, {k: v["launches"] for k, v in ks.items()}


def test_marked_unmarked_and_dropped_groups(gpu, tmp_path, monkeypatch):
    marked, plain, dropped = (tmp_path / f"{n}.gguf" for n in ("marked", "plain", "dropped"))
    build_llama_gguf(marked, SHAPE, seed=3)
    build_llama_gguf(plain, SHAPE, seed=3, fusion_marks=False)

    def drop_glu1(program, wt=None, in_place=False):
        out = mark_fusion_groups(program, wt, in_place)
        for s in out["stages"]:
            for n in s["nodes"]:
                if n.get("fuse") == "glu.1":
                    del n["fuse"]
        return out

    monkeypatch.setattr(llm, "mark_fusion_groups", drop_glu1)
    build_llama_gguf(dropped, SHAPE, seed=3)

    la, ka = decode_step(marked)
    lb, kb = decode_step(plain)
    lc, kc = decode_step(dropped)
    assert ka == kb
    assert ka["gemv_q4_0_qkv"] == ka["gemv_q4_0_glu"] == 2 and ka["gemv_q4_0_res"] == 4 and ka["gemv_q4_0_head"] == 1
    assert "swiglu" not in ka and "mul_mat" not in ka
    # layer 1's gate/up group runs as norm, multiply, two one-matrix GEMVs and SwiGLU
    assert kc["gemv_q4_0_glu"] == 1 and kc["swiglu"] == 1 and kc["gemv_q4_0"] == 2 and kc["rms_norm"] == 1
    assert "gemv_q4_0" not in ka
    np.testing.assert_array_equal(la, lb)
    np.testing.assert_array_equal(la, lc)
