"""Batched decode (include/ggml_compiler_b200.h: seq_slots, seq_copy, decode_batch, generate_batch):
several sequences per decode step, each in its own KV-cache slot at its own position, every weight
matrix streamed once per 8 sequences.

The reference decodes one sequence per model (ggml_compiler/llm.py:64), so parity is per sequence:
row i of a batched step equals, bit for bit, the program's `decode` entry run on sequence i alone,
both on the GPU and, for the reference-compiled tiny Llama, in the CPU oracle. Cases cover sequences
at different positions, row counts above the GEMV's 8 (two launches per matrix), a step whose
sequences sit in different 256-key attention windows, windows above 1024 keys (the split-KV kernel
rather than the cluster kernel), Q4_0 and Q8_0 weights, and GQA."""

import numpy as np
import pytest
from conftest import GOLDEN

from ggml_compiler_b200.llm import Decoder, LlamaShape, build_llama_gguf
from ggml_compiler_b200.runtime import BackendError, Model
from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu
GGUF = GOLDEN / "ref_llama_q8_0.gguf"  # 1 layer, d 256, 4 / 2 heads, vocab 128, 768 positions


def prompts(lengths, vocab, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).tolist() for n in lengths]


def single_sequence_logits(m, prompt, tokens):
    """The `decode` entry on one sequence alone: logits after the prompt, then after each token."""
    d = Decoder(m)
    d.restart()
    out = [d.prompt(prompt)]
    for t in tokens:
        out.append(d.step(int(t)))
    return out


def test_tiny_batch_equals_oracle_per_sequence(gpu):
    ps = prompts([5, 17, 40], 128, 3)
    with Model(GGUF) as m:
        first, start = Decoder(m).fill_slots(ps)
        oracles = []
        for p in ps:
            o = OracleGenerator(Program(GGUF))
            o.reset()
            oracles.append((o, o.feed(p)))
        np.testing.assert_array_equal(first, [int(np.argmax(l)) for _, l in oracles])
        np.testing.assert_array_equal(start, [len(p) for p in ps])
        tok, pos = first, start
        for _ in range(5):
            logits, nxt = m.decode_batch(tok, pos)
            for i, (o, _) in enumerate(oracles):
                np.testing.assert_array_equal(logits[i], o.feed([int(tok[i])]))
            np.testing.assert_array_equal(nxt, logits.argmax(axis=1))
            tok, pos = nxt, pos + 1


def test_tiny_batch_of_twelve_across_a_window_edge(gpu):
    """12 rows: each fused GEMV runs as two launches (8 + 4 rows). Two sequences start just below
    position 256, so the step's attention window grows from 256 to 512 keys mid-run."""
    lengths = [3, 9, 254, 20, 33, 64, 255, 7, 100, 2, 41, 18]
    ps = prompts(lengths, 128, 4)
    steps = 4
    with Model(GGUF) as m:
        first, start = Decoder(m).fill_slots(ps)
        toks = [first]
        rows = []
        for _ in range(steps):
            logits, nxt = m.decode_batch(toks[-1], start + len(rows))
            rows.append(logits)
            toks.append(nxt)
        for i, p in enumerate(ps):
            want = single_sequence_logits(m, p, [t[i] for t in toks[:steps]])
            assert int(np.argmax(want[0])) == first[i]
            for s in range(steps):
                np.testing.assert_array_equal(rows[s][i], want[s + 1], err_msg=f"sequence {i}, step {s}")


def test_generate_batch_equals_stepwise_and_oracle(gpu):
    ps = prompts([11, 30, 6, 52, 19], 128, 5)
    steps = 7
    with Model(GGUF) as m:
        d = Decoder(m)
        first, start = d.fill_slots(ps)
        got = m.generate_batch(first, start, steps)
        assert got.shape == (steps, len(ps))
        assert m.device_ms > 0
        # the same steps one at a time from the host (slots refilled: generate_batch moved them on)
        first2, start2 = d.fill_slots(ps)
        np.testing.assert_array_equal(first2, first)
        tok, pos = first2, start2
        for s in range(steps):
            _, tok = m.decode_batch(tok, pos)
            pos = pos + 1
            np.testing.assert_array_equal(tok, got[s])
    for i in (0, 3):
        o = OracleGenerator(Program(GGUF))
        ref, _ = o.generate(ps[i], max_new=steps + 1)
        assert [int(first[i])] + got[:, i].tolist() == ref


def test_seq_copy_round_trip(gpu):
    with Model(GGUF) as m:
        d = Decoder(m)
        d.restart()
        d.prompt([1, 2, 3, 4])
        name = "kv.0"
        before = m.read_value(name)
        m.seq_slots(2)
        m.seq_copy(1, -1)
        d.restart()
        assert not m.read_value(name).any()
        m.seq_copy(-1, 1)
        np.testing.assert_array_equal(m.read_value(name), before)


def test_batch_refusals(gpu):
    with Model(GGUF) as m:
        with pytest.raises(BackendError, match="seq_slots first"):
            m.decode_batch([1], [0])
        with pytest.raises(BackendError, match="1..16"):
            m.seq_slots(17)
        m.seq_slots(2)
        with pytest.raises(BackendError, match="n must be 1..2"):
            m.decode_batch([1, 2, 3], [0, 0, 0])
        with pytest.raises(BackendError, match="outside the KV cache"):
            m.decode_batch([1, 2], [0, 768])
        with pytest.raises(BackendError, match="slot out of range"):
            m.seq_copy(2, -1)
        with pytest.raises(BackendError, match="no entry point"):
            m.decode_batch([1, 2], [0, 1], entry="nope")
        logits, nxt = m.decode_batch([1, 2], [0, 5])  # still usable after the refusals
        assert np.isfinite(logits).all() and nxt.shape == (2,)


@pytest.mark.parametrize("wtype", ["q4_0", "q8_0"])
def test_long_windows_split_kernel(gpu, tmp_path, wtype):
    """Head size 128, 16 query / 8 K/V heads, prompts of 1100-1300 ids: attention windows of 1280
    and 1536 keys over 9 sequences, 1440-1728 chunks of 64 keys in all, so the multi-chunk kernel
    runs with several chunks per CTA (double-buffered K/V) and merges through global partials;
    9 sequences are 8 + 1 rows per GEMV (the tensor-core GEMV and the one-row GEMV)."""
    sh = LlamaShape(layers=2, d_model=2048, heads=16, kv_heads=8, head_dim=128, ffn=2048, vocab=2000,
                    rope_theta=500000.0, max_context=1536, max_prompt=512, weight_type=wtype)
    path = tmp_path / f"long_{wtype}.gguf"
    build_llama_gguf(path, sh, seed=7)
    ps = prompts([1100, 1279, 1150, 1300, 1190, 1210, 1101, 1250, 1277], sh.vocab, 6)
    steps = 3
    with Model(path) as m:
        first, start = Decoder(m).fill_slots(ps)
        toks, rows = [first], []
        for s in range(steps):
            logits, nxt = m.decode_batch(toks[-1], start + s)
            rows.append(logits)
            toks.append(nxt)
        for i in (0, 1, 3, 8):
            want = single_sequence_logits(m, ps[i], [t[i] for t in toks[:steps]])
            for s in range(steps):
                np.testing.assert_array_equal(rows[s][i], want[s + 1], err_msg=f"sequence {i}, step {s}")
    o = OracleGenerator(Program(path))
    o.reset()
    o.feed(ps[1])
    np.testing.assert_array_equal(rows[0][1], o.feed([int(toks[0][1])]))
