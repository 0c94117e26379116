"""The drop-in, end to end: the reference's own host layer, unmodified (ggml_compiler.runtime.Session,
session.py:160-306; ggml_compiler.llm.Generator, llm.py:473-634; ggml_compiler.llm.bench,
llm.py:637-683), driving this library on the B200 through $GGML_COMPILER_RT, on the GGUF the
reference compiler wrote (tests/golden/ref_llama_q8_0.gguf). Logits and greedy tokens equal the CPU
oracle's bit for bit, through the host loop and through the `generate` entry's device loop."""

import numpy as np
import pytest
from conftest import GOLDEN

from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu
GGUF = GOLDEN / "ref_llama_q8_0.gguf"


@pytest.fixture(scope="module")
def ref_session(gpu, reference_pkg):
    from ggml_compiler.runtime import Session

    s = Session(GGUF, backend="cuda")
    yield s
    s.close()


def test_reference_session_sees_the_program(ref_session):
    assert ref_session.backend_name.startswith("CUDA")
    assert set(ref_session.entries) == {"prefill", "decode", "generate"}
    assert ref_session.symbols == {"max_new": (1, 768), "s": (2, 64), "kv_blocks": (2, 3)}


def test_reference_generator_logits_match_oracle(ref_session, reference_pkg):
    ids = np.load(GOLDEN / "ref_llama_q8_0.npz")["ids"].tolist()
    g = reference_pkg.Generator(ref_session)
    o = OracleGenerator(Program(GGUF))
    g.reset()
    o.reset()
    for chunk in [ids[:20], ids[20:33]] + [[t] for t in ids[33:40]]:
        np.testing.assert_array_equal(g.feed(chunk), o.feed(chunk))


def test_reference_generator_greedy_host_and_device(ref_session, reference_pkg):
    """280 tokens from a 24-token prompt cross the KV window from 512 to 768 rows."""
    prompt = np.load(GOLDEN / "ref_llama_q8_0.npz")["ids"][:24].tolist()
    g = reference_pkg.Generator(ref_session)
    ref, _ = OracleGenerator(Program(GGUF)).generate(prompt, max_new=280)
    host = g.generate(prompt, max_new=280, stop=[])
    assert host == ref
    dev = g.generate(prompt, max_new=280, device=True)  # stops at the model's EOS id (7)
    assert dev == host[:len(dev)] and (len(dev) == 280 or dev[-1] == 7)


def test_reference_bench_runs(ref_session, reference_pkg):
    from ggml_compiler.llm import bench

    r = bench(ref_session, pp=32, tg=8, reps=1, device=True)
    assert r["pp32"] > 0 and r["tg8"] > 0
