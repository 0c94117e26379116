"""The GPU path against the CPU oracle at BASELINE's model configs (bit for bit: logits and greedy
token ids), through this package's decoder over the C ABI.

- config 1 (a 4-layer Llama, d_model 512, 8/8 heads, vocab 32000, Q8_0; the reference compiler's
  program for that shape, tests/test_program.py): a 64-token prompt (seed 1), then 32 greedy tokens
  through the host loop and through the `generate` entry's device loop.
- config 3 (the 8B shape, Q4_0, the benchmark's model): a 12-row prefill (the tensor-core GEMM path);
  then the benchmark's own workload, decode at positions 512.. over n_kv = 768: the GPU prefills the
  512-token prompt, the oracle takes over its KV cache (ggml_compiler_b200_read_value), and both
  decode 4 greedy steps. Prefilling 512 tokens on the CPU would take minutes; the 12-row prefill
  shows that the cache the GPU writes is the oracle's."""

import numpy as np
import pytest
from llm_models import config1_gguf, config1_prompt, llama8b_gguf

from ggml_compiler_b200.llm import Decoder
from ggml_compiler_b200.runtime import Model
from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def config1(gpu, tmp_path_factory):
    path = tmp_path_factory.mktemp("config1") / "config1.gguf"
    config1_gguf(path)
    m = Model(path)
    yield path, m
    m.close()


def test_config1_prompt_and_greedy_match_oracle(config1):
    path, m = config1
    ids = config1_prompt()
    d, o = Decoder(m), OracleGenerator(Program(path))
    d.restart()
    o.reset()
    np.testing.assert_array_equal(d.prompt(ids), o.feed(ids))
    ref, ref_logits = OracleGenerator(Program(path)).generate(ids, max_new=32)
    assert d.greedy(ids, 32, stop=[]) == ref
    dev = d.greedy(ids, 32, on_device=True)
    assert dev == ref[:len(dev)] and (len(dev) == 32 or dev[-1] == 2)


@pytest.fixture(scope="module")
def llama8b(gpu):
    path = llama8b_gguf()
    m = Model(path)
    yield path, m
    m.close()


def test_8b_prefill_matches_oracle(llama8b):
    path, m = llama8b
    ids = np.random.default_rng(5).integers(0, 128256, 12).tolist()
    d, o = Decoder(m), OracleGenerator(Program(path))
    d.restart()
    o.reset()
    np.testing.assert_array_equal(d.prompt(ids), o.feed(ids))


def test_8b_decode_at_768_matches_oracle(llama8b):
    path, m = llama8b
    prompt = np.random.default_rng(1).integers(0, 128256, 512).tolist()  # the benchmark's prompt
    d = Decoder(m)
    d.restart()
    tok = int(np.argmax(d.prompt(prompt)))
    p = Program(path)
    for name in p.prog["state"]:  # the KV cache the GPU wrote, handed to the oracle
        snap = m.read_value(name)
        assert snap.nbytes == p.values[name].nbytes
        p.values[name][:] = snap.view(p.values[name].dtype)
    o = OracleGenerator(p)
    o.n_past = d.ctx
    for _ in range(4):
        a, b = d.step(tok), o.feed([tok])
        np.testing.assert_array_equal(a, b)
        tok = int(np.argmax(a))
    assert d.window(d.ctx) == 768
