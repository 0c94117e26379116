"""Tensor parallelism (Model.join_tensor_parallel, ggml_compiler_b200_tp_init/_tp_connect) on 2, 4 and
8 GPUs, each rank its own process (tests/tp_worker.py), against the CPU oracle on the same GGUF.

Sharding keeps every row's arithmetic: each GEMV row and each attention head is computed by one
rank exactly as one GPU computes it, and the exchanges only move bytes. So the bar is bit-exact:
every rank's logits after each chunk equal the oracle's, and greedy tokens (host loop and the
`generate` entry's device loop) equal the oracle's. The chunks cover prefill rows that are not split
(16 and 14 tokens: tensor-core GEMM path), a 5-row chunk (split GEMVs over several activation rows)
and single-token decode steps across the first KV block.

Models: the reference-compiled tiny Llama (Q8_0; 4 query heads, 2 K/V heads: split by heads at 2
ranks, attention replicated at 4 and 8) and a synthetic 2-layer Q4_0 Llama with 8 query and 8 K/V
heads (split by heads at every size). Skipped where fewer GPUs are visible."""

import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
from conftest import GOLDEN, REPO

from oracle.interp import OracleGenerator, Program

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    import torch

    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def synthetic_q4(tmp_path_factory):
    from ggml_compiler_b200.llm import LlamaShape, build_llama_gguf

    p = tmp_path_factory.mktemp("tp") / "llama_q4_0_h8.gguf"
    build_llama_gguf(p, LlamaShape(layers=2, d_model=512, heads=8, kv_heads=8, ffn=1408, vocab=4096, max_context=768,
                                   max_prompt=32, eos=[], weight_type="q4_0"), seed=0)
    return p


def _case(vocab: int) -> dict:
    ids = np.random.default_rng(5).integers(0, vocab, 40).tolist()
    return {"chunks": [ids[:16], ids[16:30], ids[30:35]] + [[t] for t in ids[35:40]], "prompt": ids[:12], "max_new": 12}


def _oracle(path, case: dict) -> dict:
    o = OracleGenerator(Program(path))
    o.reset()
    logits = []
    for c in case["chunks"]:
        x = np.asarray(o.feed(c), np.float32)
        logits.append(x if x.ndim == 1 else x[-1])
    return {"logits": np.stack(logits), "tokens": np.array(o.generate(case["prompt"], case["max_new"])[0])}


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("model", ["golden_q8_0", "synthetic_q4_0"])
def test_tensor_parallel_matches_oracle(gpu, tmp_path, synthetic_q4, model, world):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs, {_gpus()} visible")
    path = GOLDEN / "ref_llama_q8_0.gguf" if model == "golden_q8_0" else synthetic_q4
    vocab = 128 if model == "golden_q8_0" else 4096
    case = _case(vocab)
    (tmp_path / "case.json").write_text(json.dumps(case))
    port = _free_port()
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "GGML_COMPILER_B200_TP_TIMEOUT_MS": "20000"}
    procs = [subprocess.Popen([sys.executable, str(REPO / "tests" / "tp_worker.py"), str(path), str(tmp_path), str(r),
                               str(world), str(port), str(tmp_path / "case.json")], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True) for r in range(world)]
    logs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=600)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        logs.append(out)
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{logs[r][-3000:]}"
    want = _oracle(path, case)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npz")
        np.testing.assert_array_equal(got["logits"], want["logits"], err_msg=f"rank {r}")
        np.testing.assert_array_equal(got["tokens"], want["tokens"], err_msg=f"rank {r}")
        np.testing.assert_array_equal(got["device_tokens"], want["tokens"], err_msg=f"rank {r}")


def test_absent_peer_times_out(gpu, tmp_path):
    """Failure detection without a GPU fault: rank 1 stays alive with its window mapped but never
    runs the decode step, so rank 0's first exchange waits for a flag that nothing sets. The wait
    gives up after 2 s (GGML_COMPILER_B200_TP_TIMEOUT_MS), the kernel returns, and the run reports
    the timeout through the C ABI's error string; no GPU is left waiting."""
    if _gpus() < 2:
        pytest.skip(f"needs 2 GPUs, {_gpus()} visible")
    port = _free_port()
    env = {**os.environ, "NCCL_NVLS_ENABLE": "0", "GGML_COMPILER_B200_TP_TIMEOUT_MS": "2000"}
    procs = [subprocess.Popen([sys.executable, str(REPO / "tests" / "tp_worker.py"), str(GOLDEN / "ref_llama_q8_0.gguf"),
                               str(tmp_path), str(r), "2", str(port), "absent-peer"], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    logs = [p.communicate(timeout=600)[0] for p in procs]
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{logs[r][-3000:]}"
    msg = (tmp_path / "rank0.txt").read_text()
    assert "tensor-parallel exchange timed out" in msg, msg
