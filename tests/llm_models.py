"""Causal-LM models the parity tests share (test infrastructure).

BASELINE config 1 (a 4-layer Llama, d_model 512, 8/8 heads, FFN 1408, vocab 32000, N(0, 0.02) weights
from seed 0, Q8_0 projections and output head): the transformers model is made as the reference's
golden generator makes it (tests/golden/make_llm_golden.py), and its GGUF is written by this
repository's writer, whose program tests/test_program.py pins to the one the reference compiler
wrote for this shape (tests/golden/ref_program_config1.json)."""

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def config1() -> dict:
    return json.loads((GOLDEN / "ref_program_config1.json").read_text())


def config1_shape():
    from ggml_compiler_b200.llm import LlamaShape

    c = config1()["config"]
    return LlamaShape(layers=c["num_hidden_layers"], d_model=c["hidden_size"], heads=c["num_attention_heads"],
                      kv_heads=c["num_key_value_heads"], ffn=c["intermediate_size"], vocab=c["vocab_size"],
                      rope_theta=c["rope_theta"], eps=c["rms_norm_eps"], max_context=c["max_context"],
                      max_prompt=c["max_prompt"], eos=[c["eos_token_id"]], weight_type=c["weights"])


def config1_model():
    import torch
    import transformers

    c = {k: v for k, v in config1()["config"].items() if k not in ("max_context", "max_prompt", "weights")}
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(transformers.LlamaConfig(**c)).float().eval()
    model.config._attn_implementation = "eager"
    return model


def config1_gguf(path: Path):
    """Writes config 1's GGUF to `path`; returns the transformers model it was made from."""
    from ggml_compiler_b200.llm import build_llama_gguf

    model = config1_model()
    weights = {k: v.detach().numpy() for k, v in model.state_dict().items()}
    build_llama_gguf(path, config1_shape(), weights=weights)
    return model


def config1_prompt() -> list[int]:
    """64 ids uniform in [0, 32000) from seed 1."""
    return np.random.default_rng(1).integers(0, 32000, 64).tolist()


def llama8b_gguf() -> Path:
    """BASELINE config 3's model: the 8B-shape Q4_0 GGUF the benchmark writes (same cache file, same
    bytes: seeded weights, bit-exact encoder)."""
    import os

    from ggml_compiler_b200.llm import LLAMA3_8B, build_llama_gguf

    cache = Path(os.environ.get("GCB_BENCH_CACHE", "/tmp/gcb_bench"))
    cache.mkdir(parents=True, exist_ok=True)
    p = cache / "8b_q4_0_seed0.gguf"
    if not p.exists():
        tmp = p.with_suffix(f".part{os.getpid()}")
        build_llama_gguf(tmp, LLAMA3_8B, seed=0)
        tmp.rename(p)
    return p
