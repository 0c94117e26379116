"""Generate the causal-LM golden fixtures from the reference itself (run in a container that has the
reference checkout; the GPU tests only read the files this writes).

1. ref_llama_q8_0.gguf: a random-init LlamaForCausalLM (GQA: 4 query heads, 2 K/V heads, head
   size 64) compiled by the reference compiler (`ggml_compiler.compile(causal_lm(model), opt="O3")`,
   ggml_compiler/llm.py:361-444, compiler.py:171-297) with Q8_0 projections and output head, as
   BASELINE config 1 asks (norms and embeddings f32). The reference encodes the weights through
   $GGML_COMPILER_RT's ggml_compiler_quantize, i.e. this repository's library, whose encoding is
   pinned to gguf-py by tests/test_quant.py.
2. ref_llama_q8_0.npz: transformers' fp32 logits for a seeded prompt with the weights replaced by
   their Q8_0 decodings (gguf-py dequantize, as the reference's own tests decode,
   tests/unit/test_frontend.py:303), plus transformers' greedy continuation: the reference's
   per-model oracle (tests/unit/test_llm.py:81-145).
3. ref_program_gqa2.json: the program the reference writes for a 2-layer GQA Llama (config in the
   file), to pin this repository's Llama program emitter node for node.
4. ref_program_config1.json: the same for BASELINE config 1's shape (4 layers, d_model 512, 8/8
   heads, FFN 1408, vocab 32000, Q8_0 projections and head). The GGUF itself (f32 embeddings,
   65 MB) is not kept: the tests rebuild it from the same seeded transformers model with this
   repository's writer, whose program this file pins.

    GGML_COMPILER_RT=ggml-compiler_b200/ggml_compiler_b200/lib/libggml_compiler_rt.so \
        python tests/golden/make_llm_golden.py REFERENCE_CHECKOUT
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


# tiny Llama-architecture decoder (the EOS id is transformers' Llama default)
CONFIG1 = dict(vocab_size=32000, hidden_size=512, intermediate_size=1408, num_hidden_layers=4, num_attention_heads=8,
               num_key_value_heads=8, eos_token_id=2, rope_theta=10000.0, rms_norm_eps=1e-5)


def _program(gguf_path: str) -> tuple[dict, dict]:
    import gguf

    r = gguf.GGUFReader(gguf_path)

    def field(k):
        f = r.fields[k]
        return json.loads(bytes(f.parts[f.data[0]]).decode())

    return field("ggml_compiler.program"), field("ggml_compiler.meta")


def main(ref_root: str) -> None:
    os.environ.setdefault("GGML_COMPILER_RT", str(REPO / "ggml-compiler_b200/ggml_compiler_b200/lib/libggml_compiler_rt.so"))
    sys.path.insert(0, ref_root)
    import gguf
    import torch
    import transformers

    import ggml_compiler
    from ggml_compiler.quant import DTypePolicy

    tmp = Path(tempfile.mkdtemp())
    try:
        # 1 + 2: the Q8_0 model
        cfg = dict(vocab_size=128, hidden_size=256, intermediate_size=256, num_hidden_layers=1, num_attention_heads=4,
                   num_key_value_heads=2, eos_token_id=7, rope_theta=10000.0, rms_norm_eps=1e-5)
        torch.manual_seed(0)
        model = transformers.LlamaForCausalLM(transformers.LlamaConfig(**cfg)).float().eval()
        model.config._attn_implementation = "eager"
        policy = DTypePolicy(rules=[("*_proj.weight", "q8_0"), ("lm_head.weight", "q8_0")], float="f32", fallback=[])
        art = ggml_compiler.compile(ggml_compiler.causal_lm(model, max_context=768, max_prompt=64), opt="O3",
                                    out_dir=tmp / "q8", dtype_policy=policy)
        shutil.copy(art.gguf, HERE / "ref_llama_q8_0.gguf")
        reader = gguf.GGUFReader(art.gguf)
        f = reader.fields["ggml_compiler.tensor_names"]
        names = json.loads(bytes(f.parts[f.data[0]]).decode())
        params = dict(model.named_parameters())
        with torch.no_grad():
            for t in reader.tensors:
                fqn = names.get(t.name)
                if fqn is None or t.tensor_type.name != "Q8_0":
                    continue
                back = gguf.quants.dequantize(t.data, t.tensor_type).reshape(params[fqn].shape)
                params[fqn].copy_(torch.from_numpy(np.ascontiguousarray(back)))
            ids = torch.randint(0, cfg["vocab_size"], (1, 40), generator=torch.Generator().manual_seed(1))
            logits = model(ids).logits[0].numpy()
            gen = model.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=24, do_sample=False,
                                 pad_token_id=0, eos_token_id=None)[0, 40:]
            gen_logits = model(torch.cat([ids[0], gen]).reshape(1, -1)).logits[0, 39:-1].numpy()
        np.savez(HERE / "ref_llama_q8_0.npz", ids=ids[0].numpy().astype(np.int32), logits=logits.astype(np.float32),
                 gen=gen.numpy().astype(np.int32), gen_logits=gen_logits.astype(np.float32),
                 config=json.dumps({**cfg, "max_context": 768, "max_prompt": 64, "weights": "q8_0"}))

        # 3: a 2-layer GQA program for the emitter
        cfg2 = dict(vocab_size=256, hidden_size=256, intermediate_size=384, num_hidden_layers=2, num_attention_heads=4,
                    num_key_value_heads=2, eos_token_id=7, rope_theta=500000.0, rms_norm_eps=1e-5)
        torch.manual_seed(0)
        m2 = transformers.LlamaForCausalLM(transformers.LlamaConfig(**cfg2)).float().eval()
        m2.config._attn_implementation = "eager"
        pol2 = DTypePolicy(rules=[("*_proj.weight", "q4_0"), ("lm_head.weight", "q4_0")], float="f32", fallback=[])
        art2 = ggml_compiler.compile(ggml_compiler.causal_lm(m2, max_context=1024, max_prompt=32), opt="O3",
                                     out_dir=tmp / "gqa2", dtype_policy=pol2)
        prog, meta = _program(art2.gguf)
        for s in prog["stages"]:
            for n in s["nodes"]:
                n.pop("loc", None)
                n.pop("scope", None)
        (HERE / "ref_program_gqa2.json").write_text(json.dumps(
            {"config": {**cfg2, "max_context": 1024, "max_prompt": 32, "weights": "q4_0"}, "meta": meta,
             "program": prog}, separators=(",", ":")))

        # 4: BASELINE config 1's shape
        cfg1 = CONFIG1
        torch.manual_seed(0)
        m1 = transformers.LlamaForCausalLM(transformers.LlamaConfig(**cfg1)).float().eval()
        m1.config._attn_implementation = "eager"
        pol1 = DTypePolicy(rules=[("*_proj.weight", "q8_0"), ("lm_head.weight", "q8_0")], float="f32", fallback=[])
        art1 = ggml_compiler.compile(ggml_compiler.causal_lm(m1, max_context=768, max_prompt=64), opt="O3",
                                     out_dir=tmp / "config1", dtype_policy=pol1)
        prog, meta = _program(art1.gguf)
        for s in prog["stages"]:
            for n in s["nodes"]:
                n.pop("loc", None)
                n.pop("scope", None)
        (HERE / "ref_program_config1.json").write_text(json.dumps(
            {"config": {**cfg1, "max_context": 768, "max_prompt": 64, "weights": "q8_0"}, "meta": meta,
             "program": prog}, separators=(",", ":")))
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_llm_golden.py REFERENCE_CHECKOUT (the ggml-compiler source tree)")
    main(sys.argv[1])
