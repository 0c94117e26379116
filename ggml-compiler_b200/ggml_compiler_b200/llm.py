"""Causal language models on this backend: a greedy decoder over a compiled causal LM, and an
emitter for Llama-shaped programs.

- `Decoder` feeds token ids to a program compiled by the reference's `causal_lm` (or written by
  `llama_program`): it chooses the entry (prefill for two or more ids, decode for one), builds
  positions and the additive causal mask over the smallest KV window the program allows, and runs
  greedy decoding on the host or through the program's `generate` entry (the loop on the device).
  The reference drives the same entries from its own `ggml_compiler.llm.Generator`, which runs
  unchanged over this library; the two issue the same calls for the same ids.
- `llama_program` writes the program JSON the reference's `causal_lm(model, ...)` compiles a
  LlamaForCausalLM into at -O3 (flash attention, f16 KV cache, fused rope/rms_norm/swiglu): the same
  values, stages, node lists, parameters and driver (format 3). A test checks it node for node
  against programs the reference compiler wrote. It lets 8B- and 70B-shaped models be built from
  seeded weights without materialising them as fp32 PyTorch modules.
- `build_llama_gguf` writes such a model with N(0, 0.02) weights (norm weights 1, as HF's init),
  encoding the projections and the output head with a bit-exact Q4_0 / Q8_0 encoder.
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Sequence

import numpy as np

from .fusion import mark_fusion_groups
from .gguf_write import TensorEntry, write_gguf

KV_BLOCK = 256


def call_sizes(n: int, limit: int) -> list[int]:
    """How `n` ids are fed: calls of at most `limit` ids, taken greedily, except that a call is
    shortened by one when it would leave a single id behind (a prefill call takes two or more)."""
    sizes, left = [], n
    while left:
        take = min(limit, left)
        if take > 1 and left - take == 1:
            take -= 1
        sizes.append(take)
        left -= take
    return sizes


class Decoder:
    """Greedy decoding over a causal-LM program loaded in a `runtime.Model`.

    `ctx` counts the positions filled in the program's KV cache; `restart()` empties it."""

    def __init__(self, model: Any) -> None:
        self.model = model
        self.meta = model.meta
        if self.meta.get("kind") != "causal_lm":
            raise ValueError(f"{model.path} holds no causal-LM program (metadata kind {self.meta.get('kind')!r})")
        self.ctx = 0

    def restart(self) -> None:
        self.model.clear_state()
        self.ctx = 0

    def window(self, end: int) -> int:
        """KV rows the program attends over once positions < end are filled: whole blocks, at
        least the program's minimum."""
        blk = self.meta["kv_block"]
        return max(self.meta["min_kv"], blk * ((end + blk - 1) // blk))

    def _call(self, ids: Sequence[int]) -> np.ndarray:
        n, start = len(ids), self.ctx
        if start + n > self.meta["max_context"]:
            raise ValueError(f"{start} + {n} positions exceed the program's max_context {self.meta['max_context']}")
        cols = np.arange(self.window(start + n))
        mask = np.full((1, 1, n, cols.size), -np.inf, np.float32)
        mask[0, 0][cols[None, :] <= start + np.arange(n)[:, None]] = 0.0
        toks = np.asarray(ids, np.int32).reshape(1, n)
        where = np.arange(start, start + n, dtype=np.int32)
        if n == 1:
            res = self.model.entries["decode"](token=toks, position=where, mask1=mask)["logits1"]
        else:
            res = self.model.entries["prefill"](tokens=toks, positions=where, mask=mask)["logits"]
        self.ctx += n
        return res.reshape(-1, res.shape[-1])  # [rows, vocab]: the last row, or every row (logits="all")

    def prompt(self, ids: Sequence[int]) -> np.ndarray:
        """Appends `ids` to the context; the logits after the last one ([vocab])."""
        ids, last, i = list(ids), None, 0
        for n in call_sizes(len(ids), self.meta["max_prompt"]):
            last = self._call(ids[i:i + n])
            i += n
        return last[-1]

    def step(self, token: int) -> np.ndarray:
        """Appends one token; the logits after it ([vocab])."""
        return self._call([int(token)])[-1]

    def fill_slots(self, prompts: Sequence[Sequence[int]]) -> tuple[np.ndarray, np.ndarray]:
        """Batched decode set-up: gives the model one sequence slot per prompt, prefills prompt i in
        the model's own state and copies that state into slot i. Returns each sequence's greedy
        first token and its next position (the inputs of `Model.generate_batch`)."""
        self.model.seq_slots(len(prompts))
        first, start = [], []
        for i, p in enumerate(prompts):
            self.restart()
            first.append(int(np.argmax(self.prompt(p))))
            start.append(self.ctx)
            self.model.seq_copy(i, -1)
        return np.asarray(first, np.int32), np.asarray(start, np.int32)

    def greedy(self, prompt: Sequence[int], n: int, stop: Sequence[int] | None = None,
               on_device: bool = False) -> list[int]:
        """Up to `n` greedy tokens after `prompt` from an empty context, ending early at a stop id
        (default: the model's EOS ids). on_device: the tokens after the first come from the
        program's `generate` entry, whose loop stops at the model's EOS ids."""
        self.restart()
        stops = set(self.meta["eos"] if stop is None else stop)
        first = int(np.argmax(self.prompt(prompt)))
        toks = [first]
        if first in stops or n == 1:
            return toks
        if on_device:
            room = self.meta["max_context"] - self.ctx
            self.model.bind(max_new=max(1, min(n - 1, room)))
            gen = self.model.entries["generate"]
            got = gen(first=np.array([[first]], np.int32), start=np.array([self.ctx], np.int32))["generated"].ravel()
            made = self.model.stage_calls()["decode_greedy"]
            self.ctx += made
            return toks + [int(t) for t in got[:made]]
        while len(toks) < n and toks[-1] not in stops:
            toks.append(int(np.argmax(self.step(toks[-1]))))
        return toks


# ------------------------------------------------------------------------------------------------
# Llama-shaped programs


@dataclass
class LlamaShape:
    layers: int
    d_model: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    head_dim: int | None = None
    rope_theta: float = 10000.0
    eps: float = 1e-5
    max_context: int = 1024
    max_prompt: int = 512
    eos: list[int] = field(default_factory=list)
    bos: int | None = 1
    weight_type: str = "q4_0"  # projections and output head
    embed_type: str = "f32"

    @property
    def hd(self) -> int:
        return self.head_dim or self.d_model // self.heads


# BASELINE configs 1, 3/4 and 5 (Llama-3 shapes).
TINY = LlamaShape(layers=4, d_model=512, heads=8, kv_heads=8, ffn=1408, vocab=32000, rope_theta=10000.0,
                  max_context=768, max_prompt=64, weight_type="q8_0")
LLAMA3_8B = LlamaShape(layers=32, d_model=4096, heads=32, kv_heads=8, ffn=14336, vocab=128256, rope_theta=500000.0,
                       max_context=1024, max_prompt=512, weight_type="q4_0")
LLAMA3_70B = LlamaShape(layers=80, d_model=8192, heads=64, kv_heads=8, ffn=28672, vocab=128256, rope_theta=500000.0,
                        max_context=1280, max_prompt=1024, weight_type="q4_0")


def recovered_rope_base(theta: float, d: int) -> float:
    """The freq_base the reference's fuse_rope pass recovers from HF's float32 inv_freq
    (passes/fuse_rope.py:75-91: the median of -log(inv_i) * d / (2 i) over i > 0)."""
    import torch

    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).to(dtype=torch.float) / d))
    inv = inv.double()
    i = torch.arange(len(inv), dtype=torch.float64)
    live = (inv > 0) & (i > 0)
    return math.exp(float((-torch.log(inv[live]) * d / (2 * i[live])).median()))


def _t(name: str, typ: str, ne: list[Any], shape: list[Any]) -> dict[str, Any]:
    return {"name": name, "type": typ, "ne": ne, "shape": shape}


def _stage(sh: LlamaShape, kind: str, freq_base: float) -> dict[str, Any]:
    """One stage of the program: kind is "prefill", "decode" or "decode_greedy"."""
    D, H, Hkv, d, F, V, L = sh.hd, sh.heads, sh.kv_heads, sh.d_model, sh.ffn, sh.vocab, sh.layers
    S: Any = "s" if kind == "prefill" else 1
    nkv: Any = ["*", KV_BLOCK, "kv_blocks"]
    ctx = sh.max_context
    nodes: list[dict[str, Any]] = []

    def node(op: str, src: list[str], typ: str, ne: list[Any], p: dict[str, Any] | None = None) -> str:
        nid = f"%{len(nodes)}"
        nodes.append({"id": nid, "op": op, "src": src, "type": typ, "ne": ne, "p": p or {}})
        return nid

    rope_p = {"n_dims": D, "mode": 2, "freq_base": freq_base, "freq_scale": 1.0, "attn_factor": 1.0}
    params = [_t("a.0", "i32", [S, 1, 1, 1], [1, S]), _t("a.1", "i32", [S, 1, 1, 1], [S] if kind == "prefill" else [1]),
              _t("a.2", "f32", [nkv, S, 1, 1], [1, 1, S, nkv])]
    for i in range(2 * L):
        params.append(_t(f"a.{3 + i}", "f16", [D, ctx, Hkv, 1], [Hkv, ctx, D]))
    w = 1  # GGUF weight index (w.0 is the embedding)
    x = node("reshape", ["a.0"], "i32", [S, 1, 1, 1])
    x = node("get_rows", ["w.0", x], "f32", [d, S, 1, 1])
    resid = node("reshape", [x], "f32", [d, S, 1, 1])
    mask16 = None
    outs = []
    for layer in range(L):
        wn, wq, wk, wv, wo, wn2, wg, wu, wd = (f"w.{w + k}" for k in range(9))
        w += 9
        h = node("rms_norm", [resid], "f32", [d, S, 1, 1], {"eps": sh.eps})
        h = node("mul", [h, wn], "f32", [d, S, 1, 1])
        h = node("reshape", [h], "f32", [d, S, 1, 1])
        q = node("mul_mat", [wq, h], "f32", [H * D, S, 1, 1])
        q = node("reshape", [q], "f32", [D, H, S, 1])
        k = node("mul_mat", [wk, h], "f32", [Hkv * D, S, 1, 1])
        k = node("reshape", [k], "f32", [D, Hkv, S, 1])
        v = node("mul_mat", [wv, h], "f32", [Hkv * D, S, 1, 1])
        if kind == "prefill":
            v = node("reshape", [v], "f32", [D, Hkv, S, 1])
            v = node("permute", [v], "f32", [D, S, Hkv, 1], {"axes": [0, 2, 1, 3]})
            q = node("rope", [q, "a.1"], "f32", [D, H, S, 1], rope_p)
            q = node("permute", [q], "f32", [D, S, H, 1], {"axes": [0, 2, 1, 3]})
            k = node("rope", [k, "a.1"], "f32", [D, Hkv, S, 1], rope_p)
            k = node("permute", [k], "f32", [D, S, Hkv, 1], {"axes": [0, 2, 1, 3]})
        else:
            v = node("reshape", [v], "f32", [D, 1, Hkv, 1])
            q = node("rope", [q, "a.1"], "f32", [D, H, 1, 1], rope_p)
            q = node("reshape", [q], "f32", [D, 1, H, 1])
            k = node("rope", [k, "a.1"], "f32", [D, Hkv, 1, 1], rope_p)
            k = node("reshape", [k], "f32", [D, 1, Hkv, 1])
        k = node("view", [k], "f32", [D, S, Hkv, 1], {"dim": 3, "start": 0})
        k = node("reshape", [k], "f32", [D, S, Hkv, 1])
        kc = node("set_rows", [f"a.{3 + 2 * layer}", k, "a.1"], "f16", [D, ctx, Hkv, 1])
        kview = node("view", [kc], "f16", [D, nkv, Hkv, 1], {"dim": 1, "start": 0})
        kview = node("reshape", [kview], "f16", [D, nkv, Hkv, 1])
        v = node("view", [v], "f32", [D, S, Hkv, 1], {"dim": 3, "start": 0})
        v = node("reshape", [v], "f32", [D, S, Hkv, 1])
        vc = node("set_rows", [f"a.{4 + 2 * layer}", v, "a.1"], "f16", [D, ctx, Hkv, 1])
        vview = node("view", [vc], "f16", [D, nkv, Hkv, 1], {"dim": 1, "start": 0})
        vview = node("reshape", [vview], "f16", [D, nkv, Hkv, 1])
        outs += [kc, vc]
        if mask16 is None:
            m = node("clamp", ["a.2"], "f32", [nkv, S, 1, 1], {"min": -65504.0, "max": 65504.0})
            mask16 = node("cast", [m], "f16", [nkv, S, 1, 1])
        a = node("flash_attn", [q, kview, vview, mask16], "f32", [D, H, S, 1], {"scale": 1.0 / math.sqrt(D)})
        a = node("reshape", [a], "f32", [H * D, S, 1, 1])
        o = node("mul_mat", [wo, a], "f32", [d, S, 1, 1])
        o = node("reshape", [o], "f32", [d, S, 1, 1])
        resid = node("add", [resid, o], "f32", [d, S, 1, 1])
        h = node("rms_norm", [resid], "f32", [d, S, 1, 1], {"eps": sh.eps})
        h = node("mul", [h, wn2], "f32", [d, S, 1, 1])
        h = node("reshape", [h], "f32", [d, S, 1, 1])
        g = node("mul_mat", [wg, h], "f32", [F, S, 1, 1])
        g = node("reshape", [g], "f32", [F, S, 1, 1])
        u = node("mul_mat", [wu, h], "f32", [F, S, 1, 1])
        u = node("reshape", [u], "f32", [F, S, 1, 1])
        f = node("swiglu", [g, u], "f32", [F, S, 1, 1])
        f = node("reshape", [f], "f32", [F, S, 1, 1])
        f = node("mul_mat", [wd, f], "f32", [d, S, 1, 1])
        f = node("reshape", [f], "f32", [d, S, 1, 1])
        resid = node("add", [resid, f], "f32", [d, S, 1, 1])
    h = node("rms_norm", [resid], "f32", [d, S, 1, 1], {"eps": sh.eps})
    h = node("mul", [h, f"w.{w}"], "f32", [d, S, 1, 1])
    if kind == "prefill":
        h = node("view", [h], "f32", [d, 1, 1, 1], {"dim": 1, "start": ["+", -1, "s"]})
    h = node("reshape", [h], "f32", [d, 1, 1, 1])
    logits = node("mul_mat", [f"w.{w + 1}", h], "f32", [V, 1, 1, 1])
    if kind == "decode_greedy":
        logits = node("argmax", [logits], "i32", [1, 1, 1, 1])
        res = node("reshape", [logits], "i32", [1, 1, 1, 1])
    else:
        res = node("reshape", [logits], "f32", [V, 1, 1, 1])
    return {"name": kind, "params": params, "outputs": [res] + outs, "nodes": nodes}


def llama_program(sh: LlamaShape) -> tuple[dict[str, Any], dict[str, Any]]:
    """(program JSON, metadata) of a Llama-shaped causal LM, as the reference compiles it at -O3."""
    D, Hkv, V, L, ctx = sh.hd, sh.kv_heads, sh.vocab, sh.layers, sh.max_context
    if ctx % KV_BLOCK or ctx < 3 * KV_BLOCK:
        raise ValueError(f"max_context must be a multiple of {KV_BLOCK}, at least {3 * KV_BLOCK}")
    nkv: Any = ["*", KV_BLOCK, "kv_blocks"]
    base = recovered_rope_base(sh.rope_theta, D)
    kv = [f"kv.{i}" for i in range(2 * L)]
    values = [_t(n, "f16", [D, ctx, Hkv, 1], [Hkv, ctx, D]) for n in kv]
    values += [_t("tokens", "i32", ["s", 1, 1, 1], [1, "s"]), _t("positions", "i32", ["s", 1, 1, 1], ["s"]),
               _t("mask", "f32", [nkv, "s", 1, 1], [1, 1, "s", nkv]), _t("logits", "f32", [V, 1, 1, 1], [1, 1, V]),
               _t("token", "i32", [1, 1, 1, 1], [1, 1]), _t("position", "i32", [1, 1, 1, 1], [1]),
               _t("mask1", "f32", [nkv, 1, 1, 1], [1, 1, 1, nkv]), _t("logits1", "f32", [V, 1, 1, 1], [1, 1, V]),
               _t("first", "i32", [1, 1, 1, 1], [1, 1]), _t("start", "i32", [1, 1, 1, 1], [1]),
               _t("tok", "i32", [1, 1, 1, 1], [1, 1]), _t("pos", "i32", [1, 1, 1, 1], [1]),
               _t("gmask", "f32", [nkv, 1, 1, 1], [1, 1, 1, nkv]),
               _t("generated", "i32", [1, 1, "max_new", 1], ["max_new", 1, 1])]
    pre_in, dec_in = ["tokens", "positions", "mask"], ["token", "position", "mask1"]
    prefill = [{"op": "call", "stage": "prefill", "args": pre_in + kv, "out": ["logits"] + kv}]
    decode = [{"op": "call", "stage": "decode", "args": dec_in + kv, "out": ["logits1"] + kv}]
    blocks = ctx // KV_BLOCK
    loop = {"op": "loop", "n": "max_new", "carry": [["tok", "first"]], "scalars": [], "slices": [],
            "counters": [["pos", "start"]],
            "bind": [["kv_blocks", ["max", 2, ["min", blocks, ["+", 1, ["//", "pos", KV_BLOCK]]]]]],
            "masks": [["gmask", "pos"]], "until": [["tok", list(sh.eos)]] if sh.eos else [],
            "collect": [["generated", "tok"]],
            "body": [{"op": "call", "stage": "decode_greedy", "args": ["tok", "pos", "gmask"] + kv, "out": ["tok"] + kv}]}
    program = {
        "format_version": 3,
        "symbols": [{"name": "max_new", "min": 1, "max": ctx}, {"name": "s", "min": 2, "max": sh.max_prompt},
                    {"name": "kv_blocks", "min": 2, "max": blocks}],
        "values": values,
        "inputs": pre_in,
        "outputs": ["logits"],
        "stages": [_stage(sh, "prefill", base), _stage(sh, "decode", base), _stage(sh, "decode_greedy", base)],
        "driver": prefill,
        "entries": [{"name": "prefill", "inputs": pre_in, "outputs": ["logits"], "driver": prefill},
                    {"name": "decode", "inputs": dec_in, "outputs": ["logits1"], "driver": decode},
                    {"name": "generate", "inputs": ["first", "start"], "outputs": ["generated"], "driver": [loop]}],
        "state": kv,
    }
    meta = {"kind": "causal_lm", "max_context": ctx, "max_prompt": sh.max_prompt, "kv_block": KV_BLOCK,
            "min_kv": 2 * KV_BLOCK, "vocab": V, "eos": list(sh.eos), "logits": "last", "bos": sh.bos,
            "rope": "positions"}
    return program, meta


def llama_weights(sh: LlamaShape) -> list[tuple[str, str, tuple[int, ...], str]]:
    """(GGUF name, HF name, PyTorch shape, storage type) of every weight, in the reference's order."""
    D, H, Hkv, d, F, V = sh.hd, sh.heads, sh.kv_heads, sh.d_model, sh.ffn, sh.vocab
    out = [("w.0", "model.embed_tokens.weight", (V, d), sh.embed_type)]
    k = 1
    for layer in range(sh.layers):
        p = f"model.layers.{layer}."
        for hf, shape, typ in ((p + "input_layernorm.weight", (d,), "f32"),
                               (p + "self_attn.q_proj.weight", (H * D, d), sh.weight_type),
                               (p + "self_attn.k_proj.weight", (Hkv * D, d), sh.weight_type),
                               (p + "self_attn.v_proj.weight", (Hkv * D, d), sh.weight_type),
                               (p + "self_attn.o_proj.weight", (d, H * D), sh.weight_type),
                               (p + "post_attention_layernorm.weight", (d,), "f32"),
                               (p + "mlp.gate_proj.weight", (F, d), sh.weight_type),
                               (p + "mlp.up_proj.weight", (F, d), sh.weight_type),
                               (p + "mlp.down_proj.weight", (d, F), sh.weight_type)):
            out.append((f"w.{k}", hf, shape, typ))
            k += 1
    out.append((f"w.{k}", "model.norm.weight", (d,), "f32"))
    out.append((f"w.{k + 1}", "lm_head.weight", (V, d), sh.weight_type))
    return out


def normal_weights(shape: tuple[int, ...], seed: int, index: int, std: float = 0.02) -> np.ndarray:
    """Seeded N(0, std) f32 weights for weight `index` of a synthetic model (chunked over threads)."""
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    chunk = 1 << 22
    parts = [(i, min(n, i + chunk)) for i in range(0, n, chunk)]
    seqs = np.random.SeedSequence([seed, index]).spawn(len(parts))

    def fill(j: int) -> None:
        a, b = parts[j]
        np.random.default_rng(seqs[j]).standard_normal(b - a, dtype=np.float32, out=out[a:b])
        out[a:b] *= np.float32(std)

    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
        list(ex.map(fill, range(len(parts))))
    return out.reshape(shape)


def build_llama_gguf(path: str | Path, sh: LlamaShape, seed: int = 0,
                     encoder: Callable[[np.ndarray, str], np.ndarray] | None = None,
                     weights: dict[str, np.ndarray] | None = None, fusion_marks: bool = True) -> dict[str, Any]:
    """Write a Llama-shaped model as a ggml-compiler GGUF; returns its metadata. The weights are
    `weights` (f32 arrays by Hugging Face name, e.g. a LlamaForCausalLM's state dict) or, without
    it, seeded synthetic ones. `encoder(w, type)` encodes the quantized matrices (default: this
    library's `runtime.encode`; any bit-exact Q4_0 / Q8_0 encoder writes the same bytes).
    `fusion_marks`: the program's fusable node groups carry `"fuse"` marks (fusion.py); without
    them the program is exactly the reference compiler's and the backend finds the groups itself."""
    if encoder is None:
        from .runtime import encode as encoder
    program, meta = llama_program(sh)
    if fusion_marks:
        program = mark_fusion_groups(program, {g: t for g, _, _, t in llama_weights(sh)}, in_place=True)
    entries = []
    names = {}
    for idx, (gname, hf, shape, typ) in enumerate(llama_weights(sh)):
        names[gname] = hf

        def data(shape=shape, typ=typ, idx=idx, hf=hf) -> np.ndarray:
            if weights is not None:
                w = np.ascontiguousarray(weights[hf], np.float32).reshape(shape)
            elif hf.endswith("norm.weight"):
                return np.ones(shape, np.float32)
            else:
                w = normal_weights(shape, seed, idx)
            if typ == "f32":
                return w
            if typ == "f16":
                return w.astype(np.float16)
            return encoder(w, typ)

        entries.append(TensorEntry(gname, typ, tuple(reversed(shape)), data))
    write_gguf(path, program, entries, metadata=meta, tensor_names=names,
               source={"frontend": "ggml_compiler_b200.llm.build_llama_gguf", "seed": seed})
    return meta
