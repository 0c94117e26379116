"""Causal language models over this backend: the reference's text-model host driver, and an emitter
for Llama-shaped programs.

- `causal_mask`, `Generator` and `bench` are the reference's host side for a compiled causal LM
  (ggml_compiler/llm.py:355-358, :473-634 text path, :637-683): positions, additive masks, prompt
  chunking and greedy decoding over the prefill / decode / generate entries.
- `llama_program` writes the program JSON the reference's `causal_lm(model, ...)` compiles a
  LlamaForCausalLM into at -O3 (flash attention, f16 KV cache, fused rope/rms_norm/swiglu): the same
  values, stages, node lists, parameters and driver (format 3). A test checks it node for node
  against programs the reference compiler wrote. It lets 8B- and 70B-shaped models be built from
  seeded weights without materialising them as fp32 PyTorch modules.
- `build_llama_gguf` writes such a model with N(0, 0.02) weights (norm weights 1, as HF's init),
  quantizing the projections and the output head with this library's bit-exact encoder.
"""

from __future__ import annotations

import math
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Sequence

import numpy as np

from . import runtime
from .gguf_write import TensorEntry, write_gguf

KV_BLOCK = 256


def causal_mask(n_past: int, s: int, n_kv: int) -> np.ndarray:
    """[1, 1, s, n_kv]: token i (at position n_past + i) attends to positions 0 .. n_past + i."""
    rows = n_past + np.arange(s)[:, None]
    return np.where(np.arange(n_kv)[None, :] <= rows, 0.0, -np.inf).astype(np.float32)[None, None]


class Generator:
    """Drives a compiled causal LM on the host: positions, masks, prompt chunks, greedy decoding
    (the reference's Generator, text path)."""

    def __init__(self, session: Any) -> None:
        meta = session.metadata
        if meta.get("kind") != "causal_lm":
            raise ValueError("the artifact was not compiled from ggml_compiler.causal_lm")
        self.s, self.meta = session, meta
        self.reset(state=False)

    def reset(self, state: bool = True) -> None:
        if state:
            self.s.reset()
        self.n_past = 0

    def _n_kv(self, end: int) -> int:
        block = self.meta["kv_block"]
        return max(self.meta["min_kv"], -(-end // block) * block)

    def _run(self, ids: Sequence[int]) -> np.ndarray:
        n = len(ids)
        if self.n_past + n > self.meta["max_context"]:
            raise ValueError(f"context full: {self.n_past} + {n} tokens > max_context {self.meta['max_context']}")
        n_kv = self._n_kv(self.n_past + n)
        pos = np.arange(self.n_past, self.n_past + n, dtype=np.int32)
        mask = causal_mask(self.n_past, n, n_kv)
        tok = np.asarray(ids, dtype=np.int32)[None]
        if n == 1:
            out = self.s.run(token=tok, position=pos, mask1=mask, entry="decode")["logits1"]
        else:
            out = self.s.run(tokens=tok, positions=pos, mask=mask, entry="prefill")["logits"]
        self.n_past += n
        return out[0]

    def feed(self, ids: Sequence[int]) -> np.ndarray:
        """Append tokens to the context; returns the logits after the last one ([vocab])."""
        ids = list(ids)
        step = self.meta["max_prompt"]
        rows = []
        i = 0
        while i < len(ids):
            n = min(step, len(ids) - i)
            if n == 1 or len(ids) - i - n == 1:  # never leave a lone token for a prefill of one
                n = 1 if n == 1 else n - 1
            rows.append(self._run(ids[i:i + n]))
            i += n
        out = np.concatenate(rows, axis=0)
        return out if self.meta["logits"] == "all" else out[-1]

    def generate(self, prompt: Sequence[int], max_new: int, stop: Sequence[int] | None = None,
                 device: bool = False) -> list[int]:
        """Greedy continuation of `prompt` from an empty context (device=True: the `generate` entry's
        loop runs in the runtime)."""
        self.reset()
        stop = set(self.meta["eos"] if stop is None else stop)
        logits = self.feed(prompt)
        if device:
            if "generate" not in self.s.entries:
                raise ValueError("compiled without the generate entry")
            first = int(np.argmax(logits if logits.ndim == 1 else logits[-1]))
            if first in stop or max_new == 1:
                return [first]
            room = self.meta["max_context"] - self.n_past
            self.s.set_symbol("max_new", max(1, min(max_new - 1, room)))
            out = self.s.run(first=np.array([[first]], np.int32), start=np.array([self.n_past], np.int32),
                             entry="generate")["generated"].reshape(-1)
            n = self.s.stats["stages"]["decode_greedy"]["calls"]
            self.n_past += n
            return [first] + out[:n].tolist()
        out: list[int] = []
        for _ in range(max_new):
            tok = int(np.argmax(logits if logits.ndim == 1 else logits[-1]))
            out.append(tok)
            if tok in stop or len(out) == max_new:
                break
            logits = self.feed([tok])
        return out


def bench(session: Any, pp: int = 512, tg: int = 128, reps: int = 5, seed: int = 0,
          device: bool = False) -> dict[str, float]:
    """llama-bench style tokens/s (the reference's llm.bench): pp = one prefill of `pp` tokens from an
    empty context, tg = `tg` single-token decodes; mean over `reps` runs after a warmup."""
    import time

    g = Generator(session)
    rng = np.random.default_rng(seed)
    vocab = g.meta["vocab"]
    out: dict[str, float] = {}
    if pp:
        times = []
        for r in range(reps + 1):
            ids = rng.integers(0, vocab, pp).tolist()
            g.reset()
            t = time.perf_counter()
            g.feed(ids)
            if r:
                times.append(time.perf_counter() - t)
        out[f"pp{pp}"] = pp / float(np.mean(times))
    if tg and device:
        rates = []
        session.set_symbol("max_new", tg)
        for r in range(reps + 1):
            g.reset()
            first = np.array([[int(rng.integers(0, vocab))]], np.int32)
            t = time.perf_counter()
            session.run(first=first, start=np.array([0], np.int32), entry="generate")
            dt = time.perf_counter() - t
            if r:
                rates.append(session.stats["stages"]["decode_greedy"]["calls"] / dt)
        out[f"tg{tg}"] = float(np.mean(rates))
    elif tg:
        times = []
        for r in range(reps + 1):
            g.reset()
            tok = int(rng.integers(0, vocab))
            t = time.perf_counter()
            for _ in range(tg):
                logits = g.feed([tok])
                tok = int(np.argmax(logits))
            if r:
                times.append(time.perf_counter() - t)
        out[f"tg{tg}"] = tg / float(np.mean(times))
    return out


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


def build_llama_gguf(path: str | Path, sh: LlamaShape, seed: int = 0) -> dict[str, Any]:
    """Write a seeded synthetic Llama-shaped model as a ggml-compiler GGUF; returns its metadata."""
    program, meta = llama_program(sh)
    entries = []
    names = {}
    for idx, (gname, hf, shape, typ) in enumerate(llama_weights(sh)):
        names[gname] = hf

        def data(shape=shape, typ=typ, idx=idx, hf=hf) -> np.ndarray:
            if hf.endswith("norm.weight"):
                return np.ones(shape, np.float32)
            w = normal_weights(shape, seed, idx)
            if typ == "f32":
                return w
            if typ == "f16":
                return w.astype(np.float16)
            return runtime.quantize(w, typ)

        entries.append(TensorEntry(gname, typ, tuple(reversed(shape)), data))
    write_gguf(path, program, entries, metadata=meta, tensor_names=names,
               source={"frontend": "ggml_compiler_b200.llm.build_llama_gguf", "seed": seed})
    return meta
