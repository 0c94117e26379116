"""TEST INFRASTRUCTURE ONLY: runs a ggml-compiler GGUF on the CPU oracle.

A restatement of what the reference runtime does with a program (runtime/src/ggml_compiler_rt.cpp
:250-443 load, values, call sites and driver loop; runtime/src/ops.cpp the op table), with every
arithmetic op taken from ggml_oracle.c or from single-rounding numpy float32 ufuncs. Tensors are
numpy arrays in ggml order reversed (numpy shape = (ne3, ne2, ne1, ne0)), views share memory as
ggml views do, and set_rows writes the state (the KV cache) in place.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import numpy as np

from . import BLOCK_TYPES, dequantize, lib, mul_mat, rms_norm_rows

_NP = {"f32": np.float32, "f16": np.float16, "i32": np.int32}
_QUANT = BLOCK_TYPES


class Q:
    """A quantized weight: raw GGUF rows [rows, row_bytes] with ggml ne."""

    def __init__(self, raw: np.ndarray, typ: str, ne: list[int]) -> None:
        self.raw, self.type, self.ne = raw, typ, ne


def _ne(a: np.ndarray) -> list[int]:
    return list(reversed(a.shape))


def _ev(e: Any, syms: dict[str, int]) -> int:
    if isinstance(e, int):
        return e
    if isinstance(e, str):
        return syms[e]
    op, *args = e
    vals = [_ev(a, syms) for a in args]
    acc = vals[0]
    for v in vals[1:]:
        if op == "+":
            acc += v
        elif op == "*":
            acc *= v
        elif op == "//":
            acc = acc // v
        elif op == "%":
            acc = acc % v
        elif op == "max":
            acc = max(acc, v)
        elif op == "min":
            acc = min(acc, v)
        else:
            raise ValueError(op)
    return acc


def _view(base: np.ndarray, ne: list[int], nb: list[int], offset: int) -> np.ndarray:
    return np.lib.stride_tricks.as_strided(base.reshape(-1)[offset // base.itemsize:] if offset else base,
                                           shape=tuple(reversed(ne)), strides=tuple(reversed(nb)))


def _nb(a: np.ndarray) -> list[int]:
    return list(reversed(a.strides))


class Program:
    """`act`: "q8_0" converts activations to Q8_0 blocks before a quantized matmul, as ggml's CPU
    backend does (the reference semantics); "f32" multiplies the decoded weights by the f32
    activations instead, which isolates the rest of the graph's arithmetic for pinning against
    transformers."""

    def __init__(self, gguf_path: str | Path, act: str = "q8_0") -> None:
        import gguf

        self.act = act

        r = gguf.GGUFReader(str(gguf_path))

        def s(key: str) -> Any:
            f = r.fields.get(key)
            return None if f is None else bytes(f.parts[f.data[0]]).decode()

        self.prog = json.loads(s("ggml_compiler.program"))
        meta = s("ggml_compiler.meta")
        self.meta = json.loads(meta) if meta else {}
        self.weights: dict[str, Any] = {}
        for t in r.tensors:
            ne = [int(x) for x in t.shape] + [1] * (4 - len(t.shape))
            tn = t.tensor_type.name.lower()
            if tn in _QUANT:
                self.weights[t.name] = Q(np.asarray(t.data).reshape(-1, np.asarray(t.data).shape[-1]), tn, ne)
            else:
                self.weights[t.name] = np.asarray(t.data).reshape(tuple(reversed(ne))).copy()
        self.symbols = {sy["name"]: (sy["min"], sy["max"]) for sy in self.prog["symbols"]}
        self.binding = {k: hi for k, (lo, hi) in self.symbols.items()}
        self.vspec = {v["name"]: v for v in self.prog["values"]}
        self.values: dict[str, np.ndarray] = {}
        for v in self.prog["values"]:  # storage for the largest size, viewed per binding
            self.values[v["name"]] = np.zeros(self._max_elems(v), _NP[v["type"]])
        self.stages = {st["name"]: st for st in self.prog["stages"]}
        self.entries = {e["name"]: e for e in self.prog["entries"]}
        self.calls: dict[str, int] = {}
        self._rope_cache: dict[tuple, np.ndarray] = {}
        # (stage, node id) pairs whose values the next stage runs record in `taps` (copies)
        self.tap_ids: set[tuple[str, str]] = set()
        self.taps: dict[tuple[str, str], np.ndarray] = {}

    # -- values ---------------------------------------------------------------------------------
    def _max_elems(self, v: dict[str, Any]) -> int:
        best = 0
        names = list(self.symbols)
        for mask in range(1 << len(names)):
            b = {n: (self.symbols[n][1] if (mask >> i) & 1 else self.symbols[n][0]) for i, n in enumerate(names)}
            best = max(best, int(np.prod([_ev(d, b) for d in v["ne"]])))
        return best

    def ne_of(self, name: str) -> list[int]:
        return [_ev(d, self.binding) for d in self.vspec[name]["ne"]]

    def shape_of(self, name: str) -> list[int]:
        return [_ev(d, self.binding) for d in self.vspec[name]["shape"]]

    def value(self, name: str) -> np.ndarray:
        ne = self.ne_of(name)
        return self.values[name][: int(np.prod(ne))].reshape(tuple(reversed(ne)))

    def reset(self) -> None:
        for name in self.prog.get("state", []):
            self.values[name][:] = 0

    def set_input(self, name: str, arr: np.ndarray) -> None:
        """Bind the symbols the input's shape fixes (by search, as the runtime does) and store it."""
        spec = self.vspec[name]
        arr = np.asarray(arr, _NP[spec["type"]])
        shape = list(arr.shape)
        for dim, want in zip(spec["shape"], shape):
            syms = set()

            def collect(e: Any) -> None:
                if isinstance(e, str):
                    syms.add(e)
                elif isinstance(e, list):
                    for a in e[1:]:
                        collect(a)

            collect(dim)
            if len(syms) == 1:
                (k,) = syms
                lo, hi = self.symbols[k]
                for v in range(lo, hi + 1):
                    self.binding[k] = v
                    if _ev(dim, self.binding) >= want:
                        break
        if self.shape_of(name) != shape:
            raise ValueError(f"input {name} cannot have shape {shape}")
        self.value(name)[...] = arr.reshape(self.value(name).shape)

    # -- ops ------------------------------------------------------------------------------------
    def _src(self, name: str, env: dict[str, Any]) -> Any:
        return env[name] if name in env else self.weights[name]

    def _node(self, n: dict[str, Any], s: list[Any]) -> Any:
        op, p = n["op"], dict(n.get("p", {}))
        for k in ("start", "stop"):
            if k in p and not isinstance(p[k], (int, float)):
                p[k] = _ev(p[k], self.binding)
        ne = [_ev(d, self.binding) for d in n["ne"]]
        if op == "reshape":
            x = s[0]
            if isinstance(x, Q):
                return Q(x.raw, x.type, ne)
            if x.flags["C_CONTIGUOUS"]:
                return x.reshape(tuple(reversed(ne)))
            xne, xnb = _ne(x), _nb(x)
            nb, k = [xnb[0], 0, 0, 0], 0
            for i in range(4):
                if ne[i] == 1:
                    if i:
                        nb[i] = nb[i - 1] * ne[i - 1]
                    continue
                while xne[k] == 1:
                    k += 1
                nb[i] = xnb[k]
                k += 1
            return np.lib.stride_tricks.as_strided(x, shape=tuple(reversed(ne)), strides=tuple(reversed(nb)))
        if op == "view":
            x = s[0]
            dim, start = p["dim"], p["start"]
            nb = _nb(x)
            for k in range(1, 4):
                if ne[k] == 1:
                    nb[k] = nb[k - 1] * ne[k - 1]
            idx = [slice(None)] * 4
            idx[3 - dim] = slice(start, start + ne[dim])
            sub = x[tuple(idx)]
            return np.lib.stride_tricks.as_strided(sub, shape=tuple(reversed(ne)), strides=tuple(reversed(nb)))
        if op == "permute":
            x = s[0]
            axes = p["axes"]
            xne, xnb = _ne(x), _nb(x)
            yne, ynb = [0] * 4, [0] * 4
            for i in range(4):
                yne[axes[i]], ynb[axes[i]] = xne[i], xnb[i]
            return np.lib.stride_tricks.as_strided(x, shape=tuple(reversed(yne)), strides=tuple(reversed(ynb)))
        if op == "cont":
            return np.ascontiguousarray(s[0]).reshape(tuple(reversed(ne)))
        if op == "cast":
            return np.ascontiguousarray(s[0]).astype(_NP[n["type"]])
        if op in ("add", "sub", "mul", "div"):
            a, b = s
            ar, br = np.asarray(a, np.float32), np.asarray(b, np.float32)
            reps = tuple(x // y for x, y in zip(ar.shape, br.shape))
            bt = np.tile(br, reps)
            f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide}[op]
            return f(ar, bt).astype(a.dtype)
        if op == "scale":
            x = np.asarray(s[0], np.float32)
            return (x * np.float32(p["s"])) + np.float32(p.get("b", 0.0))
        if op == "clamp":
            return np.minimum(np.maximum(s[0], np.float32(p["min"])), np.float32(p["max"])).astype(np.float32)
        if op == "rms_norm":
            return rms_norm_rows(s[0], float(p["eps"]))
        if op == "soft_max":
            x = np.ascontiguousarray(s[0], np.float32)
            out = np.empty_like(x)
            mask = s[1] if len(s) > 1 else None
            X = x.reshape(-1, x.shape[-1])
            O = out.reshape(-1, x.shape[-1])
            B3, B2, R, _ = x.shape
            for i3 in range(B3):
                for i2 in range(B2):
                    for r in range(R):
                        row = (i3 * B2 + i2) * R + r
                        mrow = None
                        if mask is not None:
                            mrow = np.ascontiguousarray(mask[i3 % mask.shape[0], i2 % mask.shape[1], r], np.float32)
                        lib().orc_soft_max(X[row].ctypes.data, mrow.ctypes.data if mrow is not None else None,
                                           x.shape[-1], float(p.get("scale", 1.0)), O[row].ctypes.data)
            return out
        if op == "mul_mat":
            a, b = s
            if isinstance(a, Q):
                K, N = a.ne[0], a.ne[1]
                A2, A3 = a.ne[2], a.ne[3]
                raw = a.raw.reshape(A3, A2, N, -1)
                wtype = a.type
            else:
                K, N, A2, A3 = _ne(a)
                raw = a
                wtype = "f16" if a.dtype == np.float16 else "f32"
            B3, B2, M, _ = b.shape
            out = np.empty((B3, B2, M, N), np.float32)
            for i3 in range(B3):
                for i2 in range(B2):
                    w = raw[i3 // (B3 // A3), i2 // (B2 // A2)]
                    if self.act == "f32" and wtype in _QUANT:
                        out[i3, i2] = mul_mat(dequantize(w, wtype, K), "f32", K, b[i3, i2])
                    else:
                        out[i3, i2] = mul_mat(w, wtype, K, b[i3, i2])
            return out
        if op == "swiglu":
            g = np.ascontiguousarray(s[0], np.float32)
            u = np.ascontiguousarray(s[1], np.float32)
            y = np.empty_like(g)
            lib().orc_swiglu(g.ctypes.data, u.ctypes.data, g.size, y.ctypes.data)
            return y
        if op == "get_rows":
            tab, idx = s
            idx = np.asarray(idx).reshape(-1)
            if isinstance(tab, Q):
                rows = dequantize(tab.raw[idx], tab.type, tab.ne[0])
                return rows.reshape(tuple(reversed(ne)))
            return np.ascontiguousarray(tab.reshape(-1, tab.shape[-1])[idx].astype(np.float32)).reshape(tuple(reversed(ne)))
        if op == "set_rows":
            dst, src, idx = s
            idx = np.asarray(idx).reshape(-1).astype(np.int64)
            dst[:, :, idx, :] = np.asarray(src).astype(dst.dtype)
            return dst
        if op == "rope":
            x, pos = s[0], np.asarray(s[1]).reshape(-1)
            nd = p["n_dims"]
            if p["mode"] != 2 or len(s) > 2:
                raise NotImplementedError("oracle rope: NEOX without frequency factors")
            table = self._rope_table(nd, p, int(pos.max()) + 1)
            xf = np.asarray(x, np.float32)  # (B, S, H, D)
            cs = table[pos]  # (S, nd/2, 2)
            c = cs[None, :, None, :, 0]
            sn = cs[None, :, None, :, 1]
            h = nd // 2
            x0, x1 = xf[..., :h], xf[..., h:nd]
            y = xf.copy()
            y[..., :h] = (x0 * c) - (x1 * sn)
            y[..., h:nd] = (x0 * sn) + (x1 * c)
            return y
        if op == "flash_attn":
            q, k, v = s[0], s[1], s[2]
            mask = s[3] if len(s) > 3 else None
            B, H, Sq, D = q.shape
            Hkv, nkv = k.shape[1], k.shape[2]
            out = np.empty((B, Sq, H, D), np.float32)
            scale = float(p["scale"])
            for b in range(B):
                for h in range(H):
                    hk = h // (H // Hkv)
                    K = np.ascontiguousarray(k[b, hk]).view(np.uint16)
                    V = np.ascontiguousarray(v[b, hk]).view(np.uint16)
                    for iq in range(Sq):
                        qr = np.ascontiguousarray(q[b, h, iq], np.float32)
                        mr = None
                        if mask is not None:
                            mr = np.ascontiguousarray(mask[b % mask.shape[0], h % mask.shape[1], iq]).view(np.uint16)
                        o = np.empty(D, np.float32)
                        lib().orc_flash_attn_row(qr.ctypes.data, K.ctypes.data, D, V.ctypes.data, D, nkv, D,
                                                 mr.ctypes.data if mr is not None else None, scale, o.ctypes.data)
                        out[b, iq, h] = o
            return out
        if op == "argmax":
            x = np.asarray(s[0], np.float32)
            return np.argmax(x.reshape(-1, x.shape[-1]), axis=-1).astype(np.int32).reshape(tuple(reversed(ne)))
        raise NotImplementedError(f"oracle: op {op}")

    def _rope_table(self, nd: int, p: dict[str, Any], npos: int) -> np.ndarray:
        key = (nd, p["freq_base"], p.get("freq_scale", 1.0), p.get("attn_factor", 1.0))
        t = self._rope_cache.get(key)
        if t is None or t.shape[0] < npos:
            n = max(npos, 4096)
            t = np.empty((n, nd // 2, 2), np.float32)
            lib().orc_rope_table(nd, float(np.float32(p["freq_base"])), float(p.get("freq_scale", 1.0)),
                                 float(p.get("attn_factor", 1.0)), None, n, t.ctypes.data)
            self._rope_cache[key] = t
        return t

    # -- driver ---------------------------------------------------------------------------------
    def run_stage(self, call: dict[str, Any]) -> None:
        st = self.stages[call["stage"]]
        env: dict[str, Any] = {}
        for prm, arg in zip(st["params"], call["args"]):
            env[prm["name"]] = self.value(arg)
        for n in st["nodes"]:
            env[n["id"]] = self._node(n, [self._src(x, env) for x in n["src"]])
            if (st["name"], n["id"]) in self.tap_ids:
                self.taps[(st["name"], n["id"])] = np.array(env[n["id"]], copy=True)
        results = [env[o] for o in st["outputs"]]
        for res, out in zip(results, call["out"]):
            dst = self.value(out)
            if isinstance(res, np.ndarray) and np.shares_memory(res, dst):
                continue
            dst[...] = np.asarray(res).reshape(dst.shape).astype(dst.dtype)
        self.calls[st["name"]] = self.calls.get(st["name"], 0) + 1

    def _run_ops(self, ops: list[dict[str, Any]]) -> None:
        for d in ops:
            if d["op"] == "call":
                self.run_stage(d)
                continue
            for dst, src in d["carry"]:
                self.value(dst)[...] = self.value(src)
            n = self.binding[d["n"]] if isinstance(d["n"], str) else d["n"]
            starts = [int(self.value(src).reshape(-1)[0]) for _, src in d.get("counters", [])]
            for dst, _ in d.get("collect", []):
                self.values[dst][:] = 0
            for i in range(n):
                for k, (name, _) in enumerate(d.get("counters", [])):
                    self.value(name).reshape(-1)[0] = starts[k] + i
                ext = dict(self.binding)
                for k, (name, _) in enumerate(d.get("counters", [])):
                    ext[name] = starts[k] + i
                for sym, e in d.get("bind", []):
                    self.binding[sym] = _ev(e, ext)
                for name, ck in d.get("masks", []):
                    pos = starts[[c[0] for c in d["counters"]].index(ck)] + i
                    m = self.value(name)
                    j = np.arange(m.size) % m.shape[-1]
                    m.reshape(-1)[:] = np.where(j <= pos, 0.0, -np.inf).astype(np.float32)
                self._run_ops(d["body"])
                for dst, src in d.get("collect", []):
                    row = self.value(src).reshape(-1)
                    self.values[dst][i * row.size:(i + 1) * row.size] = row
                stop = False
                for name, ids in d.get("until", []):
                    stop = stop or int(self.value(name).reshape(-1)[0]) in ids
                if stop:
                    break

    def run(self, entry: str, **inputs: np.ndarray) -> dict[str, np.ndarray]:
        e = self.entries[entry]
        for name in e["inputs"]:
            self.set_input(name, inputs[name])
        self.calls = {}
        self._run_ops(e["driver"])
        return {name: np.array(self.value(name)).reshape(self.shape_of(name)) for name in e["outputs"]}

    def set_symbol(self, name: str, value: int) -> None:
        self.binding[name] = value


class OracleGenerator:
    """The reference's Generator host loop (ggml_compiler/llm.py:473-634, text path) over the oracle."""

    def __init__(self, prog: Program) -> None:
        self.p, self.meta = prog, prog.meta
        self.n_past = 0

    def reset(self) -> None:
        self.p.reset()
        self.n_past = 0

    def _run(self, ids: list[int]) -> np.ndarray:
        n = len(ids)
        block = self.meta["kv_block"]
        n_kv = max(self.meta["min_kv"], -(-(self.n_past + n) // block) * block)
        pos = np.arange(self.n_past, self.n_past + n, dtype=np.int32)
        rows = self.n_past + np.arange(n)[:, None]
        mask = np.where(np.arange(n_kv)[None, :] <= rows, 0.0, -np.inf).astype(np.float32)[None, None]
        tok = np.asarray(ids, np.int32)[None]
        if n == 1:
            out = self.p.run("decode", token=tok, position=pos, mask1=mask)["logits1"]
        else:
            out = self.p.run("prefill", tokens=tok, positions=pos, mask=mask)["logits"]
        self.n_past += n
        return out[0]

    def feed(self, ids: list[int]) -> np.ndarray:
        ids = list(ids)
        step = self.meta["max_prompt"]
        rows, i = [], 0
        while i < len(ids):
            n = min(step, len(ids) - i)
            if n == 1 or len(ids) - i - n == 1:
                n = 1 if n == 1 else n - 1
            rows.append(self._run(ids[i:i + n]))
            i += n
        return np.concatenate(rows, axis=0)[-1]

    def generate(self, prompt: list[int], max_new: int) -> tuple[list[int], list[np.ndarray]]:
        """Greedy tokens and the logits each was chosen from."""
        self.reset()
        logits = self.feed(prompt)
        out, ls = [], []
        for _ in range(max_new):
            ls.append(np.asarray(logits).reshape(-1))
            tok = int(np.argmax(logits))
            out.append(tok)
            if len(out) == max_new:
                break
            logits = self.feed([tok])
        return out, ls
