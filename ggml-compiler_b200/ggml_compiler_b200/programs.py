"""Single-stage programs around one node: the isolated-op form the reference's tests and the op sweep
use (tests/helpers.py:22-28 `run_stage_on`: one stage, its inputs as program inputs, weights as
GGUF tensors). Used for the quantized GEMV/GEMM sweep and op parity tests."""

from __future__ import annotations

from pathlib import Path
from typing import Any, Sequence

import numpy as np

from . import runtime
from .gguf_write import BLOCKS, TensorEntry, write_gguf


def single_node_program(op: str, inputs: Sequence[tuple[str, str, list[int], list[int]]], src: Sequence[str],
                        out_type: str, out_ne: list[int], out_shape: list[int],
                        params: dict[str, Any] | None = None) -> dict[str, Any]:
    """One stage `main` computing node %0 = op(src...) from program inputs (name, type, ggml ne,
    PyTorch shape) and GGUF weights (names in `src` that are not inputs). The output is `out.0`."""
    names = [n for n, _, _, _ in inputs]
    pmap = {n: f"a.{i}" for i, n in enumerate(names)}
    values = [{"name": n, "type": t, "ne": list(ne), "shape": list(sh)} for n, t, ne, sh in inputs]
    values.append({"name": "out.0", "type": out_type, "ne": list(out_ne), "shape": list(out_shape)})
    stage = {"name": "main",
             "params": [{"name": pmap[n], "type": t, "ne": list(ne), "shape": list(sh)} for n, t, ne, sh in inputs],
             "outputs": ["%0"],
             "nodes": [{"id": "%0", "op": op, "src": [pmap.get(s, s) for s in src], "type": out_type, "ne": list(out_ne),
                        "p": params or {}}]}
    driver = [{"op": "call", "stage": "main", "args": names, "out": ["out.0"]}]
    return {"format_version": 3, "symbols": [], "values": values, "inputs": names, "outputs": ["out.0"],
            "stages": [stage], "driver": driver,
            "entries": [{"name": "main", "inputs": names, "outputs": ["out.0"], "driver": driver}], "state": []}


# byte offsets of the fp16 scale fields in one block of each format that has no encoder here
_SCALE_FIELDS = {"q4_1": (0, 2), "q5_0": (0,), "q5_1": (0, 2), "iq4_nl": (0,), "q4_k": (0, 2), "q5_k": (0, 2),
                 "q6_k": (208,)}
# scale field spread that gives weights of about N(0, 0.02) magnitude
SYNTHETIC_SCALE = {"q4_1": 2e-3, "q5_0": 2e-3, "q5_1": 1e-3, "iq4_nl": 2e-4, "q4_k": 3e-5, "q5_k": 2e-5, "q6_k": 1.5e-5}


def random_block_rows(typ: str, rows: int, K: int, seed: int, scale: float | None = None) -> np.ndarray:
    """Seeded synthetic `typ` rows of K values, uint8 [rows, row bytes]: random code bytes with the
    fp16 scale fields drawn from N(0, scale) (finite, so every block decodes). The stand-in for
    weights in the formats this library has no encoder for (iq4_nl, q4_k, q5_k, q6_k)."""
    blk, size = BLOCKS[typ]
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, (rows, K // blk, size), dtype=np.uint8)
    sd = SYNTHETIC_SCALE[typ] if scale is None else scale
    for off in _SCALE_FIELDS[typ]:
        h = (rng.standard_normal((rows, K // blk)) * sd).astype(np.float16)
        raw[:, :, off:off + 2] = h.view(np.uint8).reshape(rows, K // blk, 2)
    return raw.reshape(rows, -1)


def write_mul_mat(path: str | Path, w: np.ndarray, wtype: str, M: int, batch: int = 1) -> None:
    """A program y = mul_mat(W, x): W [N, K] f32 stored as `wtype`, x [batch, M, K] f32 input. A
    uint8 `w` of shape [N, row bytes] is taken as already-encoded `wtype` rows of K values (the
    formats this library has no encoder for: iq4_nl, q4_k, q5_k, q6_k)."""
    if w.dtype == np.uint8:
        blk, size = BLOCKS[wtype]
        N, K = w.shape[0], w.shape[1] // size * blk
        data = np.ascontiguousarray(w)
    elif wtype in ("q4_0", "q4_1", "q5_0", "q5_1", "q8_0"):
        N, K = w.shape
        data = runtime.encode(w, wtype)
    elif wtype == "f16":
        N, K = w.shape
        data = w.astype(np.float16)
    else:
        N, K = w.shape
        data = np.ascontiguousarray(w, np.float32)
    prog = single_node_program("mul_mat", [("x", "f32", [K, M, batch, 1], [batch, M, K])], ["w.0", "x"], "f32",
                               [N, M, batch, 1], [batch, M, N])
    write_gguf(path, prog, [TensorEntry("w.0", wtype, (K, N), data)])
