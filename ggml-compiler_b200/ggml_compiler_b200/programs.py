"""Single-stage programs around one node: the isolated-op form the reference's tests and the op sweep
use (tests/helpers.py:22-28 `run_stage_on`: one stage, its inputs as program inputs, weights as
GGUF tensors). Used for the quantized GEMV/GEMM sweep and op parity tests."""

from __future__ import annotations

from pathlib import Path
from typing import Any, Sequence

import numpy as np

from . import runtime
from .gguf_write import TensorEntry, write_gguf


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


def write_mul_mat(path: str | Path, w: np.ndarray, wtype: str, M: int, batch: int = 1) -> None:
    """A program y = mul_mat(W, x): W [N, K] f32 stored as `wtype`, x [batch, M, K] f32 input."""
    N, K = w.shape
    if wtype in ("q4_0", "q8_0"):
        data = runtime.encode(w, wtype)
    elif wtype == "f16":
        data = w.astype(np.float16)
    else:
        data = np.ascontiguousarray(w, np.float32)
    prog = single_node_program("mul_mat", [("x", "f32", [K, M, batch, 1], [batch, M, K])], ["w.0", "x"], "f32",
                               [N, M, batch, 1], [batch, M, N])
    write_gguf(path, prog, [TensorEntry("w.0", wtype, (K, N), data)])
