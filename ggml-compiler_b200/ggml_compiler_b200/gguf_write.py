"""A streaming GGUF writer for ggml-compiler programs (weights + the program JSON).

Writes the same keys the reference's emitter writes (ggml_compiler/emit/gguf_runtime.py:213-224):
general.architecture = "ggml_compiler", ggml_compiler.format_version, ggml_compiler.program,
ggml_compiler.tensor_names, ggml_compiler.source and ggml_compiler.meta. Tensor data is produced one
tensor at a time by a callback, so a multi-GB model never sits in memory twice.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Iterable

import numpy as np

GGUF_VERSION = 3
ALIGN = 32
# GGUF type ids and (block elements, block bytes) of the types this writer stores.
TYPE_IDS = {"f32": 0, "f16": 1, "q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8, "q4_k": 12, "q5_k": 13,
            "q6_k": 14, "iq4_nl": 20, "i32": 26, "bf16": 30}
BLOCKS = {"f32": (1, 4), "f16": (1, 2), "q4_0": (32, 18), "q4_1": (32, 20), "q5_0": (32, 22), "q5_1": (32, 24),
          "q8_0": (32, 34), "q4_k": (256, 144), "q5_k": (256, 176), "q6_k": (256, 210), "iq4_nl": (32, 18),
          "i32": (1, 4), "bf16": (1, 2)}

_T_U32, _T_STRING = 4, 8


@dataclass
class TensorEntry:
    name: str
    dtype: str                  # storage type name
    ne: tuple[int, ...]         # ggml order: innermost first
    data: Callable[[], np.ndarray] | np.ndarray  # bytes-like uint8 array of the stored encoding

    @property
    def nbytes(self) -> int:
        blk, size = BLOCKS[self.dtype]
        n = 1
        for d in self.ne:
            n *= d
        return n // blk * size


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str | Path, program: dict[str, Any], tensors: Iterable[TensorEntry],
               metadata: dict[str, Any] | None = None, tensor_names: dict[str, str] | None = None,
               source: dict[str, Any] | None = None) -> None:
    tensors = list(tensors)
    kv: list[tuple[str, int, bytes]] = [
        ("general.architecture", _T_STRING, _str("ggml_compiler")),
        ("ggml_compiler.format_version", _T_U32, struct.pack("<I", int(program.get("format_version", 3)))),
        ("ggml_compiler.program", _T_STRING, _str(json.dumps(program, separators=(",", ":")))),
        ("ggml_compiler.tensor_names", _T_STRING, _str(json.dumps(tensor_names or {}, separators=(",", ":")))),
        ("ggml_compiler.source", _T_STRING, _str(json.dumps(source or {"frontend": "ggml_compiler_b200"},
                                                            separators=(",", ":")))),
    ]
    if metadata:
        kv.append(("ggml_compiler.meta", _T_STRING, _str(json.dumps(metadata, separators=(",", ":")))))
    head = bytearray(b"GGUF" + struct.pack("<IQQ", GGUF_VERSION, len(tensors), len(kv)))
    for key, t, val in kv:
        head += _str(key) + struct.pack("<I", t) + val
    offset = 0
    for t in tensors:
        head += _str(t.name) + struct.pack("<I", len(t.ne)) + b"".join(struct.pack("<Q", d) for d in t.ne)
        head += struct.pack("<IQ", TYPE_IDS[t.dtype], offset)
        offset += (t.nbytes + ALIGN - 1) // ALIGN * ALIGN
    head += b"\0" * ((-len(head)) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for t in tensors:
            data = t.data() if callable(t.data) else t.data
            buf = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
            if buf.size != t.nbytes:
                raise ValueError(f"tensor {t.name}: {buf.size} bytes for a {t.dtype} {t.ne} ({t.nbytes} bytes)")
            f.write(memoryview(buf))
            f.write(b"\0" * ((-t.nbytes) % ALIGN))
