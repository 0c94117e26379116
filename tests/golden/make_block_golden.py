"""Generate the golden vectors of the other GGUF block formats the reference can store weights in
(ggml_compiler/quant/types.py:6-19: q4_1, q5_0, q5_1, iq4_nl, q4_k, q5_k, q6_k) from gguf-py 0.19
(gguf/quants.py restates ggml's block layouts and, for q4_1 / q5_0 / q5_1, its reference encoders;
it has no encoder for iq4_nl or the K-quants).

Writes tests/golden/block_formats.npz:
- `x`: edge-case rows of 256 values; `<t>` and `<t>_dec`: their gguf-py encoding and decoding for
  t in q4_1, q5_0, q5_1;
- `raw_<t>`, `dec_<t>`: seeded random blocks of every format (random bytes, the fp16 scale fields
  set to finite values) and gguf-py's decoding of them;
- `sha_<t>_4096x4096`: SHA-256 of gguf-py's encoding of the 4096 x 4096 N(0, 0.02) seed-0 matrix.
Run from the repo root:

    python tests/golden/make_block_golden.py
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = Path(__file__).resolve().parent
ENCODED = {"q4_1": T.Q4_1, "q5_0": T.Q5_0, "q5_1": T.Q5_1}
ALL = {**ENCODED, "iq4_nl": T.IQ4_NL, "q4_k": T.Q4_K, "q5_k": T.Q5_K, "q6_k": T.Q6_K}
# block bytes and the byte offsets of fp16 scale fields, per format
LAYOUT = {"q4_1": (20, 32, (0, 2)), "q5_0": (22, 32, (0,)), "q5_1": (24, 32, (0, 2)), "iq4_nl": (18, 32, (0,)),
          "q4_k": (144, 256, (0, 2)), "q5_k": (176, 256, (0, 2)), "q6_k": (210, 256, (208,))}


def edge_cases() -> np.ndarray:
    rng = np.random.default_rng(11)
    rows = [
        np.zeros(256, np.float32),
        np.linspace(-1, 1, 256, dtype=np.float32),
        np.tile(np.array([1.0, -1.0, 0.5, -0.5], np.float32), 64),
        np.tile(np.array([-3.0, 3.0, 1.5, 0.0], np.float32), 64),
        (np.arange(256, dtype=np.float32) - 128) * np.float32(1 / 127),
        rng.standard_normal(256).astype(np.float32) * np.float32(1e-6),
        rng.standard_normal(256).astype(np.float32) * np.float32(1e3),
        np.full(256, 0.25, np.float32),
        rng.standard_normal(256).astype(np.float32),
    ]
    r = np.stack(rows)
    r[8, 5] = 0.0
    r[8, 40] = -r[8].max() * 2
    return r


def random_blocks(t: str, rows: int, n: int, seed: int) -> np.ndarray:
    bs, qk, scales = LAYOUT[t]
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, (rows, n // qk, bs), dtype=np.uint8)
    for off in scales:
        h = (rng.standard_normal((rows, n // qk)) * 0.01).astype(np.float16)
        raw[:, :, off:off + 2] = h.view(np.uint8).reshape(rows, n // qk, 2)
    return raw.reshape(rows, -1)


def main() -> None:
    x = edge_cases()
    out: dict[str, np.ndarray] = {"x": x}
    for name, qt in ENCODED.items():
        enc = quants.quantize(x, qt)
        out[name] = enc
        out[f"{name}_dec"] = quants.dequantize(enc, qt)
    for i, (name, qt) in enumerate(ALL.items()):
        raw = random_blocks(name, 6, 1024, 100 + i)
        out[f"raw_{name}"] = raw
        out[f"dec_{name}"] = quants.dequantize(raw, qt)
    w = np.random.default_rng(0).standard_normal((4096, 4096), dtype=np.float32) * np.float32(0.02)
    for name, qt in ENCODED.items():
        out[f"sha_{name}_4096x4096"] = np.array(hashlib.sha256(quants.quantize(w, qt).tobytes()).hexdigest())
    np.savez_compressed(HERE / "block_formats.npz", **out)


if __name__ == "__main__":
    main()
