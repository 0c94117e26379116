"""Generate the Q4_0 / Q8_0 encoding golden vectors from gguf-py 0.19 (the encoder the reference
pins: pyproject.toml `gguf>=0.19`; gguf/quants.py Q4_0 :220-252 and Q8_0 :378-402 restate ggml's
reference quantizers bit for bit; the reference decodes its own output with them at
ggml_compiler/emit/gguf_runtime.py:268).

Writes tests/golden/quant_golden.json (digests at the full op-sweep shapes of BASELINE config 2)
and tests/golden/quant_small.npz (raw bytes of small edge-case inputs). Run from the repo root:

    python tests/golden/make_quant_golden.py
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = Path(__file__).resolve().parent

# Config 2 weight shapes, PyTorch order [out, in]: rows of `in` values.
SWEEP = [(4096, 4096), (14336, 4096), (4096, 14336)]


def weights(shape: tuple[int, int], seed: int = 0) -> np.ndarray:
    """N(0, 0.02) f32 weights from `seed` (the synthetic-weight rule used across this repo)."""
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(0.02)


def edge_cases() -> np.ndarray:
    """Rows that exercise the encoders' corner cases: zeros, ties of the max magnitude, a negative
    max, exact .5 quotients, tiny (subnormal-scale) and large values."""
    rng = np.random.default_rng(7)
    rows = [
        np.zeros(64, np.float32),
        np.linspace(-1, 1, 64, dtype=np.float32),
        np.tile(np.array([1.0, -1.0, 0.5, -0.5], np.float32), 16),
        np.tile(np.array([-3.0, 3.0, 1.5, 0.0], np.float32), 16),
        (np.arange(64, dtype=np.float32) - 32) * np.float32(1 / 127),
        rng.standard_normal(64).astype(np.float32) * np.float32(1e-6),
        rng.standard_normal(64).astype(np.float32) * np.float32(1e3),
        rng.standard_normal(64).astype(np.float32),
    ]
    r = np.stack(rows)
    r[7, 5] = 0.0
    r[7, 40] = -r[7].max() * 2  # a negative value of largest magnitude in its block
    return r


def main() -> None:
    out: dict[str, dict[str, str]] = {}
    for shape in SWEEP:
        w = weights(shape)
        key = f"{shape[0]}x{shape[1]}"
        out[key] = {}
        for name, qt in (("q4_0", T.Q4_0), ("q8_0", T.Q8_0)):
            enc = quants.quantize(w, qt)
            out[key][name] = hashlib.sha256(enc.tobytes()).hexdigest()
        out[key]["f32"] = hashlib.sha256(w.tobytes()).hexdigest()
    (HERE / "quant_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    x = edge_cases()
    np.savez(HERE / "quant_small.npz", x=x, q4_0=quants.quantize(x, T.Q4_0), q8_0=quants.quantize(x, T.Q8_0),
             q4_0_dec=quants.dequantize(quants.quantize(x, T.Q4_0), T.Q4_0),
             q8_0_dec=quants.dequantize(quants.quantize(x, T.Q8_0), T.Q8_0))


if __name__ == "__main__":
    main()
