"""TEST INFRASTRUCTURE ONLY: the CPU oracle for the B200 backend's parity tests.

`ops` binds oracle/ggml_oracle.c (the C restatement of ggml's CPU arithmetic for the LLM op subset)
and `interp.Program` runs a ggml-compiler GGUF on it. Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import this package; the product library never uses it.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "build" / "libggml_oracle.so"

_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the oracle with its Makefile (gcc) if the shared library is missing or stale."""
    src = HERE / "ggml_oracle.c"
    if not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        p, i64, f, i = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        sigs = {
            "orc_quantize": ([i, p, i64, i64, p], ctypes.c_size_t),
            "orc_dequantize": ([i, p, i64, i64, p], None),
            "orc_row_size": ([i, i64], ctypes.c_size_t),
            "orc_act_q8_0": ([p, i64, p, p], None),
            "orc_act_q8_1": ([p, i64, p, p, p], None),
            "orc_act_q8_K": ([p, i64, p, p, p], None),
            "orc_mul_mat": ([i, p, ctypes.c_size_t, i64, i64, p, i64, i64, p, i64], i),
            "orc_rms_norm": ([p, i64, f, p], None),
            "orc_soft_max": ([p, p, i64, f, p], None),
            "orc_rope_table": ([i, f, f, f, p, i64, p], None),
            "orc_rope_neox": ([p, i64, i, p, p], None),
            "orc_flash_attn_row": ([p, p, i64, p, i64, i64, i64, p, f, p], None),
            "orc_swiglu": ([p, p, i64, p], None),
            "orc_argmax": ([p, i64], ctypes.c_int32),
            "orc_expf": ([f], f),
            "orc_silu": ([f], f),
            "orc_h2f": ([ctypes.c_uint16], f),
            "orc_f2h": ([f], ctypes.c_uint16),
            "orc_set_threads": ([i], None),
            "orc_get_threads": ([], i),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q4_1": 3, "q5_0": 6, "q5_1": 7, "q8_0": 8, "q4_k": 12, "q5_k": 13,
         "q6_k": 14, "iq4_nl": 20}
BLOCK_TYPES = ("q4_0", "q4_1", "q5_0", "q5_1", "q8_0", "q4_k", "q5_k", "q6_k", "iq4_nl")


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def quantize(x: np.ndarray, type_name: str) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    rows = x.size // n
    rb = lib().orc_row_size(TYPES[type_name], n)
    out = np.empty(x.shape[:-1] + (rb,), np.uint8)
    if lib().orc_quantize(TYPES[type_name], _ptr(x), rows, n, _ptr(out)) == 0:
        raise ValueError(f"oracle cannot encode {type_name} rows of {n}")
    return out


def dequantize(raw: np.ndarray, type_name: str, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, np.uint8)
    rows = raw.size // lib().orc_row_size(TYPES[type_name], n)
    out = np.empty((rows, n), np.float32)
    lib().orc_dequantize(TYPES[type_name], _ptr(raw), rows, n, _ptr(out))
    return out


def mul_mat(w: np.ndarray, wtype: str, K: int, x: np.ndarray) -> np.ndarray:
    """y[m, n] = sum_k x[m, k] w[n, k]; w raw rows (quantized: bytes [N, row_bytes]; f32/f16 values)."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, np.float32)
    N = w.shape[0]
    M = x.shape[0]
    y = np.empty((M, N), np.float32)
    rb = w.strides[0]
    if lib().orc_mul_mat(TYPES[wtype], _ptr(w), rb, N, K, _ptr(x), K, M, _ptr(y), N) != 0:
        raise ValueError("oracle mul_mat failed")
    return y


def act_q8_0(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 32, np.uint16)
    lib().orc_act_q8_0(_ptr(x), x.size, _ptr(q), _ptr(d))
    return q, d


def act_q8_1(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Q8_1 activation blocks: codes, fp16 scale bits, fp16 d * sum(codes) bits."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 32, np.uint16)
    s = np.empty(x.size // 32, np.uint16)
    lib().orc_act_q8_1(_ptr(x), x.size, _ptr(q), _ptr(d), _ptr(s))
    return q, d, s


def act_q8_k(x: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Q8_K activation super-blocks: codes, f32 scales, int16 sums of 16 codes."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    d = np.empty(x.size // 256, np.float32)
    bs = np.empty(x.size // 16, np.int16)
    lib().orc_act_q8_K(_ptr(x), x.size, _ptr(q), _ptr(d), _ptr(bs))
    return q, d, bs


def rms_norm_rows(x: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[-1]
    flat = x.reshape(-1, n)
    out = np.empty_like(flat)
    for r in range(flat.shape[0]):
        lib().orc_rms_norm(_ptr(flat[r]), n, eps, _ptr(out[r]))
    return out.reshape(x.shape)


def expf(x: float) -> float:
    return lib().orc_expf(x)
