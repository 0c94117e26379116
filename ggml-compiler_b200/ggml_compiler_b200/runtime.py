"""ctypes bindings to this repository's libggml_compiler_rt.so (the B200 backend).

The same Python interface as the reference's ggml_compiler/runtime/session.py (Session, quantize,
has_backend, version, GgmlCompilerRuntimeError; signatures bound as at session.py:75-122), so code
written against the reference runs unchanged. The library is found through $GGML_COMPILER_RT, else
the in-tree build (ggml_compiler_b200/lib/). There is no CPU fallback: without a B200 the library
loads and encodes weights, but loading a model fails with a GgmlCompilerRuntimeError.
"""

from __future__ import annotations

import ctypes
import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

import numpy as np

_BACKENDS = {"cpu": 0, "cuda": 1, "auto": 2}
_DTYPES = {0: ("f32", np.float32), 1: ("f16", np.float16), 2: ("i32", np.int32)}
_MAX_RANK = 8
LIB_NAME = "libggml_compiler_rt.so"


class _Options(ctypes.Structure):
    _fields_ = [("backend", ctypes.c_int), ("device", ctypes.c_int), ("n_threads", ctypes.c_int),
                ("allow_cpu_fallback", ctypes.c_bool)]


class _TensorInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_int64 * _MAX_RANK), ("nbytes", ctypes.c_size_t)]


class _Stats(ctypes.Structure):
    _fields_ = [("ms_total", ctypes.c_double), ("n_calls", ctypes.c_int)]


class GgmlCompilerRuntimeError(RuntimeError):
    """An error reported by libggml_compiler_rt."""


def library_path() -> Path:
    env = os.environ.get("GGML_COMPILER_RT")
    if env:
        return Path(env)
    p = Path(__file__).resolve().parent / "lib" / LIB_NAME
    if not p.exists():
        raise RuntimeError(f"{LIB_NAME} not found: run `python -m ggml_compiler_b200.build` or set GGML_COMPILER_RT")
    return p


# Every symbol of include/ggml_compiler_rt.h that takes or returns plain C types.
_SIGS: dict[str, tuple[list[Any], Any]] = {}


def _sigs() -> dict[str, tuple[list[Any], Any]]:
    p, i, c_size, c_str = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_char_p
    return {
        "ggml_compiler_version": ([], c_str),
        "ggml_compiler_last_error": ([], c_str),
        "ggml_compiler_default_options": ([], _Options),
        "ggml_compiler_has_backend": ([i], ctypes.c_bool),
        "ggml_compiler_load": ([c_str, ctypes.POINTER(_Options)], p),
        "ggml_compiler_load_with": ([c_str, ctypes.POINTER(_Options), p, i], p),
        "ggml_compiler_quantize": ([c_str, p, ctypes.c_int64, ctypes.c_int64, p, c_size], c_size),
        "ggml_compiler_row_size": ([c_str, ctypes.c_int64], c_size),
        "ggml_compiler_free": ([p], None),
        "ggml_compiler_backend_name": ([p], c_str),
        "ggml_compiler_n_inputs": ([p], i),
        "ggml_compiler_n_outputs": ([p], i),
        "ggml_compiler_input_info": ([p, i, ctypes.POINTER(_TensorInfo)], i),
        "ggml_compiler_output_info": ([p, i, ctypes.POINTER(_TensorInfo)], i),
        "ggml_compiler_set_input": ([p, c_str, p, c_size], i),
        "ggml_compiler_n_entries": ([p], i),
        "ggml_compiler_entry_name": ([p, i], c_str),
        "ggml_compiler_entry_n_inputs": ([p, i], i),
        "ggml_compiler_entry_n_outputs": ([p, i], i),
        "ggml_compiler_entry_input_info": ([p, i, i, ctypes.POINTER(_TensorInfo)], i),
        "ggml_compiler_entry_output_info": ([p, i, i, ctypes.POINTER(_TensorInfo)], i),
        "ggml_compiler_run_entry": ([p, c_str], i),
        "ggml_compiler_reset": ([p], i),
        "ggml_compiler_metadata": ([p, c_str], c_str),
        "ggml_compiler_n_symbols": ([p], i),
        "ggml_compiler_symbol_info": ([p, i, ctypes.POINTER(c_str), ctypes.POINTER(ctypes.c_int64),
                                       ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)], i),
        "ggml_compiler_set_symbol": ([p, c_str, ctypes.c_int64], i),
        "ggml_compiler_set_input_shape": ([p, c_str, i, ctypes.POINTER(ctypes.c_int64)], i),
        "ggml_compiler_run": ([p], i),
        "ggml_compiler_get_output": ([p, c_str, p, c_size], i),
        "ggml_compiler_last_stats": ([p, ctypes.POINTER(_Stats)], i),
        "ggml_compiler_n_stages": ([p], i),
        "ggml_compiler_stage_stats": ([p, i, ctypes.POINTER(c_str), ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(ctypes.c_int)], i),
        # extensions of this backend (include/ggml_compiler_b200.h)
        "ggml_compiler_b200_stream": ([p], p),
        "ggml_compiler_b200_last_device_ms": ([p], ctypes.c_double),
        "ggml_compiler_b200_set_profiling": ([p, i], i),
        "ggml_compiler_b200_n_kernel_stats": ([p], i),
        "ggml_compiler_b200_kernel_stats": ([p, i, ctypes.POINTER(c_str), ctypes.POINTER(ctypes.c_double),
                                             ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double)], i),
        "ggml_compiler_b200_tp_init": ([p, i, i, c_size, p, c_size], i),
        "ggml_compiler_b200_tp_connect": ([p, p, c_size], i),
    }


_lib: ctypes.CDLL | None = None


def load_library() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    lib = ctypes.CDLL(str(library_path()))
    for name, (args, res) in _sigs().items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    _lib = lib
    return lib


_load = load_library


def _error() -> GgmlCompilerRuntimeError:
    return GgmlCompilerRuntimeError(_load().ggml_compiler_last_error().decode())


def version() -> str:
    return _load().ggml_compiler_version().decode()


def quantize(data: np.ndarray, type_name: str) -> np.ndarray:
    """Encode f32 data (rows along the last axis) in a ggml type; uint8 [rows..., row_bytes]."""
    lib = _load()
    x = np.ascontiguousarray(data, dtype=np.float32)
    n = x.shape[-1]
    rows = x.size // n
    row_bytes = lib.ggml_compiler_row_size(type_name.encode(), n)
    if row_bytes == 0:
        raise _error()
    out = np.empty(x.shape[:-1] + (row_bytes,), dtype=np.uint8)
    if lib.ggml_compiler_quantize(type_name.encode(), x.ctypes.data, rows, n, out.ctypes.data, out.nbytes) == 0:
        raise _error()
    return out


def row_size(type_name: str, n: int) -> int:
    return int(_load().ggml_compiler_row_size(type_name.encode(), n))


def has_backend(backend: str) -> bool:
    return bool(_load().ggml_compiler_has_backend(_BACKENDS[backend]))


@dataclass(frozen=True)
class TensorInfo:
    name: str
    shape: tuple[int, ...]
    dtype: str
    nbytes: int


class Session:
    """A loaded model. `run` takes inputs positionally or by name and returns outputs by name
    (reference ggml_compiler/runtime/session.py:160-306). Symbols are bound from the input shapes;
    `set_symbol` binds the others (a loop's trip count). State (a KV cache) persists across runs
    until `reset()`."""

    def __init__(self, path: str | os.PathLike, backend: str = "auto", device: int = 0, n_threads: int = 0,
                 allow_cpu_fallback: bool = False) -> None:
        lib = _load()
        self._m = None
        if backend not in _BACKENDS:
            raise ValueError(f"backend must be one of {sorted(_BACKENDS)}")
        opt = lib.ggml_compiler_default_options()
        opt.backend, opt.device, opt.n_threads, opt.allow_cpu_fallback = (
            _BACKENDS[backend], device, n_threads, allow_cpu_fallback)
        self._m = lib.ggml_compiler_load(os.fsencode(path), ctypes.byref(opt))
        if not self._m:
            raise _error()
        self.backend_name: str = lib.ggml_compiler_backend_name(self._m).decode()
        self._np: dict[str, np.dtype] = {}
        self.entries: dict[str, tuple[list[TensorInfo], list[TensorInfo]]] = {}
        for e in range(lib.ggml_compiler_n_entries(self._m)):
            ins = [self._info(lambda m, k, info: lib.ggml_compiler_entry_input_info(m, e, k, info), k)
                   for k in range(lib.ggml_compiler_entry_n_inputs(self._m, e))]
            outs = [self._info(lambda m, k, info: lib.ggml_compiler_entry_output_info(m, e, k, info), k)
                    for k in range(lib.ggml_compiler_entry_n_outputs(self._m, e))]
            self.entries[lib.ggml_compiler_entry_name(self._m, e).decode()] = (ins, outs)
        self.inputs, self.outputs = next(iter(self.entries.values()))
        self.symbols: dict[str, tuple[int, int]] = {}
        for k in range(lib.ggml_compiler_n_symbols(self._m)):
            name, lo, hi = ctypes.c_char_p(), ctypes.c_int64(), ctypes.c_int64()
            lib.ggml_compiler_symbol_info(self._m, k, ctypes.byref(name), ctypes.byref(lo), ctypes.byref(hi), None)
            self.symbols[name.value.decode()] = (lo.value, hi.value)

    @property
    def metadata(self) -> dict[str, Any]:
        raw = _load().ggml_compiler_metadata(self._m, b"ggml_compiler.meta")
        return json.loads(raw.decode()) if raw else {}

    def set_symbol(self, name: str, value: int) -> None:
        if _load().ggml_compiler_set_symbol(self._m, name.encode(), int(value)) != 0:
            raise _error()

    def bound(self) -> dict[str, int]:
        lib, out = _load(), {}
        for k in range(len(self.symbols)):
            name, v = ctypes.c_char_p(), ctypes.c_int64()
            lib.ggml_compiler_symbol_info(self._m, k, ctypes.byref(name), None, None, ctypes.byref(v))
            out[name.value.decode()] = v.value
        return out

    def _info(self, fn: Any, k: int) -> TensorInfo:
        info = _TensorInfo()
        if fn(self._m, k, ctypes.byref(info)) != 0:
            raise _error()
        name, (dtype, np_dtype) = info.name.decode(), _DTYPES[info.dtype]
        self._np[name] = np.dtype(np_dtype)
        return TensorInfo(name, tuple(info.shape[: info.ndim]), dtype, info.nbytes)

    def reset(self) -> None:
        if _load().ggml_compiler_reset(self._m) != 0:
            raise _error()

    def set_inputs(self, entry: str, arrays: dict[str, np.ndarray]) -> None:
        """Bind symbols from the shapes and upload every input of `entry` (host -> device)."""
        lib = _load()
        inputs, _ = self.entries[entry]
        for t in inputs:
            x = arrays[t.name]
            if not self.symbols:
                if x.shape != t.shape:
                    raise ValueError(f"input {t.name} has shape {x.shape}, the model expects {t.shape}")
                continue
            shape = (ctypes.c_int64 * max(1, x.ndim))(*x.shape)
            if lib.ggml_compiler_set_input_shape(self._m, t.name.encode(), x.ndim, shape) != 0:
                raise _error()
        for t in inputs:
            x = arrays[t.name]
            if lib.ggml_compiler_set_input(self._m, t.name.encode(), x.ctypes.data, x.nbytes) != 0:
                raise _error()

    def run_entry(self, entry: str) -> None:
        if _load().ggml_compiler_run_entry(self._m, entry.encode()) != 0:
            raise _error()

    def get_outputs(self, entry: str) -> dict[str, np.ndarray]:
        lib = _load()
        _, outputs = self.entries[entry]
        if self.symbols:
            e = list(self.entries).index(entry)
            outputs = [self._info(lambda m, k, info: lib.ggml_compiler_entry_output_info(m, e, k, info), k)
                       for k in range(len(outputs))]
        out = {}
        for t in outputs:
            y = np.empty(t.shape, dtype=self._np[t.name])
            if lib.ggml_compiler_get_output(self._m, t.name.encode(), y.ctypes.data, y.nbytes) != 0:
                raise _error()
            out[t.name] = y
        return out

    def run(self, *args: Any, entry: str | None = None, **kwargs: Any) -> dict[str, np.ndarray]:
        entry = entry or next(iter(self.entries))
        if entry not in self.entries:
            raise ValueError(f"no entry point {entry!r}; the model has {list(self.entries)}")
        inputs, _ = self.entries[entry]
        if len(args) > len(inputs):
            raise TypeError(f"{len(args)} positional inputs for an entry with {len(inputs)} inputs")
        given = {t.name: a for t, a in zip(inputs, args)}
        for k, v in kwargs.items():
            if k in given:
                raise TypeError(f"input {k} given twice")
            given[k] = v
        names = {t.name for t in inputs}
        unknown = set(given) - names
        if unknown:
            raise TypeError(f"unknown inputs {sorted(unknown)}; the model takes {[t.name for t in inputs]}")
        missing = names - set(given)
        if missing:
            raise TypeError(f"missing inputs {sorted(missing)}")
        arrays = {t.name: _as_numpy(given[t.name], self._np[t.name]) for t in inputs}
        self.set_inputs(entry, arrays)
        self.run_entry(entry)
        return self.get_outputs(entry)

    @property
    def stats(self) -> dict[str, Any]:
        lib = _load()
        st = _Stats()
        if lib.ggml_compiler_last_stats(self._m, ctypes.byref(st)) != 0:
            raise _error()
        stages = {}
        for k in range(lib.ggml_compiler_n_stages(self._m)):
            name, ms, calls = ctypes.c_char_p(), ctypes.c_double(), ctypes.c_int()
            lib.ggml_compiler_stage_stats(self._m, k, ctypes.byref(name), ctypes.byref(ms), ctypes.byref(calls))
            stages[name.value.decode()] = {"ms": ms.value, "calls": calls.value}
        return {"ms_total": st.ms_total, "n_calls": st.n_calls, "stages": stages}

    # ---- extensions of this backend (no counterpart in the reference's Session)

    @property
    def stream(self) -> int:
        """The CUDA stream (cudaStream_t as an int) every launch of this session goes to."""
        return int(_load().ggml_compiler_b200_stream(self._m) or 0)

    @property
    def last_device_ms(self) -> float:
        """Device time of the last run or run_entry, CUDA events around all its launches."""
        return float(_load().ggml_compiler_b200_last_device_ms(self._m))

    def set_profiling(self, on: bool) -> None:
        """Per-launch timing (each launch synchronised, no CUDA graphs) while on; clears the stats."""
        if _load().ggml_compiler_b200_set_profiling(self._m, int(bool(on))) != 0:
            raise _error()

    def kernel_stats(self) -> dict[str, dict[str, float]]:
        """Per kernel family, since profiling was switched on: total ms, launches and algorithmic bytes."""
        lib = _load()
        out = {}
        for k in range(lib.ggml_compiler_b200_n_kernel_stats(self._m)):
            name, ms, n, b = ctypes.c_char_p(), ctypes.c_double(), ctypes.c_int(), ctypes.c_double()
            lib.ggml_compiler_b200_kernel_stats(self._m, k, ctypes.byref(name), ctypes.byref(ms), ctypes.byref(n),
                                                ctypes.byref(b))
            out[name.value.decode()] = {"ms": ms.value, "launches": n.value, "bytes": b.value}
        return out

    def tensor_parallel(self, rank: int, world: int, all_gather: Callable[[bytes], list[bytes]],
                        window_bytes: int = 0) -> None:
        """Join a tensor-parallel group of `world` processes, one GPU each, that loaded the same
        program (ggml_compiler_b200_tp_init / _tp_connect). `all_gather(b)` returns every rank's
        bytes in rank order (for example `torch_all_gather()`); call before the first run, on every
        rank. Afterwards every rank must make the same runs; results equal one GPU's."""
        lib = _load()
        h = ctypes.create_string_buffer(256)
        n = lib.ggml_compiler_b200_tp_init(self._m, rank, world, window_bytes, h, len(h))
        if n < 0:
            raise _error()
        handles = exchange_handles(h.raw[:n], rank, world, all_gather)
        if lib.ggml_compiler_b200_tp_connect(self._m, handles, len(handles)) != 0:
            raise _error()

    def close(self) -> None:
        if getattr(self, "_m", None):
            _load().ggml_compiler_free(self._m)
            self._m = None

    def __enter__(self) -> "Session":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()

    def __del__(self) -> None:
        self.close()


def exchange_handles(mine: bytes, rank: int, world: int, all_gather: Callable[[bytes], list[bytes]]) -> bytes:
    """Every rank's window handle, concatenated in rank order, checked for shape."""
    got = list(all_gather(bytes(mine)))
    if len(got) != world:
        raise ValueError(f"all_gather returned {len(got)} handles for a group of {world}")
    if got[rank] != mine or any(len(g) != len(mine) for g in got):
        raise ValueError("all_gather must return every rank's handle, in rank order, all of one size")
    return b"".join(got)


def torch_all_gather(group: Any = None) -> Callable[[bytes], list[bytes]]:
    """An all_gather for Session.tensor_parallel over an initialised torch.distributed group."""
    import torch.distributed as dist

    def gather(b: bytes) -> list[bytes]:
        out: list[Any] = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, b, group=group)
        return out

    return gather


def _as_numpy(x: Any, dtype: np.dtype) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(x).astype(dtype, copy=False))
