"""Python handle on libggml_compiler_rt.so, the B200 backend for ggml-compiler programs.

The library exports the reference runtime's C ABI (include/ggml_compiler_rt.h), so the reference's
own Python front end (ggml_compiler.runtime.Session, ggml_compiler.llm.Generator) drives it when
$GGML_COMPILER_RT names it. This module is this repository's own, smaller binding, used by the
tests, the benchmark and smoke(): a `Model` owns one loaded program; each of its entry points is an
`Entry` that uploads host arrays, runs, and fetches the results; the backend's extensions (device
timing, per-kernel statistics, tensor parallelism) are methods of `Model`.

The library is looked up in $GGML_COMPILER_RT, else in the in-tree build (ggml_compiler_b200/lib/).
There is no CPU fallback: without a B200 the library still encodes weights, but loading fails.
"""

from __future__ import annotations

import ctypes as C
import json
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable

import numpy as np

LIB_NAME = "libggml_compiler_rt.so"
BACKEND_CUDA = 1  # ggml_compiler_backend: CPU 0, CUDA 1, AUTO 2
_NP_OF_DTYPE = (np.float32, np.float16, np.int32)  # ggml_compiler_dtype F32, F16, I32


class BackendError(RuntimeError):
    """A call into libggml_compiler_rt returned an error; the message is the library's."""


# Layouts of the ABI's structs (include/ggml_compiler_rt.h).
class COptions(C.Structure):
    _fields_ = [("backend", C.c_int), ("device", C.c_int), ("n_threads", C.c_int), ("allow_cpu_fallback", C.c_bool)]


class CTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int), ("shape", C.c_int64 * 8),
                ("nbytes", C.c_size_t)]


class CStats(C.Structure):
    _fields_ = [("ms_total", C.c_double), ("n_calls", C.c_int)]


def _prototypes() -> dict[str, tuple[Any, list[Any]]]:
    """name -> (result type, argument types) for every exported function this module calls."""
    vp, i32, i64, sz, s = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_char_p
    P = C.POINTER
    proto: dict[str, tuple[Any, list[Any]]] = {
        "version": (s, []), "last_error": (s, []), "default_options": (COptions, []), "has_backend": (C.c_bool, [i32]),
        "load": (vp, [s, P(COptions)]), "load_with": (vp, [s, P(COptions), vp, i32]), "free": (None, [vp]),
        "quantize": (sz, [s, vp, i64, i64, vp, sz]), "row_size": (sz, [s, i64]),
        "backend_name": (s, [vp]), "metadata": (s, [vp, s]),
        "n_inputs": (i32, [vp]), "n_outputs": (i32, [vp]),
        "input_info": (i32, [vp, i32, P(CTensorInfo)]), "output_info": (i32, [vp, i32, P(CTensorInfo)]),
        "n_entries": (i32, [vp]), "entry_name": (s, [vp, i32]),
        "entry_n_inputs": (i32, [vp, i32]), "entry_n_outputs": (i32, [vp, i32]),
        "entry_input_info": (i32, [vp, i32, i32, P(CTensorInfo)]),
        "entry_output_info": (i32, [vp, i32, i32, P(CTensorInfo)]),
        "run_entry": (i32, [vp, s]), "run": (i32, [vp]), "reset": (i32, [vp]),
        "n_symbols": (i32, [vp]), "symbol_info": (i32, [vp, i32, P(s), P(i64), P(i64), P(i64)]),
        "set_symbol": (i32, [vp, s, i64]), "set_input_shape": (i32, [vp, s, i32, P(i64)]),
        "set_input": (i32, [vp, s, vp, sz]), "get_output": (i32, [vp, s, vp, sz]),
        "last_stats": (i32, [vp, P(CStats)]), "n_stages": (i32, [vp]),
        "stage_stats": (i32, [vp, i32, P(s), P(C.c_double), P(i32)]),
        # this backend's extensions (include/ggml_compiler_b200.h)
        "b200_stream": (vp, [vp]), "b200_last_device_ms": (C.c_double, [vp]), "b200_set_profiling": (i32, [vp, i32]),
        "b200_n_kernel_stats": (i32, [vp]),
        "b200_kernel_stats": (i32, [vp, i32, P(s), P(C.c_double), P(i32), P(C.c_double)]),
        "b200_tp_init": (i32, [vp, i32, i32, sz, vp, sz]), "b200_tp_connect": (i32, [vp, vp, sz]),
        "b200_value_bytes": (i64, [vp, s]), "b200_read_value": (i32, [vp, s, vp, sz]),
        "b200_write_value": (i32, [vp, s, vp, sz]),
        "b200_seq_slots": (i32, [vp, i32]), "b200_seq_copy": (i32, [vp, i32, i32]),
        "b200_decode_batch": (i32, [vp, s, i32, vp, vp, vp, vp]),
        "b200_generate_batch": (i32, [vp, s, i32, vp, vp, i32, vp]),
    }
    return {"ggml_compiler_" + k: v for k, v in proto.items()}


_LIB: C.CDLL | None = None


def library_path() -> Path:
    if os.environ.get("GGML_COMPILER_RT"):
        return Path(os.environ["GGML_COMPILER_RT"])
    built = Path(__file__).resolve().parent / "lib" / LIB_NAME
    if not built.exists():
        raise FileNotFoundError(f"{built} is missing: build it with `python -m ggml_compiler_b200.build`")
    return built


def load_library() -> C.CDLL:
    """The product library with every prototype bound (loaded once per process)."""
    global _LIB
    if _LIB is None:
        handle = C.CDLL(str(library_path()))
        for name, (res, args) in _prototypes().items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _LIB = handle
    return _LIB


_RETURNS_HANDLE = ("load", "entry_name", "backend_name")


def _call(fn: str, *args: Any) -> Any:
    """Calls ggml_compiler_<fn>. A negative int result, or NULL from a function that returns a
    handle or a name, is the library's error convention and becomes a BackendError."""
    out = getattr(load_library(), "ggml_compiler_" + fn)(*args)
    failed = out is None if fn in _RETURNS_HANDLE else type(out) is int and out < 0
    if failed:
        raise BackendError(load_library().ggml_compiler_last_error().decode())
    return out


def version() -> str:
    return load_library().ggml_compiler_version().decode()


def cuda_available() -> bool:
    return bool(load_library().ggml_compiler_has_backend(BACKEND_CUDA))


def encoded_row_bytes(type_name: str, n: int) -> int:
    """Bytes of one row of `n` values encoded as `type_name` (0 if the type cannot hold it)."""
    return int(load_library().ggml_compiler_row_size(type_name.encode(), n))


def encode(values: np.ndarray, type_name: str) -> np.ndarray:
    """Rows (the last axis) of f32 values in a ggml block format, through the library's encoder:
    uint8 [..., encoded_row_bytes]."""
    x = np.ascontiguousarray(values, np.float32)
    width = encoded_row_bytes(type_name, x.shape[-1])
    if not width:
        raise BackendError(load_library().ggml_compiler_last_error().decode())
    out = np.empty(x.shape[:-1] + (width,), np.uint8)
    if not load_library().ggml_compiler_quantize(type_name.encode(), x.ctypes.data, x.size // x.shape[-1],
                                                 x.shape[-1], out.ctypes.data, out.nbytes):
        raise BackendError(load_library().ggml_compiler_last_error().decode())
    return out


@dataclass(frozen=True)
class Port:
    """An input or output of an entry point, at the program's current symbol binding."""

    name: str
    dtype: Any
    shape: tuple[int, ...]
    nbytes: int

    @staticmethod
    def of(info: CTensorInfo) -> "Port":
        return Port(info.name.decode(), np.dtype(_NP_OF_DTYPE[info.dtype]), tuple(info.shape[: info.ndim]), info.nbytes)


class Entry:
    """One entry point of a loaded program (prefill, decode, generate, ...)."""

    def __init__(self, model: "Model", index: int) -> None:
        self.model, self.index = model, index
        self.name = _call("entry_name", model.handle, index).decode()

    def _ports(self, outputs: bool) -> list[Port]:
        h, e = self.model.handle, self.index
        count = _call("entry_n_outputs" if outputs else "entry_n_inputs", h, e)
        ports = []
        for k in range(count):
            info = CTensorInfo()
            _call("entry_output_info" if outputs else "entry_input_info", h, e, k, C.byref(info))
            ports.append(Port.of(info))
        return ports

    @property
    def inputs(self) -> list[Port]:
        return self._ports(False)

    @property
    def outputs(self) -> list[Port]:
        """The outputs at the binding in force now (after the inputs of a run were uploaded)."""
        return self._ports(True)

    def upload(self, arrays: dict[str, Any]) -> None:
        """Copies every input of this entry from host arrays; symbolic dims bind from their shapes."""
        ports = self.inputs
        given, wanted = set(arrays), {p.name for p in ports}
        if given != wanted:
            raise KeyError(f"entry {self.name} takes {sorted(wanted)}, got {sorted(given)}")
        host = {p.name: np.ascontiguousarray(np.asarray(arrays[p.name]), p.dtype) for p in ports}
        h = self.model.handle
        if self.model.symbol_range:
            for name, a in host.items():
                dims = (C.c_int64 * max(1, a.ndim))(*a.shape)
                _call("set_input_shape", h, name.encode(), a.ndim, dims)
        for name, a in host.items():
            _call("set_input", h, name.encode(), a.ctypes.data, a.nbytes)

    def launch(self) -> None:
        _call("run_entry", self.model.handle, self.name.encode())

    def fetch(self) -> dict[str, np.ndarray]:
        out = {}
        for p in self.outputs:
            y = np.empty(p.shape, p.dtype)
            _call("get_output", self.model.handle, p.name.encode(), y.ctypes.data, y.nbytes)
            out[p.name] = y
        return out

    def __call__(self, **arrays: Any) -> dict[str, np.ndarray]:
        self.upload(arrays)
        self.launch()
        return self.fetch()


class Model:
    """A ggml-compiler GGUF loaded on one B200 (ggml_compiler_load with the CUDA backend)."""

    def __init__(self, path: str | os.PathLike, device: int = 0) -> None:
        opts = load_library().ggml_compiler_default_options()
        opts.backend, opts.device = BACKEND_CUDA, device
        self.handle = _call("load", os.fsencode(path), C.byref(opts))
        self.path = Path(path)
        self.entries = {e.name: e for e in (Entry(self, k) for k in range(_call("n_entries", self.handle)))}
        self.symbol_range: dict[str, tuple[int, int]] = {}
        for k in range(_call("n_symbols", self.handle)):
            name, lo, hi = C.c_char_p(), C.c_int64(), C.c_int64()
            _call("symbol_info", self.handle, k, C.byref(name), C.byref(lo), C.byref(hi), None)
            self.symbol_range[name.value.decode()] = (lo.value, hi.value)

    # -- the program ------------------------------------------------------------------------------
    @property
    def backend(self) -> str:
        return _call("backend_name", self.handle).decode()

    @property
    def meta(self) -> dict[str, Any]:
        """The program's own metadata (GGUF key ggml_compiler.meta), {} if it has none."""
        raw = load_library().ggml_compiler_metadata(self.handle, b"ggml_compiler.meta")
        return json.loads(raw) if raw else {}

    def symbols(self) -> dict[str, int]:
        vals = {}
        for k, name in enumerate(self.symbol_range):
            v = C.c_int64()
            _call("symbol_info", self.handle, k, None, None, None, C.byref(v))
            vals[name] = v.value
        return vals

    def bind(self, **values: int) -> None:
        """Binds symbols that no input shape fixes (a loop's trip count `max_new`)."""
        for name, v in values.items():
            _call("set_symbol", self.handle, name.encode(), int(v))

    def clear_state(self) -> None:
        """Zeroes the program's state values (the KV cache)."""
        _call("reset", self.handle)

    def stage_calls(self) -> dict[str, int]:
        """Calls of each stage in the last entry run (a device loop's iterations, for one)."""
        out = {}
        for k in range(_call("n_stages", self.handle)):
            name, ms, n = C.c_char_p(), C.c_double(), C.c_int()
            _call("stage_stats", self.handle, k, C.byref(name), C.byref(ms), C.byref(n))
            out[name.value.decode()] = n.value
        return out

    def wall_ms(self) -> float:
        st = CStats()
        _call("last_stats", self.handle, C.byref(st))
        return st.ms_total

    # -- this backend's extensions ---------------------------------------------------------------------
    @property
    def stream(self) -> int:
        """The cudaStream_t (as an int) of every launch of this model."""
        return int(_call("b200_stream", self.handle) or 0)

    @property
    def device_ms(self) -> float:
        """Device time of the last entry run: CUDA events on the model's stream around its launches."""
        return float(_call("b200_last_device_ms", self.handle))

    def profile(self, on: bool) -> None:
        """On: every launch timed on its own (synchronised, no CUDA graphs); the statistics restart."""
        _call("b200_set_profiling", self.handle, int(bool(on)))

    def kernel_table(self) -> dict[str, dict[str, float]]:
        """Per kernel family since profiling was switched on: ms, launches, algorithmic bytes."""
        table = {}
        for k in range(_call("b200_n_kernel_stats", self.handle)):
            name, ms, n, b = C.c_char_p(), C.c_double(), C.c_int(), C.c_double()
            _call("b200_kernel_stats", self.handle, k, C.byref(name), C.byref(ms), C.byref(n), C.byref(b))
            table[name.value.decode()] = {"ms": ms.value, "launches": n.value, "bytes": b.value}
        return table

    def read_value(self, name: str) -> np.ndarray:
        """The whole device storage of value `name` (a KV cache, for one) as bytes."""
        out = np.empty(int(_call("b200_value_bytes", self.handle, name.encode())), np.uint8)
        _call("b200_read_value", self.handle, name.encode(), out.ctypes.data, out.nbytes)
        return out

    def write_value(self, name: str, data: np.ndarray) -> None:
        """Overwrites the whole device storage of value `name` with `data`'s bytes."""
        a = np.ascontiguousarray(data)
        _call("b200_write_value", self.handle, name.encode(), a.ctypes.data, a.nbytes)

    # ---- batched decode (several sequences per decode step; include/ggml_compiler_b200.h)

    def seq_slots(self, n: int) -> None:
        """Gives the model n (1..16) sequence slots, each a zeroed copy of its state (the KV caches)."""
        _call("b200_seq_slots", self.handle, n)

    def seq_copy(self, dst: int, src: int) -> None:
        """Copies the whole state from slot src to slot dst; -1 is the model's own state (the one the
        entries use)."""
        _call("b200_seq_copy", self.handle, dst, src)

    def decode_batch(self, tokens: Any, positions: Any, entry: str = "decode") -> tuple[np.ndarray, np.ndarray]:
        """One decode step for the sequences in slots 0..n-1: token i at position i of sequence i.
        Returns (logits [n, vocab], greedy tokens [n])."""
        tok = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(-1))
        pos = np.ascontiguousarray(np.asarray(positions, np.int32).reshape(-1))
        if tok.shape != pos.shape:
            raise ValueError("one position per token")
        n = tok.size
        vocab = self._vocab()
        logits = np.empty((n, vocab), np.float32)
        nxt = np.empty(n, np.int32)
        _call("b200_decode_batch", self.handle, entry.encode(), n, tok.ctypes.data, pos.ctypes.data, logits.ctypes.data,
              nxt.ctypes.data)
        return logits, nxt

    def generate_batch(self, first: Any, start: Any, steps: int, entry: str = "decode") -> np.ndarray:
        """`steps` greedy steps for the sequences in slots 0..n-1 from token first[i] at position
        start[i], each step's tokens fed back on the device. Returns the tokens [steps, n]."""
        f = np.ascontiguousarray(np.asarray(first, np.int32).reshape(-1))
        st = np.ascontiguousarray(np.asarray(start, np.int32).reshape(-1))
        if f.shape != st.shape:
            raise ValueError("one start position per sequence")
        out = np.empty((steps, f.size), np.int32)
        _call("b200_generate_batch", self.handle, entry.encode(), f.size, f.ctypes.data, st.ctypes.data, steps,
              out.ctypes.data)
        return out

    def _vocab(self) -> int:
        """Rows of the decode entry's logits output."""
        if getattr(self, "_vocab_rows", None) is None:
            e = self.entries["decode"]
            self._vocab_rows = int(np.prod(e.outputs[0].shape))
        return self._vocab_rows

    def join_tensor_parallel(self, rank: int, world: int, all_gather: Callable[[bytes], list[bytes]],
                             window_bytes: int = 0) -> None:
        """Makes this process rank `rank` of `world` (one GPU each, every rank with the same program
        loaded): exports this rank's exchange window, gathers every rank's handle with `all_gather`
        (bytes -> list of every rank's bytes, rank order) and maps the peers' windows. Every rank
        must then make the same entry runs; results equal one GPU's."""
        buf = C.create_string_buffer(256)
        n = _call("b200_tp_init", self.handle, rank, world, window_bytes, buf, len(buf))
        joined = joined_handles(buf.raw[:n], rank, world, all_gather)
        _call("b200_tp_connect", self.handle, joined, len(joined))

    def close(self) -> None:
        if getattr(self, "handle", None):
            load_library().ggml_compiler_free(self.handle)
            self.handle = None

    def __enter__(self) -> "Model":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()

    def __del__(self) -> None:
        self.close()


def joined_handles(mine: bytes, rank: int, world: int, all_gather: Callable[[bytes], list[bytes]]) -> bytes:
    """Every rank's exchange-window handle in rank order, concatenated; checks what came back."""
    every = [bytes(b) for b in all_gather(bytes(mine))]
    if len(every) != world or every[rank] != mine or len({len(b) for b in every}) != 1:
        raise ValueError(f"all_gather must return {world} handles of one size in rank order, "
                         f"this rank's ({rank}) at its place")
    return b"".join(every)


def torch_all_gather(group: Any = None) -> Callable[[bytes], list[bytes]]:
    """An all_gather of bytes over an initialised torch.distributed process group."""
    import torch.distributed as dist

    def gather(b: bytes) -> list[bytes]:
        got: list[Any] = [None] * dist.get_world_size(group)
        dist.all_gather_object(got, b, group=group)
        return got

    return gather
