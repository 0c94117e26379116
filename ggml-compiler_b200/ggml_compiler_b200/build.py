"""Build libggml_compiler_rt.so (the B200 backend) in-tree with nvcc for sm_100a.

    python -m ggml_compiler_b200.build          # from ggml-compiler_b200/, or via __graft_entry__.build()

Objects go to ggml-compiler_b200/_build/ (rebuilt when a source or header changes); the library to
ggml-compiler_b200/ggml_compiler_b200/lib/libggml_compiler_rt.so.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # ggml-compiler_b200/
REPO = ROOT.parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "lib" / "libggml_compiler_rt.so"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: no multiply-add contraction, so every kernel rounds exactly as its source says.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
              "-DGGML_COMPILER_RT_BUILD", f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cpp"), *CSRC.glob("*.cu"), *CSRC.glob("kernels/*.cu")])


def _headers_mtime() -> float:
    hs = [*CSRC.glob("*.h"), *CSRC.glob("kernels/*.cuh"), *CSRC.glob("kernels/*.h"), *INCLUDE.glob("*.h")]
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, hdr_time: float, extra: list[str]) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "_") + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if os.environ.get("GCB_PTXAS_VERBOSE"):
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    hdr = _headers_mtime()
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, hdr, extra or []), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
