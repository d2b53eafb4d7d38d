"""Compile the native library (CUDA kernels for sm_100a + the C++ engine + the
C ABI) in-tree into ``grande_b200/libomg_b200.so``.

    python -m grande_b200.build [-v] [--force]

Objects go to ``grande_b200/_build/``; a source is recompiled when it, or any
header in ``csrc/``, is newer than its object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "_build"
LIB = HERE / "libomg_b200.so"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(CSRC), "-I", str(INCLUDE)]
CU_FLAGS = ARCH + COMMON + ["-lineinfo", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
CXX_FLAGS = COMMON + ["-Xcompiler", "-pthread", "-Wno-deprecated-gpu-targets"]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = OUT / (src.name + ".o")
    if not force and obj.exists():
        if obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
            return obj
    flags = CU_FLAGS if src.suffix == ".cu" else CXX_FLAGS
    cmd = [NVCC, *flags, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"nvcc failed on {src.name}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-Xcompiler", "-pthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
