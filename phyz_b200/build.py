"""Build recipe of libphyzb200.so (the C-ABI stepper) for sm_100a.

The library is built in-tree (phyz_b200/libphyzb200.so) with nvcc directly:
the CUDA sources and the host C++ of the C ABI link into one shared object
with the CUDA runtime linked statically, so the object has no dependency on
torch and can be loaded by any host (ctypes, a Rust FFI crate, C++).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libphyzb200.so"
SOURCES = ["stepper.cu", "capi.cu", "flops.cpp", "peaks.cu"]
HEADERS = ["pz_types.cuh", "pz_model.cuh", "pz_world.cuh", "pz_launch.h", "pz_pack.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / s for s in SOURCES + HEADERS] + [PKG.parent / "include" / "phyzb.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [
        nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-Wno-unknown-pragmas", "-o", str(LIB) + ".tmp",
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
