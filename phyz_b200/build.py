"""Build recipe of libphyzb200.so (the C-ABI stepper) for sm_100a.

The library is built in-tree (phyz_b200/libphyzb200.so) with nvcc directly:
the CUDA sources and the host C++ of the C ABI link into one shared object
with the CUDA runtime linked statically, so the object has no dependency on
torch and can be loaded by any host (ctypes, a Rust FFI crate, C++).

The rollout kernel has one instantiation per (precision, feature set);
rollout_variants.cu is compiled once per pair and every object compiles in
parallel (objects under phyz_b200/_build/).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libphyzb200.so"
OBJ = PKG / "_build"
SOURCES = ["stepper.cu", "capi.cu", "capi_policy.cu", "capi_train.cu", "policy.cu", "train.cu", "flops.cpp",
           "peaks.cu", "capi_noalloc.cu"]
VARIANT_SOURCE = "rollout_variants.cu"
FEAT_COUNT = 64  # pz_variants.h; bit 8 only with bit 4, bits 16 and 32 only with bit 2 (feat_valid)
VARIANTS = [(t, f) for t in ("float", "double") for f in range(FEAT_COUNT)
            if not (f & 8 and not f & 4) and not (f & 16 and not f & 2) and not (f & 32 and not f & 2)]
HEADERS = ["pz_types.cuh", "pz_model.cuh", "pz_world.cuh", "pz_launch.h", "pz_pack.h", "pz_variants.h",
           "stepper_kernels.cuh", "pz_policy.h", "capi_internal.h", "pz_mlp.cuh", "pz_train.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wno-unknown-pragmas"]


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


def _jobs() -> list[tuple[Path, list[str]]]:
    jobs = []
    for s in SOURCES:
        jobs.append((OBJ / (s + ".o"), [str(CSRC / s)]))
    for t, f in VARIANTS:
        jobs.append((OBJ / f"rollout_{t}_{f}.o", [f"-DPZ_VARIANT_T={t}", f"-DPZ_VARIANT_FEAT={f}",
                                                  str(CSRC / VARIANT_SOURCE)]))
    return jobs


def build(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / s for s in SOURCES + HEADERS + [VARIANT_SOURCE]] + [PKG.parent / "include" / "phyzb.h"]
    if not force and not _stale(LIB, deps):
        return LIB
    OBJ.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(job):
        out, args = job
        cmd = [cc, *ARCH, *FLAGS, "-c", "-o", str(out), *args]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        return out, cmd, r

    workers = max(1, min(len(_jobs()), os.cpu_count() or 1))
    with ThreadPoolExecutor(workers) as ex:
        results = list(ex.map(compile_one, _jobs()))
    failed = False
    for out, cmd, r in results:
        if verbose or r.returncode != 0:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        failed = failed or r.returncode != 0
    if failed:
        raise RuntimeError("nvcc failed (see above)")
    link = [cc, *ARCH, "-shared", "-o", str(LIB) + ".tmp", *[str(o) for o, _, _ in results]]
    subprocess.run(link, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
