"""The rollout launch planner on the host (no GPU): the tile shape and the
slice-mode shape that pz::pick_launch derives from a layout's scratch words,
Tensor-Memory columns and a kernel's registers, and pz::plan_slices' choice
between tile mode and slice mode (and its run length) for a launch, against
the numbers worked out by hand for the configs the bench runs.

* C2 f32 (96 shared-memory words and 256 Tensor-Memory columns per world,
  206 registers): tile blocks of 224 worlds (1.98 waves of 65536 worlds run
  as 2), slice shape 256 worlds (8 warps, still 2 per SM sub-partition);
  65536 x 1000 runs in slice mode as 4 runs of 250 steps (7 rounds of jobs:
  1757 step-times against 2000).
* C2 f64 (512 columns per world): 128-world blocks, 3.46 waves; 2 runs of 500
  steps (3507 against 4000).
* One wave of worlds, one step, PHYZB_SLICES=0, a variant without slice mode
  and a job count past the 32-bit queue counter all stay in tile mode;
  PHYZB_SLICES=1 runs a launch in runs of a third of its steps."""
import ctypes as C
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = tmp_path_factory.mktemp("plan_host") / "plan_host.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", str(ROOT / "phyz_b200" / "csrc"), "-I",
                    str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(ROOT / "tests" / "cpp" / "plan_host.cpp"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.plan_host.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_int,
                              C.c_int, C.POINTER(C.c_int)]
    return lib


def plan(lib, *, tm=1, esz=4, scratch=96, model_bytes=12288, nworld=65536, tmem_cols=256, regs=206,
         can_slice=1, nsteps=1000, force=-1):
    out = (C.c_int * 8)()
    assert lib.plan_host(tm, esz, scratch, model_bytes, nworld, tmem_cols, regs, can_slice, nsteps, force, out) == 0
    return dict(zip(("W", "grid", "blocks", "slice_W", "slice_grid", "chunk", "run_W", "run_grid"), list(out)))


def test_c2_f32_headline(lib, monkeypatch):
    monkeypatch.delenv("PHYZB_WORLDS_PER_BLOCK", raising=False)
    p = plan(lib)
    assert (p["W"], p["grid"], p["blocks"]) == (224, 148, 1), p
    assert (p["slice_W"], p["slice_grid"]) == (256, 148), p
    assert (p["chunk"], p["run_W"], p["run_grid"]) == (250, 256, 148), p


def test_c2_f64(lib, monkeypatch):
    monkeypatch.delenv("PHYZB_WORLDS_PER_BLOCK", raising=False)
    p = plan(lib, esz=8, tmem_cols=512, regs=255)
    assert (p["W"], p["slice_W"]) == (128, 128), p
    assert p["chunk"] == 500, p


def test_tile_mode_cases(lib, monkeypatch):
    monkeypatch.delenv("PHYZB_WORLDS_PER_BLOCK", raising=False)
    assert plan(lib, nworld=4096)["chunk"] == 0  # one wave: nothing to share
    assert plan(lib, nsteps=1)["chunk"] == 0
    assert plan(lib, force=0)["chunk"] == 0
    p = plan(lib, can_slice=0)
    assert p["slice_W"] == 0 and p["chunk"] == 0, p
    # a job count past the 32-bit queue counter
    assert plan(lib, nworld=1 << 36)["chunk"] == 0


def test_forced_runs(lib, monkeypatch):
    monkeypatch.delenv("PHYZB_WORLDS_PER_BLOCK", raising=False)
    # 300 worlds: 32-world tile blocks on 10 SMs (one warp per SM), so the
    # slice shape is 4 warps; the 10 warp tiles need 3 such blocks
    p = plan(lib, nworld=300, nsteps=12, force=1)
    assert (p["W"], p["grid"]) == (32, 10), p
    assert p["chunk"] == 4 and p["run_W"] == 128 and p["run_grid"] == 3, p
    assert plan(lib, nworld=300, nsteps=2, force=1)["chunk"] == 1
    assert plan(lib, nworld=300, nsteps=10000, force=1)["chunk"] == 512


def test_slice_shape_keeps_warps_per_scheduler(lib, monkeypatch):
    """The slice shape never puts more warps on an SM sub-partition than the
    tile shape: a tile block of 4 warps (1 per sub-partition) gets a 4-warp
    slice shape even where 8 would fit."""
    monkeypatch.setenv("PHYZB_WORLDS_PER_BLOCK", "128")
    p = plan(lib)
    assert p["W"] == 128 and p["slice_W"] == 128, p
