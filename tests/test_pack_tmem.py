"""Tensor-Memory records in the packed scratch layout (pz_pack.h), on the
host: with a budget, every relabelled hinge gets an 8-column record (16 in
f64) and, when they fit beside those, every collidable body's contact
wrench too (its shared-memory slots are then not allocated); records never
overlap and stay inside the budget; impulse contact and a body plane keep
the wrenches in shared memory; without a budget nothing moves.

C4 (humanoid, 10 contact shapes, 21 relabelled hinges): 272 shared
words per world without records; with a 256-column budget, 168 + 80 = 248
columns and 212 words. C3 (quadruped, 4 feet, 8 hinges): 64 + 32 = 96
columns and 130 words."""
import ctypes as C
import subprocess
from pathlib import Path

import pytest

from phyz_b200 import configs

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = tmp_path_factory.mktemp("pack_host") / "pack_host.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", str(ROOT / "phyz_b200" / "csrc"), "-I",
                    str(ROOT / "include"), str(ROOT / "tests" / "cpp" / "pack_host.cpp"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.pack_host.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]
    return lib


def pack(lib, name, contact=1, plane_body=-1, f64=0, budget=0):
    m = configs.CONFIGS[name].builder()
    cm, keep = m.to_c()
    out = (C.c_int * 6)()
    lib.pack_host(C.addressof(cm), m.nv, contact, plane_body, f64, budget, out)
    return dict(zip(("scratch", "tmem_cols", "t_f", "s_f", "t_rec", "top"), list(out)))


def test_humanoid_wrenches_join_the_hinge_records(lib):
    base = pack(lib, "c4_humanoid")
    assert base["tmem_cols"] == 0 and base["t_f"] == 0 and base["s_f"] == 10, base
    p = pack(lib, "c4_humanoid", budget=256)
    assert p["t_rec"] == 21 and p["t_f"] == 10 and p["s_f"] == 0, p
    assert p["tmem_cols"] == 21 * 8 + 10 * 8 == 248 and p["top"] == p["tmem_cols"] <= 256, p
    assert p["scratch"] == base["scratch"] - 21 * 8 - 10 * 6 == 212, (base, p)


def test_quadruped(lib):
    p = pack(lib, "c3_quadruped", budget=512)
    assert (p["t_rec"], p["t_f"], p["s_f"], p["tmem_cols"], p["scratch"]) == (8, 4, 0, 96, 130), p


def test_f64_records_are_16_columns(lib):
    p = pack(lib, "c4_humanoid", f64=1, budget=512)
    assert p["tmem_cols"] == 21 * 16 + 10 * 16 == 496 and p["top"] == 496, p
    # at 256 columns the hinges alone do not fit: no records at all
    q = pack(lib, "c4_humanoid", f64=1, budget=256)
    assert q["tmem_cols"] == 0 and q["t_f"] == 0 and q["t_rec"] == 0, q


def test_wrenches_stay_in_shared_memory(lib):
    # hinges fit but the wrenches would not: the hinges move, the wrenches stay
    p = pack(lib, "c4_humanoid", budget=170)
    assert p["t_rec"] == 21 and p["t_f"] == 0 and p["s_f"] == 10, p
    # impulse contact and a body plane keep them in shared memory
    for kw in ({"contact": 2}, {"plane_body": 0}):
        q = pack(lib, "c4_humanoid", budget=256, **kw)
        assert q["t_rec"] == 21 and q["t_f"] == 0 and q["s_f"] >= 10, (kw, q)
    # no contact: no wrenches anywhere
    n = pack(lib, "c4_humanoid", contact=0, budget=256)
    assert n["t_f"] == 0 and n["s_f"] == 0, n
