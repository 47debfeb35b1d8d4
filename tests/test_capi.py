"""The C-ABI library without a GPU: it loads, exports every entry point
include/phyzb.h declares, its structs match the header, and it reports the
absence of a device as an error instead of computing anything."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

from phyz_b200 import _lib, configs
from phyz_b200.batch_sim import BatchSim

HEADER = Path(__file__).resolve().parents[1] / "include" / "phyzb.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(phyzb_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_abi_version_and_struct_sizes():
    lib = _lib.load()
    assert lib.phyzb_abi_version() == 1
    # sizes of the C structs, counted from include/phyzb.h on LP64
    assert C.sizeof(_lib.PhyzbBody) == 8 + 8 * (1 + 3 + 6 + 9 + 3 + 3 + 4) + 8 + 8 * 5 + 8 + 8 * (6 + 3 + 9)
    assert C.sizeof(_lib.PhyzbModel) == 48
    assert C.sizeof(_lib.PhyzbPdDof) == 32


def test_no_device_is_an_error_not_a_fallback():
    lib = _lib.load()
    if lib.phyzb_device_count() > 0:
        pytest.skip("a device is present")
    with pytest.raises(_lib.PhyzbError) as e:
        BatchSim(configs.double_pendulum(), 8)
    assert e.value.code == _lib.ERR_NO_DEVICE


def test_invalid_models_are_rejected_before_device_use():
    lib = _lib.load()
    m = configs.double_pendulum()
    m.bodies[1].parent = 1  # not topological
    cm, keep = m.to_c()
    h = C.c_void_p()
    assert lib.phyzb_create(C.byref(cm), 4, 0, 1, C.byref(h)) == _lib.ERR_INVALID
    assert b"topological" in lib.phyzb_last_error()
    big = configs.chain(33)
    cm, keep = big.to_c()
    assert lib.phyzb_create(C.byref(cm), 4, 0, 1, C.byref(h)) == _lib.ERR_TOO_LARGE
    m = configs.double_pendulum()
    m.bodies[0].inertia.mass = float("nan")
    cm, keep = m.to_c()
    assert lib.phyzb_create(C.byref(cm), 4, 0, 1, C.byref(h)) == _lib.ERR_INVALID


def test_null_handle_is_an_error():
    lib = _lib.load()
    assert lib.phyzb_step(None, 1) == _lib.ERR_INVALID
    assert lib.phyzb_destroy(None) == _lib.PHYZB_OK


def test_reference_rng_stream():
    """world_seed / KernelRng restate policy_pipeline.rs:417-457: check the
    SplitMix64 mixing against a direct scalar evaluation."""
    from phyz_b200.rng import KernelRng, world_seed
    M = (1 << 64) - 1

    def ws(seed, w):
        z = (seed + 0x9E3779B97F4A7C15 * (w + 1)) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        z = z ^ (z >> 31)
        return z or 1

    assert [int(x) for x in world_seed(7, range(5))] == [ws(7, w) for w in range(5)]
    r = KernelRng(7, [3])
    x = ws(7, 3)
    for _ in range(4):
        x ^= (x << 13) & M
        x ^= x >> 7
        x ^= (x << 17) & M
        assert int(r.next_u64()[0]) == x
    u = KernelRng(1, np.arange(20000)).uniform()
    assert 0.49 < u.mean() < 0.51 and u.min() >= 0.0 and u.max() < 1.0
