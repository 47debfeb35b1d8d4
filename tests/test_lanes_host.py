"""One world split over lanes (pz_lanes.h, pz_lanes_sweep.cuh), run on the
host in f64 by tests/cpp/lanes_host.cpp: each lane steps its sub-model (the
trunk, then its share of the limbs) with the kernel's own sweep functions,
and the limbs' contributions to trunk bodies are summed over the lanes where
the device uses warp shuffles. The result must be the oracle's (the split
changes only the order of those sums), for the quadruped and the humanoid
at 2, 4 and 8 lanes, with penalty contact; chains do not split. No GPU is
involved; tests/test_gpu_lanes.py runs the device kernel."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from phyz_b200 import configs

ROOT = Path(__file__).resolve().parents[1]
D = C.POINTER(C.c_double)


@pytest.fixture(scope="module")
def lib(tmp_path_factory):
    so = tmp_path_factory.mktemp("lanes_host") / "lanes_host.so"
    subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-I", str(ROOT / "phyz_b200" / "csrc"), "-I",
                    str(ROOT / "include"), str(ROOT / "tests" / "cpp" / "lanes_host.cpp"), "-o", str(so)],
                   check=True)
    lib = C.CDLL(str(so))
    lib.host_rollout_lanes.argtypes = [C.c_void_p, C.c_int, D, D, D, C.c_int, C.c_int, C.c_double, C.c_double,
                                       C.c_double, C.c_double, C.c_int]
    return lib


def run(lib, name, lanes, n=12, steps=100):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    q0, v0 = configs.initial_state(name, m, range(n))
    c = np.ascontiguousarray(0.5 * np.random.default_rng(3).standard_normal((n, m.nv)) * configs.actuated(m))
    cm, keep = m.to_c()
    q, v = q0.copy(), v0.copy()
    dp = lambda a: a.ctypes.data_as(D)  # noqa: E731
    contact = cfg.contact is not None
    nt = lib.host_rollout_lanes(C.addressof(cm), n, dp(q), dp(v), dp(c), steps, int(contact), 0.0, 1.0, 1e4, 100.0,
                                lanes)
    return m, q0, v0, c, contact, q, v, nt


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
@pytest.mark.parametrize("lanes", [2, 4, 8])
def test_lanes_match_oracle(lib, oracle, name, lanes):
    m, q0, v0, c, contact, q, v, nt = run(lib, name, lanes)
    assert nt == {"c3_quadruped": 1, "c4_humanoid": 3}[name]  # torso; pelvis, abdomen, chest
    gains = (0.0, 1.0, [1e4] * m.nbodies, [100.0] * m.nbodies) if contact else None
    qo, vo, _, _ = oracle.rollout(m, q0, v0, c, nsteps=100, contact=gains, nthreads=4)
    assert np.all(np.isfinite(q)) and np.all(np.isfinite(v))
    np.testing.assert_allclose(q, qo, rtol=0, atol=1e-10)
    np.testing.assert_allclose(v, vo, rtol=0, atol=1e-9)


@pytest.mark.parametrize("name", ["c1_double_pendulum", "c2_chain32"])
def test_chains_do_not_split(lib, name):
    assert run(lib, name, 4, n=2, steps=1)[-1] == -1
