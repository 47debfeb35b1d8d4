"""The library's flop counter (phyz_b200/csrc/flops.cpp, the kernel's own
step code run on the host with a counting scalar) built for the host:

* a rollout counted from real states with the ground far below (no contact
  force) equals the steady-state count of one world-step that the roofline
  has used (phyzb_flops_per_world_step), for C1-C4;
* counted as a model-specialized kernel executes (products with zero table
  constants left out), every config does less work than the generic count;
* with the feet on the ground the count grows by the contact force law."""
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
    so = tmp_path_factory.mktemp("flops") / "flops_host.so"
    subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", "-I", str(ROOT / "phyz_b200" / "csrc"), "-I",
                    str(ROOT / "include"), str(ROOT / "tests" / "cpp" / "flops_host.cpp"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.host_flops.argtypes = [C.c_void_p, C.c_int, C.c_double, C.c_double, C.c_double, C.c_double, C.c_int, D, D,
                               D, C.c_longlong, C.c_int, C.c_int, D]
    return lib


def count(lib, name, ground=None, specialized=False, steps=50, n=8, q0=None):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    cm, keep = m.to_c()
    if q0 is None:
        q0, v0 = configs.initial_state(name, m, range(n))
    else:
        v0 = np.zeros_like(q0)
    sched = np.ascontiguousarray(configs.control_schedule(name, m, range(n), steps))
    contact = 1 if cfg.contact else 0
    k, d = (cfg.contact[1], cfg.contact[2]) if cfg.contact else (0.0, 0.0)
    out = np.zeros(2)
    dp = lambda a: a.ctypes.data_as(D)  # noqa: E731
    if ground is None:  # the per-step count of the roofline
        lib.host_flops(C.addressof(cm), contact, k, d, 0.0, 1.0, 16, None, None, None, 0, 0, 0, dp(out))
    else:
        lib.host_flops(C.addressof(cm), contact, k, d, ground, 1.0, 16, dp(np.ascontiguousarray(q0)),
                       dp(np.ascontiguousarray(v0)), dp(sched), q0.shape[0], steps, int(specialized), dp(out))
    return out


@pytest.mark.parametrize("name", list(configs.CONFIGS))
def test_rollout_count_without_contact_force_equals_step_count(lib, name):
    per_step = count(lib, name)
    rolled = count(lib, name, ground=-1e9)
    # equal up to the few state-dependent branches (small-angle forms of the
    # exp/log maps) a real trajectory takes
    assert rolled[0] == pytest.approx(per_step[0], rel=1e-3)
    spec = count(lib, name, ground=-1e9, specialized=True)
    assert 0.5 * per_step[0] < spec[0] < per_step[0]


def test_contact_force_law_is_counted_where_feet_touch(lib):
    m = configs.quadruped()
    n = 8
    q0, _ = configs.initial_state("c3_quadruped", m, range(n))
    q0[:, 5] = 0.42  # feet pressed into the ground
    q0[:, 6:] = 0.0
    far = count(lib, "c3_quadruped", ground=-1e9, q0=q0, n=n)
    touching = count(lib, "c3_quadruped", ground=0.0, q0=q0, n=n)
    assert touching[0] > far[0] + 4 * 10  # four feet, tens of flops each
