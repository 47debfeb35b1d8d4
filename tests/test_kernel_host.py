"""The rollout kernel's source checked against the oracle on the CPU.

tests/cpp/kernel_host.cpp compiles the kernel's own step functions
(pz_world.cuh) for the host in f64 and steps worlds one at a time. Built as
the generic kernel evaluates them, and with PZ_KSKIP, where every product
with a zero model-table constant is left out the way a model-specialized
kernel leaves it out at compile time: both match the f64 oracle on C1-C4
(penalty contact where the config has it) over 100 steps, and each other.
No GPU is involved; the device kernels themselves are checked by the -m gpu
tests."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np
import pytest

from phyz_b200 import configs

ROOT = Path(__file__).resolve().parents[1]
D = C.POINTER(C.c_double)
NAMES = ["c1_double_pendulum", "c2_chain32", "c3_quadruped", "c4_humanoid"]


@pytest.fixture(scope="module")
def kernels(tmp_path_factory):
    out = {}
    d = tmp_path_factory.mktemp("kernel_host")
    for tag, flags in (("generic", []), ("kskip", ["-DPZ_KSKIP=1"])):
        so = d / f"kernel_host_{tag}.so"
        subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", *flags,
                        "-I", str(ROOT / "phyz_b200" / "csrc"), str(ROOT / "tests" / "cpp" / "kernel_host.cpp"),
                        "-o", str(so)], check=True)
        lib = C.CDLL(str(so))
        lib.host_rollout.argtypes = [C.c_void_p, C.c_int, D, D, D, C.c_int, C.c_int, C.c_double, C.c_double,
                                     C.c_double, C.c_double, C.c_int]
        lib.host_set_heightfield.argtypes = [C.c_int, C.c_int, C.c_double, C.c_double, C.c_double, C.c_double,
                                             C.POINTER(C.c_float)]
        out[tag] = lib
    return out


def host_run(lib, name, n=16, steps=100, impulse=False):
    cfg = configs.CONFIGS[name]
    m = cfg.builder()
    q0, v0 = configs.initial_state(name, m, range(n))
    if impulse:  # root heights at which the feet stand on the ground through the run
        lo, hi = {"c3_quadruped": (0.45, 0.6), "c4_humanoid": (0.9, 1.05)}[name]
        q0[:, 5] = np.linspace(lo, hi, n)
    c = 0.5 * np.random.default_rng(1).standard_normal((n, m.nv)) * configs.actuated(m)
    cm, keep = m.to_c()
    q, v = q0.copy(), v0.copy()
    dp = lambda a: a.ctypes.data_as(D)  # noqa: E731
    contact = cfg.contact is not None
    mode = 2 if impulse else int(contact)
    feat = lib.host_rollout(C.addressof(cm), n, dp(q), dp(v), dp(np.ascontiguousarray(c)), steps, mode,
                            0.0, 1.0, 1e4, 100.0, 16)
    assert feat >= 0
    return m, q0, v0, c, contact, q, v


@pytest.mark.parametrize("name", NAMES)
def test_kernel_source_matches_oracle(kernels, oracle, name):
    runs = {tag: host_run(lib, name) for tag, lib in kernels.items()}
    m, q0, v0, c, contact, _, _ = runs["generic"]
    gains = (0.0, 1.0, [1e4] * m.nbodies, [100.0] * m.nbodies) if contact else None
    qo, vo, _, _ = oracle.rollout(m, q0, v0, c, nsteps=100, contact=gains, nthreads=4)
    for tag, (_, _, _, _, _, q, v) in runs.items():
        assert np.all(np.isfinite(q)) and np.all(np.isfinite(v)), tag
        np.testing.assert_allclose(q, qo, rtol=0, atol=1e-11, err_msg=tag)
        np.testing.assert_allclose(v, vo, rtol=0, atol=1e-10, err_msg=tag)
    np.testing.assert_allclose(runs["kskip"][5], runs["generic"][5], rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", ["c3_quadruped", "c4_humanoid"])
def test_kernel_source_impulse_matches_oracle(kernels, oracle, name):
    """Impulse mode (16 sweeps per step, the kept backward state and the
    wrench responses): the kernel source against the oracle's full re-sweep
    formulation, from a cold start, with the feet on the ground."""
    runs = {tag: host_run(lib, name, impulse=True) for tag, lib in kernels.items()}
    m, q0, v0, c, _, _, _ = runs["generic"]
    qo, vo, _, _, _ = oracle.rollout_impulse(m, q0, v0, c, nsteps=100, contact=(0.0, 1.0), sweeps=16, nthreads=4)
    for tag, (_, _, _, _, _, q, v) in runs.items():
        assert np.all(np.isfinite(q)) and np.all(np.isfinite(v)), tag
        # the staged law is discontinuous (friction clamp, margin): rounding
        # may send a world down another branch, as in the GPU impulse tests
        ok = np.max(np.abs(q - qo), axis=1) < 1e-8
        assert ok.mean() >= 0.9, (tag, ok.mean(), np.abs(q - qo).max())


def test_kernel_source_terrain_matches_oracle(kernels, oracle):
    """Penalty contact over a heightfield (full world frames, bilinear
    terrain and its gradient normal): the kernel source against the oracle
    on the quadruped walking over bumps."""
    from phyz_b200 import Heightfield

    rng = np.random.default_rng(3)
    hf = Heightfield.new((-2.0, -2.0, -0.05), 0.25, 17, 17)
    hf.heights[:] = (0.08 * rng.standard_normal(17 * 17)).astype(np.float32)
    h = np.ascontiguousarray(hf.heights, np.float32)
    try:
        for lib in kernels.values():
            lib.host_set_heightfield(17, 17, *hf.origin, hf.cell, h.ctypes.data_as(C.POINTER(C.c_float)))
        runs = {tag: host_run(lib, "c3_quadruped") for tag, lib in kernels.items()}
        m, q0, v0, c, _, _, _ = runs["generic"]
        oracle.set_heightfield(hf)
        qo, vo, _, _ = oracle.rollout(m, q0, v0, c, nsteps=100, contact=(0.0, 1.0, [1e4] * m.nbodies,
                                                                         [100.0] * m.nbodies), nthreads=4)
    finally:
        oracle.set_heightfield(None)
        for lib in kernels.values():
            lib.host_set_heightfield(0, 0, 0.0, 0.0, 0.0, 1.0, None)
    for tag, (_, _, _, _, _, q, v) in runs.items():
        assert np.all(np.isfinite(q)) and np.all(np.isfinite(v)), tag
        np.testing.assert_allclose(q, qo, rtol=0, atol=1e-10, err_msg=tag)
