"""The C++ host mirror (include/phyzb.hpp) compiles against the C ABI and
behaves like the reference's BatchSim: Err without a device, and on a
device a rollout equal to the f64 oracle's."""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def host_binary(tmp_path_factory):
    from phyz_b200 import build

    build.build()
    out = tmp_path_factory.mktemp("cpp") / "batchsim_host"
    lib_dir = ROOT / "phyz_b200"
    subprocess.run(["g++", "-std=c++17", "-O2", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "cpp" / "batchsim_host.cpp"), "-o", str(out),
                    f"-L{lib_dir}", "-l:libphyzb200.so", f"-Wl,-rpath,{lib_dir}"], check=True)
    return out


def run(binary, *args):
    r = subprocess.run([str(binary), *map(str, args)], capture_output=True, text=True, check=True)
    return json.loads(r.stdout)


def test_cpp_host_reports_missing_device(host_binary):
    from phyz_b200 import _lib

    if _lib.load().phyzb_device_count() > 0:
        pytest.skip("a device is present")
    out = run(host_binary, 8, 10)
    assert out["error"] == _lib.ERR_NO_DEVICE


@pytest.mark.gpu
def test_cpp_host_rollout_matches_oracle(host_binary, oracle):
    from phyz_b200 import configs

    n, steps = 8, 100
    out = run(host_binary, n, steps)
    assert "error" not in out, out
    assert out["contacts_err"] == -4
    t = np.arange(n) / n
    q0 = np.stack([0.2 + 1.2 * t, -0.4 + 0.8 * t], 1)
    qo, _, _, _ = oracle.rollout(configs.double_pendulum(), q0, np.zeros_like(q0), np.zeros_like(q0), steps)
    assert np.max(np.abs(np.array(out["q"]) - qo)) < 1e-10
