"""The model-specialized kernel's source compiles for sm_100a, on the CPU.

NVRTC needs no GPU: for a few models the packed table is turned into the
specialized translation unit (pz_spec.h, through tests/cpp/spec_source.cpp)
and compiled with the options spec.cu uses, against the kernel headers in
phyz_b200/csrc. This catches a header change that breaks run-time
compilation (a host-only include, a construct NVRTC rejects) before a GPU
run would, and checks that the compiled kernel spills nothing."""
import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

from phyz_b200 import configs

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "phyz_b200" / "csrc"


def nvrtc():
    for name in ("libnvrtc.so.12", "libnvrtc.so"):
        try:
            return C.CDLL(name)
        except OSError:
            continue
    pytest.skip("libnvrtc is not available")


@pytest.fixture(scope="module")
def helper(tmp_path_factory):
    so = tmp_path_factory.mktemp("spec") / "spec_source.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", "-I", str(CSRC),
                    str(ROOT / "tests" / "cpp" / "spec_source.cpp"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.spec_source_for.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_char_p, C.c_int,
                                    C.c_char_p, C.c_int]
    return lib


@pytest.mark.parametrize("name,contact,f64,W,sliced", [
    ("c1_double_pendulum", 0, 1, 32, 0),
    ("c3_quadruped", 1, 0, 128, 0),
    ("c3_quadruped", 1, 0, 128, 1),  # the slice-mode twin
    ("c3_quadruped", 2, 0, 224, 0),
])
def test_specialized_source_compiles(helper, name, contact, f64, W, sliced):
    nv_lib = nvrtc()
    m = configs.CONFIGS[name].builder()
    cm, keep = m.to_c()
    src = C.create_string_buffer(1 << 22)
    kname = C.create_string_buffer(256)
    n = helper.spec_source_for(C.addressof(cm), m.nv, contact, f64, W, sliced, src, len(src), kname, len(kname))
    assert n > 0
    prog = C.c_void_p()
    assert nv_lib.nvrtcCreateProgram(C.byref(prog), src.value, b"spec.cu", 0, None, None) == 0
    assert nv_lib.nvrtcAddNameExpression(prog, kname.value) == 0
    opts = [b"-arch=sm_100a", b"-std=c++17", b"-lineinfo", b"-I" + str(CSRC).encode(), b"--ptxas-options=-v"]
    rc = nv_lib.nvrtcCompileProgram(prog, len(opts), (C.c_char_p * len(opts))(*opts))
    size = C.c_size_t()
    nv_lib.nvrtcGetProgramLogSize(prog, C.byref(size))
    log = C.create_string_buffer(size.value)
    nv_lib.nvrtcGetProgramLog(prog, log)
    text = log.value.decode(errors="replace")
    nv_lib.nvrtcDestroyProgram(C.byref(prog))
    assert rc == 0, text[-4000:]
    # the specialized rollout kernel (the first entry ptxas reports) spills nothing
    m_spill = re.search(r"Compiling entry function '[^']*rollout_kernel[^']*'.*?(\d+) bytes spill stores, "
                        r"(\d+) bytes spill loads", text, re.S)
    assert m_spill, text[-2000:]
    assert m_spill.group(1) == "0" and m_spill.group(2) == "0", text[-2000:]
