"""The Rust FFI crate (crates/phyz-b200-sys) against the C header it binds.

No Rust toolchain exists in this image, so the crate is checked by reading
it: every `#[repr(C)]` struct's field offsets and size (computed with C's
layout rules, which repr(C) follows) equal those the C compiler gives for
the same struct of include/phyzb.h; every function of the header is
declared in the crate's extern block with the same parameter count and
corresponding types; every constant equals its #define."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
LIB_RS = ROOT / "crates" / "phyz-b200-sys" / "src" / "lib.rs"
HEADER = ROOT / "include" / "phyzb.h"

PRIM = {"i8": 1, "u8": 1, "i16": 2, "u16": 2, "i32": 4, "u32": 4, "f32": 4, "i64": 8, "u64": 8, "f64": 8,
        "c_int": 4, "c_char": 1, "usize": 8, "isize": 8}


def rust_structs():
    src = LIB_RS.read_text()
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*(?:#\[derive\([^)]*\)\]\s*)?pub struct (\w+)\s*\{(.*?)\n\}", src, re.S):
        name, body = m.group(1), m.group(2)
        fields = re.findall(r"pub (\w+):\s*([^,\n]+),", body)
        if fields:
            out[name] = [(f, t.strip()) for f, t in fields]
    return out


def size_align(t):
    t = t.strip()
    if t.startswith("*"):
        return 8, 8
    m = re.fullmatch(r"\[(.+);\s*(\d+)\]", t)
    if m:
        s, a = size_align(m.group(1))
        return s * int(m.group(2)), a
    return PRIM[t], PRIM[t]


def repr_c_layout(fields):
    off, align, offs = 0, 1, {}
    for f, t in fields:
        s, a = size_align(t)
        off = (off + a - 1) // a * a
        offs[f] = off
        off += s
        align = max(align, a)
    return offs, (off + align - 1) // align * align


@pytest.fixture(scope="module")
def c_layout(tmp_path_factory):
    structs = rust_structs()
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "phyzb.h"', "int main(void) {"]
    for name, fields in structs.items():
        lines.append(f'  printf("%s size %zu\\n", "{name}", sizeof({name}));')
        for f, _ in fields:
            lines.append(f'  printf("%s.%s %zu\\n", "{name}", "{f}", offsetof({name}, {f}));')
    lines += ["  return 0;", "}"]
    d = tmp_path_factory.mktemp("ffi")
    (d / "probe.c").write_text("\n".join(lines) + "\n")
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(d / "probe.c"), "-o", str(d / "probe")],
                   check=True)
    out = subprocess.run([str(d / "probe")], check=True, capture_output=True, text=True).stdout
    res = {}
    for ln in out.splitlines():
        key, val = ln.rsplit(" ", 1)
        res[key] = int(val)
    return structs, res


def test_every_header_struct_is_bound():
    hdr = HEADER.read_text()
    named = set(re.findall(r"typedef struct(?: \w+)? \{.*?\} (\w+);", hdr, re.S))
    assert named <= set(rust_structs()), named - set(rust_structs())


def test_struct_layouts_match_the_c_compiler(c_layout):
    structs, c = c_layout
    assert len(structs) >= 14
    for name, fields in structs.items():
        offs, size = repr_c_layout(fields)
        assert c[f"{name} size"] == size, (name, c[f"{name} size"], size)
        for f, _ in fields:
            assert c[f"{name}.{f}"] == offs[f], (name, f, c[f"{name}.{f}"], offs[f])


def c_prototypes():
    s = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for ret, name, args in re.findall(r"\n((?:const )?[a-z_0-9]+\s*\**)\s*(phyzb_\w+)\s*\(([^;]*)\);", s):
        args = " ".join(args.split())
        params = [] if args in ("", "void") else [a.strip() for a in args.split(",")]
        protos[name] = (ret.replace(" ", ""), params)
    return protos


def rust_functions():
    src = LIB_RS.read_text()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    block = re.sub(r"//[^\n]*", "", block)
    out = {}
    for name, args, ret in re.findall(r"pub fn (phyzb_\w+)\s*\((.*?)\)\s*(?:->\s*([^;]+))?;", block, re.S):
        params = [a.strip() for a in " ".join(args.split()).split(",") if a.strip()]
        out[name] = ([p.split(":", 1)[1].strip() for p in params], (ret or "()").strip())
    return out


C_TO_RUST = {"int": "c_int", "int32_t": "i32", "int64_t": "i64", "uint64_t": "u64", "uint32_t": "u32",
             "uint8_t": "u8", "double": "f64", "float": "f32", "void": "c_void", "char": "c_char"}


def c_param_to_rust(p):
    """`const double* q` -> `*const f64`; struct params keep their name."""
    p = p.replace("struct ", "")
    m = re.fullmatch(r"(const\s+)?([a-z_0-9]+)\s*(\**)\s*\w*", p)
    assert m, p
    const, base, stars = m.group(1), m.group(2), m.group(3)
    t = C_TO_RUST.get(base, base)
    for k in range(len(stars)):
        t = ("*const " if (const and k == 0) else "*mut ") + t
    return t


def test_every_function_is_declared_with_matching_types():
    protos, funcs = c_prototypes(), rust_functions()
    assert len(protos) >= 69
    missing = sorted(set(protos) - set(funcs))
    assert not missing, missing
    extra = sorted(set(funcs) - set(protos))
    assert not extra, extra
    for name, (ret, params) in protos.items():
        rparams, rret = funcs[name]
        assert len(rparams) == len(params), (name, params, rparams)
        for cp, rp in zip(params, rparams):
            assert c_param_to_rust(cp) == rp.replace("  ", " "), (name, cp, rp)
        want_ret = {"int": "c_int", "constchar*": "*const c_char"}[ret]
        assert rret == want_ret, (name, ret, rret)


def test_constants_match_the_header():
    defines = {}
    for name, val in re.findall(r"#define (PHYZB_\w+) ([^\n/]+)", HEADER.read_text()):
        val = val.strip()
        if re.fullmatch(r"[()\-\d<\s]+", val):
            defines[name] = eval(val)  # integer literals and shifts only
    consts = {n: eval(v.replace("_", "")) for n, v in
              re.findall(r"pub const (PHYZB_\w+): \w+ = ([^;]+);", LIB_RS.read_text())}
    assert set(defines) == set(consts), set(defines) ^ set(consts)
    for n, v in defines.items():
        assert consts[n] == v, (n, v, consts[n])
