"""The Rust binding (rust/weaver-sys) against the C header, on CPU: no Rust
toolchain is needed, the two files are parsed.  Every exported function of
include/weaver_cuda.h has an extern "C" declaration with the same parameters
in the same order and corresponding types, and the mirrored structs list the
same fields in the same order (the reference's #[repr(C)] types,
nexus-core/src/types.rs:150-396, are what the header mirrors)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "weaver_cuda.h")
SYS_RS = os.path.join(ROOT, "rust", "weaver-sys", "src", "lib.rs")

SCALARS = {"int": "c_int", "uint8_t": "u8", "uint16_t": "u16", "uint32_t": "u32", "uint64_t": "u64",
           "size_t": "usize", "float": "f32", "char": "c_char", "void": "c_void"}


def _strip_c_comments(s):
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    return re.sub(r"//[^\n]*", " ", s)


def c_type_to_rust(t):
    t = " ".join(t.split())
    stars = t.count("*")
    base = t.replace("*", " ").split()
    const = "const" in base
    base = [w for w in base if w != "const"]
    assert len(base) == 1, t
    name = SCALARS.get(base[0], base[0])
    if stars == 0:
        return name
    out = ("*const " if const else "*mut ") + name
    for _ in range(stars - 1):
        out = "*mut " + out
    return out


def c_functions():
    src = _strip_c_comments(open(HEADER).read())
    fns = {}
    for ret, name, params in re.findall(r"WEAVER_EXPORT\s+([\w\s\*]+?)\s*\b(\w+)\s*\(([^)]*)\)\s*;", src, re.S):
        ps = []
        params = " ".join(params.split())
        if params and params != "void":
            for p in params.split(","):
                p = p.strip()
                m = re.match(r"(.*?)(\w+)$", p)
                ps.append(c_type_to_rust(m.group(1)))
        r = c_type_to_rust(ret)
        fns[name] = (None if r == "c_void" else r, ps)
    return fns


def rust_functions():
    src = open(SYS_RS).read()
    block = re.search(r'extern "C"\s*\{(.*?)\n\}', src, re.S).group(1)
    fns = {}
    for name, params, ret in re.findall(r"pub fn (\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, re.S):
        ps = []
        params = " ".join(params.split())
        if params:
            for p in params.split(","):
                p = p.strip()
                if not p:
                    continue
                ps.append(" ".join(p.split(":", 1)[1].split()))
        fns[name] = (ret.strip() if ret else None, ps)
    return fns


def test_every_exported_function_is_bound_with_the_same_signature():
    c, r = c_functions(), rust_functions()
    assert len(c) >= 25
    assert set(c) == set(r), (sorted(set(c) - set(r)), sorted(set(r) - set(c)))
    for name, (ret, params) in c.items():
        assert r[name][0] == ret, (name, ret, r[name][0])
        assert r[name][1] == params, (name, params, r[name][1])


STRUCTS = ["weaver_sparse_code", "weaver_params", "weaver_model_dims", "weaver_loom_descriptor",
           "weaver_fabric_regions", "weaver_shape", "weaver_views"]


def _c_struct_fields(src, name):
    body = re.search(r"typedef struct " + name + r"\s*\{(.*?)\}\s*" + name + r"\s*;", src, re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        m = re.match(r"(.*?)\s*((?:\w+\s*(?:\[\d+\])?\s*,\s*)*\w+\s*(?:\[\d+\])?)$", decl, re.S)
        for f in m.group(2).split(","):
            fields.append(re.sub(r"\[.*\]", "", f).strip())
    return fields


def _rust_struct_fields(src, name):
    body = re.search(r"pub struct " + name + r"\s*\{(.*?)\}", src, re.S).group(1)
    return re.findall(r"pub (\w+)\s*:", body)


@pytest.mark.parametrize("name", STRUCTS)
def test_mirrored_structs_have_the_same_fields(name):
    c_src = _strip_c_comments(open(HEADER).read())
    r_src = open(SYS_RS).read()
    assert _c_struct_fields(c_src, name) == _rust_struct_fields(r_src, name)


def test_crates_are_complete():
    for rel in ("rust/weaver-sys/Cargo.toml", "rust/weaver-sys/build.rs", "rust/weaver-sys/src/lib.rs",
                "rust/weaver/Cargo.toml", "rust/weaver/src/lib.rs"):
        assert os.path.exists(os.path.join(ROOT, rel)), rel
    wrapper = open(os.path.join(ROOT, "rust", "weaver", "src", "lib.rs")).read()
    for api in ("pub fn new(_metallib_path: &str) -> Result<Self, String>", "pub fn decode(",
                "pub fn device_name(&self) -> String", "pub fn max_threads_per_threadgroup(&self) -> u64"):
        assert api in wrapper, api
