"""The Rust binding of the C ABI (rust/crates/engine/src/cuda/ffi.rs) against the
header (include/w4a8.h): the same entry points, argument counts and argument
types, so a maintainer who drops the backend into crates/engine gets a binding
that matches the library.  The Rust files are not compiled here (no cargo)."""

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "w4a8.h")
FFI = os.path.join(ROOT, "rust", "crates", "engine", "src", "cuda", "ffi.rs")

# C type -> Rust type of the binding
C2RUST = {
    "const void*": "*const c_void", "void*": "*mut c_void", "void**": "*mut *mut c_void",
    "const float*": "*const f32", "float*": "*mut f32", "float": "f32",
    "const int8_t*": "*const i8", "int8_t*": "*mut i8",
    "const uint32_t*": "*const u32", "uint32_t*": "*mut u32",
    "uint64_t*": "*mut u64", "int32_t*": "*mut i32", "int32_t": "i32", "int": "c_int", "size_t": "usize",
    "const w4a8_weight*": "*const w4a8_weight", "w4a8_weight*": "*mut w4a8_weight",
    "w4a8_xchg*": "*mut w4a8_xchg", "w4a8_xchg**": "*mut *mut w4a8_xchg",
    "w4a8_status": "w4a8_status", "const char*": "*const c_char", "void": None,
}


def _norm_c(t):
    t = re.sub(r"\s+", " ", t.strip())
    return re.sub(r"\s*\*", "*", t)


def header_decls():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for m in re.finditer(r"W4A8_API\s+([\w\s\*]+?)\s*\b(w4a8_\w+)\s*\(([^)]*)\)\s*;", src):
        ret, name, args = _norm_c(m.group(1)), m.group(2), m.group(3).strip()
        params = []
        if args and args != "void":
            for a in args.split(","):
                a = _norm_c(a)
                pm = re.match(r"(.*?[\s\*])(\w+)$", a)
                params.append(_norm_c(pm.group(1)))
        out[name] = (ret, params)
    return out


def rust_decls():
    src = open(FFI).read()
    block = src[src.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    out = {}
    for m in re.finditer(r"pub fn (w4a8_\w+)\((.*?)\)(?:\s*->\s*([^;]+))?;", block, flags=re.S):
        name, args, ret = m.group(1), m.group(2), (m.group(3) or "").strip() or None
        params = []
        for a in [x.strip() for x in args.split(",") if x.strip()]:
            params.append(re.sub(r"\s+", " ", a.split(":", 1)[1].strip()))
        out[name] = (ret, params)
    return out


def test_every_header_entry_point_is_bound():
    h, r = header_decls(), rust_decls()
    assert len(h) >= 30
    assert sorted(h) == sorted(r), (set(h) ^ set(r))


def test_signatures_match():
    h, r = header_decls(), rust_decls()
    for name, (cret, cparams) in h.items():
        rret, rparams = r[name]
        assert len(cparams) == len(rparams), name
        assert C2RUST[cret] == rret, (name, cret, rret)
        for i, (c, rs) in enumerate(zip(cparams, rparams)):
            assert c in C2RUST, (name, c)
            assert C2RUST[c] == rs, (name, i, c, rs)


def test_struct_and_constants():
    src = open(FFI).read()
    hdr = open(HEADER).read()
    fields = re.search(r"pub struct w4a8_weight \{(.*?)\}", src, flags=re.S).group(1)
    assert [f.split(":")[0].strip().replace("pub ", "") for f in fields.split(",") if f.strip()] == \
        ["q", "s", "n", "k", "group", "has_min"]
    for const in ["W4A8_GEMV_MAX_M", "W4A8_XCHG_HANDLE_BYTES", "W4A8_XCHG_MAX_RANKS", "W4A8_XCHG_MAX_TOKENS"]:
        cval = int(re.search(rf"#define {const} (\d+)", hdr).group(1))
        rval = int(re.search(rf"pub const {const}: \w+ = (\d+);", src).group(1))
        assert cval == rval, const
    for name, val in [("W4A8_OK", 0), ("W4A8_EINVAL", 1), ("W4A8_ECUDA", 2), ("W4A8_ENCCL", 3),
                      ("W4A8_ETIMEOUT", 4), ("W4A8_ENOTSUP", 5), ("W4A8_STORE", 0), ("W4A8_ADD", 1),
                      ("W4A8_SWIGLU", 2), ("W4A8_ACT_GROUP32", 0), ("W4A8_ACT_TOKEN", 1)]:
        assert re.search(rf"{name}\s*=\s*{val}\b", hdr), name
        assert re.search(rf"pub const {name}: \w+ = {val};", src), name
