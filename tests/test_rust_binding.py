"""The Rust crate ffi/rust/pp-b200-sys against the C header, on the CPU.

No Rust toolchain is needed: both files are parsed.  Every function the
header declares must appear in the crate's extern block with the same
number of arguments and the corresponding Rust type for each argument and
the return value; every struct must have the same fields in the same order
with corresponding types; every #define constant must have a `pub const`
of the same value."""
from __future__ import annotations

import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pp_b200.h")
CRATE = os.path.join(ROOT, "ffi", "rust", "pp-b200-sys")

SCALARS = {"uint32_t": "u32", "int32_t": "i32", "uint64_t": "u64", "size_t": "usize", "float": "f32",
           "uint8_t": "u8", "void": "c_void", "char": "c_char"}


def _strip_c_comments(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    return re.sub(r"^\s*#[^\n]*", " ", text, flags=re.M)  # preprocessor lines


def _rust_type(c: str) -> str:
    c = " ".join(c.replace("*", " * ").split())
    const = c.startswith("const ")
    if const:
        c = c[len("const "):]
    stars = c.count("*")
    base = c.replace("*", "").strip()
    r = SCALARS.get(base, base)
    for i in range(stars):
        r = ("*const " if const and i == 0 else "*mut ") + r
    return r


def _split_param(p: str) -> tuple[str, str]:
    p = " ".join(p.replace("*", " * ").split())
    m = re.match(r"(.*?)(\w+)$", p)
    return m.group(1).strip(), m.group(2)


def header_functions() -> dict[str, tuple[str, list[str]]]:
    text = _strip_c_comments(open(HEADER).read())
    out = {}
    for ret, name, args in re.findall(r"([A-Za-z_][\w\s\*]*?)\s*\b(pp_b200_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        args = " ".join(args.split())
        params = [] if args in ("", "void") else [_rust_type(_split_param(a)[0]) for a in args.split(",")]
        out[name] = (_rust_type(ret.strip()), params)
    return out


def header_structs() -> dict[str, list[tuple[str, str]]]:
    text = _strip_c_comments(open(HEADER).read())
    out = {}
    for body, name in re.findall(r"typedef struct \w+\s*\{(.*?)\}\s*(\w+)\s*;", text, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            arr = re.match(r"(.*?)\s*\[(\d+)\]$", decl)
            n = None
            if arr:
                decl, n = arr.group(1), arr.group(2)
            t, f = _split_param(decl)
            rt = _rust_type(t)
            fields.append((f, f"[{rt}; {n}]" if n else rt))
        out[name] = fields
    return out


def header_constants() -> dict[str, int]:
    text = open(HEADER).read()
    return {n: int(v, 0) for n, v in re.findall(r"#define\s+(PP_\w+)\s+(0x[0-9a-fA-F]+|\d+)u?\b", text)}


def _rust_source() -> str:
    text = open(os.path.join(CRATE, "src", "lib.rs")).read()
    text = re.sub(r"//[^\n]*", " ", text)
    return text


def rust_functions() -> dict[str, tuple[str, list[str]]]:
    text = _rust_source()
    block = re.search(r'extern "C"\s*\{(.*?)\n\}', text, flags=re.S).group(1)
    out = {}
    for name, args, ret in re.findall(r"pub fn (\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        params = [] if not args.strip() else [" ".join(a.split(":", 1)[1].split()) for a in args.split(",")
                                                if a.strip()]
        out[name] = (" ".join(ret.split()) if ret else "()", params)
    return out


def rust_structs() -> dict[str, list[tuple[str, str]]]:
    text = _rust_source()
    out = {}
    for name, body in re.findall(r"#\[repr\(C\)\]\s*(?:#\[derive\([^)]*\)\]\s*)?pub struct (\w+)\s*\{(.*?)\}", text,
                                 flags=re.S):
        out[name] = [(f, " ".join(t.split())) for f, t in re.findall(r"pub (\w+):\s*([^,]+),", body)]
    return out


def rust_constants() -> dict[str, int]:
    return {n: int(v.replace("_", ""), 0) for n, v in
            re.findall(r"pub const (PP_\w+):\s*\w+\s*=\s*(0x[0-9a-fA-F_]+|\d+);", _rust_source())}


def test_crate_files_exist():
    for rel in ("Cargo.toml", "build.rs", os.path.join("src", "lib.rs"), os.path.join("src", "int8_kv_ops.rs")):
        assert os.path.exists(os.path.join(CRATE, rel)), rel
    cargo = open(os.path.join(CRATE, "Cargo.toml")).read()
    assert 'links = "pp_b200"' in cargo
    assert "rustc-link-lib=dylib=pp_b200" in open(os.path.join(CRATE, "build.rs")).read()


def test_every_header_function_is_bound_with_matching_types():
    c, r = header_functions(), rust_functions()
    assert len(c) == len(set(c)) >= 28
    assert set(c) == set(r), f"only in header: {set(c) - set(r)}; only in crate: {set(r) - set(c)}"
    for name, (ret, params) in c.items():
        rret, rparams = r[name]
        assert rret == ret, f"{name}: return {rret} != {ret}"
        assert rparams == params, f"{name}: {rparams} != {params}"


def test_structs_have_the_header_layout():
    c, r = header_structs(), rust_structs()
    assert set(c) == {"PpKvArena", "PpAttnParams", "PpFloatKv", "PpQkvRope"}
    assert set(c) <= set(r)
    for name, fields in c.items():
        assert r[name] == fields, f"{name}: {r[name]} != {fields}"


def test_constants_have_the_header_values():
    c, r = header_constants(), rust_constants()
    assert c and set(c) == set(r), set(c) ^ set(r)
    for n, v in c.items():
        assert r[n] == v, n


def test_the_binding_matches_the_python_binding(pp):
    assert set(rust_functions()) == set(pp._native.EXPORTED)
