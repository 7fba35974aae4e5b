"""The Rust -sys crate (bindings/rust/trs-sys) against include/trs.h.

No Rust toolchain exists in this image, so the crate cannot be compiled here;
instead every declaration is checked against the header it binds: each C
function has exactly one `extern "C"` declaration with the same parameters in
the same order and the corresponding Rust types (and no declaration binds a
function the header lacks), every enumerator and constant has the header's
value, and the #[repr(C)] structs have the header's fields in order."""
from __future__ import annotations

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "trs.h"
CRATE = ROOT / "bindings" / "rust" / "trs-sys" / "src" / "lib.rs"

SCALARS = {"void": "c_void", "char": "c_char", "int32_t": "i32", "int64_t": "i64", "uint64_t": "u64",
           "size_t": "usize", "double": "f64", "uint8_t": "u8", "trs_view": "trs_view", "trs_scalar": "trs_scalar",
           "trs_ew_program": "trs_ew_program", "trs_comm": "trs_comm", "trs_stream": "trs_stream",
           "trs_status": "trs_status"}


def c_to_rust(ctype: str) -> str:
    """A C parameter or return type as the crate spells it: `const T*` is
    `*const T`, `T*` is `*mut T`, `T**` is `*mut *mut T`."""
    t = " ".join(ctype.split())
    const = t.startswith("const ")
    if const:
        t = t[6:]
    stars = t.count("*")
    base = SCALARS[t.replace("*", "").strip()]
    if stars == 0:
        return base
    out = ("*const " if const else "*mut ") + base
    for _ in range(stars - 1):
        out = "*mut " + out
    return out


def header_functions() -> dict[str, tuple[str, list[str]]]:
    s = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"\n((?:const\s+)?[a-z_0-9]+\s*\**)\s*(trs_[a-z0-9_]+)\(([^;]*?)\);", s,
                                      flags=re.S):
        args = " ".join(args.split())
        types = []
        if args != "void":
            for a in args.split(","):
                a = a.strip()
                arr = re.match(r"(.*?)(\w+)\[\d+\]$", a)  # an array parameter is a pointer
                types.append(c_to_rust(arr.group(1) + "*" if arr else re.match(r"(.*?)(\w+)$", a).group(1)))
        r = c_to_rust(ret)
        out[name] = ("" if r == "c_void" else r, types)
    return out


def crate_functions() -> dict[str, tuple[str, list[str]]]:
    s = CRATE.read_text()
    block = s[s.index('extern "C" {'):]
    block = block[: block.index("\n}\n")]
    out = {}
    for name, params, ret in re.findall(r"pub fn (trs_\w+)\(([^)]*)\)(?:\s*->\s*([^;]+))?;", block):
        types = [p.split(":", 1)[1].strip() for p in params.split(",") if p.strip()]
        assert name not in out, f"{name} declared twice"
        out[name] = ((ret or "").strip(), types)
    return out


def test_every_header_function_is_bound_with_the_same_signature():
    hdr, crate = header_functions(), crate_functions()
    assert len(hdr) >= 50
    missing = sorted(set(hdr) - set(crate))
    extra = sorted(set(crate) - set(hdr))
    assert not missing, f"not bound: {missing}"
    assert not extra, f"bound but not in trs.h: {extra}"
    for name, (ret, types) in hdr.items():
        assert crate[name] == (ret, types), (name, crate[name], (ret, types))


def header_constants() -> dict[str, int]:
    s = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    consts = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (TRS_[A-Z_]+) (\d+)", s)}
    for body in re.findall(r"typedef enum \w+ \{(.*?)\}", s, flags=re.S):
        for name, val in re.findall(r"(TRS_\w+)\s*=\s*(\d+)", body):
            consts[name] = int(val)
    return consts


def test_constants_match_the_header():
    s = CRATE.read_text()
    crate = {n: int(v) for n, v in re.findall(r"pub const (TRS_\w+): \w+ = (\d+);", s)}
    hdr = header_constants()
    assert len(hdr) > 40
    for name, val in hdr.items():
        assert crate.get(name) == val, (name, crate.get(name), val)


def struct_fields_c(name: str) -> list[tuple[str, str]]:
    s = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, s, flags=re.S).group(1)
    out = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        arr = re.match(r"(.+?)\s*(\w+)\[(\w+)\]$", decl)
        if arr:
            out.append((arr.group(2), f"[{c_to_rust(arr.group(1))}; {arr.group(3)}]"))
        else:
            m = re.match(r"(.+?)\s*(\w+)$", decl)
            out.append((m.group(2), c_to_rust(m.group(1))))
    return out


def struct_fields_rust(name: str) -> list[tuple[str, str]]:
    s = CRATE.read_text()
    body = re.search(r"pub struct %s \{(.*?)\}" % name, s, flags=re.S).group(1)
    return [(n, t.strip()) for n, t in re.findall(r"pub (\w+): ([^,]+),", body)]


def test_repr_c_structs_match_the_header():
    for name in ("trs_view", "trs_scalar", "trs_ew_program"):
        assert struct_fields_rust(name) == struct_fields_c(name), name
    assert "#[repr(C)]\n#[derive(Clone, Copy, Debug)]\npub struct trs_view" in CRATE.read_text()
