"""The Rust crate (dial-8b-orin_b200/dial-cuda) against the C header.

There is no Rust toolchain in this image, so the crate is not built here; this
test checks what a build would rely on: its `extern "C"` block declares every
DIAL_API function of include/dial_cuda.h with the same parameter kinds in the
same order (pointer constness, integer and float widths, structs by value),
its #[repr(C)] structs list the header's fields in order, and its build.rs
compiles csrc/*.cu for sm_100a only.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dial_cuda.h")
CRATE = os.path.join(ROOT, "dial-8b-orin_b200", "dial-cuda")

C_SCALAR = {"int64_t": "i64", "int32_t": "i32", "int": "i32", "size_t": "usize", "float": "f32",
            "double": "f64", "dial_status": "i32", "dial_dtype": "i32", "dial_ggml_type": "i32",
            "uint64_t": "u64", "dial_stream": "stream"}
RS_SCALAR = {"i64": "i64", "i32": "i32", "c_int": "i32", "usize": "usize", "f32": "f32", "f64": "f64",
             "dial_status": "i32", "dial_dtype": "i32", "dial_ggml_type": "i32", "u64": "u64",
             "dial_stream": "stream"}


def _c_kind(t: str) -> str:
    t = " ".join(t.replace("*", " * ").split())
    stars = t.count("*")
    base = t.replace("*", "").replace("const", "").split()
    if stars:
        return ("const*" if t.startswith("const") else "mut*") * stars if stars == 1 else \
            ("mut*" + ("const*" if t.startswith("const") else "mut*"))
    if base[-1] in C_SCALAR:
        return C_SCALAR[base[-1]]
    return "struct:" + base[-1]


def _rs_kind(t: str) -> str:
    t = t.strip()
    if t.startswith("*mut *mut"):
        return "mut*mut*"
    if t.startswith("*const"):
        return "const*"
    if t.startswith("*mut"):
        return "mut*"
    if t in RS_SCALAR:
        return RS_SCALAR[t]
    return "struct:" + t


def _split_args(a: str):
    a = a.strip()
    if not a or a == "void":
        return []
    return [x.strip() for x in a.split(",")]


def header_functions():
    s = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"DIAL_API\s+([\w\s\*]+?)\s*\b(dial_\w+)\s*\(([^;]*?)\)\s*;", s, flags=re.S):
        kinds = []
        for a in _split_args(" ".join(args.split())):
            m = re.match(r"(.*?)(\w+)$", a)
            kinds.append(_c_kind(m.group(1)))
        out[name] = kinds
    return out


def crate_functions():
    s = open(os.path.join(CRATE, "src", "lib.rs")).read()
    block = s[s.index('extern "C" {'):]
    block = block[:block.index("\n}\n")]
    block = re.sub(r"//[^\n]*", "", block)
    out = {}
    for name, args in re.findall(r"pub fn (dial_\w+)\(([^)]*)\)", block, flags=re.S):
        kinds = []
        for a in _split_args(" ".join(args.split())):
            kinds.append(_rs_kind(a.split(":", 1)[1]))
        out[name] = kinds
    return out


def test_every_entry_point_is_declared_with_the_same_parameters():
    h, r = header_functions(), crate_functions()
    assert len(h) >= 39
    assert sorted(h) == sorted(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name in h:
        assert h[name] == r[name], (name, h[name], r[name])


def test_repr_c_structs_follow_the_header():
    hs = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    rs = open(os.path.join(CRATE, "src", "lib.rs")).read()
    for name, body in re.findall(r"typedef struct (dial_\w+) \{(.*?)\} \1;", hs, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            for piece in decl.split(","):  # "int a, b[4]" -> a, b
                fields.append(re.findall(r"(\w+)\s*(?:\[[^\]]*\])?\s*$", piece.strip())[0])
        m = re.search(r"pub struct " + name + r" \{(.*?)\n\}", rs, flags=re.S)
        assert m, f"{name} missing from lib.rs"
        rfields = re.findall(r"pub (\w+):", m.group(1))
        assert rfields == fields, (name, fields, rfields)
    assert "pub struct dial_stage_comm" in rs  # opaque


def test_build_script_compiles_for_sm_100a_only():
    b = open(os.path.join(CRATE, "build.rs")).read()
    assert "arch=compute_100a,code=sm_100a" in b
    assert "csrc" in b and '"cu"' in b
    code = "\n".join(l for l in b.splitlines() if not l.strip().startswith("//"))
    assert "nvrtc" not in code.lower() and "triton" not in code.lower()
    cargo = open(os.path.join(CRATE, "Cargo.toml")).read()
    assert 'links = "dial_cuda"' in cargo
