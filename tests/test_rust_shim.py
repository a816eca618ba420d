"""The Rust bindings crate (an-operating-system-for-ai-models-and-tensor-
inference_b200/rust/myos_cuda_sys) against include/myos_cuda.h: every C
function has an extern declaration with the same name, the same number of
arguments and the same pointer / value kind per argument, and the repr(C)
structs have the C structs' fields in order. No Rust toolchain is needed
(the crate itself is not compiled here)."""
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "myos_cuda.h")
CRATE = os.path.join(REPO, "an-operating-system-for-ai-models-and-tensor-inference_b200", "rust",
                     "myos_cuda_sys")


def c_functions():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b[\w\s\*]*?\b(myos_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        name, args = m.group(1), " ".join(m.group(2).split())
        params = [] if args in ("", "void") else [a.strip() for a in args.split(",")]
        out[name] = ["ptr" if ("*" in p or "[" in p) else "val" for p in params]
    return out


def rust_functions():
    text = open(os.path.join(CRATE, "src", "lib.rs")).read()
    block = text[text.index('extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    out = {}
    for m in re.finditer(r"pub fn (myos_[a-z0-9_]+)\(([^)]*)\)", block):
        args = m.group(2).strip()
        params = [] if not args else [a.split(":", 1)[1].strip() for a in args.split(",")]
        out[m.group(1)] = ["ptr" if p.startswith("*") else "val" for p in params]
    return out


def c_struct(name):
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, text, flags=re.S).group(1)
    return [re.sub(r"\[.*\]", "", f.split()[-1]) for f in body.split(";") if f.strip()]


def rust_struct(name):
    text = open(os.path.join(CRATE, "src", "lib.rs")).read()
    body = re.search(r"pub struct %s \{(.*?)\}" % name, text, flags=re.S).group(1)
    return [f.split(":")[0].replace("pub", "").strip() for f in body.split(",") if ":" in f]


def test_every_c_function_has_a_matching_rust_declaration():
    c, r = c_functions(), rust_functions()
    assert len(c) >= 30
    assert set(c) == set(r), (sorted(set(c) - set(r)), sorted(set(r) - set(c)))
    for name, kinds in c.items():
        assert r[name] == kinds, (name, kinds, r[name])


def test_structs_match_field_for_field():
    for s in ("myos_shape", "myos_opts", "myos_tp", "myos_tp_part"):
        assert c_struct(s) == rust_struct(s), s


def test_status_codes_match():
    text = open(HEADER).read()
    c = dict((n, int(v)) for n, v in re.findall(r"(MYOS_(?:OK|ERR_[A-Z_]+))\s*=\s*(\d+)", text))
    rs = open(os.path.join(CRATE, "src", "lib.rs")).read()
    r = dict((n, int(v)) for n, v in re.findall(r"pub const (MYOS_(?:OK|ERR_[A-Z_]+)): c_int = (\d+);", rs))
    assert c == r


def test_build_script_targets_sm100a():
    b = open(os.path.join(CRATE, "build.rs")).read()
    assert "arch=compute_100a,code=sm_100a" in b
    srcs = re.findall(r'"([a-z0-9_]+\.(?:cu|cpp))"', b)
    import build as pkg_build
    assert sorted(srcs) == sorted(pkg_build.CUDA_SOURCES)
