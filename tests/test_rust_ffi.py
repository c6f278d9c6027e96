"""The Rust binding (crates/cuda-ffi) against the C header (include/qw_qmm.h):
every entry point the header declares is in the crate's extern "C" block
and nothing else is; each has the same arity, the same parameter names and
Rust types that match the C types; qw_array / qw_qmm_op and the status,
dtype and size constants have the same layout and values; and the
mlxcel-core patch is well formed (hunk sizes match their lines) and routes
UnifiedLinear::forward's quantized arm (layers.rs:2025) through the crate.
cargo is not installed here, so the crate is checked as text."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qw_qmm.h")
CRATE = os.path.join(ROOT, "crates", "cuda-ffi", "src", "lib.rs")
PATCH = os.path.join(ROOT, "crates", "cuda-ffi", "patches", "mlxcel-core-cuda.patch")

# C parameter / return type -> Rust type in the binding
C_TO_RUST = {
    "const qw_array*": "*const QwArray",
    "qw_array*": "*mut QwArray",
    "int": "c_int",
    "int64_t": "i64",
    "const char*": "*const c_char",
    "void*": "*mut c_void",
    "const qw_qmm_op*": "*const QwQmmOp",
    "qw_allreduce**": "*mut *mut QwAllreduce",
    "qw_allreduce*": "*mut QwAllreduce",
    "unsigned char*": "*mut u8",
    "const unsigned char*": "*const u8",
    "unsigned int*": "*mut u32",
    "int64_t*": "*mut i64",
}


def _strip_c_comments(s):
    return re.sub(r"/\*.*?\*/", " ", s, flags=re.S)


def c_functions():
    src = _strip_c_comments(open(HEADER).read())
    out = {}
    for m in re.finditer(r"\b(int|const char\*)\s+(qw_\w+)\s*\(([^)]*)\)\s*;", src):
        ret, name, params = m.group(1), m.group(2), m.group(3)
        args = []
        for p in [p.strip() for p in params.split(",")]:
            if p in ("", "void"):
                continue
            pm = re.match(r"(.*?)(\w+)$", p.replace(" *", "* ").strip())
            ctype = re.sub(r"\s+", " ", pm.group(1).strip()).replace(" *", "*")
            args.append((pm.group(2), ctype))
        out[name] = (ret, args)
    return out


def rust_functions():
    src = open(CRATE).read()
    block = re.search(r'extern "C" \{(.*?)\n\}', src, flags=re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (qw_\w+)\((.*?)\)\s*->\s*([^;]+);", block, flags=re.S):
        name, params, ret = m.group(1), m.group(2), m.group(3).strip()
        args = []
        for p in [p.strip() for p in re.sub(r"\s+", " ", params).split(",")]:
            if not p:
                continue
            pname, ptype = [t.strip() for t in p.split(":", 1)]
            args.append((pname, ptype))
        out[name] = (ret, args)
    return out


def test_same_entry_points():
    c, r = c_functions(), rust_functions()
    assert len(c) >= 20
    assert set(c) == set(r), (sorted(set(c) - set(r)), sorted(set(r) - set(c)))


@pytest.mark.parametrize("name", sorted(c_functions()))
def test_signature_matches(name):
    cret, cargs = c_functions()[name]
    rret, rargs = rust_functions()[name]
    assert {"int": "c_int", "const char*": "*const c_char"}[cret] == rret
    assert len(cargs) == len(rargs), f"{name}: arity {len(cargs)} vs {len(rargs)}"
    for (cn, ct), (rn, rt) in zip(cargs, rargs):
        assert cn == rn, f"{name}: parameter {cn} is {rn} in Rust"
        assert C_TO_RUST[ct] == rt, f"{name}({cn}): C {ct} vs Rust {rt}"


def _c_struct(name):
    src = _strip_c_comments(open(HEADER).read())
    body = re.search(r"typedef struct %s \{(.*?)\}" % name, src, flags=re.S).group(1)
    return [re.sub(r"\s+", " ", f.strip()) for f in body.split(";") if f.strip()]


def _rust_struct(name):
    src = open(CRATE).read()
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, src, flags=re.S).group(1)
    return [re.sub(r"\s+", " ", f.strip().rstrip(",")) for f in body.strip().splitlines() if f.strip()]


def test_array_descriptor_layout():
    assert _c_struct("qw_array") == ["void* data", "int32_t dtype", "int32_t ndim", "int64_t shape[4]",
                                     "int64_t strides[4]"]
    assert _rust_struct("QwArray") == ["pub data: *mut c_void", "pub dtype: i32", "pub ndim: i32",
                                       "pub shape: [i64; 4]", "pub strides: [i64; 4]"]
    assert "#[repr(C)]\n#[derive(Clone, Copy, Debug)]\npub struct QwArray" in open(CRATE).read()


def test_chain_op_layout():
    assert _c_struct("qw_qmm_op") == ["const qw_array* x", "const qw_array* w", "const qw_array* scales",
                                      "const qw_array* biases", "qw_array* y"]
    assert _rust_struct("QwQmmOp") == ["pub x: *const QwArray", "pub w: *const QwArray",
                                       "pub scales: *const QwArray", "pub biases: *const QwArray",
                                       "pub y: *mut QwArray"]


def test_constants_match():
    hdr = _strip_c_comments(open(HEADER).read())
    crate = open(CRATE).read()
    consts = dict(re.findall(r"\b(QW_[A-Z0-9_]+) = (\d+)", hdr))
    consts.update(re.findall(r"#define (QW_[A-Z_]+) (\d+)", hdr))
    rust = dict(re.findall(r"pub const (QW_[A-Z0-9_]+): \w+ = (\d+);", crate))
    assert len(consts) >= 12
    for k, v in consts.items():
        assert rust.get(k) == v, f"{k}: C {v}, Rust {rust.get(k)}"


def test_patch_is_well_formed():
    text = open(PATCH).read()
    files = re.findall(r"^\+\+\+ b/(\S+)$", text, flags=re.M)
    assert "crates/mlxcel-core/src/layers.rs" in files and "crates/mlxcel-core/src/cuda_linear.rs" in files
    # every hunk adds exactly the lines its header announces and removes none
    hunks = re.split(r"^(@@ .* @@)$", text, flags=re.M)
    for hdr, body in zip(hunks[1::2], hunks[2::2]):
        m = re.match(r"@@ -(\d+),0 \+(\d+)(?:,(\d+))? @@", hdr)
        assert m, hdr
        want = int(m.group(3) or 1)
        lines = [l for l in body.split("\n") if l.startswith("+") and not l.startswith("+++")]
        lines = lines[:want]
        assert len(lines) == want, hdr
        assert not re.search(r"^-(?!--)", body.split("\n--- ")[0], flags=re.M), hdr
    assert re.search(r"^@@ -2025,0 ", text, flags=re.M), "the dispatch sits at the head of the Quantized arm"
    assert "cuda_linear::forward(x, weight, bias.as_ref())" in text
