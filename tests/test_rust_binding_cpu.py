"""The Rust binding (rust/src/ffi.rs) declares every entry point of
include/krikil_cuda.h with the same parameter and return types.

No Rust toolchain is available on these machines, so the crate is not compiled
here; this test parses both files and compares the declarations one for one
(C type -> the Rust type an `extern "C"` block must use), which catches a
missing or mistyped binding after a change of the header.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_TO_RUST = {
    "void": None,
    "int": "c_int",
    "float": "c_float",
    "size_t": "usize",
    "int64_t": "i64",
    "uint64_t": "u64",
    "const char*": "*const c_char",
    "const float*": "*const c_float",
    "float*": "*mut c_float",
    "double*": "*mut c_double",
    "int*": "*mut c_int",
    "int32_t*": "*mut i32",
    "const int32_t*": "*const i32",
    "int64_t*": "*mut i64",
    "uint32_t*": "*mut u32",
    "const uint32_t*": "*const u32",
    "uint64_t*": "*mut u64",
    "const uint64_t*": "*const u64",
    "const uint8_t*": "*const u8",
    "void*": "*mut c_void",
    "void**": "*mut *mut c_void",
    "krk_model*": "*mut krk_model",
    "const krk_model*": "*const krk_model",
    "krk_model**": "*mut *mut krk_model",
    "krk_state*": "*mut krk_state",
    "const krk_state*": "*const krk_state",
    "krk_state**": "*mut *mut krk_state",
}


def _norm_c(t: str) -> str:
    t = re.sub(r"\s+", " ", t.strip())
    return re.sub(r"\s*\*", "*", t)


def header_decls():
    src = open(os.path.join(ROOT, "include", "krikil_cuda.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"KRK_API\s+([\w\s\*]+?)\s*\b(krk_\w+)\s*\(([^)]*)\)\s*;", src, flags=re.S):
        ps = []
        if params.strip() not in ("", "void"):
            for p in params.split(","):
                p = p.strip()
                m = re.match(r"(.*?)(\w+)$", p, flags=re.S)
                ps.append(_norm_c(m.group(1)))
        out[name] = (_norm_c(ret), ps)
    return out


def rust_decls():
    src = open(os.path.join(ROOT, "rust", "src", "ffi.rs")).read()
    body = src[src.index('extern "C" {'):]
    out = {}
    for name, params, ret in re.findall(r"pub fn (krk_\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+?))?\s*;", body, flags=re.S):
        ps = []
        for p in params.split(","):
            p = p.strip()
            if p:
                ps.append(re.sub(r"\s+", " ", p.split(":", 1)[1].strip()))
        out[name] = (ret.strip() if ret else None, ps)
    return out


def test_every_header_entry_point_is_bound_with_matching_types():
    h, r = header_decls(), rust_decls()
    assert len(h) == open(os.path.join(ROOT, "include", "krikil_cuda.h")).read().count("\nKRK_API "), sorted(h)
    missing = sorted(set(h) - set(r))
    assert not missing, f"not declared in rust/src/ffi.rs: {missing}"
    extra = sorted(set(r) - set(h))
    assert not extra, f"declared in rust/src/ffi.rs but not in the header: {extra}"
    for name, (ret, ps) in h.items():
        rret, rps = r[name]
        assert C_TO_RUST[ret] == rret, (name, ret, rret)
        assert len(ps) == len(rps), (name, ps, rps)
        for i, (c, rust) in enumerate(zip(ps, rps)):
            assert C_TO_RUST[c] == rust, (name, i, c, rust)


def test_rust_constants_match_the_header():
    hdr = open(os.path.join(ROOT, "include", "krikil_cuda.h")).read()
    ffi = open(os.path.join(ROOT, "rust", "src", "ffi.rs")).read()
    for name, val in re.findall(r"#define (KRK_[A-Z_0-9]+) \(?([0-9][0-9 <]*)\)?", hdr):
        m = re.search(rf"pub const {name}: \w+ = ([^;]+);", ffi)
        assert m, name
        assert eval(m.group(1)) == eval(val), (name, m.group(1), val)
    for name, val in re.findall(r"\b(KRK_[A-Z_]+)\s*=\s*(\d+)", hdr):
        m = re.search(rf"pub const {name}: \w+ = (\d+);", ffi)
        assert m and int(m.group(1)) == int(val), name
