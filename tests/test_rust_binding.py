"""The Rust declarations of the C ABI (include/kestrel_cuda_sys.rs, the
`kestrel-cuda-sys` crate's lib.rs for Kestrel, whose backends sit behind
`InferenceSession`, crates/kestrel-backends/src/lib.rs:60-74) against the
header include/kestrel_cuda.h.

There is no Rust toolchain here, so the file is checked by parsing: the same
functions in both, the same parameters in the same order with the Rust type
the C type maps to (`int` -> c_int, `const float*` -> *const f32,
`kc_ctx**` -> *mut *mut kc_ctx, `char x[128]` -> *mut c_char, ...), the same
return types, and every constant of the header's enums with its value. A
header change that the Rust side misses fails here."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "kestrel_cuda.h"
RUST = ROOT / "include" / "kestrel_cuda_sys.rs"

C_TO_RUST = {"int": "c_int", "int64_t": "i64", "uint64_t": "u64", "int32_t": "i32", "uint32_t": "u32",
             "int8_t": "i8", "float": "f32", "double": "f64", "char": "c_char", "void": "c_void",
             "kc_ctx": "kc_ctx"}


def c_type_to_rust(c):
    c = " ".join(c.split())
    const = c.startswith("const ")
    if const:
        c = c[len("const "):]
    stars = c.count("*")
    base = c.replace("*", "").strip()
    rust = C_TO_RUST[base]
    if stars == 0:
        return rust
    rust = ("*const " if const else "*mut ") + rust
    for _ in range(stars - 1):
        rust = "*mut " + rust
    return rust


def header_functions():
    src = re.sub(r"/\*.*?\*/", " ", HEADER.read_text(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"KC_API\s+([^;(]*?)\b(kc_\w+)\s*\(([^)]*)\)\s*;", src, flags=re.S):
        args = " ".join(args.split())
        params = []
        if args not in ("", "void"):
            for p in args.split(","):
                p = p.strip()
                m = re.fullmatch(r"(.*?)(\w+)\s*\[\d+\]", p)  # array parameter: a pointer
                if m:
                    params.append((m.group(2), c_type_to_rust(m.group(1).strip() + "*")))
                    continue
                m = re.fullmatch(r"(.*?[\s*])(\w+)", p)
                assert m, p
                params.append((m.group(2), c_type_to_rust(m.group(1))))
        ret = ret.strip()
        out[name] = (params, None if ret == "void" else c_type_to_rust(ret))
    return out


def header_constants():
    src = re.sub(r"/\*.*?\*/", " ", HEADER.read_text(), flags=re.S)
    out = {}
    for body in re.findall(r"enum\s*\{(.*?)\}", src, flags=re.S):
        for item in body.split(","):
            item = item.strip()
            if item:
                m = re.fullmatch(r"(KC_\w+)\s*=\s*(-?\d+)", item)
                assert m, f"enumerator without an explicit value: {item}"
                out.setdefault(m.group(1), int(m.group(2)))
    return out


def rust_source():
    # line comments out, doc comments included
    return re.sub(r"//[^\n]*", "", RUST.read_text())


def rust_functions():
    src = rust_source()
    m = re.search(r'unsafe\s+extern\s+"C"\s*\{(.*?)\n\}', src, flags=re.S)
    assert m, "no extern block"
    out = {}
    for name, args, ret in re.findall(r"pub\s+fn\s+(kc_\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+?))?\s*;", m.group(1),
                                      flags=re.S):
        params = []
        args = " ".join(args.split())
        if args:
            for p in args.split(","):
                pn, pt = p.split(":", 1)
                params.append((pn.strip(), " ".join(pt.split())))
        assert name not in out, f"{name} declared twice"
        out[name] = (params, " ".join(ret.split()) if ret else None)
    return out


def rust_constants():
    out = {}
    for name, ty, val in re.findall(r"pub\s+const\s+(\w+)\s*:\s*(\w+)\s*=\s*(-?\d+)\s*;", rust_source()):
        assert ty == "c_int", (name, ty)
        assert name not in out, f"{name} defined twice"
        out[name] = int(val)
    return out


def test_same_functions():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 40
    assert sorted(h) == sorted(r), {"only in the header": sorted(set(h) - set(r)),
                                    "only in the Rust file": sorted(set(r) - set(h))}


@pytest.mark.parametrize("name", sorted(header_functions()))
def test_same_signature(name):
    hp, hr = header_functions()[name]
    rp, rr = rust_functions()[name]
    assert [n for n, _ in rp] == [n for n, _ in hp], name
    assert [t for _, t in rp] == [t for _, t in hp], name
    assert rr == hr, name


def test_same_constants():
    h, r = header_constants(), rust_constants()
    assert len(h) >= 60
    assert r == h


def test_rust_file_is_balanced_and_links_the_library():
    src = rust_source()
    for a, b in ("{}", "()", "[]"):
        assert src.count(a) == src.count(b), a + b
    assert '#[link(name = "kestrel_cuda")]' in RUST.read_text()
    assert "#[repr(C)]" in src and "pub struct kc_ctx" in src


def test_exported_symbols_are_declared_in_rust():
    """Every entry point the built library exports has a Rust declaration."""
    from kestrel_b200.cuda import LIB_PATH
    if not Path(LIB_PATH).exists():
        pytest.skip("library not built")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name in rust_functions():
        assert hasattr(lib, name), name
