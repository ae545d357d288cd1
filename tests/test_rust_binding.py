"""The Rust `-sys` crate (qmm-sys/src/lib.rs) against the C header
(include/qmm.h), on the CPU: the same symbols, each with the same arguments
(names, order, C types mapped to Rust) and return type; the same struct
layouts; the same constant values.  cargo is not part of this toolchain, so
this is the check that the crate a Rust host (image-forger's quant.rs, the
`mlx-qmm` op of src/quant.rs:411-503) would link matches the library."""
import os
import re

from qwen_imager_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qmm.h")
CRATE = os.path.join(ROOT, "qmm-sys", "src", "lib.rs")

SCALARS = {"int64_t": "i64", "int32_t": "i32", "uint64_t": "u64", "uint32_t": "u32", "uint16_t": "u16",
           "float": "f32", "void": "c_void", "char": "c_char", "qmm_status": "qmm_status",
           "qmm_weight": "qmm_weight", "qmm_epilogue": "qmm_epilogue", "qmm_tp_peers": "qmm_tp_peers",
           "qmm_tp_norm": "qmm_tp_norm"}
ARRAY_LENGTHS = {"QMM_TP_MAX_RANKS": 8}


def _strip_c_comments(text):
    return re.sub(r"/\*.*?\*/", "", text, flags=re.S)


def _c_type(t):
    t = " ".join(t.replace("*", " * ").split())
    const = t.startswith("const ")
    if const:
        t = t[len("const "):]
    stars = t.count("*")
    base = t.replace("*", "").strip()
    rust = SCALARS[base]
    for _ in range(stars):
        rust = ("*const " if const else "*mut ") + rust
    return rust


def _c_param(p):
    p = " ".join(p.split())
    arr = re.match(r"(.*?)(\w+)\s*\[(\w+)\]$", p)
    if arr:  # a fixed-size array field: [T; N] in Rust
        n = arr.group(3)
        n = ARRAY_LENGTHS.get(n, n)
        return arr.group(2), f"[{_c_type(arr.group(1))}; {n}]"
    m = re.match(r"(.*?)(\w+)$", p)
    return m.group(2), _c_type(m.group(1))


def header_api():
    text = _strip_c_comments(open(HEADER).read())
    funcs = {}
    for ret, name, args in re.findall(r"QMM_API\s+((?:const\s+)?\w+\s*\*?)\s*(qmm_\w+)\s*\(([^)]*)\)\s*;", text):
        args = " ".join(args.split())
        params = [] if args in ("void", "") else [_c_param(a) for a in args.split(",")]
        funcs[name] = (params, _c_type(ret))
    structs = {}
    for body, name in re.findall(r"typedef struct \w+ \{([^}]*)\}\s*(\w+);", text):
        structs[name] = [_c_param(f) for f in body.split(";") if f.strip()]
    consts = {k: int(v, 0) for k, v in re.findall(r"#define\s+(QMM_[A-Z_0-9]+)\s+(0x[0-9a-fA-F]+|\d+)\b", text)}
    for body in re.findall(r"typedef enum \w+ \{([^}]*)\}", text):
        for k, v in re.findall(r"(QMM_\w+)\s*=\s*(\d+)", body):
            consts[k] = int(v)
    return funcs, structs, consts


def _rust_type(t):
    return " ".join(t.split())


def crate_api():
    text = re.sub(r"//.*", "", open(CRATE).read())
    block = re.search(r'extern "C" \{(.*?)\n\}', text, re.S).group(1)
    funcs = {}
    for name, args, ret in re.findall(r"pub fn (qmm_\w+)\s*\(([^)]*)\)\s*(?:->\s*([^;]+))?;", block):
        params = []
        for a in args.split(","):
            if a.strip():
                n, t = a.split(":", 1)
                params.append((n.strip(), _rust_type(t)))
        funcs[name] = (params, _rust_type(ret) if ret else "c_void")
    structs = {}
    for name, body in re.findall(r"pub struct (\w+) \{(.*?)\n\}", text, re.S):
        fields = []
        for f in re.findall(r"pub (\w+): ([^\n]+?),\s*$", body, re.M):
            fields.append((f[0], _rust_type(f[1])))
        structs[name] = fields
    consts = {k: int(v, 0) for k, v in re.findall(r"pub const (QMM_\w+): \w+ = (0x[0-9a-fA-F]+|\d+);", text)}
    return funcs, structs, consts


def test_every_header_function_is_bound_with_the_same_signature():
    hf, _, _ = header_api()
    rf, _, _ = crate_api()
    assert sorted(hf) == sorted(rf)
    for name, (params, ret) in hf.items():
        rparams, rret = rf[name]
        assert [t for _, t in rparams] == [t for _, t in params], name
        assert [n for n, _ in rparams] == [n for n, _ in params], name
        assert rret == ret, (name, rret, ret)


def test_structs_have_the_same_layout():
    _, hs, _ = header_api()
    _, rs, _ = crate_api()
    assert sorted(hs) == sorted(rs) == ["qmm_epilogue", "qmm_tp_norm", "qmm_tp_peers", "qmm_weight"]
    for name, fields in hs.items():
        assert rs[name] == fields, name


def test_constants_have_the_same_values():
    _, _, hc = header_api()
    _, _, rc = crate_api()
    assert set(hc) <= set(rc), sorted(set(hc) - set(rc))
    for k, v in hc.items():
        assert rc[k] == v, k


def test_crate_binds_what_the_python_binding_binds():
    rf, _, _ = crate_api()
    assert sorted(rf) == sorted(_lib.EXPORTED_SYMBOLS)


def test_crate_links_the_in_tree_library():
    build = open(os.path.join(ROOT, "qmm-sys", "build.rs")).read()
    assert "rustc-link-lib=dylib=qmm" in build and "_build" in build
    assert 'links = "qmm"' in open(os.path.join(ROOT, "qmm-sys", "Cargo.toml")).read()
