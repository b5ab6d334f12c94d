"""The Rust side of the drop-in boundary (tpt_spark_b200/rust/, for tpt-spark's
src-tauri/src/engine/cuda_ffi.rs and cuda_engine.rs) against the C ABI it binds.

No cargo or rustc exists here, so the Rust files are not compiled; this test reads them as
text and checks engine/cuda_ffi.rs against include/tptc.h symbol by symbol: every exported
function declared once with the same parameter count, the two structs with the same fields
in the same order, and the status / type constants with the same values."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tptc.h")
RUST = os.path.join(ROOT, "tpt_spark_b200", "rust")


def _strip_c_comments(s):
    s = re.sub(r"/\*.*?\*/", " ", s, flags=re.S)
    return re.sub(r"//[^\n]*", " ", s)


def _split_params(params):
    params = params.strip()
    if params in ("", "void"):
        return []
    return [p.strip() for p in params.split(",") if p.strip()]


def c_functions():
    src = _strip_c_comments(open(HEADER).read())
    out = {}
    for m in re.finditer(r"TPTC_API\s+[\w\s\*]+?\b(tptc_\w+)\s*\(([^)]*)\)\s*;", src):
        assert m.group(1) not in out, m.group(1)
        out[m.group(1)] = len(_split_params(m.group(2)))
    return out


def c_struct_fields(name):
    src = _strip_c_comments(open(HEADER).read())
    m = re.search(r"typedef struct \{([^}]*)\}\s*" + name + r"\s*;", src)
    assert m, name
    fields = []
    for decl in m.group(1).split(";"):
        decl = decl.strip()
        if not decl:
            continue
        decl = re.sub(r"\[[^\]]*\]", "", decl)  # array sizes
        parts = decl.split(None, 1)
        fields += [f.strip() for f in parts[1].split(",")]
    return fields


def c_constants():
    src = open(HEADER).read()
    out = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (TPTC_(?:OK|ERR_\w+|TYPE_\w+))\s+\(?(-?\d+)\)?", src)}
    for m in re.finditer(r"(TPTC_(?:SHARD|FUSED)_\w+)\s*=\s*(\d+)", src):
        out[m.group(1)] = int(m.group(2))
    return out


def rust_source():
    return open(os.path.join(RUST, "engine", "cuda_ffi.rs")).read()


def rust_functions():
    src = re.sub(r"//[^\n]*", " ", rust_source())
    block = re.search(r'extern "C"\s*\{(.*)\n\}', src, flags=re.S)
    assert block, "no extern block"
    out = {}
    for m in re.finditer(r"pub fn (tptc_\w+)\s*\(([^)]*)\)", block.group(1)):
        assert m.group(1) not in out, m.group(1)
        out[m.group(1)] = len(_split_params(m.group(2)))
    return out


def rust_struct_fields(name):
    src = rust_source()
    m = re.search(r"pub struct " + name + r"\s*\{(.*?)\n\}", src, flags=re.S)
    assert m, name
    return re.findall(r"pub (\w+)\s*:", m.group(1))


def rust_constants():
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"pub const (TPTC_\w+): c_int = (-?\d+);", rust_source())}


def test_every_c_function_is_bound_with_its_arity():
    c, r = c_functions(), rust_functions()
    assert len(c) > 40
    assert sorted(c) == sorted(r), (sorted(set(c) - set(r)), sorted(set(r) - set(c)))
    for name, n in c.items():
        assert r[name] == n, f"{name}: {n} parameters in tptc.h, {r[name]} in cuda_ffi.rs"


def test_structs_match_field_for_field():
    for name in ("tptc_model_info", "tptc_infer_params"):
        assert c_struct_fields(name) == rust_struct_fields(name), name


def test_constants_match():
    c, r = c_constants(), rust_constants()
    assert len(c) >= 25
    assert c == r


def test_rust_files_state_they_are_not_compiled_here():
    for rel in ("engine/cuda_ffi.rs", "engine/cuda_engine.rs", "build_cuda.rs", "commands_cuda.rs"):
        head = open(os.path.join(RUST, rel)).read(600)
        assert "Not compiled here" in head, rel
