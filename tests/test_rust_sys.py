"""CPU check of the Rust sys crate (mlx-rs_b200/crates/mlxr-cuda-sys) against
the C header: every #[repr(C)] struct has the header's fields in the same
order with matching types, and every entry point the header declares is
bound with the same argument types. There is no Rust toolchain in this
image, so the crate is checked as text."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "mlxr_moe.h")
LIB = os.path.join(ROOT, "mlx-rs_b200", "crates", "mlxr-cuda-sys", "src", "lib.rs")

C2RUST = {
    "int32_t": "i32", "int": "c_int", "float": "f32", "int64_t": "i64", "uint32_t": "u32", "uint64_t": "u64",
    "size_t": "usize", "void": "c_void", "char": "c_char", "mlxr_cu_dtype": "c_int",
}


def _strip_c_comments(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def _strip_rust_comments(s):
    return re.sub(r"//[^\n]*", "", s)


def c_type_to_rust(t):
    t = " ".join(t.split())
    ptrs = t.count("*")
    base = t.replace("*", "").replace("const", "").strip()
    const_ptr = t.startswith("const") or " const" in t.split("*")[0]
    rbase = C2RUST.get(base, base)
    if ptrs == 0:
        return rbase
    if ptrs == 1:
        return ("*const " if const_ptr else "*mut ") + rbase
    # void* const* / void** (pointer to pointer)
    inner = "*mut " + rbase
    if ptrs == 2 and "const" in t.split("*")[1]:
        return "*const " + inner
    return ("*const " if const_ptr else "*mut ") + inner


def split_params(s):
    out, depth, cur = [], 0, ""
    for ch in s:
        if ch == "(":
            depth += 1
        elif ch == ")":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    if cur.strip():
        out.append(cur)
    return [p.strip() for p in out if p.strip() and p.strip() != "void"]


def c_structs():
    h = _strip_c_comments(open(HDR).read())
    res = {}
    for m in re.finditer(r"typedef struct (\w+) \{(.*?)\} (\w+);", h, re.S):
        fields = []
        for decl in m.group(2).split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            mm = re.match(r"(.*?)(\w+)$", decl)
            fields.append((mm.group(2), c_type_to_rust(mm.group(1))))
        res[m.group(3)] = fields
    return res


def c_functions():
    h = _strip_c_comments(open(HDR).read())
    res = {}
    for m in re.finditer(r"MLXR_CU_API\s+([\w\s\*]+?)\s*\b(mlxr_cu_\w+)\s*\((.*?)\);", h, re.S):
        params = []
        for p in split_params(m.group(3)):
            mm = re.match(r"(.*?)(\w+)$", " ".join(p.split()))
            params.append(c_type_to_rust(mm.group(1)))
        res[m.group(2)] = (c_type_to_rust(m.group(1)), params)
    return res


def rust_structs():
    r = _strip_rust_comments(open(LIB).read())
    res = {}
    for m in re.finditer(r"#\[repr\(C\)\][^\n]*\npub struct (\w+) \{(.*?)\}", r, re.S):
        fields = []
        for f in m.group(2).split(","):
            f = " ".join(f.split())
            if not f:
                continue
            mm = re.match(r"pub (\w+): (.+)$", f)
            fields.append((mm.group(1), mm.group(2)))
        res[m.group(1)] = fields
    return res


def rust_functions():
    r = _strip_rust_comments(open(LIB).read())
    body = r[r.index('extern "C" {'):]
    res = {}
    for m in re.finditer(r"pub fn (\w+)\((.*?)\)\s*(->\s*([\w\*\s]+))?;", body, re.S):
        params = [" ".join(p.split(":", 1)[1].split()) for p in split_params(m.group(2))]
        ret = " ".join(m.group(4).split()) if m.group(4) else "c_void"
        res[m.group(1)] = (ret, params)
    return res


def test_structs_match_header_field_by_field():
    cs, rs = c_structs(), rust_structs()
    assert set(cs) == {"mlxr_cu_moe_config", "mlxr_cu_qlinear", "mlxr_cu_moe_weights", "mlxr_cu_moe_routing"}
    for name, fields in cs.items():
        assert name in rs, f"{name} missing from the sys crate"
        assert rs[name] == fields, f"{name}: header {fields} vs crate {rs[name]}"


def test_every_entry_point_is_bound_with_the_same_signature():
    cf, rf = c_functions(), rust_functions()
    assert len(cf) >= 30
    missing = sorted(set(cf) - set(rf))
    assert not missing, f"entry points not bound in the sys crate: {missing}"
    for name, (ret, params) in cf.items():
        rret, rparams = rf[name]
        assert rret == ret, f"{name}: return {ret} vs {rret}"
        assert rparams == params, f"{name}: header {params} vs crate {rparams}"


def test_crate_files_present():
    d = os.path.dirname(os.path.dirname(LIB))
    cargo = open(os.path.join(d, "Cargo.toml")).read()
    assert 'name = "mlxr-cuda-sys"' in cargo and 'links = "mlxr_moe"' in cargo
    build = open(os.path.join(d, "build.rs")).read()
    assert "rustc-link-lib=dylib=mlxr_moe" in build
