"""The Rust `-sys` crate (crates/tmoe-sys) against the C header it binds.

There is no Rust toolchain here, so the crate is not compiled; this test holds its raw
declarations to include/tmoe.h instead: every exported function in the header's order with the
same parameter names and the Rust types that match the C types, the same struct fields in the same
order, and the same constants.  The header itself is held to the library's exports by test_abi."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tmoe.h")
RAW = os.path.join(ROOT, "crates", "tmoe-sys", "src", "raw.rs")

C_TO_RUST = {"int": "c_int", "int32_t": "i32", "int64_t": "i64", "uint32_t": "u32", "uint64_t": "u64",
             "size_t": "usize", "double": "f64", "float": "f32", "void": "c_void", "char": "c_char"}
RUST_KEYWORDS = {"type": "ty", "in": "r#in"}


def c_to_rust(t):
    t = " ".join(t.split())
    const = t.startswith("const ")
    if const:
        t = t[len("const "):]
    stars = t.count("*")
    base = t.replace("*", "").strip()
    r = C_TO_RUST.get(base, base)
    if stars == 0:
        return r
    r = ("*const " if const else "*mut ") + r
    return "*mut " * (stars - 1) + r


def split_decl(d):
    m = re.match(r"(.*?[\s*])(\w+)$", " ".join(d.split()))
    return m.group(1).strip(), m.group(2)


def header():
    s = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    fns = []
    for ret, args in re.findall(r"TMOE_API\s+([^;]*?)\s*\(([^;]*?)\)\s*;", s, flags=re.S):
        rt, name = split_decl(ret)
        params = []
        if " ".join(args.split()) != "void":
            for a in args.split(","):
                t, n = split_decl(a)
                params.append((RUST_KEYWORDS.get(n, n), c_to_rust(t)))
        fns.append((name, params, None if rt == "void" else c_to_rust(rt)))
    structs = {}
    for body, name in re.findall(r"typedef struct \{(.*?)\}\s*(\w+);", s, flags=re.S):
        fields = []
        for decl in body.split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            m = re.match(r"((?:const )?[\w]+\s*\**)\s*(.*)$", decl)
            ctype = m.group(1)
            for f in m.group(2).split(","):
                f = f.strip()
                stars = f.count("*")
                fields.append((f.strip("* "), c_to_rust(ctype + "*" * stars)))
        structs[name] = fields
    consts = dict(re.findall(r"#define (TMOE_\w+)\s+(-?\d+)", open(HEADER).read()))
    return fns, structs, consts


def rust():
    s = open(RAW).read()
    block = s[s.index('extern "C" {'):]
    fns = []
    for name, params, ret in re.findall(r"pub fn (\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        ps = []
        for p in [p.strip() for p in params.split(",") if p.strip()]:
            n, t = p.split(":", 1)
            ps.append((n.strip(), " ".join(t.split())))
        fns.append((name, ps, ret.strip() if ret else None))
    structs = {}
    for name, body in re.findall(r"pub struct (\w+) \{(.*?)\}", s, flags=re.S):
        structs[name] = [(f.strip(), " ".join(t.split())) for f, t in
                         re.findall(r"pub (\w+):\s*([^,]+),", body)]
    consts = dict(re.findall(r"pub const (TMOE_\w+): c_int = (-?\d+);", s))
    return fns, structs, consts


def test_every_header_function_is_declared_in_order_with_matching_types():
    h_fns, _, _ = header()
    r_fns, _, _ = rust()
    assert [f[0] for f in r_fns] == [f[0] for f in h_fns]
    for (name, hp, hr), (_, rp, rr) in zip(h_fns, r_fns):
        assert rp == hp, f"{name}: parameters {rp} != header {hp}"
        assert rr == hr, f"{name}: returns {rr} != header {hr}"


def test_structs_and_constants_match_the_header():
    _, h_structs, h_consts = header()
    _, r_structs, r_consts = rust()
    for name in ("tmoe_config", "tmoe_expert_tensors", "tmoe_trace_info"):
        assert r_structs[name] == h_structs[name], name
    h_consts.pop("TMOE_H", None)
    assert r_consts == h_consts


def test_safe_layer_wraps_the_entry_points_the_builder_calls():
    lib = open(os.path.join(ROOT, "crates", "tmoe-sys", "src", "lib.rs")).read()
    for fn in ("tmoe_create", "tmoe_layer", "tmoe_route", "tmoe_experts", "tmoe_mul_mat_id", "tmoe_ep_layer",
               "tmoe_streamed_layer", "tmoe_slots_create", "tmoe_comm_init", "tmoe_gguf_open", "tmoe_check"):
        assert f"raw::{fn}(" in lib, fn
