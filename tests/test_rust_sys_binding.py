"""The Rust -sys crate (kivi-cache-rs_b200/rust/kivi-cache-sys) against the C
header: every function of include/kivi_gpu.h has exactly one extern "C"
declaration with the same parameter count and ABI-equivalent types, and the
#[repr(C)] structs list the header's fields in order.  (No Rust toolchain is
available here; this keeps the bindings from drifting when the header
changes.)"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kivi_gpu.h")
LIBRS = os.path.join(ROOT, "kivi-cache-rs_b200", "rust", "kivi-cache-sys", "src", "lib.rs")

SCALARS = {"int32_t": "i32", "uint32_t": "u32", "uint64_t": "u64", "float": "f32",
           "double": "f64", "char": "c_char", "void": "c_void"}


def c_to_rust(t):
    """ABI-equivalent Rust type of a C parameter or return type (None = void)."""
    toks = " ".join(t.replace("*", " * ").split()).split()
    const = toks[0] == "const"
    if const:
        toks = toks[1:]
    base = SCALARS.get(toks[0], toks[0])
    levels, cur = [], const
    rest = toks[1:]
    while rest:
        assert rest[0] == "*", t
        levels.append(cur)
        cur, rest = False, rest[1:]
        if rest and rest[0] == "const":
            cur, rest = True, rest[1:]
    if not levels and base == "c_void":
        return None
    out = base
    for c in levels:
        out = ("*const " if c else "*mut ") + out
    return out


def header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(
            r"^\s*((?:const\s+)?[a-z_0-9]+\s*\**)\s*\b(kivi_[a-z_0-9]+)\s*\(([^;]*?)\)\s*;", src,
            flags=re.M):
        args = " ".join(args.split())
        params = [] if args in ("void", "") else [p.strip() for p in args.split(",")]
        types = [c_to_rust(re.match(r"(.*?)[A-Za-z_][A-Za-z_0-9]*$", p).group(1)) for p in params]
        out[name] = (types, c_to_rust(ret))
    return out


def rust_functions():
    src = open(LIBRS).read()
    block = src[src.index('extern "C" {'):]
    out = {}
    for name, args, ret in re.findall(r"pub fn (kivi_[a-z_0-9]+)\(([^)]*)\)\s*(?:->\s*([^;]+))?;",
                                      block):
        params = [p.strip() for p in args.split(",") if p.strip()]
        types = [" ".join(p.split(":", 1)[1].split()) for p in params]
        out[name] = (types, " ".join(ret.split()) if ret else None)
    return out


def test_every_header_function_is_bound_with_the_same_signature():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 60
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, (types, ret) in h.items():
        assert r[name] == (types, ret), (name, r[name], (types, ret))


def _c_struct_fields(name):
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), src, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if decl:
            fields.append(re.match(r".*?([A-Za-z_][A-Za-z_0-9]*)(\[[^\]]*\])?$", decl).group(1))
    return fields


def _rust_struct_fields(name):
    src = open(LIBRS).read()
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, src, flags=re.S).group(1)
    return re.findall(r"pub ([a-z_0-9]+):", body)


def test_repr_c_structs_follow_the_header_field_order():
    for name in ("kivi_error", "kivi_config", "kivi_memory_report", "kivi_cache_state",
                 "kivi_budget_snapshot", "kivi_prefix_footprint", "kivi_quality_upgrade",
                 "kivi_flush_check"):
        assert _c_struct_fields(name) == _rust_struct_fields(name), name


def test_status_codes_match():
    src = open(HEADER).read()
    rs = open(LIBRS).read()
    for name, val in re.findall(r"(KIVI_(?:OK|ERR_[A-Z_]+))\s*=\s*(\d+)", src):
        assert re.search(r"pub const %s: i32 = %s;" % (name, val), rs), name
