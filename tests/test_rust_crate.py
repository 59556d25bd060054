"""The barracuda-cuda-sys crate (crates/barracuda-cuda-sys/src/lib.rs) must
declare the C ABI of include/barracuda_fhe.h one to one: every function with
the same name, argument count and argument types, the same return type, the
same struct layouts and constants.  There is no Rust toolchain in this image,
so the check reads both files as text; the library's exports are checked
against the header in test_capi.py."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "barracuda_fhe.h")
CRATE = os.path.join(ROOT, "crates", "barracuda-cuda-sys")
LIB_RS = os.path.join(CRATE, "src", "lib.rs")

# C type -> Rust FFI type
C2RUST = {
    "void": None,
    "int": "c_int",
    "int32_t": "i32",
    "int64_t": "i64",
    "uint32_t": "u32",
    "uint64_t": "u64",
    "size_t": "usize",
    "double *": "*mut f64",
    "int *": "*mut c_int",
    "void *": "*mut c_void",
    "const void *": "*const c_void",
    "void **": "*mut *mut c_void",
    "uint64_t *": "*mut u64",
    "const uint64_t *": "*const u64",
    "bc_ctx *": "*mut bc_ctx",
    "const bc_ctx *": "*const bc_ctx",
    "bc_ctx **": "*mut *mut bc_ctx",
    "bc_plan *": "*mut bc_plan",
    "const bc_plan *": "*const bc_plan",
    "bc_plan **": "*mut *mut bc_plan",
    "const bc_layout *": "*const bc_layout",
    "bc_plan_info *": "*mut bc_plan_info",
    "const char *": "*const c_char",
}


def _norm_c(t):
    t = " ".join(t.replace("*", " * ").split())
    return t.replace("* *", "**").replace(" *", " *")


def header_functions():
    h = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"\n((?:const )?[a-z_0-9]+ \*?)\s*(bc_[a-z0-9_]+)\(([^;]*?)\);", h):
        params = []
        if args.strip() != "void":
            for a in args.split(","):
                a = " ".join(a.split())
                m = re.match(r"(.*?)(\w+)$", a)
                typ = _norm_c(m.group(1).strip())
                params.append((m.group(2), typ))
        out[name] = (_norm_c(ret.strip()), params)
    return out


def crate_functions():
    src = open(LIB_RS).read()
    block = re.search(r'extern "C" \{(.*?)\n    \}', src, flags=re.S).group(1)
    block = re.sub(r"//[^\n]*", "", block)
    out = {}
    for name, args, ret in re.findall(r"pub fn (bc_\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        params = []
        for a in [x for x in args.split(",") if x.strip()]:
            n, t = a.split(":", 1)
            params.append((n.strip(), " ".join(t.split())))
        out[name] = ((ret or "").strip() or None, params)
    return out


def test_crate_files_exist():
    for f in ("Cargo.toml", "build.rs", os.path.join("src", "lib.rs")):
        assert os.path.exists(os.path.join(CRATE, f)), f
    toml = open(os.path.join(CRATE, "Cargo.toml")).read()
    assert 'name = "barracuda-cuda-sys"' in toml and 'links = "barracuda_fhe"' in toml
    assert "rustc-link-lib=dylib=barracuda_fhe" in open(os.path.join(CRATE, "build.rs")).read()


def test_every_header_function_is_declared_with_the_same_signature():
    h, r = header_functions(), crate_functions()
    assert len(h) >= 60
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, (ret, params) in h.items():
        rret, rparams = r[name]
        assert C2RUST[ret] == rret, (name, ret, rret)
        assert len(params) == len(rparams), (name, params, rparams)
        for (cn, ct), (rn, rt) in zip(params, rparams):
            assert cn == rn, (name, cn, rn)
            assert C2RUST[ct] == rt, (name, cn, ct, rt)


def test_structs_and_constants_match():
    h = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    src = open(LIB_RS).read()
    for struct in ("bc_layout", "bc_plan_info"):
        cfields = re.findall(r"(\w+) (\w+);", re.search(r"typedef struct %s \{(.*?)\}" % struct, h, re.S).group(1))
        rfields = re.findall(r"pub (\w+): (\w+),", re.search(r"pub struct %s \{(.*?)\}" % struct, src, re.S).group(1))
        assert [(n, C2RUST[t]) for t, n in cfields] == rfields, struct
    for name, val in re.findall(r"(BC_\w+) = (\d+)", h):
        assert re.search(r"pub const %s: c_int = %s;" % (name, val), src), name
    assert re.search(r"#define BC_ABI_VERSION (\d+)", h).group(1) == \
        re.search(r"pub const BC_ABI_VERSION: c_int = (\d+);", src).group(1)
    assert "(1u << 21)" in h and "BC_POLYMUL_STATIC_MAX_COEFFS: u32 = 1 << 21;" in src


def test_unsafe_stays_in_this_crate():
    """The safe layer wraps every call; the constructors' validation keeps the
    reference's messages (the crate's own Rust tests pin two)."""
    src = open(LIB_RS).read()
    assert "pub mod safe" in src and "impl Drop for Context" in src and "impl Drop for Plan" in src
    for op in ("fhe_ntt", "fhe_intt", "fhe_pointwise_mul", "fhe_fast_poly_mul"):
        assert f"pub fn {op}(" in src and f"pub fn {op}_check(" in src, op
