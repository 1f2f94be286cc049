"""The Rust FFI crate (rust/rustgears-cuda-sys) against the C ABI it binds
(include/rg_npu.h): the same entry points with the same argument and return types,
the same #[repr(C)] field names, types and order, and the same enum and flag values.
No Rust toolchain exists on these machines, so this parse-level check is what keeps
the crate from drifting from the header."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rg_npu.h")
CRATE = os.path.join(ROOT, "rust", "rustgears-cuda-sys", "src", "lib.rs")

SCALARS = {"int32_t": "i32", "int64_t": "i64", "uint64_t": "u64", "uint8_t": "u8", "int8_t": "i8", "float": "f32",
           "char": "c_char", "void": "c_void", "rg_status": "rg_status"}


def _strip_c(src):
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.sub(r"//[^\n]*", "", src)


def c_type_to_rust(t: str) -> str:
    """A C parameter / field type (pointer stars, const, and array parameters) in Rust."""
    t = " ".join(t.split())
    arr = re.match(r"^(const\s+)?(\w+)\s+\w+\[\d+\]$", t)   # `uint8_t id[128]` as a parameter
    if arr:
        return ("*const " if arr.group(1) else "*mut ") + SCALARS.get(arr.group(2), arr.group(2))
    const = t.startswith("const ")
    if const:
        t = t[len("const "):]
    stars = t.count("*")
    base = t.replace("*", "").strip()
    base = SCALARS.get(base, base)
    if stars == 0:
        return base
    out = base
    for i in range(stars):
        out = ("*const " if (const and i == stars - 1) else "*mut ") + out
    return out


def header_functions():
    src = _strip_c(open(HEADER).read())
    fns = {}
    for m in re.finditer(r"^\s*((?:const\s+)?[a-z_0-9]+\s*\**)\s*(rg_[a-z_0-9]+)\s*\(([^)]*)\);", src, flags=re.M):
        ret, name, args = m.group(1).strip(), m.group(2), " ".join(m.group(3).split())
        params = []
        if args != "void":
            for a in args.split(","):
                a = a.strip()
                if re.search(r"\[\d+\]$", a):
                    params.append(c_type_to_rust(a))
                else:
                    params.append(c_type_to_rust(re.sub(r"\s*\b\w+$", "", a)))   # drop the parameter name
        fns[name] = (c_type_to_rust(ret) if ret != "void" else None, params)
    return fns


def crate_functions():
    src = open(CRATE).read()
    block = src[src.index('extern "C" {'):]
    fns = {}
    for m in re.finditer(r"pub fn (rg_\w+)\((.*?)\)\s*(?:->\s*([^;]+))?;", block, flags=re.S):
        name, args, ret = m.group(1), " ".join(m.group(2).split()), m.group(3)
        params = [a.split(":", 1)[1].strip() for a in args.split(",") if a.strip()]
        fns[name] = (ret.strip() if ret else None, params)
    return fns


def header_structs():
    src = _strip_c(open(HEADER).read())
    out = {}
    for m in re.finditer(r"typedef struct (rg_\w+) \{(.*?)\} \1;", src, flags=re.S):
        fields = []
        for decl in m.group(2).split(";"):
            decl = " ".join(decl.split())
            if not decl:
                continue
            dm = re.match(r"^((?:const\s+)?\w+\s*\**)\s*(.*)$", decl)
            base, names = dm.group(1), dm.group(2)
            for nm in names.split(","):
                nm = nm.strip()
                stars = nm.count("*")
                nm = nm.replace("*", "").strip()
                arr = re.match(r"^(\w+)\[(\d+)\]$", nm)
                if arr:
                    fields.append((arr.group(1), f"[{SCALARS.get(base.strip(), base.strip())}; {arr.group(2)}]"))
                else:
                    fields.append((nm, c_type_to_rust(base + "*" * stars)))
        out[m.group(1)] = fields
    return out


def crate_structs():
    src = open(CRATE).read()
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*(?:#\[derive\([^)]*\)\]\s*)?pub struct (rg_\w+) \{(.*?)\n\}", src, flags=re.S):
        fields = [(fm.group(1), " ".join(fm.group(2).split()))
                  for fm in re.finditer(r"pub (\w+): ([^,\n]+),", m.group(2))]
        out[m.group(1)] = fields
    return out


def header_constants():
    src = _strip_c(open(HEADER).read())
    consts = {}
    for body in re.findall(r"typedef enum \w+ \{(.*?)\}", src, flags=re.S):
        for nm, v in re.findall(r"(RG_\w+)\s*=\s*(\d+)", body):
            consts[nm] = int(v)
    for nm, v in re.findall(r"#define (RG_\w+) (\d+)\b", src):
        consts[nm] = int(v)
    for nm, v, sh in re.findall(r"#define (RG_\w+) \((\d+)u << (\d+)\)", src):
        consts[nm] = int(v) << int(sh)
    return consts


def crate_constants():
    src = open(CRATE).read()
    out = {}
    for nm, v in re.findall(r"pub const (RG_\w+): \w+ = ([^;]+);", src):
        v = v.strip()
        sh = re.match(r"^(\d+) << (\d+)$", v)
        out[nm] = int(sh.group(1)) << int(sh.group(2)) if sh else int(v)
    return out


def test_every_entry_point_is_declared_with_the_same_types():
    h, r = header_functions(), crate_functions()
    assert len(h) >= 35
    assert set(h) == set(r), f"only in the header: {set(h) - set(r)}; only in the crate: {set(r) - set(h)}"
    for name, (ret, params) in h.items():
        rret, rparams = r[name]
        assert len(params) == len(rparams), f"{name}: {len(params)} C arguments, {len(rparams)} Rust"
        assert params == rparams, f"{name}: {params} != {rparams}"
        assert ret == rret, f"{name}: returns {ret} in C, {rret} in Rust"


def test_repr_c_structs_match_field_for_field():
    h, r = header_structs(), crate_structs()
    assert {"rg_layer_spec", "rg_session_options", "rg_profile", "rg_op_record", "rg_op_info", "rg_rng"} <= set(h)
    for name, fields in h.items():
        assert name in r, f"{name} has no #[repr(C)] struct in the crate"
        assert fields == r[name], f"{name}: {fields} != {r[name]}"


def test_enum_and_flag_values_match():
    h, r = header_constants(), crate_constants()
    for group in ("RG_OK", "RG_ERR_", "RG_LAYER_", "RG_ACT_", "RG_PREC_", "RG_SESSION_", "RG_TRACE_", "RG_RUN_"):
        names = [n for n in h if n.startswith(group)]
        assert names, group
        for n in names:
            assert n in r, f"{n} missing from the crate"
            assert r[n] == h[n], f"{n}: {h[n]} in C, {r[n]} in Rust"
    assert r["RG_NPU_ABI_VERSION"] == h["RG_NPU_ABI_VERSION"]
    assert r["RG_LINEAR_NOALLOC_MAX_BYTES"] == h["RG_LINEAR_NOALLOC_MAX_BYTES"] == 16 << 20


def test_wrapper_uses_only_declared_entry_points():
    """The reference-side wrapper (rust/device-cuda/cuda.rs) calls nothing the crate lacks."""
    src = open(os.path.join(ROOT, "rust", "device-cuda", "cuda.rs")).read()
    used = set(re.findall(r"sys::(rg_\w+)\(", src))
    assert used and used <= set(crate_functions())
