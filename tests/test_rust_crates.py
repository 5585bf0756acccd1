"""The Rust crates (crates/sketchpad-b200-sys, crates/sketchpad-b200) against the C header.

This image has no Rust toolchain, so the crates cannot be compiled here; these checks read
them as text:
  * the -sys crate declares every function of include/sketchpad_b200.h, and nothing else,
    with the same argument count and the Rust type that matches each C type;
  * its constants equal the header's enum values;
  * the safe crate calls only functions the -sys crate declares.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SYS = os.path.join(ROOT, "crates", "sketchpad-b200-sys", "src", "lib.rs")
SAFE = os.path.join(ROOT, "crates", "sketchpad-b200", "src", "lib.rs")
HDR = os.path.join(ROOT, "include", "sketchpad_b200.h")

C_TO_RUST = {
    "const void*": "*const c_void", "void*": "*mut c_void", "int64_t": "i64", "int": "c_int",
    "float": "c_float", "double": "c_double", "size_t": "usize",
    "const float*": "*const c_float", "float*": "*mut c_float", "const uint8_t*": "*const u8",
    "uint8_t*": "*mut u8", "int8_t*": "*mut i8", "uint16_t*": "*mut u16",
    "void**": "*mut *mut c_void", "int*": "*mut c_int", "const char*": "*const c_char",
    "const int64_t[4]": "*const i64", "int64_t[4]": "*mut i64", "int64_t[8]": "*mut i64",
    "char*": "*mut c_char", "int64_t*": "*mut i64", "uint64_t*": "*mut u64",
    "const uint8_t**": "*mut *const u8",
}


def header_functions():
    src = re.sub(r"/\*.*?\*/", "", open(HDR).read(), flags=re.S)
    out = {}
    for ret, name, args in re.findall(r"([A-Za-z_][\w\s\*]*?)\b(sp_\w+)\s*\(([^;]*?)\)\s*;", src,
                                      flags=re.S):
        a = " ".join(args.split())
        types = []
        for p in ([] if a == "void" else a.split(",")):
            m = re.match(r"\s*(.*?)\s*(\w+)\s*(\[\d\])?\s*$", p)
            types.append(" ".join(m.group(1).split()) + (m.group(3) or ""))
        out[name] = (" ".join(ret.split()), types)
    return out


def rust_functions():
    src = re.sub(r"//[^\n]*", "", open(SYS).read())
    block = src[src.index('extern "C"'):]
    out = {}
    for name, args, ret in re.findall(r"pub fn (sp_\w+)\s*\((.*?)\)\s*(?:->\s*([^;]+))?;", block,
                                      flags=re.S):
        types = [" ".join(p.split(":", 1)[1].split()) for p in args.split(",") if p.strip()]
        out[name] = (" ".join(ret.split()) if ret else "", types)
    return out


def test_sys_crate_declares_the_header_exactly():
    h, r = header_functions(), rust_functions()
    assert len(h) >= 40
    assert set(h) == set(r), (sorted(set(h) - set(r)), sorted(set(r) - set(h)))
    for name, (cret, cargs) in h.items():
        rret, rargs = r[name]
        assert len(cargs) == len(rargs), name
        for i, (c, rs) in enumerate(zip(cargs, rargs)):
            assert C_TO_RUST[c] == rs, f"{name} argument {i}: C {c} vs Rust {rs}"
        assert C_TO_RUST[cret] == rret, f"{name} return: C {cret} vs Rust {rret}"


def test_sys_crate_constants_match_the_header():
    hdr = open(HDR).read()
    consts = dict(re.findall(r"\b(SP_[A-Z0-9_]+)\s*=\s*(-?\d+)", hdr))
    consts["SP_ABI_VERSION"] = re.search(r"#define SP_ABI_VERSION (\d+)", hdr).group(1)
    rs = dict(re.findall(r"pub const (SP_[A-Z0-9_]+): c_int = (-?\d+);", open(SYS).read()))
    assert set(consts) == set(rs), (sorted(set(consts) - set(rs)), sorted(set(rs) - set(consts)))
    for k, v in consts.items():
        assert int(rs[k]) == int(v), k


def test_safe_crate_calls_only_declared_functions():
    used = set(re.findall(r"sys::(sp_\w+)\s*\(", open(SAFE).read()))
    assert used and used <= set(rust_functions())
    # the reference's operator names are kept
    src = open(SAFE).read()
    for name in ("pub fn flash_attention(", "pub fn flash_attention_masked(",
                 "pub fn groupnorm_silu(", "pub fn groupnorm(", "pub fn dequantize_q8_0(",
                 "pub struct GpuQuantizedLinear", "pub fn from_bytes(", "pub fn quantize_fp8(",
                 "pub struct FlashAttentionOptions", "pub struct GroupNormSiLuOptions"):
        assert name in src, name
