"""The Rust crate's bindings (crates/mold-b200/src/ffi.rs) against the C header: every MB_API
entry point is declared with the same number of parameters, the #[repr(C)] structs have the
header's fields in the header's order, and lib.rs calls only declared functions. (No Rust
toolchain exists in this image, so the crate is checked as text.)"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = open(os.path.join(ROOT, "include", "mold_b200.h")).read()
FFI = open(os.path.join(ROOT, "crates", "mold-b200", "src", "ffi.rs")).read()
LIB = open(os.path.join(ROOT, "crates", "mold-b200", "src", "lib.rs")).read()


def _strip_c(s):
    return re.sub(r"/\*.*?\*/", "", s, flags=re.S)


def header_fns():
    out = {}
    for ret, args in re.findall(r"MB_API\s+([^;]+?)\s*\(([^;]*?)\)\s*;", _strip_c(HDR), flags=re.S):
        name = re.match(r".*?(\w+)$", " ".join(ret.split())).group(1)
        a = " ".join(args.split())
        out[name] = 0 if a in ("", "void") else len(a.split(","))
    return out


def rust_fns():
    block = FFI[FFI.index('extern "C" {'):]
    out = {}
    for name, params in re.findall(r"pub fn (\w+)\((.*?)\)\s*->", block, flags=re.S):
        p = [x for x in (s.strip() for s in params.split(",")) if x]
        out[name] = len(p)
    return out


def test_every_entry_point_is_bound_with_its_arity():
    h, r = header_fns(), rust_fns()
    assert len(h) >= 40
    assert set(h) == set(r), (set(h) ^ set(r))
    for n in h:
        assert h[n] == r[n], (n, h[n], r[n])


def _c_struct_fields(tag):
    body = re.search(r"typedef struct \{([^{}]*?)\}\s*" + tag + ";", _strip_c(HDR), flags=re.S).group(1)
    return re.findall(r"(\w+)(?:\[\d+\])?;", body)


def _rust_struct_fields(name):
    body = re.search(r"pub struct " + name + r" \{(.*?)\n\}", FFI, flags=re.S).group(1)
    return re.findall(r"pub (\w+):", body)


def test_repr_c_structs_match_header():
    for c, rs in (("mb_flux_config", "MbFluxConfig"), ("mb_qwen_config", "MbQwenConfig"), ("mb_inpaint", "MbInpaint")):
        assert _c_struct_fields(c) == _rust_struct_fields(rs), c


def test_lib_calls_only_declared_functions():
    called = set(re.findall(r"ffi::(mb_\w+)\(", LIB))
    assert called and called <= set(rust_fns())
    # the seams the crate promises are present
    for sym in ("struct B200QMatMul", "impl Module for B200QMatMul", "struct B200Flux", "struct B200Qwen",
                "mb_flux_denoise_ex", "mb_qwen_denoise_ex", "mb_flux_load_gguf"):
        assert sym in LIB, sym
