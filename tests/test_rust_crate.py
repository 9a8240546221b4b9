"""The Rust binding crate (crates/rxla-b200) against the C header, on the CPU.

No cargo exists in this image, so the crate's own `cargo test` cannot run
here; this test checks what can go stale without a compiler: every
`extern "C"` item of src/ffi.rs is a function the header declares, with the
same number of parameters and a matching return kind, every header function
has a binding, the #[repr(C)] structs list the header's fields in the
header's order, and the constants carry the header's values.
"""
import re

from tests.conftest import ROOT

HEADER = (ROOT / "include" / "rxla_b200.h").read_text()
FFI = (ROOT / "crates" / "rxla-b200" / "src" / "ffi.rs").read_text()


def _header_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER, flags=re.S)
    out = {}
    for m in re.finditer(r"\n((?:const )?[a-z_0-9]+)\s*\*?\s*(rxla_b200_[a-z0-9_]+)\s*\(([^;]*)\);", text):
        ret, name, params = m.group(1), m.group(2), " ".join(m.group(3).split())
        n = 0 if params in ("void", "") else params.count(",") + 1
        out[name] = (ret, n)
    return out


def _rust_functions():
    block = FFI[FFI.index('extern "C" {'):]
    block = re.sub(r"//[^\n]*", "", block)
    out = {}
    for m in re.finditer(r"pub fn (rxla_b200_[a-z0-9_]+)\s*\((.*?)\)\s*(->\s*([^;]+))?;", block, re.S):
        params = " ".join(m.group(2).split()).rstrip(", ")
        n = 0 if not params else params.count(":")
        out[m.group(1)] = (m.group(4).strip() if m.group(4) else "()", n)
    return out


def test_every_binding_matches_a_header_function():
    h, r = _header_functions(), _rust_functions()
    assert h and r
    assert sorted(h) == sorted(r), (sorted(set(h) ^ set(r)))
    for name, (ret, n) in h.items():
        rret, rn = r[name]
        assert n == rn, f"{name}: {n} parameters in the header, {rn} in ffi.rs"
        want = {"int32_t": "i32", "void": "()", "const char": "*const c_char"}.get(ret, ret)
        assert rret == want, f"{name}: returns {ret} in the header, {rret} in ffi.rs"


def _c_struct_fields(name):
    body = re.search(r"typedef struct " + name + r" \{(.*?)\} " + name + ";", HEADER, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        # the declared names are the last identifier of each declarator
        for part in decl.split(","):
            fields.append(re.search(r"(\w+)\s*$", part).group(1))
    return fields


def _rust_struct_fields(name):
    body = re.search(r"pub struct " + name + r" \{(.*?)\n\}", FFI, re.S).group(1)
    return re.findall(r"pub (\w+):", body)


def test_structs_keep_the_header_field_order():
    for name in ("rxla_b200_paged_decode_args", "rxla_b200_gated_delta_args",
                 "rxla_b200_decoder_config",
                 "rxla_b200_xla_linear_config", "rxla_b200_xla_attention_config"):
        assert _c_struct_fields(name) == _rust_struct_fields(name), name


def test_constants_carry_the_header_values():
    enums = {m.group(1): int(m.group(2)) for m in
             re.finditer(r"(RXLA_B200_\w+)\s*=\s*(-?\d+)", HEADER)}
    rust = {m.group(1): int(m.group(2).replace("_", ""), 0) for m in
            re.finditer(r"pub const (RXLA_B200_\w+): \w+ = (-?[0-9a-fA-Fx_]+);", FFI)}
    for name, value in enums.items():
        assert rust.get(name) == value, name
    for name in ("RXLA_B200_XLA_LINEAR_MAGIC", "RXLA_B200_XLA_ATTENTION_MAGIC"):
        hv = int(re.search(rf"#define {name} (0x[0-9A-Fa-f]+)u", HEADER).group(1), 16)
        assert rust[name] == hv, name
    assert rust["RXLA_B200_COMM_ID_BYTES"] == 128
    # the scratch limit is an expression on both sides: evaluate both
    h = re.search(r"#define RXLA_B200_NOALLOC_SCRATCH_BYTES \(([^)]*)\)", HEADER).group(1)
    r = re.search(r"pub const RXLA_B200_NOALLOC_SCRATCH_BYTES: u32 = ([^;]*);", FFI).group(1)
    ev = lambda e: eval(re.sub(r"(\d+)u\b", r"\1", e), {"__builtins__": {}})
    assert ev(h) == ev(r) == 16 * 1024 * 1024
