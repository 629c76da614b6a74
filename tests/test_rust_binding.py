"""The Rust crate's raw bindings (rs-gallium_b200/crates/gallium-b200/src/ffi.rs)
against the C header, without a Rust toolchain: every struct field in the same
order with the corresponding type, every function the header declares bound
with the same number of parameters, and the same ABI version."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gallium_b200.h")
FFI = os.path.join(ROOT, "rs-gallium_b200", "crates", "gallium-b200", "src", "ffi.rs")

C_TO_RUST = {
    "uint32_t": "u32", "int32_t": "i32", "int64_t": "i64", "float": "f32",
    "const void*": "*const c_void", "const uint8_t*": "*const u8", "const float*": "*const f32",
    "const uint16_t*": "*const u16", "const gb_moe_desc*": "*const gb_moe_desc",
    "const gb_decoder_layer*": "*const gb_decoder_layer",
}


def _c_struct(src, name):
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), src, re.S).group(1)
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = " ".join(decl.split())
        if not decl:
            continue
        m = re.match(r"(const \w+\*|\w+) (.+)", decl)
        ctype, names = m.group(1), m.group(2)
        for n in names.split(","):
            fields.append((n.strip(), C_TO_RUST[ctype]))
    return fields


def _rust_struct(src, name):
    body = re.search(r"pub struct %s \{(.*?)\n\}" % name, src, re.S).group(1)
    return [(m.group(1), m.group(2).strip()) for m in
            re.finditer(r"pub (\w+): ([^,]+),", body)]


def test_structs_match_the_header_field_for_field():
    h, r = open(HEADER).read(), open(FFI).read()
    for name in ("gb_moe_desc", "gb_moe_info", "gb_decoder_layer", "gb_decoder_desc"):
        assert _rust_struct(r, name) == _c_struct(h, name), name


def test_every_function_is_bound_with_its_arity():
    h, r = open(HEADER).read(), open(FFI).read()
    h = re.sub(r"/\*.*?\*/", "", h, flags=re.S)
    c_fns = {m.group(1): (m.group(2).count(",") + 1 if m.group(2).strip() not in ("", "void") else 0)
             for m in re.finditer(r"^(?:int|const char\*) (gb_\w+)\((.*?)\);", h, re.S | re.M)}
    ext = re.search(r'extern "C" \{(.*?)\n\}', r, re.S).group(1)
    r_fns = {m.group(1): (m.group(2).count(":")) for m in
             re.finditer(r"pub fn (gb_\w+)\((.*?)\)", ext, re.S)}
    assert c_fns == r_fns


def test_abi_version_and_enums_agree():
    h, r = open(HEADER).read(), open(FFI).read()
    ver = re.search(r"#define GB_ABI_VERSION (\d+)", h).group(1)
    assert re.search(r"GB_ABI_VERSION: c_int = %s;" % ver, r)
    for name, val in re.findall(r"\b(GB_(?:ROUTER|ACT|FMT|DTYPE|PATH|ERR)_\w+) = (\d+)", h):
        assert re.search(r"pub const %s: \w+ = %s;" % (name, val), r), name
