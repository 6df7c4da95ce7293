"""The Rust crate's FFI mirror (crates/backends/backend-cuda/src/ffi.rs)
against the C header it binds, checked on CPU since no Rust toolchain is in
this image:

- every #[repr(C)] struct has the C struct's fields, in order, at the same
  offsets and with the same total size: the Rust layout is computed by the
  repr(C) rules from the declared field types, the C layout is measured by
  compiling a program with gcc against include/starlight_cuda.h;
- every function of the `extern "C"` block is declared in include/*.h with
  the same number of parameters, the same kind of each parameter (pointer,
  32-bit or 64-bit integer, float) and the same kind of result;
- every `pub const` has the value the header gives the same name."""
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FFI = os.path.join(ROOT, "crates", "backends", "backend-cuda", "src", "ffi.rs")
HEADER = os.path.join(ROOT, "include", "starlight_cuda.h")

RUST_SCALARS = {"u8": (1, "u8"), "i8": (1, "u8"), "u16": (2, "u16"), "i16": (2, "u16"),
                "u32": (4, "u32"), "i32": (4, "i32"), "c_int": (4, "i32"), "f32": (4, "f32"),
                "u64": (8, "u64"), "i64": (8, "u64"), "usize": (8, "u64"), "f64": (8, "f64")}
C_SCALARS = {"int": "i32", "int32_t": "i32", "uint32_t": "u32", "unsigned": "u32",
             "uint64_t": "u64", "int64_t": "u64", "size_t": "u64", "float": "f32",
             "double": "f64", "uint16_t": "u16", "uint8_t": "u8"}


def _strip_comments(text, rust=True):
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _rust_source():
    return _strip_comments(open(FFI).read())


def _consts(src):
    return {m.group(1): int(m.group(2), 0)
            for m in re.finditer(r"pub const (\w+)\s*:\s*\w+\s*=\s*([0-9xa-fA-F]+)\s*;", src)}


def _rust_structs(src):
    out = {}
    for m in re.finditer(r"#\[repr\(C\)\]\s*(?:#\[[^\]]*\]\s*)*pub struct (\w+)\s*\{(.*?)\}",
                         src, flags=re.S):
        fields = []
        for f in m.group(2).split(","):
            f = f.strip()
            if not f:
                continue
            fm = re.match(r"(?:pub\s+)?(\w+)\s*:\s*(.+)$", f)
            assert fm, f
            fields.append((fm.group(1), fm.group(2).strip()))
        out[m.group(1)] = fields
    return out


def _rust_size_align(ty, consts):
    ty = ty.strip()
    if ty.startswith("*"):
        return 8, 8
    am = re.match(r"\[\s*(\w+)\s*;\s*(\w+)\s*\]$", ty)
    if am:
        size, align = _rust_size_align(am.group(1), consts)
        n = int(am.group(2)) if am.group(2).isdigit() else consts[am.group(2)]
        return size * n, align
    size = RUST_SCALARS[ty][0]
    return size, size


def _rust_layout(fields, consts):
    off, offsets, max_align = 0, [], 1
    for _, ty in fields:
        size, align = _rust_size_align(ty, consts)
        off = (off + align - 1) // align * align
        offsets.append(off)
        off += size
        max_align = max(max_align, align)
    return offsets, (off + max_align - 1) // max_align * max_align


def _snake(name):
    return re.sub(r"(?<!^)(?=[A-Z])", "_", name).lower()


def _c_layouts(structs):
    """{c_name: ([offsets], size)} measured by gcc."""
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for rname, fields in structs.items():
        c = _snake(rname)
        for fname, _ in fields:
            lines.append(f'printf("{c} {fname} %zu\\n", offsetof({c}, {fname}));')
        lines.append(f'printf("{c} __size %zu\\n", sizeof({c}));')
    lines.append("return 0; }")
    with tempfile.TemporaryDirectory() as tmp:
        src, exe = os.path.join(tmp, "l.c"), os.path.join(tmp, "l")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-o", exe, src], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    res = {}
    for line in out.splitlines():
        c, f, v = line.split()
        offs, size = res.setdefault(c, ([], None))
        if f == "__size":
            res[c] = (offs, int(v))
        else:
            offs.append(int(v))
    return res


def _split_params(params):
    params = params.strip()
    if not params or params == "void":
        return []
    return [p.strip() for p in params.split(",")]


def _rust_kind(ty):
    ty = ty.strip()
    if ty.startswith("*"):
        return "ptr"
    if ty in RUST_SCALARS:
        return RUST_SCALARS[ty][1]
    return "struct " + _snake(ty)  # a #[repr(C)] struct passed by value


def _c_kind(decl):
    decl = re.sub(r"\bconst\b", "", decl).strip()
    if "*" in decl or "[" in decl:
        return "ptr"
    ty = decl.split()[0]  # "uint32_t name" or a bare type
    return C_SCALARS[ty] if ty in C_SCALARS else "struct " + ty


def _rust_functions(src):
    block = re.search(r'extern "C"\s*\{(.*?)\n\}', src, flags=re.S).group(1)
    out = {}
    for m in re.finditer(r"pub fn (\w+)\s*\((.*?)\)\s*(->\s*([^;]+))?;", block, flags=re.S):
        params = [p.split(":", 1)[1] for p in _split_params(m.group(2)) if p]
        ret = _rust_kind(m.group(4)) if m.group(4) else "void"
        out[m.group(1)] = ([_rust_kind(p) for p in params], ret)
    return out


def _c_functions():
    out = {}
    for h in os.listdir(os.path.join(ROOT, "include")):
        if not h.endswith(".h"):
            continue
        text = _strip_comments(open(os.path.join(ROOT, "include", h)).read())
        for m in re.finditer(r"^([A-Za-z_][\w \*]*?)\b(slc_\w+)\s*\(([^)]*)\)\s*;", text,
                             flags=re.M):
            ret = m.group(1).strip()
            ret_kind = "void" if ret == "void" else ("ptr" if "*" in ret else
                                                    C_SCALARS[ret.replace("const", "").split()[0]])
            out[m.group(2)] = ([_c_kind(p) for p in _split_params(m.group(3))], ret_kind)
    return out


def test_ffi_file_exists():
    assert os.path.exists(FFI)


def test_repr_c_structs_match_the_header_layout():
    src = _rust_source()
    consts = _consts(src)
    structs = _rust_structs(src)
    # Opaque handles (zero-sized private field) have no C layout to match.
    structs = {k: v for k, v in structs.items() if not (len(v) == 1 and v[0][0] == "_private")}
    assert {"SlcError", "SlcValue", "SlcBufferRef", "SlcOp", "SlcCapabilities"} <= set(structs)
    measured = _c_layouts(structs)
    for rname, fields in structs.items():
        offsets, size = _rust_layout(fields, consts)
        c_offsets, c_size = measured[_snake(rname)]
        assert offsets == c_offsets, (rname, offsets, c_offsets)
        assert size == c_size, (rname, size, c_size)


def test_extern_functions_match_the_header_declarations():
    rust = _rust_functions(_rust_source())
    c = _c_functions()
    assert len(rust) >= 15
    for name, (params, ret) in rust.items():
        assert name in c, f"{name} is not declared in include/*.h"
        c_params, c_ret = c[name]
        assert params == c_params, (name, params, c_params)
        assert ret == c_ret, (name, ret, c_ret)


def test_constants_match_the_header():
    header = _strip_comments(open(HEADER).read())
    for name, value in _consts(_rust_source()).items():
        m = re.search(rf"\b{name}\s*=\s*([0-9xa-fA-F]+)", header) or \
            re.search(rf"#define\s+{name}\s+([0-9xa-fA-F]+)u?", header)
        assert m, f"{name} is not defined in the header"
        assert int(m.group(1), 0) == value, (name, value, m.group(1))


@pytest.mark.parametrize("rust,c", [("*mut SlcDevice", "slc_device *device"),
                                    ("u64", "uint64_t len"), ("c_int", "int rank"),
                                    ("SlcBufferRef", "slc_buffer_ref weights")])
def test_kind_mapping(rust, c):
    assert _rust_kind(rust) == _c_kind(c)


def test_lib_uses_only_names_the_ffi_declares():
    lib = _strip_comments(open(os.path.join(os.path.dirname(FFI), "lib.rs")).read())
    src = _rust_source()
    declared = set(re.findall(r"pub (?:fn|struct|const) (\w+)", src))
    used = set(re.findall(r"ffi::(\w+)", lib))
    assert used and used <= declared, sorted(used - declared)
