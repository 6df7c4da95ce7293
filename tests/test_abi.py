"""CPU-side checks of the C ABI: the library exists, loads without a GPU, and
exports every entry point declared in include/*.h; the Python mirror binds
the same names; the ABI enums keep the sl-ir discriminants."""
import ctypes
import glob
import os
import re

import pytest

from starlight_b200 import device as D

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(slc_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


@pytest.fixture(scope="module")
def lib():
    from starlight_b200 import build
    build.build()
    return ctypes.CDLL(D.library_path())


def test_header_declares_core_trait_functions():
    names = declared_functions()
    for n in ["slc_allocate_f32", "slc_allocate_u32", "slc_upload_f32", "slc_upload_u32",
              "slc_download_f32", "slc_download_u32", "slc_dispatch", "slc_synchronize",
              "slc_device_create", "slc_device_destroy"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, f"undefined in libslc.so: {missing}"


def test_python_binding_covers_declared_symbols():
    assert set(D.exported_symbols()) <= declared_functions()


def test_library_exports_no_private_cxx_symbols(lib):
    # Everything but the C ABI is built with hidden visibility.
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", D.library_path()], capture_output=True,
                         text=True).stdout
    exported = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert all(n.startswith("slc_") for n in exported), [n for n in exported if not n.startswith("slc_")][:5]


def test_opcode_discriminants_match_sl_ir():
    # docs/ARCH-0004 section 5.1: #[repr(u16)] declaration order.
    order = ["MatMulNT", "MatMulNN", "Softmax", "SoftmaxCausal", "RmsNorm", "Rope", "Silu", "Mul",
             "Add", "Scale", "Gather", "LastToken", "KvAppend", "SplitHeads", "MergeHeads",
             "CausalAttention", "SwiGlu", "RmsNormMatMul"]
    for i, name in enumerate(order):
        assert D.OpCode[name] == i
    text = open(os.path.join(ROOT, "include", "starlight_cuda.h")).read()
    assert "SLC_OP_RMS_NORM_MATMUL = 17" in text and "SLC_OP_MATMUL_NT = 0" in text


def test_status_names(lib):
    lib.slc_status_name.restype = ctypes.c_char_p
    assert lib.slc_status_name(0) == b"Ok"
    assert lib.slc_status_name(6) == b"Execution"
    assert lib.slc_status_name(7) == b"Unimplemented"


def test_device_create_fails_cleanly_without_gpu(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    d = ctypes.c_void_p()
    lib.slc_device_create.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
    rc = lib.slc_device_create(0, ctypes.byref(d))
    assert rc != 0 and not d.value


def test_quant_storage_arithmetic():
    assert D.quant_storage_words(4, 688, D.QuantFormat.Int4) == (4 * 344 + 3) // 4
    assert D.quant_storage_words(3, 5, D.QuantFormat.Int8) == 4
    assert D.quant_groups(688, 32) == 22
