"""The C-ABI library loads and exports every entry point include/moe_gemm.h declares; host-side
argument checks answer without a GPU."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "moe_gemm.h"
LIB = REPO / "cute-moe-train_b200" / "cutlass_op" / "bf16_grouped_mm" / "libmoe_gemm.so"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(mgf_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "mgf_grouped_gemm_launch" in names and "mgf_device_status" in names
    assert len(names) >= 4


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} not exported by {LIB.name}"


def test_status_strings_and_version():
    lib = ctypes.CDLL(str(LIB))
    lib.mgf_status_string.restype = ctypes.c_char_p
    assert lib.mgf_version() >= 100
    assert lib.mgf_status_string(0) == b"ok"
    assert b"alignment" in lib.mgf_status_string(-3) or b"aligned" in lib.mgf_status_string(-3)


def test_null_descriptor_rejected():
    lib = ctypes.CDLL(str(LIB))
    assert lib.mgf_grouped_gemm_launch(None, None) == -1


def test_ctypes_descriptor_layouts_match_the_library():
    """The ctypes mirrors of mgf_gemm_desc (the reference-side binding ctypes_ext.py and the no-alloc
    test's) have the size the library was compiled with."""
    import importlib.util

    lib = ctypes.CDLL(str(LIB))
    lib.mgf_gemm_desc_size.restype = ctypes.c_size_t
    for name, path in (("t_no_alloc", REPO / "tests" / "test_zz_no_alloc.py"),
                       ("t_ctypes_ext", REPO / "cute-moe-train_b200" / "ctypes_ext.py")):
        spec = importlib.util.spec_from_file_location(name, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)  # ctypes_ext also checks its own layout at import
        assert ctypes.sizeof(mod.MgfGemmDesc) == lib.mgf_gemm_desc_size(), name
