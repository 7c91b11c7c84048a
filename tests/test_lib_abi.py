"""The C-ABI library builds, loads without a GPU, and exports every entry point
declared in include/microgen_b200.h (no compute calls)."""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "microgen_b200.h")


def declared_symbols() -> list[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(mg_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from microgen_b200 import build, _lib
    build.build()
    return ctypes.CDLL(_lib.LIB_PATH)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "mg_i8_linear" in syms and "mg_paged_decode_attn" in syms and "mg_quantize_rows_i8" in syms
    assert len(syms) >= 15


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, f"declared in the header but not exported: {missing}"


def test_binding_table_matches_header():
    from microgen_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared_symbols()


def test_non_compute_entry_points(lib):
    from microgen_b200 import _lib
    L = _lib.load()
    assert L.mg_abi_version() == 1
    assert L.mg_status_string(0) == b"ok"
    assert L.mg_status_string(4) == b"bounded device wait timed out"
    # argument validation happens before any CUDA call
    assert L.mg_quantize_rows_i8(None, -1, 4, None, None, None) == _lib.MG_ERR_INVALID_ARG
    assert L.mg_i8_linear(None, 1, 15, 16, None, None, None, 8, None, 8, 0, None) == _lib.MG_ERR_INVALID_ARG
    out = ctypes.c_size_t(123)
    assert L.mg_paged_attn_workspace_bytes(4, 24, 8, 96, 10, 0, ctypes.byref(out)) == _lib.MG_ERR_UNSUPPORTED
