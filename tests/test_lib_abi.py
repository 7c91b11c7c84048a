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


def test_argument_errors_of_later_entry_points(lib):
    """Bad arguments come back as MG_ERR_INVALID_ARG before any CUDA call (no GPU needed)."""
    from microgen_b200 import _lib
    L = _lib.load()
    bad = _lib.MG_ERR_INVALID_ARG
    h = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(L.mg_comm_handle_bytes())
    assert L.mg_comm_handle_bytes() > 0
    assert L.mg_comm_create(0, 0, 16, ctypes.byref(h), handle) == bad          # world < 1
    assert L.mg_comm_create(2, 2, 16, ctypes.byref(h), handle) == bad          # rank >= world
    assert L.mg_comm_create(0, 9, 16, ctypes.byref(h), handle) == bad          # world > 8
    assert L.mg_comm_open(None, handle) == bad
    assert L.mg_comm_destroy(None) == bad
    assert L.mg_i8_linear_packed_rowpar(None, 1, 128, 128, None, None, 128, None, 0, None) == bad
    assert L.mg_rowpar_reduce_norm(None, None, None, 1, 128, 1, None, None, ctypes.c_float(1e-5), None,
                                   None) == bad
    assert L.mg_argmax_rows(None, 1, 8, 8, None, None) == bad
    assert L.mg_vocab_argmax(None, None, 1, 8, 8, 0, None, None) == bad        # no communicator
    assert L.mg_argmax_rows(None, 1, 8, 4, None, None) == bad                   # ld < n
    assert L.mg_paged_decode_attn(None, None, None, 1, None, 1, None, 1, 24, 7, 128, 0, ctypes.c_float(1.0),
                                  None, None, 0, None) == bad                   # hq % hkv != 0
