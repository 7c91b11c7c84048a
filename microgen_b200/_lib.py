"""ctypes binding of libmicrogen_b200.so (the C ABI in include/microgen_b200.h).

The library is loaded on first use from this package directory. A missing or
unloadable library raises immediately: the decode path has no CPU fallback.
"""

from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmicrogen_b200.so")

MG_OK = 0
MG_ERR_INVALID_ARG = 1
MG_ERR_UNSUPPORTED = 2
MG_ERR_CUDA = 3
MG_ERR_TIMEOUT = 4
MG_ERR_DEVICE = 5

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_ADD_F32 = 2
EPI_SWIGLU_BF16 = 3
EPI_GELU_BF16 = 4

_p, _i, _i64, _f, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t

# name -> argtypes (restype is int for every entry point unless listed in _RESTYPES)
SIGNATURES = {
    "mg_abi_version": [],
    "mg_status_string": [_i],
    "mg_last_cuda_error": [],
    "mg_device_error": [_p, _i, C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "mg_quantize_rows_i8": [_p, _i64, _i64, _p, _p, _p],
    "mg_i8_linear": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _p],
    "mg_i8_linear_simt": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _p],
    "mg_i8_linear_tc": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _i, _p],
    "mg_i8_packed_bytes": [_i64, _i64],
    "mg_i8_pack_weights": [_p, _i64, _i64, _p, _p],
    "mg_i8_linear_packed": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _i, _p],
    "mg_i8_linear_sk_workspace_bytes": [_i64],
    "mg_i8_linear_packed_sk": [_p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _i64, _i, _p, _sz, _p],
    "mg_i8_linear_packed_rowpar_sk": [_p, _i64, _i64, _i64, _p, _p, _i64, _p, _p, _sz, _p],
    "mg_comm_handle_bytes": [],
    "mg_comm_create": [_i, _i, _i64, C.POINTER(C.c_void_p), _p],
    "mg_comm_open": [_p, _p],
    "mg_comm_destroy": [_p],
    "mg_i8_linear_packed_rowpar": [_p, _i64, _i64, _i64, _p, _p, _i64, _p, _i, _p],
    "mg_rowpar_reduce_norm": [_p, _p, _p, _i, _i, _i, _p, _p, _f, _p, _p],
    "mg_rope_kv_append": [_p, _i64, _p, _p, _i, _p, _i, _i, _i, _i, _p, _p, _p, _i64, _p],
    "mg_rope_kv_append_kv8": [_p, _i64, _p, _p, _i, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _i64, _p],
    "mg_paged_attn_workspace_bytes": [_i, _i, _i, _i, _i, _i, C.POINTER(C.c_size_t)],
    "mg_paged_decode_attn": [_p, _p, _p, _i64, _p, _i, _p, _i, _i, _i, _i, _i, _f, _p, _p, _sz, _p],
    "mg_paged_decode_attn_kv8": [_p, _p, _p, _p, _p, _i64, _p, _i, _p, _i, _i, _i, _i, _i, _f, _p, _p, _sz, _p],
    "mg_paged_decode_attn_noalloc": [_p, _p, _p, _i64, _p, _i, _p, _i, _i, _i, _i, _i, _f, _p, _p],
    "mg_embed": [_p, _p, _p, _p, _i, _i, _i64, _i, _p, _p],
    "mg_rmsnorm": [_p, _p, _i, _i, _f, _p, _p],
    "mg_layernorm": [_p, _p, _p, _i, _i, _f, _p, _p],
    "mg_argmax_rows": [_p, _i, _i64, _i64, _p, _p],
    "mg_vocab_argmax": [_p, _p, _i, _i64, _i64, _i64, _p, _p],
    "mg_decode_advance": [_p, _p, _p, _p, _p, _p, _i, _i, _p],
    "mg_decode_block_workspace_bytes": [_p, C.POINTER(C.c_size_t)],
    "mg_decode_block": [_p, _p, _p, _sz, _p],
    "mg_decode_block_diag": [_p, _i],
    "mg_decode_block_trace": [_p, _i],
}
_RESTYPES = {"mg_status_string": C.c_char_p, "mg_i8_packed_bytes": C.c_int64,
             "mg_i8_linear_sk_workspace_bytes": C.c_int64}

# entry points that launch one kernel per call
LAUNCHING = {"mg_quantize_rows_i8", "mg_i8_linear", "mg_i8_linear_simt", "mg_i8_linear_tc", "mg_rope_kv_append",
             "mg_i8_pack_weights", "mg_i8_linear_packed", "mg_paged_decode_attn_noalloc",
             "mg_i8_linear_packed_rowpar", "mg_rowpar_reduce_norm", "mg_i8_linear_packed_sk",
             "mg_i8_linear_packed_rowpar_sk",
             "mg_paged_decode_attn", "mg_embed", "mg_rmsnorm", "mg_layernorm", "mg_argmax_rows",
             "mg_decode_advance", "mg_decode_block", "mg_vocab_argmax", "mg_rope_kv_append_kv8",
             "mg_paged_decode_attn_kv8"}
LAUNCHES = [0]  # kernels launched (or captured) through call() in this process

_lock = threading.Lock()
_lib = None


class MGError(RuntimeError):
    """A C-ABI entry point returned a nonzero status."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} (status {status}){detail}")


def load() -> C.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m microgen_b200.build` "
                                   "(the decode path has no CPU fallback)")
            lib = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    try:
        return load().mg_status_string(int(status)).decode()
    except Exception:
        return "unknown"


def call(name: str, *args) -> None:
    """Call an entry point; raise MGError (TimeoutError for MG_ERR_TIMEOUT) on a nonzero status."""
    rc = getattr(load(), name)(*args)
    if rc == MG_OK and name in LAUNCHING:
        LAUNCHES[0] += 1
    if rc != MG_OK:
        detail = ""
        if rc == MG_ERR_CUDA:
            detail = f"; cudaError {load().mg_last_cuda_error()}"
        if rc == MG_ERR_TIMEOUT:
            raise TimeoutError(f"{name}: bounded device wait timed out")
        raise MGError(name, rc, detail)


def device_error(stream_handle: int = 0, clear: bool = True) -> tuple[int, int]:
    code, info = C.c_int(0), C.c_int(0)
    call("mg_device_error", C.c_void_p(stream_handle), 1 if clear else 0, C.byref(code), C.byref(info))
    return code.value, info.value


def check_device(stream_handle: int = 0) -> None:
    """Raise if a kernel recorded a device-side error since the last check."""
    code, info = device_error(stream_handle, clear=True)
    if code == MG_ERR_TIMEOUT:
        raise TimeoutError(f"device wait timed out (site {info})")
    if code != MG_OK:
        raise RuntimeError(f"device-side check failed: {status_string(code)} (site {info})")
