"""ctypes binding of ``libbsattn.so`` -- the C ABI declared in ``include/bsattn.h``.

There is no fallback: if the library is missing or does not export the ABI, loading raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from .build import LIB_PATH

_c_int, _c_void_p, _c_size_t = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t

# name -> (restype, argtypes); must match include/bsattn.h
SIGNATURES = {
    "bsattn_workspace_bytes": (_c_size_t, []),
    "bsattn_version": (_c_int, []),
    "bsattn_set_timeout_ns": (None, [ctypes.c_uint64]),
    "bsattn_test_unsignalled_wait": (None, [_c_int]),
    "bsattn_setup": (_c_int, []),
    "bsattn_strerror": (ctypes.c_char_p, [_c_int]),
    "bsattn_fwd": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p,          # q, k, v
        _c_void_p, _c_void_p,                     # o, lse
        _c_void_p, _c_void_p, _c_void_p,          # row_ptr, col_idx, seq_lens
        _c_int, _c_int, _c_int, _c_int,           # B, H, T, D
        ctypes.c_int64, ctypes.c_int64, _c_int,   # rp_stride_bh, ci_stride_bh, max_nnz
        ctypes.c_float, _c_int,                   # scale, dtype_flags
        _c_void_p, _c_size_t, _c_void_p,          # workspace, bytes, stream
    ]),
    "bsattn_check_error": (_c_int, [_c_void_p, _c_void_p, ctypes.POINTER(_c_int)]),
    "bsattn_fwd_plan": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p,          # q, k, v
        _c_void_p, _c_void_p,                     # o, lse
        _c_void_p, _c_void_p, _c_void_p,          # row_ptr, col_idx, seq_lens
        _c_int, _c_int, _c_int, _c_int,           # B, H, T, D
        ctypes.c_int64, ctypes.c_int64, _c_int,   # rp_stride_bh, ci_stride_bh, max_nnz
        ctypes.c_float, _c_int,                   # scale, dtype_flags
        _c_void_p, _c_int,                        # plan (device), plan_grid
        _c_void_p, _c_size_t, _c_void_p,          # workspace, bytes, stream
    ]),
    "bsattn_fwd_window": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p,          # q, k, v
        _c_void_p, _c_void_p, _c_void_p,          # o, lse, seq_lens
        _c_int, _c_int, _c_int, _c_int,           # B, H, T, D
        _c_int, _c_int,                           # window, global_blocks
        ctypes.c_float, _c_int,                   # scale, dtype_flags
        _c_void_p, _c_int,                        # plan (device), plan_grid
        _c_void_p, _c_size_t, _c_void_p,          # workspace, bytes, stream
    ]),
    "bsattn_plan_window": (_c_int, [_c_void_p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                    _c_void_p, _c_size_t]),
    "bsattn_plan_bytes": (_c_int, [_c_int, _c_int, _c_int, _c_int, ctypes.POINTER(_c_size_t)]),
    "bsattn_plan": (_c_int, [_c_void_p, ctypes.c_int64, _c_void_p, _c_int, _c_int, _c_int, _c_int,
                             _c_int, _c_void_p, _c_size_t]),
    "bsattn_bf16_to_f16": (_c_int, [_c_void_p, _c_void_p, ctypes.c_int64, _c_void_p]),
    "bsattn_csr_nnz": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int,
                                ctypes.POINTER(ctypes.c_int64)]),
    "bsattn_build_csr": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, ctypes.c_uint64,
                                  _c_int, _c_void_p, _c_void_p, ctypes.c_int64, _c_void_p]),
    "bsattn_ipc_export": (_c_int, [_c_void_p, _c_void_p, ctypes.POINTER(ctypes.c_uint64)]),
    "bsattn_ipc_open": (_c_int, [_c_void_p, ctypes.c_uint64, ctypes.POINTER(_c_void_p)]),
    "bsattn_ipc_close": (_c_int, [_c_void_p, ctypes.c_uint64]),
    "bsattn_peer_copy": (_c_int, [_c_void_p, _c_void_p, _c_size_t, _c_void_p]),
    "bsattn_fwd_noalloc": (_c_int, [
        _c_void_p, _c_void_p, _c_void_p,          # q, k, v
        _c_void_p, _c_void_p,                     # o, lse
        _c_void_p, _c_void_p, _c_void_p,          # row_ptr, col_idx, seq_lens
        _c_int, _c_int, _c_int, _c_int,           # B, H, T, D
        ctypes.c_int64, ctypes.c_int64, _c_int,   # rp_stride_bh, ci_stride_bh, max_nnz
        ctypes.c_float, _c_int,                   # scale, dtype_flags
        _c_void_p, _c_void_p,                     # status (device or pinned host int*), stream
    ]),
}

# error codes (include/bsattn.h)
OK = 0
E_SHAPE, E_ALIGN, E_NULL, E_WORKSPACE, E_CUDA, E_TMA, E_DEVICE, E_CSR, E_TIMEOUT, E_DTYPE = (
    -1, -2, -3, -4, -5, -6, -7, -8, -9, -10)
E_PLAN = -11
OUT_F16, OUT_BF16, IN_BF16 = 0, 1, 2
CSR_WINDOW, CSR_PREFIX_WINDOW, CSR_RETRIEVAL = 0, 1, 2

_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load the in-tree kernel library once; raise if it is absent (no CPU fallback)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing; build it with `python -m usagi_b200.build` "
                "(the block-sparse attention path has no non-CUDA fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)  # AttributeError if the ABI is incomplete
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def strerror(code: int) -> str:
    return load().bsattn_strerror(int(code)).decode()
