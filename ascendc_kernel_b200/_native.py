"""ctypes binding of the in-tree CUDA library ``lib/libdsa_b200.so``.

The library is the only compute path: if it is missing or fails to load,
:func:`lib` raises; there is no fallback implementation. Every entry point
returns a ``dsa_status_t``; :func:`check` turns a non-zero status into a
``DsaError`` carrying the status name and the last CUDA error code.
"""

from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "lib", "libdsa_b200.so")

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_size_t = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/dsa_b200.h
SIGNATURES = {
    "dsa_status_string": (ctypes.c_char_p, [_i32]),
    "dsa_last_cuda_error": (_i32, []),
    "dsa_device_error_read": (_i32, [_i32, ctypes.POINTER(ctypes.c_uint), _i32]),
    "dsa_version": (_i32, []),
    "dsa_sinkhorn_fwd": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _i32, _f32, _c_void_p]),
    "dsa_sparse_attn_fwd": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i32, _c_void_p, _c_void_p,
                                   _i64, _i64, _i32, _i32, _i32, _i32, _f32, _c_void_p]),
    "dsa_indexer_qproj_rope": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64,
                                      _i32, _i32, _i32, _i32, _i64, _c_void_p, _size_t,
                                      _c_void_p]),
    "dsa_indexer_wproj_workspace_bytes": (_size_t, [_i64, _i32]),
    "dsa_indexer_wproj": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i32, _i32, _f32,
                                 _c_void_p, _size_t, _c_void_p]),
    "dsa_indexer_score_topk": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p, _i64,
                                      _i64, _i32, _i32, _i64, _i32, _i64, _i32, _i64,
                                      _c_void_p, _size_t, _c_void_p]),
    "dsa_indexer_score_workspace_bytes": (_size_t, [_i64, _i64, _i64, _i32]),
    "dsa_indexer_workspace_bytes": (_size_t, [_i64, _i64, _i32, _i32, _i64, _i32]),
    "dsa_indexer_overlap_extra_bytes": (_size_t, [_i64, _i32, _i32]),
    "dsa_indexer_fwd": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                               _c_void_p, _i64, _c_void_p, _c_void_p, _size_t, _i64, _i64, _i32,
                               _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i64, _f32,
                               _c_void_p]),
    "dsa_indexer_fwd_noalloc": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                       _c_void_p, _c_void_p, _i64, _c_void_p, _i64, _i64, _i32,
                                       _i32, _i32, _i32, _i32, _i32, _i64, _i32, _i64, _f32,
                                       _c_void_p]),
    "dsa_indexer_fp8_quant_rows": (_i32, [_c_void_p, _i64, _i64, _i64, _i32, _c_void_p,
                                          _c_void_p, _c_void_p, _c_void_p, _c_void_p]),
    "dsa_indexer_score_topk_fp8": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                          _c_void_p, _i64, _i64, _i32, _i32, _i64, _i32, _i64,
                                          _i32, _i64, _c_void_p]),
    "dsa_indexer_fp8_workspace_bytes": (_size_t, [_i64, _i64, _i32, _i32, _i64]),
    "dsa_indexer_fwd_fp8": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                   _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _size_t,
                                   _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i64, _i32,
                                   _i64, _f32, _c_void_p]),
    "dsa_kv_cache_write": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                                  _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i32, _i32, _i32,
                                  _i64, _i32, _c_void_p]),
    "dsa_chain_workspace_bytes": (_size_t, [_i64, _i64, _i32, _i32, _i64]),
    "dsa_chain_fwd": (_i32, [_c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _c_void_p,
                             _c_void_p, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _i32,
                             _i64, _i32, _i64, _f32, _c_void_p, _c_void_p, _i32, _i32, _i32,
                             _c_void_p, _f32, _c_void_p, _c_void_p, _size_t, _c_void_p]),
}

_LIB = None


class DsaError(RuntimeError):
    """A dsa_* entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, cuda_err: int):
        self.status = status
        self.cuda_error = cuda_err
        name = lib().dsa_status_string(status).decode()
        super().__init__(f"{fn} failed: {name} (status {status}, last CUDA error {cuda_err})")


def lib() -> ctypes.CDLL:
    """Loads the CUDA library once and declares every C-ABI signature."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m ascendc_kernel_b200.build` "
                "(this package has no non-CUDA fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(fn: str, status: int) -> None:
    if status != 0:
        raise DsaError(fn, status, lib().dsa_last_cuda_error())


def call(fn: str, *args) -> None:
    """Calls entry point `fn` and raises DsaError on a non-zero status."""
    check(fn, getattr(lib(), fn)(*args))


def device_error(device: int, clear: bool = True) -> int:
    """Synchronizes `device` and returns (then clears) its device error word."""
    code = ctypes.c_uint(0)
    check("dsa_device_error_read", lib().dsa_device_error_read(device, ctypes.byref(code),
                                                                1 if clear else 0))
    return int(code.value)
