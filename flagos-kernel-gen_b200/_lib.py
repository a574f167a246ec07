"""ctypes binding of the in-tree C-ABI library ``lib/libw4a8moe.so``.

The library is the product path: there is no Python, Triton or CPU fallback.
Loading fails loudly (``ImportError``) when the library has not been built, and
every call that returns a non-zero status raises ``RuntimeError`` with the
library's message (``w4a8_last_error``).
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libw4a8moe.so")

W4A8_OK = 0
W4A8_ERR_INVALID = 1
W4A8_ERR_CUDA = 2
W4A8_ERR_DEVICE = 3

KERNEL_AUTO = 0
KERNEL_TC = 1
KERNEL_SIMT = 2
KERNEL_GEMV = 3

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/w4a8moe.h
SIGNATURES = {
    "w4a8_abi_version": (ctypes.c_int, []),
    "w4a8_last_error": (ctypes.c_char_p, []),
    "w4a8_group_gemm_moe": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                           _i64, _i64, _p]),
    "w4a8_group_gemm_moe_ex": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                              _i64, _i64, _i64, _i32, _p, _p]),
    "w4a8_group_gemm_moe_combine": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _p, _i64, _i64,
                                                   _i64, _i64, _i64, _i64, _i32, _p]),
    "w4a8_combine_finish": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _p]),
    "w4a8_group_gemm_moe_hint": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                                _i64, _i64, _i64, _p]),
    "w4a8_ep_exchange": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i32, _i64, _p, _p, _p]),
    "w4a8_ep_dispatch": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _p,
                                        _i64, _i64, _i64, _p, _p]),
    "w4a8_ep_dispatch_dedup": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p,
                                              _p, _i64, _i64, _i64, _i64, _p, _p]),
    "w4a8_ep_replicate": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _p]),
    "w4a8_ep_barrier": (ctypes.c_int, [_p, _i64, _i64, _i64, _i32, _p]),
    "w4a8_prepack_weights": (ctypes.c_int, [_p, _p, _i64, _i64, _p]),
    "w4a8_group_gemm_moe_prepacked": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                                     _i64, _i64, _i64, _i32, _p, _p]),
    "w4a8_group_gemm_moe_rows": (ctypes.c_int, [_p, _i64, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64,
                                                _i64, _i64, _p]),
    "w4a8_ep_row_addresses": (ctypes.c_int, [_p, _p, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "w4a8_ep_return": (ctypes.c_int, [_p, _i64, _i64, _p, _p, _i64, _i64, _p, _i64, _p]),
    "w4a8_act_quant": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "w4a8_quant_scatter": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _i64, _p, _p, _p]),
    "w4a8_router_topk": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _i32, _i32, _p, _p, _p, _i64, _i64, _p, _i64,
                                        _p, _p]),
    "w4a8_moe_align_workspace_size": (_sz, [_i64, _i64, _i64]),
    "w4a8_moe_align": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _sz, _p]),
    "w4a8_silu_mul_requant": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _p]),
    "w4a8_silu_mul_requant_rows": (ctypes.c_int, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "w4a8_moe_combine": (ctypes.c_int, [_p, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "w4a8_gather_rows": (ctypes.c_int, [_p, _i64, _p, _i64, _i64, _p, _i64, _p]),
    "w4a8_moe_align_noalloc": (ctypes.c_int, [_p, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p]),
    "w4a8_selftest_wait_timeout": (ctypes.c_int, [_i64, _p, _p]),
    "w4a8_device_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int32), _i32, _p]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Returns the loaded library, loading it on first use."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: the CUDA library has not been built "
            "(run __graft_entry__.build() or python flagos-kernel-gen_b200/build.py)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != W4A8_OK:
        msg = load().w4a8_last_error().decode("utf-8", "replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")
