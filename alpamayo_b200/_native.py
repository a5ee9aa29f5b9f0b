"""Locate and load the in-tree native libraries.

``libparo_b200.so`` exports the C ABI of ``include/paro_b200.h``;
``libparo_torch.so`` registers the ``torch.ops.paro_b200`` operators on top
of it.  There is no fallback: if the libraries are missing, importing the
package raises with the command that builds them.
"""
from __future__ import annotations

import ctypes
import os

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(PKG_DIR, "lib")
CORE_LIB = os.path.join(LIB_DIR, "libparo_b200.so")
TORCH_LIB = os.path.join(LIB_DIR, "libparo_torch.so")

_capi = None
_ops_loaded = False


def _missing(path):
    raise ImportError(
        f"alpamayo_b200 native library not found: {path}\n"
        "build it with:  python alpamayo_b200/csrc/build.py")


def load_ops() -> None:
    """Register torch.ops.paro_b200.* (idempotent)."""
    global _ops_loaded
    if _ops_loaded:
        return
    for p in (CORE_LIB, TORCH_LIB):
        if not os.path.exists(p):
            _missing(p)
    # load the C ABI first so the shim's DT_NEEDED entry resolves to this copy
    ctypes.CDLL(CORE_LIB, mode=ctypes.RTLD_GLOBAL)
    torch.ops.load_library(TORCH_LIB)
    _ops_loaded = True


def capi() -> ctypes.CDLL:
    """The C ABI as a ctypes library with argument types declared."""
    global _capi
    if _capi is not None:
        return _capi
    if not os.path.exists(CORE_LIB):
        _missing(CORE_LIB)
    L = ctypes.CDLL(CORE_LIB, mode=ctypes.RTLD_GLOBAL)
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    sigs = {
        "paro_status_string": (ctypes.c_char_p, [i32]),
        "paro_version": (i32, []),
        "paro_last_cuda_error": (ctypes.c_char_p, []),
        "paro_prepare_rotation": (i32, [vp, vp, i32, i32, i32, vp, vp, vp]),
        "paro_rotation_table_words": (sz, [i32, i32]),
        "paro_prepare_rotation_matrices": (i32, [vp, i32, vp]),
        "paro_rotate": (i32, [vp, i32, i64, i32, vp, vp, i32, vp, i32, i32, vp, vp]),
        "paro_rotq_int8": (i32, [vp, i32, i64, i32, vp, vp, i32, i32, i32, vp, vp, vp]),
        "paro_rotq_int8_workspace_size": (sz, [i64, i32, i32]),
        "paro_rotq_int8_ws": (i32, [vp, i32, i64, i32, vp, vp, i32, i32, i32, vp, vp, vp, sz, vp]),
        "paro_quant_int8": (i32, [vp, i32, i64, i32, vp, vp, vp]),
        "paro_packed_weight_bytes": (sz, [i32, i32]),
        "paro_prepare_weights": (i32, [vp, vp, vp, i32, i32, i32, vp, vp]),
        "paro_prepare_weights_awq": (i32, [vp, vp, vp, i32, i32, vp, vp]),
        "paro_w4a8_gemm_workspace_size": (sz, [i64, i32, i32]),
        "paro_w4a8_gemm": (i32, [vp, vp, i64, i32, i32, vp, vp, i32, vp, i32, vp, sz, vp]),
        "paro_w4a8_gemm_path": (i32, [i64, i32, i32]),
        "paro_w4a8_gemm_route_workspace_size": (sz, [i32, i64, i32, i32]),
        "paro_w4a8_gemm_route": (i32, [i32, vp, vp, i64, i32, i32, vp, vp, i32, vp, i32, vp, sz, vp]),
        "paro_w4a8_linear_workspace_size": (sz, [i64, i32, i32]),
        "paro_w4a8_linear_scratch_size": (sz, [i64, i32, i32, i32]),
        "paro_w4a8_linear": (i32, [vp, i32, i64, i32, i32, vp, vp, i32, vp, vp, i32, vp, i32, vp, sz, vp, sz, vp]),
        "paro_device_error_word": (i32, [i32]),
        "paro_selftest_wait_timeout": (i32, [ctypes.c_longlong, vp]),
        "paro_w4a8_linear_prologue_scratch_size": (sz, [i32, i64, i32, i32, i32]),
        "paro_w4a8_linear_prologue": (i32, [i32, vp, vp, vp, vp, ctypes.c_float, i64, i32, i32, vp, vp, i32, vp, vp,
                                            i32, vp, i32, vp, sz, vp, sz, vp]),
        "paro_w4a8_linear_group_workspace_size": (sz, [i64, i32, vp, i32]),
        "paro_w4a8_linear_group_scratch_size": (sz, [i32, i64, i32, vp, i32, i32]),
        "paro_w4a8_linear_group": (i32, [i32, vp, i32, vp, vp, vp, ctypes.c_float, i64, i32, i32, vp, vp, vp, i32,
                                         vp, vp, i32, vp, i32, vp, sz, vp, sz, vp]),
        "paro_w4a8_gemm_noalloc": (i32, [vp, vp, i64, i32, i32, vp, vp, i32, vp, i32, vp]),
        "paro_w4a8_gemm_multicast": (i32, [vp, vp, i64, i32, i32, vp, vp, i32, vp, vp]),
        "paro_add_rmsnorm": (i32, [vp, vp, vp, i64, i32, ctypes.c_float, vp, vp]),
        "paro_silu_mul": (i32, [vp, i64, i32, vp, vp]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _capi = L
    return L


_shim = None


def shim() -> ctypes.CDLL:
    """The torch operator shim as a ctypes library (its few extern "C"
    helpers, e.g. paro_torch_reset_workspaces)."""
    global _shim
    if _shim is None:
        load_ops()
        _shim = ctypes.CDLL(TORCH_LIB)
        _shim.paro_torch_reset_workspaces.restype = ctypes.c_int
        _shim.paro_torch_reset_workspaces.argtypes = []
    return _shim


DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
