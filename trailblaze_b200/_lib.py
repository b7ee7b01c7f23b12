"""ctypes binding of libtb_cuda_sm100.so (the C ABI in include/tb_gguf_dequant.h).

This is the binding a Python caller of the reference's C ABI would write; it
adds nothing on top of the library.  Loading fails loudly when the shared
library is missing: there is no fallback implementation of any kind.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtb_cuda_sm100.so")

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m trailblaze_b200.build` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    L = ctypes.CDLL(LIB_PATH)
    c_int, c_void_p, c_size_t = ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t
    fp = ctypes.POINTER(ctypes.c_float)
    sig = {
        "tb_cuda_init": (c_int, []),
        "tb_cuda_upload_tensor": (c_void_p, [c_void_p, c_size_t]),
        "tb_cuda_free_tensor": (None, [c_void_p]),
        "tb_cuda_upload_x": (c_int, [fp, c_int]),
        "tb_cuda_set_snap": (None, [c_void_p]),
        "tb_cuda_matvec_device": (c_int, [c_void_p, c_int, c_int, c_int, fp, fp]),
        "tb_cuda_sync_all": (None, []),
        "tb_cuda_cleanup": (None, []),
        "tb_cuda_matvec_dev": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
        "tb_cuda_dequant_dev": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p]),
        "tb_cuda_qtype_info": (c_int, [c_int, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
        "tb_cuda_last_error": (c_int, []),
        "tb_cuda_launch_count": (ctypes.c_ulonglong, []),
        "tb_cuda_version": (ctypes.c_char_p, []),
        "tb_cuda_matvec_device_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, fp, fp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def exported_symbols() -> list[str]:
    """Names the header declares (checked against the .so's dynamic symbols by the tests)."""
    return [
        "tb_cuda_init", "tb_cuda_upload_tensor", "tb_cuda_free_tensor", "tb_cuda_upload_x",
        "tb_cuda_set_snap", "tb_cuda_matvec_device", "tb_cuda_sync_all", "tb_cuda_cleanup",
        "tb_cuda_matvec_dev", "tb_cuda_dequant_dev", "tb_cuda_qtype_info", "tb_cuda_last_error",
        "tb_cuda_launch_count", "tb_cuda_version", "tb_cuda_matvec_device_noalloc",
    ]
