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


class DecConfig(ctypes.Structure):
    """tb_dec_config (include/tb_gguf_dequant.h, part 3)."""
    _fields_ = [(n, ctypes.c_int) for n in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim",
                                            "ffn_dim", "vocab", "max_ctx")] + \
               [("rope_base", ctypes.c_float), ("norm_eps", ctypes.c_float), ("quirks", ctypes.c_int)]


class DecLayer(ctypes.Structure):
    """tb_dec_layer (include/tb_gguf_dequant.h, part 3)."""
    _fields_ = [("w_qkv", ctypes.c_void_p), ("qkv_qtype", ctypes.c_int),
                ("w_o", ctypes.c_void_p), ("o_qtype", ctypes.c_int),
                ("w_gate_up", ctypes.c_void_p), ("gate_up_qtype", ctypes.c_int),
                ("w_down", ctypes.c_void_p), ("down_qtype", ctypes.c_int),
                ("attn_norm", ctypes.c_void_p), ("ffn_norm", ctypes.c_void_p),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p)]


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
        "tb_cuda_set_matvec_arith": (c_int, [c_int]),
        "tb_cuda_arena_create": (c_void_p, [c_size_t]),
        "tb_cuda_arena_upload": (c_void_p, [c_void_p, c_void_p, c_size_t]),
        "tb_cuda_arena_upload_rows": (c_void_p, [c_void_p, c_void_p, c_size_t, c_int, c_int]),
        "tb_cuda_arena_upload_cols": (c_void_p, [c_void_p, c_void_p, c_int, c_size_t, c_size_t, c_size_t]),
        "tb_cuda_arena_used": (c_size_t, [c_void_p]),
        "tb_cuda_arena_destroy": (None, [c_void_p]),
        "tb_cuda_get_matvec_arith": (c_int, []),
        "tb_cuda_matvec_device_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, fp, fp]),
        "tb_cuda_matvec_fused_dev": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_int,
                                             c_void_p, c_void_p, ctypes.c_float, c_void_p, c_int, c_void_p]),
        "tb_cuda_qgemm_dev": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_void_p]),
        "tb_cuda_matvec_experts_dev": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                               c_void_p, c_int, c_int, c_void_p]),
        "tb_cuda_sample_dev": (c_int, [c_void_p, c_int, c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float, c_void_p,
                                       c_void_p]),
        "tb_cuda_dec_create": (c_void_p, [ctypes.POINTER(DecConfig)]),
        "tb_cuda_dec_set_layer": (c_int, [c_void_p, c_int, ctypes.POINTER(DecLayer)]),
        "tb_cuda_dec_set_head": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int]),
        "tb_cuda_dec_kv": (c_void_p, [c_void_p, c_int, c_int]),
        "tb_cuda_dec_kv_copy": (c_int, [c_void_p, c_int, c_int, c_int, c_int, fp, c_int]),
        "tb_cuda_dec_read": (c_int, [c_void_p, c_int, fp, c_int]),
        "tb_cuda_dec_create_tp": (c_void_p, [ctypes.POINTER(DecConfig), c_int, c_int]),
        "tb_cuda_dec_tp_handle": (c_int, [c_void_p, c_void_p]),
        "tb_cuda_dec_tp_connect": (c_int, [c_void_p, c_void_p]),
        "tb_cuda_dec_create_moe": (c_void_p, [ctypes.POINTER(DecConfig), c_int, c_int]),
        "tb_cuda_dec_create_moe_tp": (c_void_p, [ctypes.POINTER(DecConfig), c_int, c_int, c_int, c_int]),
        "tb_cuda_dec_set_moe_layer": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int]),
        "tb_cuda_dec_step": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_int), fp]),
        "tb_cuda_dec_prefill": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int, c_int, ctypes.POINTER(c_int), fp]),
        "tb_cuda_dec_generate": (c_int, [c_void_p, c_int, c_int, c_int, ctypes.POINTER(c_int), fp, fp]),
        "tb_cuda_dec_set_sampling": (c_int, [c_void_p, ctypes.c_float, c_int, ctypes.c_float]),
        "tb_cuda_dec_generate_u": (c_int, [c_void_p, c_int, c_int, c_int, fp, ctypes.POINTER(c_int), fp, fp]),
        "tb_cuda_dec_destroy": (None, [c_void_p]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def exported_symbols() -> list[str]:
    """Names the header declares (checked against the .so's dynamic symbols by the tests)."""
    return sorted([
        "tb_cuda_init", "tb_cuda_upload_tensor", "tb_cuda_free_tensor", "tb_cuda_upload_x",
        "tb_cuda_set_snap", "tb_cuda_matvec_device", "tb_cuda_sync_all", "tb_cuda_cleanup",
        "tb_cuda_matvec_dev", "tb_cuda_dequant_dev", "tb_cuda_qtype_info", "tb_cuda_last_error",
        "tb_cuda_launch_count", "tb_cuda_version", "tb_cuda_set_matvec_arith", "tb_cuda_get_matvec_arith",
        "tb_cuda_arena_create", "tb_cuda_arena_upload", "tb_cuda_arena_upload_rows", "tb_cuda_arena_upload_cols",
        "tb_cuda_arena_used", "tb_cuda_arena_destroy",
        "tb_cuda_matvec_device_noalloc",
        "tb_cuda_matvec_fused_dev", "tb_cuda_matvec_experts_dev", "tb_cuda_sample_dev", "tb_cuda_qgemm_dev", "tb_cuda_dec_create", "tb_cuda_dec_set_layer", "tb_cuda_dec_set_head",
        "tb_cuda_dec_kv", "tb_cuda_dec_kv_copy", "tb_cuda_dec_read", "tb_cuda_dec_create_tp",
        "tb_cuda_dec_tp_handle", "tb_cuda_dec_tp_connect", "tb_cuda_dec_create_moe", "tb_cuda_dec_create_moe_tp", "tb_cuda_dec_set_moe_layer",
        "tb_cuda_dec_step", "tb_cuda_dec_prefill", "tb_cuda_dec_generate", "tb_cuda_dec_set_sampling", "tb_cuda_dec_generate_u",
        "tb_cuda_dec_destroy",
    ])
