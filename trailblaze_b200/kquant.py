"""Python mirror of the Trailblaze dequant ABI (layer4/tb_gguf_dequant.h).

Method names and argument meaning follow the C entry points one for one
(tb_cuda_init, tb_cuda_upload_tensor, tb_cuda_matvec_device, ...), and so does
error behaviour: calls return the C return code (1 / 0, pointer / 0) instead of
raising, exactly like the reference's callers see them, except where a Python
caller would have no way to see a failure (a ctypes argument error raises).
Every compute call goes to libtb_cuda_sm100.so.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import qtypes as Q
from ._lib import lib

_fp = ctypes.POINTER(ctypes.c_float)


def _fptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


class KQuantLib:
    """Thin wrapper over the C ABI (one per process; the library is process-global)."""

    def __init__(self):
        self.L = lib()

    # ---- part 1: the reference ABI ------------------------------------------------
    def tb_cuda_init(self) -> int:
        return self.L.tb_cuda_init()

    def tb_cuda_upload_tensor(self, host: np.ndarray) -> int:
        host = np.ascontiguousarray(host)
        p = self.L.tb_cuda_upload_tensor(host.ctypes.data_as(ctypes.c_void_p), host.nbytes)
        return int(p or 0)

    def tb_cuda_free_tensor(self, d_ptr: int) -> None:
        self.L.tb_cuda_free_tensor(ctypes.c_void_p(d_ptr) if d_ptr else None)

    def tb_cuda_upload_x(self, x: np.ndarray) -> int:
        x = np.ascontiguousarray(x, dtype=np.float32)
        return self.L.tb_cuda_upload_x(_fptr(x), x.size)

    def tb_cuda_set_snap(self, snap_ptr: int | None) -> None:
        self.L.tb_cuda_set_snap(ctypes.c_void_p(snap_ptr) if snap_ptr else None)

    def tb_cuda_matvec_device(self, W_dev: int, qtype: int, M: int, K: int,
                              x: np.ndarray | None, out: np.ndarray) -> int:
        if x is not None:
            x = np.ascontiguousarray(x, dtype=np.float32)
        return self.L.tb_cuda_matvec_device(ctypes.c_void_p(W_dev), qtype, M, K, _fptr(x), _fptr(out))

    def tb_cuda_matvec_device_noalloc(self, W_dev: int, qtype: int, M: int, K: int,
                                      x: np.ndarray, out: np.ndarray) -> int:
        """The allocation-free blocking variant (static device staging, bounded M and K)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert out.dtype == np.float32 and out.flags.c_contiguous
        return self.L.tb_cuda_matvec_device_noalloc(ctypes.c_void_p(W_dev), qtype, M, K, _fptr(x), _fptr(out))

    def tb_cuda_sync_all(self) -> None:
        self.L.tb_cuda_sync_all()

    def tb_cuda_cleanup(self) -> None:
        self.L.tb_cuda_cleanup()

    # ---- part 2: device-pointer entry points ------------------------------------------
    def tb_cuda_matvec_dev(self, W_dev: int, qtype: int, M: int, K: int, d_x: int, d_y: int,
                           stream: int = 0) -> int:
        return self.L.tb_cuda_matvec_dev(ctypes.c_void_p(W_dev), qtype, M, K, ctypes.c_void_p(d_x),
                                         ctypes.c_void_p(d_y), ctypes.c_void_p(stream or None))

    def tb_cuda_qgemm_dev(self, W_dev: int, qtype: int, N: int, K: int, d_a_bf16: int, T: int, d_c: int,
                          stream: int = 0) -> int:
        """Prefill GEMM C[T][N] = A[T][K] (bf16) x dequant(W)^T on the tensor cores."""
        return self.L.tb_cuda_qgemm_dev(ctypes.c_void_p(W_dev), qtype, N, K, ctypes.c_void_p(d_a_bf16), T,
                                        ctypes.c_void_p(d_c), ctypes.c_void_p(stream or None))

    def tb_cuda_matvec_fused_dev(self, W_dev: int, qtype: int, M: int, K: int, d_x: int, d_y: int,
                                 xmode: int = 0, d_x2: int = 0, d_norm_w: int = 0, eps: float = 0.0,
                                 d_res: int = 0, ymode: int = 0, stream: int = 0) -> int:
        v = lambda p: ctypes.c_void_p(p) if p else None  # noqa: E731
        return self.L.tb_cuda_matvec_fused_dev(ctypes.c_void_p(W_dev), qtype, M, K, v(d_x), v(d_y), xmode,
                                               v(d_x2), v(d_norm_w), ctypes.c_float(eps), v(d_res), ymode,
                                               v(stream))

    def tb_cuda_matvec_experts_dev(self, W_dev: int, qtype: int, M: int, K: int, n_experts: int, d_ids: int,
                                   n_sel: int, d_x: int, x_stride: int, d_y: int, y_stride: int, ymode: int = 0,
                                   stream: int = 0) -> int:
        v = lambda p: ctypes.c_void_p(p) if p else None  # noqa: E731
        return self.L.tb_cuda_matvec_experts_dev(ctypes.c_void_p(W_dev), qtype, M, K, n_experts, v(d_ids), n_sel,
                                                 v(d_x), x_stride, v(d_y), y_stride, ymode, v(stream))

    def tb_cuda_sample_dev(self, d_logits: int, vocab: int, top_k: int, top_p: float, temperature: float, u: float,
                           d_token: int, stream: int = 0) -> int:
        v = lambda p: ctypes.c_void_p(p) if p else None  # noqa: E731
        return self.L.tb_cuda_sample_dev(v(d_logits), vocab, top_k, top_p, temperature, u, v(d_token), v(stream))

    def tb_cuda_dequant_dev(self, W_dev: int, qtype: int, M: int, K: int, d_out: int, sem: int = 0,
                            stream: int = 0) -> int:
        return self.L.tb_cuda_dequant_dev(ctypes.c_void_p(W_dev), qtype, M, K, ctypes.c_void_p(d_out),
                                          sem, ctypes.c_void_p(stream or None))

    def tb_cuda_qtype_info(self, qtype: int) -> tuple[int, int] | None:
        bw, bb = ctypes.c_int(), ctypes.c_int()
        if not self.L.tb_cuda_qtype_info(qtype, ctypes.byref(bw), ctypes.byref(bb)):
            return None
        return bw.value, bb.value

    def tb_cuda_last_error(self) -> int:
        return self.L.tb_cuda_last_error()

    def tb_cuda_launch_count(self) -> int:
        return int(self.L.tb_cuda_launch_count())

    def tb_cuda_version(self) -> str:
        return self.L.tb_cuda_version().decode()

    def tb_cuda_set_matvec_arith(self, mode: int) -> int:
        return int(self.L.tb_cuda_set_matvec_arith(mode))

    def tb_cuda_get_matvec_arith(self) -> int:
        return int(self.L.tb_cuda_get_matvec_arith())

    # ---- convenience ------------------------------------------------------------------
    def matvec(self, W_dev: int, qtype: int, M: int, K: int, x: np.ndarray) -> np.ndarray:
        """Blocking y = dequant(W) @ x through tb_cuda_matvec_device; raises on a 0 return."""
        out = np.empty(M, dtype=np.float32)
        if not self.tb_cuda_matvec_device(W_dev, qtype, M, K, x, out):
            raise RuntimeError(f"tb_cuda_matvec_device failed ({Q.NAMES.get(qtype, qtype)} {M}x{K})")
        return out


_singleton: KQuantLib | None = None


def load() -> KQuantLib:
    global _singleton
    if _singleton is None:
        _singleton = KQuantLib()
    return _singleton
