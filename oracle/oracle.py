"""ctypes access to the parity checker (TEST INFRASTRUCTURE ONLY).

  * liboracle.so          — tb_oracle.c, the C restatement of the reference's
                             decode semantics (see tb_oracle.h for citations).
  * _ref/libtbref_*.so    — the reference's own CPU code (layer4/tb_gguf.c,
                             src/tb_analog_dispatch.c) compiled from its sources,
                             plus ref_mt.c's thread-split timer.
  * _ref/libtbref_cuda.so — the reference's CUDA kernels built for sm_100a.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module.  The shipped library never loads any of these files.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
SEM_CUDA, SEM_GGUF_C, SEM_DISPATCH = 0, 1, 2

_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_vp = ctypes.c_void_p


def build(ref: str | None = None) -> None:
    """Run oracle/Makefile (liboracle.so always; _ref/ when the reference tree exists).

    The reference checkout is `ref`, else $TB_REFERENCE_DIR, else none (the
    prebuilt _ref/ files are used as they are)."""
    cmd = ["make", "-s", "-C", HERE]
    ref = ref or os.environ.get("TB_REFERENCE_DIR")
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd + ["oracle"], check=True)
    subprocess.run(cmd + ["ref"], check=True)


def _p(a):
    return a.ctypes.data_as(_vp)


class Oracle:
    def __init__(self):
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        L.tbo_h2f.restype = ctypes.c_float
        L.tbo_h2f.argtypes = [ctypes.c_uint16]
        L.tbo_bf2f.restype = ctypes.c_float
        L.tbo_bf2f.argtypes = [ctypes.c_uint16]
        L.tbo_dequant_block.argtypes = [ctypes.c_int, ctypes.c_int, _vp, _fp]
        L.tbo_dequant_rows.argtypes = [ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _fp]
        L.tbo_matvec_f64.argtypes = [ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _fp, _dp]
        L.tbo_matvec_f32_seq.argtypes = [ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _fp, _fp]
        L.tbo_row_bytes.restype = ctypes.c_size_t
        L.tbo_row_bytes.argtypes = [ctypes.c_int, ctypes.c_int]
        self.L = L

    def h2f(self, h: int) -> float:
        return self.L.tbo_h2f(h)

    def bf2f(self, b: int) -> float:
        return self.L.tbo_bf2f(b)

    def dequant(self, qtype: int, W: np.ndarray, M: int, K: int, sem: int = SEM_CUDA) -> np.ndarray:
        out = np.empty(M * K, dtype=np.float32)
        W = np.ascontiguousarray(W)
        assert self.L.tbo_dequant_rows(qtype, sem, _p(W), M, K, out.ctypes.data_as(_fp)) == 1
        return out.reshape(M, K)

    def matvec_f64(self, qtype: int, W: np.ndarray, M: int, K: int, x: np.ndarray,
                   sem: int = SEM_CUDA) -> np.ndarray:
        y = np.empty(M, dtype=np.float64)
        W = np.ascontiguousarray(W)
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert self.L.tbo_matvec_f64(qtype, sem, _p(W), M, K, x.ctypes.data_as(_fp), y.ctypes.data_as(_dp)) == 1
        return y

    def matvec_f32_seq(self, qtype: int, W: np.ndarray, M: int, K: int, x: np.ndarray,
                       sem: int = SEM_GGUF_C) -> np.ndarray:
        y = np.empty(M, dtype=np.float32)
        W = np.ascontiguousarray(W)
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert self.L.tbo_matvec_f32_seq(qtype, sem, _p(W), M, K, x.ctypes.data_as(_fp), y.ctypes.data_as(_fp)) == 1
        return y


def host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return all(t in flags for t in ("avx512f", "avx512bw", "avx512dq", "avx512vl", "avx512_vnni"))
    except OSError:
        return False


class Reference:
    """The reference's own CPU routines, built from its sources into _ref/."""

    def __init__(self, variant: str | None = None):
        if variant is None:
            variant = "avx512" if host_has_avx512() else "avx2"
        path = os.path.join(REF_DIR, f"libtbref_{variant}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing (built by oracle/Makefile from the reference tree)")
        L = ctypes.CDLL(path)
        L.tb_gguf_dequant_row.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _fp]
        L.tb_gguf_dequant_matvec.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, _fp]
        for n in ("tb_dot_q4k_scalar", "tb_dot_q3k_scalar", "tb_dot_q8_scalar"):
            getattr(L, n).restype = ctypes.c_float
            getattr(L, n).argtypes = [_vp, ctypes.c_int, _fp]
        L.tbr_time_matvec.restype = ctypes.c_double
        L.tbr_time_matvec.argtypes = [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_size_t, _fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        self.L = L
        self.variant = variant
        self.path = path

    def dequant_row(self, qtype: int, W: np.ndarray, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        W = np.ascontiguousarray(W)
        self.L.tb_gguf_dequant_row(_p(W), qtype, n, out.ctypes.data_as(_fp))
        return out

    def dequant_matvec(self, qtype: int, W: np.ndarray, M: int, K: int, x: np.ndarray) -> np.ndarray:
        y = np.empty(M, dtype=np.float32)
        W = np.ascontiguousarray(W)
        x = np.ascontiguousarray(x, dtype=np.float32)
        self.L.tb_gguf_dequant_matvec(_p(W), qtype, M, K, x.ctypes.data_as(_fp), y.ctypes.data_as(_fp))
        return y

    def dot_scalar(self, name: str, row: np.ndarray, K: int, x: np.ndarray) -> float:
        row = np.ascontiguousarray(row)
        x = np.ascontiguousarray(x, dtype=np.float32)
        return float(getattr(self.L, name)(_p(row), K, x.ctypes.data_as(_fp)))

    def time_matvec(self, path: int, qtype: int, W: np.ndarray, M: int, K: int, row_bytes: int,
                    x: np.ndarray, nthreads: int, reps: int) -> tuple[float, np.ndarray]:
        y = np.empty(M, dtype=np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        t = self.L.tbr_time_matvec(path, _p(W), qtype, M, K, row_bytes, x.ctypes.data_as(_fp),
                                   y.ctypes.data_as(_fp), nthreads, reps,
                                   1 if self.variant == "avx512" else 0)
        return t, y


class ReferenceCuda:
    """The reference's unmodified CUDA kernels (tb_gguf_dequant.cu) built for sm_100a,
    plus tbr_cuda_launch (oracle/ref_cuda_launch.cu): one kernel launch on device
    pointers at the reference's default geometry, stream-ordered, for timing."""

    def __init__(self):
        path = os.path.join(REF_DIR, "libtbref_cuda.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        if hasattr(L, "tbr_cuda_launch"):
            L.tbr_cuda_launch.restype = ctypes.c_int
            L.tbr_cuda_launch.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]
        L.tb_cuda_init.restype = ctypes.c_int
        L.tb_cuda_upload_tensor.restype = _vp
        L.tb_cuda_upload_tensor.argtypes = [_vp, ctypes.c_size_t]
        L.tb_cuda_free_tensor.argtypes = [_vp]
        L.tb_cuda_matvec_device.restype = ctypes.c_int
        L.tb_cuda_matvec_device.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _fp, _fp]
        L.tb_cuda_set_snap.argtypes = [_vp]
        self.L = L
