"""Pins of oracle/sample_ref.py against the reference's own samplers
(tb_sample_top_p / tb_sample_top_k, layer1/tb_tensor.c:436-540), compiled from
its sources into oracle/_ref/libtbref_infer.so (CPU only).  The reference draws
u with rand(); the test seeds the C library's generator, reads the value the
sampler will see, seeds it again and runs the sampler."""
import ctypes
import os

import numpy as np
import pytest

from oracle import sample_ref as S

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libtbref_infer.so")
RAND_MAX = 2147483647   # glibc


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libtbref_infer.so not built")
    L = ctypes.CDLL(LIB)
    fp = ctypes.POINTER(ctypes.c_float)
    L.tb_sample_top_p.argtypes = [fp, ctypes.c_int, ctypes.c_float, ctypes.c_float]
    L.tb_sample_top_k.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    libc = ctypes.CDLL("libc.so.6")
    return L, libc


def _u(libc, seed):
    libc.srand(seed)
    return float(np.float32(libc.rand()) / (np.float32(RAND_MAX) + np.float32(1.0)))


@pytest.mark.parametrize("case", range(12))
def test_top_p_matches_reference(ref, case):
    L, libc = ref
    rng = np.random.default_rng(100 + case)
    V = [50, 1000, 5000, 32000][case % 4]
    lg = (rng.standard_normal(V) * (1 + case % 3)).astype(np.float32)
    p, t = [0.9, 0.5, 0.99][case % 3], [1.0, 0.7, 1.3, 0.005][case % 4]
    u = _u(libc, 7 + case)
    libc.srand(7 + case)
    want = L.tb_sample_top_p(lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V, p, t)
    assert S.sample_top_p(lg, p, t, u) == want


@pytest.mark.parametrize("case", range(12))
def test_top_k_matches_reference(ref, case):
    L, libc = ref
    rng = np.random.default_rng(200 + case)
    V = [64, 1000, 8000][case % 3]
    lg = (rng.standard_normal(V) * 2).astype(np.float32)
    k = [1, 5, 40, 10000][case % 4]
    t = [1.0, 0.8, 0.0][case % 3]
    u = _u(libc, 30 + case)
    libc.srand(30 + case)
    want = L.tb_sample_top_k(lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V, k, t)
    assert S.sample_top_k(lg, k, t, u) == want


def test_top_k_tie_order_differs_from_reference(ref):
    """A recorded divergence: among equal logits at the k boundary the reference's
    selection sort swaps elements and keeps the later index (logits [2, 2, 3], k = 2:
    indices 2 and 1), while the oracle and the device keep the lower index (2 and 0).
    With u below the first candidate's probability both pick index 2; above it, the
    reference picks 1 and the oracle 0."""
    L, libc = ref
    lg = np.array([2.0, 2.0, 3.0], dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    seed = next(s for s in range(1000) if _u(libc, s) > 0.9)
    u = _u(libc, seed)
    libc.srand(seed)
    want = L.tb_sample_top_k(lg.ctypes.data_as(fp), 3, 2, 1.0)
    assert want == 1
    assert S.sample_top_k(lg, 2, 1.0, u) == 0
