"""Pins of oracle/decode_ref.py against the reference's own decode-step code,
compiled from its sources into oracle/_ref/libtbref_infer.so (CPU only).

  tb_rms_norm    layer1/tb_tensor.c:194-199
  tb_rope_apply  layer4/tb_infer.c:142-155
  tb_swiglu      layer4/tb_infer.c:130-135
  tb_attention   layer1/tb_tensor.c:303-409 (with tb_kvcache_alloc, :tb_tensor.h:68-78)

The reference computes in fp32, the oracle in fp64, so agreement is to fp32
rounding (about 1e-6 relative), not bit for bit.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import decode_ref as D

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libtbref_infer.so")

fp = ctypes.POINTER(ctypes.c_float)


class KVCache(ctypes.Structure):
    """TB_KVCache, layer1/tb_tensor.h:68-78."""
    _fields_ = [("keys", ctypes.POINTER(fp)), ("vals", ctypes.POINTER(fp)), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("seq_len", ctypes.c_int), ("branch_id", ctypes.c_int), ("epoch", ctypes.c_int32)]


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libtbref_infer.so not built")
    L = ctypes.CDLL(LIB)
    L.tb_rms_norm.argtypes = [fp, fp, fp, ctypes.c_int, ctypes.c_float]
    L.tb_rope_apply.argtypes = [fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    L.tb_swiglu.argtypes = [fp, fp, fp, ctypes.c_int]
    L.tb_kvcache_alloc.restype = ctypes.POINTER(KVCache)
    L.tb_kvcache_alloc.argtypes = [ctypes.c_int] * 5 + [ctypes.c_int32]
    L.tb_kvcache_free.argtypes = [ctypes.POINTER(KVCache)]
    L.tb_attention.argtypes = [fp, fp, fp, ctypes.POINTER(KVCache), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, fp]
    return L


def p(a):
    return a.ctypes.data_as(fp)


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def test_rms_norm_pinned(ref):
    rng = np.random.default_rng(1)
    x = rng.standard_normal(4096).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float32)
    out = np.zeros_like(x)
    ref.tb_rms_norm(p(x), p(w), p(out), 4096, 1e-6)
    assert rel(out, D.rms_norm(x, w, 1e-6)) < 2e-6


@pytest.mark.parametrize("pos", [0, 7, 1000, 4096])
def test_rope_pinned(ref, pos):
    rng = np.random.default_rng(pos)
    q = rng.standard_normal(128).astype(np.float32)
    k = rng.standard_normal(128).astype(np.float32)
    q2, k2 = q.copy(), k.copy()
    ref.tb_rope_apply(p(q2), p(k2), 128, pos, 1e6)
    assert rel(q2, D.rope(q, pos, 1e6, 128)) < 2e-6
    assert rel(k2, D.rope(k, pos, 1e6, 128)) < 2e-6


def test_swiglu_pinned(ref):
    rng = np.random.default_rng(2)
    g = (3 * rng.standard_normal(3000)).astype(np.float32)
    u = rng.standard_normal(3000).astype(np.float32)
    out = np.zeros_like(g)
    ref.tb_swiglu(p(g), p(u), p(out), 3000)
    assert rel(out, D.swiglu(g, u)) < 2e-6


@pytest.mark.parametrize("NH,NK,T", [(8, 2, 1), (8, 2, 77), (32, 8, 300), (32, 4, 65)])
def test_attention_pinned(ref, NH, NK, T):
    """tb_attention appends k, v at seq_len and attends over seq_len + 1 positions."""
    HD, max_seq = 128, 512
    rng = np.random.default_rng(NH * 1000 + T)
    c = ref.tb_kvcache_alloc(1, NK, HD, max_seq, 0, 0)
    assert c
    try:
        pre_k = rng.standard_normal((NK, T - 1, HD)).astype(np.float32)
        pre_v = rng.standard_normal((NK, T - 1, HD)).astype(np.float32)
        kp = np.ctypeslib.as_array(c.contents.keys[0], shape=(NK * max_seq * HD,)).reshape(NK, max_seq, HD)
        vp = np.ctypeslib.as_array(c.contents.vals[0], shape=(NK * max_seq * HD,)).reshape(NK, max_seq, HD)
        kp[:, :T - 1] = pre_k
        vp[:, :T - 1] = pre_v
        c.contents.seq_len = T - 1
        q = rng.standard_normal((NH, HD)).astype(np.float32)
        k = rng.standard_normal((NK, HD)).astype(np.float32)
        v = rng.standard_normal((NK, HD)).astype(np.float32)
        out = np.zeros((NH, HD), dtype=np.float32)
        ref.tb_attention(p(q), p(k), p(v), c, 0, NH, NK, HD, p(out))
        kc = np.concatenate([pre_k, k[:, None]], axis=1).astype(np.float64)
        vc = np.concatenate([pre_v, v[:, None]], axis=1).astype(np.float64)
        assert rel(out, D.attention(q.astype(np.float64), kc, vc, NH, NK)) < 2e-6
        assert c.contents.seq_len == T   # layer 0 advances the counter
    finally:
        ref.tb_kvcache_free(c)
