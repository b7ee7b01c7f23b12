"""The allocation-free blocking entry point, tb_cuda_matvec_device_noalloc.

It must give the same result as tb_cuda_matvec_device (same kernel, same
inputs, so bit-identical) on two calls in a row, whether this file runs alone
or after the other GPU tests, and it must reject shapes larger than its static
buffers without launching anything.
"""
import numpy as np
import pytest

from trailblaze_b200 import qtypes as Q, synth

pytestmark = pytest.mark.gpu

MAX_K, MAX_M = 65536, 262144   # the static buffer sizes stated in the header


def _upload(kq, W):
    d = kq.tb_cuda_upload_tensor(W)
    assert d
    return d


@pytest.mark.parametrize("qt,M,K", [(Q.Q4_K, 512, 4096), (Q.Q6_K, 300, 2560), (Q.Q8_0, 77, 1056)])
def test_noalloc_matches_blocking_entry_twice(kq, qt, M, K):
    W = synth.weights(qt, M, K, seed=61, tensor=qt)
    d = _upload(kq, W)
    try:
        for call in range(2):   # two calls in a row, different x each time
            x = synth.activations(K, seed=62 + call)
            ref = np.zeros(M, dtype=np.float32)
            got = np.full(M, np.nan, dtype=np.float32)
            assert kq.tb_cuda_matvec_device(d, qt, M, K, x, ref) == 1
            assert kq.tb_cuda_matvec_device_noalloc(d, qt, M, K, x, got) == 1
            np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    finally:
        kq.tb_cuda_free_tensor(d)


def test_noalloc_long_rows_then_short(kq):
    """A long row (half the static x buffer), then a short shape again."""
    for qt, M, K in [(Q.Q8_0, 8, MAX_K // 2), (Q.Q4_K, 16, 256)]:
        W = synth.weights(qt, M, K, seed=63, tensor=qt)
        x = synth.activations(K, seed=64)
        d = _upload(kq, W)
        try:
            ref = np.zeros(M, dtype=np.float32)
            got = np.zeros(M, dtype=np.float32)
            assert kq.tb_cuda_matvec_device(d, qt, M, K, x, ref) == 1
            assert kq.tb_cuda_matvec_device_noalloc(d, qt, M, K, x, got) == 1
            np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
        finally:
            kq.tb_cuda_free_tensor(d)


def test_noalloc_rejects_oversize_and_bad_args(kq):
    W = synth.weights(Q.Q4_K, 1, 256, seed=65, tensor=1)
    d = _upload(kq, W)
    try:
        x = np.zeros(MAX_K + 256, dtype=np.float32)
        out = np.zeros(MAX_M + 1, dtype=np.float32)
        # rejected on the host before any copy or launch
        assert kq.tb_cuda_matvec_device_noalloc(d, Q.Q4_K, 1, MAX_K + 256, x, out) == 0
        assert kq.tb_cuda_matvec_device_noalloc(d, Q.Q4_K, MAX_M + 1, 256, x, out) == 0
        assert kq.tb_cuda_matvec_device_noalloc(d, Q.Q4_K, 1, 100, x, out) == 0     # K % 256
        assert kq.tb_cuda_matvec_device_noalloc(d, 99, 1, 256, x, out) == 0         # unknown qtype
        assert kq.tb_cuda_last_error() == 0
    finally:
        kq.tb_cuda_free_tensor(d)
