"""The model arena (tb_cuda_arena_*): whole tensors, a rank's row range and a
rank's K-column slice uploaded through pinned staging arrive byte for byte
(several staging chunks included), sub-ranges are 256-byte aligned, a full arena
refuses an upload, and a matvec on an uploaded K slice equals the oracle's
matvec of that slice (the tensor-parallel o / down shard)."""
import ctypes

import numpy as np
import pytest

from oracle.oracle import SEM_CUDA
from trailblaze_b200 import qtypes as Q, shard, synth

pytestmark = pytest.mark.gpu


def _read(ptr, n):
    """n device bytes at ptr, copied to the host with the CUDA runtime."""
    import torch
    from cuda.bindings import runtime as rt
    torch.cuda.synchronize()
    host = np.empty(n, dtype=np.uint8)
    err, = rt.cudaMemcpy(host.ctypes.data, ptr, n, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert err == rt.cudaError_t.cudaSuccess
    return host


def test_arena_uploads_whole_rows_and_cols(kq):
    L = kq.L
    rng = np.random.default_rng(3)
    big = rng.integers(0, 256, 80 << 20, dtype=np.uint8)          # three staging chunks
    qt, M, K = Q.Q6_K, 300, 4096
    W = synth.weights(qt, M, K, seed=12, tensor=qt)
    rb = Q.row_bytes(qt, K)
    a = L.tb_cuda_arena_create(256 << 20)
    assert a
    try:
        p1 = L.tb_cuda_arena_upload(a, big.ctypes.data, big.nbytes)
        p2 = L.tb_cuda_arena_upload_rows(a, W.ctypes.data, rb, 37, 211)
        b_lo, b_hi = 4 * Q.geometry(qt)[1], 12 * Q.geometry(qt)[1]   # blocks [4, 12) of every row
        p3 = L.tb_cuda_arena_upload_cols(a, W.ctypes.data, M, rb, b_lo, b_hi)
        assert p1 and p2 and p3
        assert p1 % 256 == 0 and p2 % 256 == 0 and p3 % 256 == 0
        np.testing.assert_array_equal(_read(p1, big.nbytes), big)
        np.testing.assert_array_equal(_read(p2, 174 * rb), shard.row_slice(W, qt, M, K, 37, 211))
        cols = np.ascontiguousarray(shard.k_slice(W, qt, M, K, 4 * 256, 12 * 256))
        np.testing.assert_array_equal(_read(p3, cols.nbytes), cols)
        assert L.tb_cuda_arena_used(a) >= big.nbytes + 174 * rb + cols.nbytes
        assert not L.tb_cuda_arena_upload(a, big.ctypes.data, 200 << 20)   # full: refused
        # the K slice as a tensor-parallel shard: its matvec equals the oracle's on the slice
        import torch
        from oracle.oracle import Oracle
        x = synth.activations(2048, seed=5)
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty(M, device="cuda")
        assert kq.tb_cuda_matvec_dev(p3, qt, M, 2048, dx.data_ptr(), dy.data_ptr(), 0) == 1
        torch.cuda.synchronize()
        ref = Oracle().matvec_f64(qt, cols, M, 2048, x, SEM_CUDA)
        y = dy.cpu().numpy().astype(np.float64)
        assert np.linalg.norm(y - ref) / np.linalg.norm(ref) <= 2e-5
    finally:
        L.tb_cuda_arena_destroy(a)
