"""GPU parity of the prefill GEMM (tb_cuda_qgemm_dev, tcgen05 bf16 MMA with
fp32 accumulation) against the oracle.

The GEMM rounds the exactly dequantised weights to bf16 (round to nearest
even) and multiplies them with bf16 activations, the products exact and the
sums fp32.  So the reference is oracle dequant -> bf16 -> fp64 products and
sums: rel L2 <= 2e-5 (fp32 accumulation only).  Against the unrounded weights
the bf16 rounding of W costs about 1e-3 relative; <= 4e-3 is asserted.
Shapes: T = 16, 128 and 512 tokens (one and two MMAs per K step), several
128-row tiles, and a single tile with split K (partial sums added into C).
Q6_K rows must be a multiple of 16 bytes (K a multiple of 2048) for the
weight tensor map."""
import numpy as np
import pytest

from trailblaze_b200 import qtypes as Q, synth

pytestmark = pytest.mark.gpu


def bf16_round(x):
    """float32 -> bf16 (round to nearest even) -> float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    return (r.astype(np.uint32) << 16).view(np.float32)


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


CASES = [(Q.Q4_K, 256, 512, 16), (Q.Q4_K, 384, 1024, 128), (Q.Q4_K, 256, 768, 512), (Q.Q4_K, 128, 2048, 32),
         (Q.Q6_K, 256, 2048, 16), (Q.Q6_K, 384, 2048, 128), (Q.Q6_K, 256, 4096, 512), (Q.Q6_K, 128, 4096, 48)]


@pytest.mark.parametrize("qt,N,K,T", CASES)
def test_qgemm_matches_oracle(kq, qt, N, K, T):
    import torch
    from oracle.oracle import Oracle
    W = synth.weights(qt, N, K, seed=N + K + T, tensor=qt)
    Wd = Oracle().dequant(qt, W, N, K)                      # exact fp32 weights
    rng = np.random.default_rng(T)
    A = bf16_round(rng.standard_normal((T, K)).astype(np.float32))
    ref_bf = A.astype(np.float64) @ bf16_round(Wd).astype(np.float64).T
    ref = A.astype(np.float64) @ Wd.astype(np.float64).T
    dW = torch.from_numpy(W).cuda()
    dA = torch.from_numpy(A).cuda().to(torch.bfloat16)      # exact: A holds bf16 values
    dC = torch.full((T, N), float("nan"), dtype=torch.float32, device="cuda")
    assert kq.tb_cuda_qgemm_dev(dW.data_ptr(), qt, N, K, dA.data_ptr(), T, dC.data_ptr()) == 1
    torch.cuda.synchronize()
    C = dC.cpu().numpy()
    assert np.isfinite(C).all()
    assert rel_l2(C, ref_bf) <= 2e-5, rel_l2(C, ref_bf)
    assert rel_l2(C, ref) <= 4e-3
    assert kq.tb_cuda_last_error() == 0


def test_qgemm_rejects_unsupported(kq):
    import torch
    W = torch.zeros(Q.row_bytes(Q.Q4_K, 512) * 128, dtype=torch.uint8, device="cuda")
    A = torch.zeros((16, 512), dtype=torch.bfloat16, device="cuda")
    C = torch.zeros((16, 128), dtype=torch.float32, device="cuda")
    assert kq.tb_cuda_qgemm_dev(W.data_ptr(), Q.Q8_0, 128, 512, A.data_ptr(), 16, C.data_ptr()) == 0   # type
    assert kq.tb_cuda_qgemm_dev(W.data_ptr(), Q.Q4_K, 100, 512, A.data_ptr(), 16, C.data_ptr()) == 0   # N % 128
    assert kq.tb_cuda_qgemm_dev(W.data_ptr(), Q.Q4_K, 128, 512, A.data_ptr(), 24, C.data_ptr()) == 0   # T % 16
    W6 = torch.zeros(Q.row_bytes(Q.Q6_K, 512) * 128, dtype=torch.uint8, device="cuda")
    assert kq.tb_cuda_qgemm_dev(W6.data_ptr(), Q.Q6_K, 128, 512, A.data_ptr(), 16, C.data_ptr()) == 0  # 420-B rows
