"""Parity at the BASELINE model widths (configs 3, 4 and 5), against the oracle.

- Config 3: a Qwen3-8B-width dense decoder (hidden 4096, 32 q / 8 kv heads,
  head_dim 128, FFN 12288, vocabulary 151936; Q4_K weights, Q6_K ffn_down and
  output), 2 layers, one step at context 4096 over an N(0,1) fp32 cache, in
  the reference's order: logits (1e-3 relative L2) and the greedy token, the
  last layer's q|k|v, attention output, x2 and SwiGLU activation.
- Config 4: a Qwen3-30B-A3B-width routed decoder (hidden 2048, 32 q / 4 kv
  heads, 128 experts of FFN 768, top 8; Q4_K experts, Q6_K attention and
  output, fp32 router), 2 layers, one step at context 2048: router logits,
  the selected experts, their SwiGLU activations, logits and the token.
- Config 5: the prefill GEMM at 12288 x 4096 and 4096 x 12288 for T = 16,
  128, 512, Q4_K and Q6_K, against oracle dequant -> bf16 -> fp64 products.
The oracle keeps these tensors as raw bytes and dequantises them chunk by
chunk (oracle/decode_ref.py LazyMat), so its float64 matrices never exist."""
import numpy as np
import pytest

from oracle.decode_ref import DecodeOracle
from trailblaze_b200 import qtypes as Q, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def _prefill(m, dec, orc, n, seed):
    rng = np.random.default_rng(seed)
    for li in range(m.n_layers):
        for which in (0, 1):
            a = rng.standard_normal((m.n_kv_heads, n, m.head_dim)).astype(np.float32)
            dec.load_kv(li, which, a)
            (orc.kc if which == 0 else orc.vc)[li, :, :n] = a


def test_config3_qwen3_8b_width_decode(kq):
    from test_gpu_decode import GpuDecoder, check_token, make_model
    ctx = 4096
    m = make_model(n_layers=2, hidden=4096, nh=32, nk=8, ffn=12288, vocab=151936, max_ctx=ctx + 4, seed=33)
    dec, orc = GpuDecoder(kq, m, True), DecodeOracle(m, quirks=True, lazy=True)
    try:
        _prefill(m, dec, orc, ctx, seed=3)
        lg, nxt = dec.step(12345, ctx)
        lr, _ = orc.step(12345, ctx)
        check_token(lg, nxt, lr)
        H, NH, NK, F = m.hidden, m.n_heads, m.n_kv_heads, m.ffn_dim
        assert rel_l2(dec.read(2, (NH + 2 * NK) * 128), orc.last["qkv"]) <= TOL
        assert rel_l2(dec.read(3, NH * 128), orc.last["att"]) <= TOL
        assert rel_l2(dec.read(1, H), orc.last["x2"]) <= TOL
        assert rel_l2(dec.read(4, F), orc.last["act"]) <= TOL
    finally:
        dec.close()


def test_config4_qwen3_30b_a3b_width_decode(kq):
    from test_gpu_decode import check_token
    from test_gpu_moe import GpuMoeDecoder, make_moe_model
    ctx = 2048
    m = make_moe_model(n_layers=2, hidden=2048, nh=32, nk=4, ffn=768, n_exp=128, top_k=8, vocab=151936,
                       max_ctx=ctx + 4, seed=44)
    dec, orc = GpuMoeDecoder(kq, m), DecodeOracle(m, quirks=True, lazy=True)
    try:
        _prefill(m, dec, orc, ctx, seed=4)
        lg, nxt = dec.step(777, ctx)
        lr, _ = orc.step(777, ctx)
        E, k, F = m.n_experts, m.top_k, m.ffn_dim
        last = orc.last
        assert rel_l2(dec.read(6, E), last["router"]) <= TOL
        ids = dec.read(8, k).view(np.int32)
        order = sorted(range(k), key=lambda i: (-last["wts"][i], last["ids"][i]))
        assert list(ids) == [last["ids"][i] for i in order], (ids, last["ids"], last["wts"])
        acts = dec.read(9, k * F).reshape(k, F)
        for r, i in enumerate(order):
            assert rel_l2(acts[r], last["acts"][i]) <= TOL
        check_token(lg, nxt, lr)
    finally:
        dec.close()


@pytest.mark.parametrize("qt", [Q.Q4_K, Q.Q6_K], ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("N,K", [(12288, 4096), (4096, 12288)])
def test_config5_prefill_gemm_full_shapes(kq, qt, N, K):
    import torch
    from oracle.oracle import Oracle
    from test_gpu_qgemm import bf16_round
    W = synth.weights(qt, N, K, seed=N + K, tensor=qt)
    Wb = bf16_round(Oracle().dequant(qt, W, N, K)).astype(np.float64)
    dW = torch.from_numpy(W).cuda()
    for T in (16, 128, 512):
        rng = np.random.default_rng(T)
        A = bf16_round(rng.standard_normal((T, K)).astype(np.float32))
        ref = A.astype(np.float64) @ Wb.T
        dA = torch.from_numpy(A).cuda().to(torch.bfloat16)
        dC = torch.full((T, N), float("nan"), dtype=torch.float32, device="cuda")
        assert kq.tb_cuda_qgemm_dev(dW.data_ptr(), qt, N, K, dA.data_ptr(), T, dC.data_ptr()) == 1
        torch.cuda.synchronize()
        C = dC.cpu().numpy()
        assert np.isfinite(C).all()
        assert rel_l2(C, ref) <= 2e-5, (T, rel_l2(C, ref))
        assert kq.tb_cuda_last_error() == 0
