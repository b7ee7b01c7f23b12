"""Batched prefill (tb_cuda_dec_prefill) against the oracle, then decode.

The oracle (oracle/decode_ref.py DecodeOracle.prefill) restates the prefill
one token at a time with the tensor-core GEMM's roundings: bf16 activations
into the projections and bf16-rounded weights, norms, attention and the
residual exact.  Checks: the last prompt token's logits (1e-3 relative L2) and
greedy token, the K and V cache rows written for every prompt position, and a
chain of decode steps after the prompt (the oracle following the GPU's
tokens).  Prompts of 40 tokens (one chunk, padded to 48 rows) and 530 tokens
(two chunks), from position 0 and after a cached prefix, in both orders."""
import ctypes

import numpy as np
import pytest

from oracle.decode_ref import DecodeOracle

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("n,pos0,quirks", [(40, 0, True), (530, 0, True), (40, 17, False)])
def test_prefill_then_decode_matches_oracle(kq, n, pos0, quirks):
    from test_gpu_decode import GpuDecoder, check_token, make_model
    m = make_model(n_layers=2, hidden=512, nh=8, nk=2, ffn=2048, vocab=1000, max_ctx=pos0 + n + 8, seed=71)
    dec, orc = GpuDecoder(kq, m, quirks), DecodeOracle(m, quirks=quirks)
    try:
        if pos0:
            rng = np.random.default_rng(5)
            for li in range(m.n_layers):
                for which in (0, 1):
                    a = rng.standard_normal((m.n_kv_heads, pos0, m.head_dim)).astype(np.float32)
                    dec.load_kv(li, which, a)
                    (orc.kc if which == 0 else orc.vc)[li, :, :pos0] = a
        toks = np.random.default_rng(n).integers(0, m.vocab, n).astype(np.int32)
        nxt = ctypes.c_int(-1)
        lg = np.zeros(m.vocab, dtype=np.float32)
        ip = ctypes.POINTER(ctypes.c_int)
        assert kq.L.tb_cuda_dec_prefill(dec.d, toks.ctypes.data_as(ip), n, pos0, ctypes.byref(nxt),
                                        lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float))) == 1
        lr, _ = orc.prefill(list(toks), pos0)
        check_token(lg, nxt.value, lr)
        for li in range(m.n_layers):
            for which in (0, 1):
                got = dec.read_kv(li, which, pos0, n)
                want = (orc.kc if which == 0 else orc.vc)[li, :, pos0:pos0 + n]
                assert rel_l2(got, want) <= TOL, (li, which, rel_l2(got, want))
        # decode continues after the prompt; the oracle follows the GPU's tokens
        tok = nxt.value
        for i in range(3):
            lgd, nd = dec.step(tok, pos0 + n + i)
            lrd, _ = orc.step(tok, pos0 + n + i)
            check_token(lgd, nd, lrd)
            tok = nd
    finally:
        dec.close()


def test_prefill_refuses_unsupported(kq):
    from test_gpu_decode import GpuDecoder, make_model
    m = make_model(n_layers=1, hidden=512, nh=8, nk=2, ffn=1024, vocab=300, max_ctx=64, seed=3)   # Q6_K down, K=1024
    dec = GpuDecoder(kq, m, True)
    try:
        toks = np.arange(8, dtype=np.int32)
        ip = ctypes.POINTER(ctypes.c_int)
        nxt = ctypes.c_int(-1)
        assert kq.L.tb_cuda_dec_prefill(dec.d, toks.ctypes.data_as(ip), 8, 0, ctypes.byref(nxt), None) == 0
    finally:
        dec.close()
