"""GPU parity of the decode step (tb_cuda_matvec_fused_dev, tb_cuda_dec_*) against
the numpy restatement of tb_layer_forward / tb_infer_decode (oracle/decode_ref.py).

Tolerance: the step's logits within 1e-3 relative L2 of the fp64 oracle (the
matvec bar); the appended cache rows within 1e-4.  The greedy token must be
the oracle's argmax, or tie with it within the logits' tolerance.
"""
import ctypes

import numpy as np
import pytest

from oracle.decode_ref import DecodeModel, DecodeOracle
from trailblaze_b200 import qtypes as Q, synth
from trailblaze_b200._lib import DecConfig, DecLayer

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def make_model(n_layers=2, hidden=512, nh=8, nk=2, ffn=768, vocab=1000, max_ctx=96, qk_norm=True, seed=5):
    rng = np.random.default_rng(seed)
    HD = 128
    m = DecodeModel(n_layers, hidden, nh, nk, HD, ffn, vocab, max_ctx, rope_base=1e6, norm_eps=1e-6)
    t = 0

    def W(qt, M, K):
        nonlocal t
        t += 1
        return synth.weights(qt, M, K, seed=seed, tensor=t)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    m.emb, m.emb_qt = W(Q.Q4_K, vocab, hidden), Q.Q4_K
    m.lm, m.lm_qt = W(Q.Q6_K, vocab, hidden), Q.Q6_K
    m.out_norm = norm(hidden)
    for _ in range(n_layers):
        m.layers.append(dict(
            wqkv=W(Q.Q4_K, (nh + 2 * nk) * HD, hidden), qkv_qt=Q.Q4_K,
            wo=W(Q.Q4_K, hidden, nh * HD), o_qt=Q.Q4_K,
            wgu=W(Q.Q4_K, 2 * ffn, hidden), gu_qt=Q.Q4_K,
            wd=W(Q.Q6_K, hidden, ffn), d_qt=Q.Q6_K,
            attn_norm=norm(hidden), ffn_norm=norm(hidden),
            q_norm=norm(HD) if qk_norm else None, k_norm=norm(HD) if qk_norm else None))
    return m


class GpuDecoder:
    """The library's decoder loaded with a DecodeModel's tensors (device copies kept alive here)."""

    def __init__(self, kq, m: DecodeModel, quirks: bool):
        import torch
        self.kq, self.m, self.keep = kq, m, []
        L = kq.L
        cfg = DecConfig(m.n_layers, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim, m.vocab,
                        m.max_ctx, m.rope_base, m.norm_eps, 1 if quirks else 0)
        self.d = L.tb_cuda_dec_create(ctypes.byref(cfg))
        assert self.d

        def dev(a):
            t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
            self.keep.append(t)
            return t.data_ptr()

        for li, w in enumerate(m.layers):
            lw = DecLayer(dev(w["wqkv"]), w["qkv_qt"], dev(w["wo"]), w["o_qt"], dev(w["wgu"]), w["gu_qt"],
                          dev(w["wd"]), w["d_qt"], dev(w["attn_norm"]), dev(w["ffn_norm"]),
                          dev(w["q_norm"]) if w["q_norm"] is not None else None,
                          dev(w["k_norm"]) if w["k_norm"] is not None else None)
            assert L.tb_cuda_dec_set_layer(self.d, li, ctypes.byref(lw)) == 1
        assert L.tb_cuda_dec_set_head(self.d, dev(m.emb), m.emb_qt, dev(m.out_norm), dev(m.lm), m.lm_qt) == 1

    def load_kv(self, li, which, arr):   # arr [NK][n][HD]
        a = np.ascontiguousarray(arr, dtype=np.float32)
        fp = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        assert self.kq.L.tb_cuda_dec_kv_copy(self.d, li, which, 0, a.shape[1], fp, 1) == 1

    def read_kv(self, li, which, p0, n):
        out = np.zeros((self.m.n_kv_heads, n, self.m.head_dim), dtype=np.float32)
        fp = out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        assert self.kq.L.tb_cuda_dec_kv_copy(self.d, li, which, p0, n, fp, 0) == 1
        return out

    def read(self, which, n):
        out = np.zeros(n, dtype=np.float32)
        assert self.kq.L.tb_cuda_dec_read(self.d, which, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n) == 1
        return out

    def step(self, token, pos):
        nxt = ctypes.c_int(-1)
        logits = np.zeros(self.m.vocab, dtype=np.float32)
        assert self.kq.L.tb_cuda_dec_step(self.d, token, pos, ctypes.byref(nxt),
                                          logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))) == 1
        return logits, nxt.value

    def close(self):
        self.kq.L.tb_cuda_dec_destroy(self.d)


def prefill(m, dec, orc, n, seed=9):
    rng = np.random.default_rng(seed)
    for li in range(m.n_layers):
        for which in (0, 1):
            a = rng.standard_normal((m.n_kv_heads, n, m.head_dim)).astype(np.float32)
            dec.load_kv(li, which, a)
            (orc.kc if which == 0 else orc.vc)[li, :, :n] = a


def check_token(logits_gpu, nxt, logits_ref):
    assert rel_l2(logits_gpu, logits_ref) <= TOL, rel_l2(logits_gpu, logits_ref)
    best = float(np.max(logits_ref))
    scale = float(np.linalg.norm(logits_ref)) / np.sqrt(logits_ref.size)
    assert logits_ref[nxt] >= best - 10 * TOL * scale, (nxt, int(np.argmax(logits_ref)))


@pytest.mark.parametrize("quirks", [True, False])
def test_decode_step_matches_oracle(kq, quirks):
    m = make_model()
    dec, orc = GpuDecoder(kq, m, quirks), DecodeOracle(m, quirks=quirks)
    try:
        pos = 40
        prefill(m, dec, orc, pos)
        lg, nxt = dec.step(17, pos)
        lr, _ = orc.step(17, pos)
        check_token(lg, nxt, lr)
        H, NH, NK, F = m.hidden, m.n_heads, m.n_kv_heads, m.ffn_dim
        assert rel_l2(dec.read(2, (NH + 2 * NK) * 128), orc.last["qkv"]) <= TOL
        assert rel_l2(dec.read(3, NH * 128), orc.last["att"]) <= TOL
        assert rel_l2(dec.read(1, H), orc.last["x2"]) <= TOL
        assert rel_l2(dec.read(4, F), orc.last["act"]) <= TOL
        assert kq.L.tb_cuda_dec_read(dec.d, 6, None, 0) == 0
        for li in range(m.n_layers):   # the rows appended at pos: rotated/normed k, raw v
            assert rel_l2(dec.read_kv(li, 0, pos, 1)[:, 0], orc.kc[li, :, pos]) <= 1e-4
            assert rel_l2(dec.read_kv(li, 1, pos, 1)[:, 0], orc.vc[li, :, pos]) <= 1e-4
    finally:
        dec.close()


@pytest.mark.parametrize("nh,nk", [(32, 8), (28, 4), (32, 4), (12, 4), (4, 4)])
def test_decode_long_context(kq, nh, nk):
    """Chunks of several streamed blocks of cached positions, query heads per
    KV head 4, 7, 8 (the Qwen3-30B-A3B shape), 3 and 1 (padded to 4, 8, 8, 4
    and 1 in the score reduction)."""
    m = make_model(n_layers=1, hidden=256, nh=nh, nk=nk, ffn=256, vocab=300, max_ctx=4736, seed=nh + nk)
    dec, orc = GpuDecoder(kq, m, False), DecodeOracle(m, quirks=False)
    try:
        pos = 4700
        prefill(m, dec, orc, pos, seed=nh)
        lg, nxt = dec.step(5, pos)
        lr, _ = orc.step(5, pos)
        check_token(lg, nxt, lr)
        assert rel_l2(dec.read_kv(0, 0, pos, 1)[:, 0], orc.kc[0, :, pos]) <= 1e-4
        # the attention output itself (the logits barely see it at this context)
        assert rel_l2(dec.read(3, nh * 128), orc.last["att"]) <= TOL
    finally:
        dec.close()


def test_decode_first_token_and_no_qk_norm(kq):
    m = make_model(qk_norm=False, seed=6)
    dec, orc = GpuDecoder(kq, m, True), DecodeOracle(m, quirks=True)
    try:
        lg, nxt = dec.step(3, 0)   # empty cache: attends to itself only
        lr, _ = orc.step(3, 0)
        check_token(lg, nxt, lr)
    finally:
        dec.close()


def test_decode_chain_feeds_back_argmax(kq):
    """Four tokens in a row, each step fed the previous argmax (device-resident)."""
    m = make_model(seed=7)
    dec, orc = GpuDecoder(kq, m, True), DecodeOracle(m, quirks=True)
    try:
        pos0 = 20
        prefill(m, dec, orc, pos0)
        toks = (ctypes.c_int * 4)()
        logits = np.zeros(m.vocab, dtype=np.float32)
        assert kq.L.tb_cuda_dec_generate(dec.d, 11, pos0, 4, toks,
                                         logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), None) == 1
        tok = 11
        for i in range(4):   # the oracle follows the GPU's own tokens
            lr, _ = orc.step(tok, pos0 + i)
            best = float(np.max(lr))
            scale = float(np.linalg.norm(lr)) / np.sqrt(lr.size)
            assert lr[toks[i]] >= best - 10 * TOL * scale
            tok = toks[i]
        assert rel_l2(logits, lr) <= TOL
    finally:
        dec.close()


def _gen_u(kq, dec, token, pos, u, vocab):
    """tb_cuda_dec_generate_u: (tokens, last logits), or None when the call returns 0."""
    u = np.ascontiguousarray(u, dtype=np.float32)
    toks = (ctypes.c_int * u.size)()
    logits = np.zeros(vocab, dtype=np.float32)
    fp = ctypes.POINTER(ctypes.c_float)
    if kq.L.tb_cuda_dec_generate_u(dec.d, token, pos, u.size, u.ctypes.data_as(fp), toks,
                                   logits.ctypes.data_as(fp), None) != 1:
        return None
    return list(toks), logits


def _oracle_pick(logits, temp, k, p, u):
    from oracle.sample_ref import sample_top_k, sample_top_p
    return sample_top_k(logits, k, temp, u) if k > 0 else sample_top_p(logits, p, temp, u)


# (temperature, top_k, top_p): top-k, nucleus, and top-k >= vocab (nucleus 0.95)
SAMPLING = [(0.8, 40, 0.0), (0.7, 0, 0.9), (1.3, 0, 0.5), (0.9, 5000, 0.0)]


@pytest.mark.parametrize("temp,k,p", SAMPLING)
def test_decode_sampled_step_matches_sampler_oracle(kq, temp, k, p):
    """The step's sampler (tb_infer.c:1031-1038) picks what the reference's
    tb_sample_top_k / tb_sample_top_p pick from the step's own logits for the
    same variate; switching from greedy leaves the logits bit-identical."""
    m = make_model(seed=11)
    dec, orc = GpuDecoder(kq, m, True), DecodeOracle(m, quirks=True)
    try:
        pos = 30
        prefill(m, dec, orc, pos)
        lg, _ = dec.step(9, pos)
        assert kq.L.tb_cuda_dec_set_sampling(dec.d, temp, k, p) == 1
        for u in (0.0, 0.13, 0.5, 0.77, 0.999):
            r = _gen_u(kq, dec, 9, pos, [u], m.vocab)
            assert r is not None
            toks, logits = r
            assert np.array_equal(logits, lg)
            assert toks[0] == _oracle_pick(logits, temp, k, p, u), (u, toks[0])
    finally:
        dec.close()


def test_decode_sampled_chain_uses_each_variate(kq):
    """Four sampled steps back to back (one graph replay each) equal four
    single steps fed the same tokens and variates: step i draws u[i] and
    advances the position."""
    m = make_model(seed=12, vocab=600)
    dec, orc = GpuDecoder(kq, m, True), DecodeOracle(m, quirks=True)
    try:
        pos0 = 10
        prefill(m, dec, orc, pos0)
        assert kq.L.tb_cuda_dec_set_sampling(dec.d, 1.5, 0, 0.98) == 1
        u = [0.91, 0.05, 0.42, 0.66]
        chain, last = _gen_u(kq, dec, 4, pos0, u, m.vocab)
        tok = 4
        for i in range(4):
            toks, logits = _gen_u(kq, dec, tok, pos0 + i, [u[i]], m.vocab)
            assert toks[0] == chain[i] == _oracle_pick(logits, 1.5, 0, 0.98, u[i]), (i, toks[0], chain[i])
            tok = toks[0]
        assert np.array_equal(logits, last)
    finally:
        dec.close()


def test_decode_sampling_settings(kq):
    m = make_model(seed=13, n_layers=1)
    dec = GpuDecoder(kq, m, True)
    L = kq.L
    try:
        lg, greedy = dec.step(2, 0)
        assert L.tb_cuda_dec_set_sampling(dec.d, 0.8, 0, 0.0) == 0      # nucleus needs p in (0, 1]
        assert L.tb_cuda_dec_set_sampling(dec.d, 0.8, 0, 1.5) == 0
        assert L.tb_cuda_dec_set_sampling(dec.d, 0.8, 999, 0.0) == 1    # top-k below the vocabulary
        nxt = ctypes.c_int(-1)
        assert L.tb_cuda_dec_step(dec.d, 2, 0, ctypes.byref(nxt), None) == 0   # sampling needs the variates
        assert _gen_u(kq, dec, 2, 0, [1.0], m.vocab) is None                  # u outside [0, 1)
        assert _gen_u(kq, dec, 2, 0, [-0.1], m.vocab) is None
        assert _gen_u(kq, dec, 2, 0, [0.3], m.vocab) is not None
        # temperatures below 0.01 are greedy again, as in the reference
        assert L.tb_cuda_dec_set_sampling(dec.d, 0.005, 40, 0.9) == 1
        lg2, g2 = dec.step(2, 0)
        assert g2 == greedy and np.array_equal(lg2, lg)
        toks, _ = _gen_u(kq, dec, 2, 0, [0.7], m.vocab)                       # u ignored when greedy
        assert toks[0] == greedy
    finally:
        dec.close()


def test_fused_matvec_modes(kq):
    import torch
    rng = np.random.default_rng(3)
    M, K = 300, 1024
    W = synth.weights(Q.Q4_K, M, K, seed=3, tensor=1)
    from oracle.oracle import Oracle
    Wd = Oracle().dequant(Q.Q4_K, W, M, K).astype(np.float64)
    x = rng.standard_normal(K).astype(np.float32)
    x2 = rng.standard_normal(K).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    res = rng.standard_normal(M).astype(np.float32)
    dW, dx, dx2, dnw, dres = (torch.from_numpy(a).cuda() for a in (W, x, x2, nw, res))
    dy = torch.zeros(M, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    xd = x.astype(np.float64)
    cases = [
        (0, None, (Wd @ xd) + res),
        (1, None, Wd @ (xd / np.sqrt(np.mean(xd * xd) + 1e-5) * nw) + res),
        (2, None, Wd @ ((xd / (1 + np.exp(-xd))) * x2) + res),
    ]
    for xmode, _, ref in cases:
        assert kq.tb_cuda_matvec_fused_dev(dW.data_ptr(), Q.Q4_K, M, K, dx.data_ptr(), dy.data_ptr(), xmode,
                                           dx2.data_ptr(), dnw.data_ptr(), 1e-5, dres.data_ptr(), ymode=0,
                                           stream=st) == 1
        torch.cuda.synchronize()
        assert rel_l2(dy.cpu().numpy(), ref) <= 3e-4, xmode
    # (gate, up) row pairs: y[i] = silu(row 2i . x') * (row 2i+1 . x'), RMSNorm input
    xn = xd / np.sqrt(np.mean(xd * xd) + 1e-5) * nw
    ref = (Wd[0::2] @ xn / (1 + np.exp(-(Wd[0::2] @ xn)))) * (Wd[1::2] @ xn)
    dy.zero_()
    assert kq.tb_cuda_matvec_fused_dev(dW.data_ptr(), Q.Q4_K, M, K, dx.data_ptr(), dy.data_ptr(), 1, 0,
                                       dnw.data_ptr(), 1e-5, 0, ymode=1, stream=st) == 1
    torch.cuda.synchronize()
    assert rel_l2(dy.cpu().numpy()[:M // 2], ref) <= 3e-4
    # the pair mode rejects an odd row count and a residual
    assert kq.tb_cuda_matvec_fused_dev(dW.data_ptr(), Q.Q4_K, M - 1, K, dx.data_ptr(), dy.data_ptr(), 0, 0, 0,
                                       0.0, 0, ymode=1, stream=st) == 0
    assert kq.tb_cuda_matvec_fused_dev(dW.data_ptr(), Q.Q4_K, M, K, dx.data_ptr(), dy.data_ptr(), 0, 0, 0,
                                       0.0, dres.data_ptr(), ymode=1, stream=st) == 0
    assert kq.tb_cuda_last_error() == 0
