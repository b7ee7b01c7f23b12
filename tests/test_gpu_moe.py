"""GPU parity of the mixture-of-experts path against the oracle.

- tb_cuda_matvec_experts_dev: the selected experts of a packed expert tensor
  in one launch, ids read on the device, against the fp64 oracle matvec of the
  same expert's rows (1e-3 relative L2, the matvec bar); shared and per-expert
  x, SwiGLU row pairs, and an id out of range (error word 2, nothing written).
- tb_cuda_dec_create_moe / _set_moe_layer: a routed decode step against the
  numpy restatement of tb_layer_forward's MoE branch (oracle/decode_ref.py):
  the router logits, the selected experts and their weights, their SwiGLU
  activations, the logits and the greedy token, then a chain of steps.
"""
import ctypes

import numpy as np
import pytest

from oracle.decode_ref import DecodeModel, DecodeOracle
from oracle.oracle import Oracle
from trailblaze_b200 import qtypes as Q, synth
from trailblaze_b200._lib import DecConfig, DecLayer

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("qt,M,K,ymode,per_x", [
    (Q.Q4_K, 256, 512, 0, False), (Q.Q4_K, 512, 768, 1, False), (Q.Q6_K, 384, 256, 0, True),
    (Q.Q4_K, 1024, 256, 0, True), (Q.Q8_0, 128, 512, 0, True)])
def test_expert_matvec_matches_oracle(kq, qt, M, K, ymode, per_x):
    import torch
    E, ids = 8, [5, 0, 7, 2]
    n = len(ids)
    W = synth.weights(qt, E * M, K, seed=31, tensor=qt)
    rb = Q.matrix_bytes(qt, M, K)
    xs = np.stack([synth.activations(K, seed=40 + g) for g in range(n if per_x else 1)])
    out = M // 2 if ymode == 1 else M
    dW = torch.from_numpy(W).cuda()
    dx = torch.from_numpy(xs.reshape(-1)).cuda()
    dids = torch.tensor(ids, dtype=torch.int32, device="cuda")
    dy = torch.full((n * out,), float("nan"), device="cuda")
    assert kq.tb_cuda_matvec_experts_dev(dW.data_ptr(), qt, M, K, E, dids.data_ptr(), n, dx.data_ptr(),
                                         K if per_x else 0, dy.data_ptr(), out, ymode) == 1
    torch.cuda.synchronize()
    assert kq.L.tb_cuda_last_error() == 0
    y = dy.cpu().numpy().reshape(n, out)
    o = Oracle()
    for g, e in enumerate(ids):
        ref = o.matvec_f64(qt, W[e * rb:(e + 1) * rb], M, K, xs[g if per_x else 0])
        if ymode == 1:
            gt, up = ref[0::2], ref[1::2]
            ref = (gt / (1.0 + np.exp(-gt))) * up
        assert rel_l2(y[g], ref) <= TOL, (g, e, rel_l2(y[g], ref))


def test_expert_matvec_bad_id_sets_error(kq):
    import torch
    qt, E, M, K = Q.Q4_K, 4, 256, 256
    W = torch.from_numpy(synth.weights(qt, E * M, K, seed=3, tensor=1)).cuda()
    x = torch.from_numpy(synth.activations(K, seed=4)).cuda()
    dids = torch.tensor([1, E + 3], dtype=torch.int32, device="cuda")
    dy = torch.full((2 * M,), 7.0, device="cuda")
    assert kq.tb_cuda_matvec_experts_dev(W.data_ptr(), qt, M, K, E, dids.data_ptr(), 2, x.data_ptr(), 0,
                                         dy.data_ptr(), M, 0) == 1
    torch.cuda.synchronize()
    assert kq.L.tb_cuda_last_error() == 2
    y = dy.cpu().numpy()
    assert np.all(y[M:] == 7.0)            # the bad expert's outputs are untouched
    assert np.all(np.isfinite(y[:M]))      # the good one ran
    assert kq.L.tb_cuda_last_error() == 0  # read once, then cleared
    # argument checks on the host
    assert kq.tb_cuda_matvec_experts_dev(W.data_ptr(), qt, M, K + 1, E, dids.data_ptr(), 2, x.data_ptr(), 0,
                                         dy.data_ptr(), M, 0) == 0
    assert kq.tb_cuda_matvec_experts_dev(W.data_ptr(), qt, M, K, E, dids.data_ptr(), 2, x.data_ptr(), 0,
                                         dy.data_ptr(), M - 1, 0) == 0


def make_moe_model(n_layers=2, hidden=512, nh=8, nk=2, ffn=256, n_exp=16, top_k=4, vocab=1000, max_ctx=96,
                   seed=8):
    rng = np.random.default_rng(seed)
    HD = 128
    m = DecodeModel(n_layers, hidden, nh, nk, HD, ffn, vocab, max_ctx, rope_base=1e6, norm_eps=1e-6,
                    n_experts=n_exp, top_k=top_k)
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
            wqkv=W(Q.Q6_K, (nh + 2 * nk) * HD, hidden), qkv_qt=Q.Q6_K,
            wo=W(Q.Q6_K, hidden, nh * HD), o_qt=Q.Q6_K,
            wr=W(Q.F32, n_exp, hidden), r_qt=Q.F32,
            wgu_e=W(Q.Q4_K, n_exp * 2 * ffn, hidden), gue_qt=Q.Q4_K,
            wd_e=W(Q.Q4_K, n_exp * hidden, ffn), de_qt=Q.Q4_K,
            attn_norm=norm(hidden), ffn_norm=norm(hidden), q_norm=norm(HD), k_norm=norm(HD)))
    return m


class GpuMoeDecoder:
    def __init__(self, kq, m: DecodeModel, quirks: bool = True):
        import torch
        self.kq, self.m, self.keep = kq, m, []
        L = kq.L
        cfg = DecConfig(m.n_layers, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim, m.vocab,
                        m.max_ctx, m.rope_base, m.norm_eps, 1 if quirks else 0)
        self.d = L.tb_cuda_dec_create_moe(ctypes.byref(cfg), m.n_experts, m.top_k)
        assert self.d

        def dev(a):
            t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
            self.keep.append(t)
            return t.data_ptr()

        for li, w in enumerate(m.layers):
            lw = DecLayer(dev(w["wqkv"]), w["qkv_qt"], dev(w["wo"]), w["o_qt"], None, 0, None, 0,
                          dev(w["attn_norm"]), dev(w["ffn_norm"]), dev(w["q_norm"]), dev(w["k_norm"]))
            assert L.tb_cuda_dec_set_layer(self.d, li, ctypes.byref(lw)) == 1
            assert L.tb_cuda_dec_set_moe_layer(self.d, li, dev(w["wr"]), w["r_qt"], dev(w["wgu_e"]), w["gue_qt"],
                                               dev(w["wd_e"]), w["de_qt"]) == 1
        assert L.tb_cuda_dec_set_head(self.d, dev(m.emb), m.emb_qt, dev(m.out_norm), dev(m.lm), m.lm_qt) == 1

    def load_kv(self, li, which, arr):
        a = np.ascontiguousarray(arr, dtype=np.float32)
        assert self.kq.L.tb_cuda_dec_kv_copy(self.d, li, which, 0, a.shape[1],
                                             a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 1) == 1

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


def test_moe_decode_matches_oracle(kq):
    from test_gpu_decode import check_token
    m = make_moe_model()
    dec, orc = GpuMoeDecoder(kq, m), DecodeOracle(m, quirks=True)
    try:
        pos = 30
        rng = np.random.default_rng(9)
        for li in range(m.n_layers):
            for which in (0, 1):
                a = rng.standard_normal((m.n_kv_heads, pos, m.head_dim)).astype(np.float32)
                dec.load_kv(li, which, a)
                (orc.kc if which == 0 else orc.vc)[li, :, :pos] = a
        lg, nxt = dec.step(17, pos)
        lr, _ = orc.step(17, pos)
        E, k, F = m.n_experts, m.top_k, m.ffn_dim
        last = orc.last
        assert rel_l2(dec.read(6, E), last["router"]) <= TOL
        ids = dec.read(8, k).view(np.int32)
        wts = dec.read(7, k)
        # the same experts; the GPU lists them by probability, the reference in scan order
        order = sorted(range(k), key=lambda i: (-last["wts"][i], last["ids"][i]))
        assert list(ids) == [last["ids"][i] for i in order], (ids, last["ids"], last["wts"])
        # weights: softmax of logits that carry the matvec's error (a few 1e-5 of their scale)
        assert np.allclose(wts, [last["wts"][i] for i in order], rtol=1e-3, atol=1e-6)
        acts = dec.read(9, k * F).reshape(k, F)
        for r, i in enumerate(order):
            assert rel_l2(acts[r], last["acts"][i]) <= TOL
        check_token(lg, nxt, lr)
        # a chain: the oracle follows the GPU's tokens
        tok = nxt
        for i in range(3):
            lg, nxt = dec.step(tok, pos + 1 + i)
            lr, _ = orc.step(tok, pos + 1 + i)
            check_token(lg, nxt, lr)
            tok = nxt
    finally:
        dec.close()


def test_moe_decoder_rejects_bad_setup(kq):
    m = make_moe_model(n_layers=1)
    cfg = DecConfig(m.n_layers, m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim, m.vocab, m.max_ctx,
                    m.rope_base, m.norm_eps, 1)
    L = kq.L
    assert not L.tb_cuda_dec_create_moe(ctypes.byref(cfg), 300, 8)     # more experts than the router kernel holds
    assert not L.tb_cuda_dec_create_moe(ctypes.byref(cfg), 16, 17)     # top_k > n_experts
    d = L.tb_cuda_dec_create(ctypes.byref(cfg))                        # a dense decoder takes no expert tensors
    assert d
    try:
        assert L.tb_cuda_dec_set_moe_layer(d, 0, ctypes.c_void_p(16), 0, ctypes.c_void_p(16), 12,
                                           ctypes.c_void_p(16), 12) == 0
    finally:
        L.tb_cuda_dec_destroy(d)
    d = L.tb_cuda_dec_create_moe(ctypes.byref(cfg), 16, 4)
    assert d
    try:   # a step before the experts are set is refused on the host
        nxt = ctypes.c_int(-1)
        assert L.tb_cuda_dec_step(d, 1, 0, ctypes.byref(nxt), None) == 0
    finally:
        L.tb_cuda_dec_destroy(d)
