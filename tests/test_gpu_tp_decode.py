"""Tensor-parallel decode on two GPUs (tb_cuda_dec_create_tp / _tp_handle /
_tp_connect) against the whole-model numpy oracle (oracle/decode_ref.py).

Two processes, one per GPU, each hold their shard of the same model
(trailblaze_b200.shard.tp_layer); they exchange CUDA IPC handles through a
gloo process group and then run the decode step, whose o / down partials and
greedy pairs cross NVLink by peer stores.  Checks: the same token on both
ranks, equal to the oracle's argmax within the logits' tolerance; each rank's
logits equal the oracle's vocabulary slice and its attention output the
oracle's heads (1e-3 relative L2); the appended cache rows of its kv heads;
a chain of steps keeps the exchange counters in step.  Skipped with fewer
than two GPUs."""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3
WORLD = 2
SHAPE = dict(n_layers=2, hidden=512, nh=8, nk=2, ffn=1024, vocab=1000, max_ctx=96, seed=21)


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _model():
    from test_gpu_decode import make_model
    return make_model(**SHAPE)


def _prefill(m, n, seed=9):
    """[layer][which] -> [NK][n][HD] fp32, the same on every rank."""
    rng = np.random.default_rng(seed)
    return [[rng.standard_normal((m.n_kv_heads, n, m.head_dim)).astype(np.float32) for _ in (0, 1)]
            for _ in range(m.n_layers)]


def _rank_main(rank, port, out, pos, token, chain):
    import datetime

    import torch
    import torch.distributed as dist
    from trailblaze_b200 import load, shard
    from trailblaze_b200._lib import DecConfig, DecLayer
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=120))
    dec, kq = None, None
    try:
        kq = load()
        assert kq.tb_cuda_init() == 1
        L = kq.L
        m = _model()
        H, NH, NK, HD, F, V = m.hidden, m.n_heads, m.n_kv_heads, m.head_dim, m.ffn_dim, m.vocab
        cfg = DecConfig(m.n_layers, H, NH, NK, HD, F, V, m.max_ctx, m.rope_base, m.norm_eps, 1)
        dec = L.tb_cuda_dec_create_tp(ctypes.byref(cfg), rank, WORLD)
        assert dec
        keep = []

        def dev(a):
            t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
            keep.append(t)
            return t.data_ptr()

        for li, w in enumerate(m.layers):
            s = shard.tp_layer(w, H, NH, NK, HD, F, rank, WORLD)
            lw = DecLayer(dev(s["wqkv"]), s["qkv_qt"], dev(s["wo"]), s["o_qt"], dev(s["wgu"]), s["gu_qt"],
                          dev(s["wd"]), s["d_qt"], dev(w["attn_norm"]), dev(w["ffn_norm"]),
                          dev(w["q_norm"]), dev(w["k_norm"]))
            assert L.tb_cuda_dec_set_layer(dec, li, ctypes.byref(lw)) == 1
        vl = V // WORLD
        lm = shard.row_slice(m.lm, m.lm_qt, V, H, rank * vl, (rank + 1) * vl)
        assert L.tb_cuda_dec_set_head(dec, dev(m.emb), m.emb_qt, dev(m.out_norm), dev(lm), m.lm_qt) == 1
        nk = NK // WORLD
        for li, pair in enumerate(_prefill(m, pos)):
            for which, a in enumerate(pair):
                loc = np.ascontiguousarray(a[rank * nk:(rank + 1) * nk])
                assert L.tb_cuda_dec_kv_copy(dec, li, which, 0, pos, loc.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                             1) == 1
        h = (ctypes.c_ubyte * 64)()
        assert L.tb_cuda_dec_tp_handle(dec, h) == 1
        hs = [None] * WORLD
        dist.all_gather_object(hs, bytes(h))
        allh = (ctypes.c_ubyte * (64 * WORLD)).from_buffer_copy(b"".join(hs))
        assert L.tb_cuda_dec_tp_connect(dec, allh) == 1
        dist.barrier()
        nxt = ctypes.c_int(-1)
        logits = np.zeros(vl, dtype=np.float32)
        ok = L.tb_cuda_dec_step(dec, token, pos, ctypes.byref(nxt), logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        att = np.zeros(NH // WORLD * HD, dtype=np.float32)
        L.tb_cuda_dec_read(dec, 3, att.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), att.size)
        krow = np.zeros((nk, 1, HD), dtype=np.float32)
        L.tb_cuda_dec_kv_copy(dec, m.n_layers - 1, 0, pos, 1, krow.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 0)
        dist.barrier()
        toks = (ctypes.c_int * chain)()
        last = np.zeros(vl, dtype=np.float32)
        ok2 = L.tb_cuda_dec_generate(dec, nxt.value, pos + 1, chain, toks,
                                     last.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), None)
        out.put((rank, int(ok), nxt.value, logits, att, krow[:, 0], int(ok2), list(toks), last))
    except Exception as e:   # the parent asserts on what arrives
        out.put((rank, -1, repr(e)))
        raise
    finally:
        if dec and kq:
            kq.L.tb_cuda_dec_destroy(dec)
        dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < WORLD, reason="needs two GPUs")
def test_tp2_decode_matches_whole_model():
    import torch.multiprocessing as mp
    from oracle.decode_ref import DecodeOracle
    from test_gpu_decode import check_token, rel_l2
    pos, token, chain = 40, 17, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_main, args=(r, 29651, q, pos, token, chain)) for r in range(WORLD)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(WORLD)], key=lambda t: t[0])
    for p in ps:
        p.join(timeout=120)
    for r in res:
        assert r[1] == 1, r
    for p in ps:
        assert p.exitcode == 0
    m = _model()
    orc = DecodeOracle(m, quirks=True)
    for li, pair in enumerate(_prefill(m, pos)):
        orc.kc[li, :, :pos] = pair[0]
        orc.vc[li, :, :pos] = pair[1]
    lr, _ = orc.step(token, pos)
    nxt = res[0][2]
    assert all(r[2] == nxt for r in res)   # every rank takes the same token
    logits = np.concatenate([r[3] for r in res])
    check_token(logits, nxt, lr)
    nh, nk, HD = m.n_heads // WORLD, m.n_kv_heads // WORLD, m.head_dim
    att = orc.last["att"]
    for r in res:
        rk = r[0]
        assert rel_l2(r[4], att[rk * nh * HD:(rk + 1) * nh * HD]) <= TOL
        assert rel_l2(r[5], orc.kc[m.n_layers - 1, rk * nk:(rk + 1) * nk, pos]) <= 1e-4
    # the chain: the oracle follows the GPU's own tokens
    assert all(r[6] == 1 for r in res)
    assert all(r[7] == res[0][7] for r in res)
    tok = nxt
    for i in range(chain):
        lr, _ = orc.step(tok, pos + 1 + i)
        best = float(np.max(lr))
        scale = float(np.linalg.norm(lr)) / np.sqrt(lr.size)
        assert lr[res[0][7][i]] >= best - 10 * TOL * scale
        tok = res[0][7][i]
    assert rel_l2(np.concatenate([r[8] for r in res]), lr) <= TOL
