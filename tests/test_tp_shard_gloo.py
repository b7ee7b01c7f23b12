"""Tensor-parallel shards of a decode layer (trailblaze_b200.shard.tp_layer,
k_slice, row_slice) on CPU, with world-size-2 gloo ranks: each rank's K-slice
matvec partial, summed by an all-reduce, reproduces the whole matvec, and the
row shards concatenate to the whole output.  The partial sums are what the
library's tensor-parallel decoder exchanges over NVLink."""
import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from trailblaze_b200 import qtypes as Q, shard, synth


def _deq(qt, W, M, K):
    from oracle.oracle import Oracle
    return Oracle().dequant(qt, W, M, K).astype(np.float64)


def test_k_slice_and_row_slice_on_block_boundaries():
    M, K = 6, 1024
    W = synth.weights(Q.Q6_K, M, K, seed=1, tensor=1)
    full = _deq(Q.Q6_K, W, M, K)
    assert np.array_equal(_deq(Q.Q6_K, np.ascontiguousarray(shard.k_slice(W, Q.Q6_K, M, K, 256, 768)), M, 512),
                          full[:, 256:768])
    assert np.array_equal(_deq(Q.Q6_K, shard.row_slice(W, Q.Q6_K, M, K, 2, 5), 3, K), full[2:5])
    with pytest.raises(ValueError):
        shard.k_slice(W, Q.Q6_K, M, K, 100, 512)


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, NH, NK, HD, F = 512, 8, 2, 128, 1024
        t = 0

        def W(qt, M, K):
            nonlocal t
            t += 1
            return synth.weights(qt, M, K, seed=11, tensor=t)

        w = dict(wqkv=W(Q.Q4_K, (NH + 2 * NK) * HD, H), qkv_qt=Q.Q4_K, wo=W(Q.Q4_K, H, NH * HD), o_qt=Q.Q4_K,
                 wgu=W(Q.Q4_K, 2 * F, H), gu_qt=Q.Q4_K, wd=W(Q.Q6_K, H, F), d_qt=Q.Q6_K)
        s = shard.tp_layer(w, H, NH, NK, HD, F, rank, world)
        rng = np.random.default_rng(3)
        att = rng.standard_normal(NH * HD)
        act = rng.standard_normal(F)
        nh, f = NH // world, F // world
        # K-sharded o and down: partials summed across ranks
        po = _deq(Q.Q4_K, s["wo"], H, nh * HD) @ att[rank * nh * HD:(rank + 1) * nh * HD]
        pd = _deq(Q.Q6_K, s["wd"], H, f) @ act[rank * f:(rank + 1) * f]
        to, td = torch.from_numpy(po), torch.from_numpy(pd)
        dist.all_reduce(to)
        dist.all_reduce(td)
        # row-sharded qkv (q rows of this rank's heads first) and gate/up pairs
        x = rng.standard_normal(H)
        qkv = _deq(Q.Q4_K, s["wqkv"], (nh + 2 * (NK // world)) * HD, H) @ x
        gu = _deq(Q.Q4_K, s["wgu"], 2 * f, H) @ x
        out.put((rank, to.numpy(), td.numpy(), qkv, gu))
    finally:
        dist.destroy_process_group()


def test_tp_partials_sum_to_whole_layer_gloo():
    world, port = 2, 29641
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda t: t[0])
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    H, NH, NK, HD, F = 512, 8, 2, 128, 1024
    t = 0

    def W(qt, M, K):
        nonlocal t
        t += 1
        return synth.weights(qt, M, K, seed=11, tensor=t)

    wqkv, wo, wgu, wd = W(Q.Q4_K, (NH + 2 * NK) * HD, H), W(Q.Q4_K, H, NH * HD), W(Q.Q4_K, 2 * F, H), W(Q.Q6_K, H, F)
    rng = np.random.default_rng(3)
    att, act, x = rng.standard_normal(NH * HD), rng.standard_normal(F), rng.standard_normal(H)
    o_full = _deq(Q.Q4_K, wo, H, NH * HD) @ att
    d_full = _deq(Q.Q6_K, wd, H, F) @ act
    for _, o, d, _, _ in res:   # every rank holds the same reduced vector
        assert np.allclose(o, o_full, rtol=1e-12, atol=1e-9)
        assert np.allclose(d, d_full, rtol=1e-12, atol=1e-9)
    qkv_full = _deq(Q.Q4_K, wqkv, (NH + 2 * NK) * HD, H) @ x
    nh, nk = NH // world, NK // world
    q = np.concatenate([r[3][:nh * HD] for r in res])
    k = np.concatenate([r[3][nh * HD:(nh + nk) * HD] for r in res])
    v = np.concatenate([r[3][(nh + nk) * HD:] for r in res])
    assert np.allclose(np.concatenate([q, k, v]), qkv_full, rtol=1e-12, atol=1e-9)
    gu_full = _deq(Q.Q4_K, wgu, 2 * F, H) @ x
    assert np.allclose(np.concatenate([r[4] for r in res]), gu_full, rtol=1e-12, atol=1e-9)
