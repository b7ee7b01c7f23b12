"""Multi-GPU decode against the single-GPU decode of the same model.

Tensor-parallel dense decode (tb_cuda_dec_create_tp) and expert-parallel routed
decode (tb_cuda_dec_create_moe_tp) at 2 and 4 ranks, one process per GPU, each
rank holding its share of one seeded model (trailblaze_b200.decoder.
synthetic_model cuts the shares from the whole tensors).  Rank 0 also decodes
the whole model on its own GPU with the single-device decoder, which the
single-GPU tests check against the numpy oracle.  Checks: every rank takes the
same tokens, equal to the single-device tokens, and the gathered logits of the
last step match (1e-4 relative L2; only the rounding order of the partial sums
differs), greedy and sampled (each rank gathers the whole vocabulary and samples
it with the same variate).  At 4 ranks the 2 kv heads are each held by two ranks.

Failure detection: after a joint step one rank skips the next step while
staying alive (it would free the memory its peers store into if it exited);
the other rank's bounded waits run out (the decoder's error word 1), its step
returns 0, and a plain matvec afterwards still works.  No GPU fault is
involved: the missing contributions are made on the host.

Skipped with fewer GPUs than ranks."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _shape(kind):
    from trailblaze_b200 import qtypes as Q
    from trailblaze_b200.decoder import ModelShape
    if kind.startswith("dense"):
        return ModelShape(2, 512, 8, 2, 128, 1024, 1024)
    return ModelShape(2, 512, 8, 2, 128, 256, 1024, w_qt=Q.Q4_K, out_qt=Q.Q6_K, n_experts=16, top_k=4,
                      attn_qt=Q.Q6_K)


CTX, NTOK = 48, 6


def _worker(rank, world, port, q, kind, fail):
    import datetime

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    dec = None
    try:
        from trailblaze_b200 import load, qtypes as Q, synth
        from trailblaze_b200.decoder import synthetic_model
        kq = load()
        assert kq.tb_cuda_init() == 1
        shape = _shape(kind)
        dec = synthetic_model(shape, max_ctx=CTX + 2 * NTOK + 8, ctx=CTX, rank=rank, world=world)
        hs = [None] * world
        dist.all_gather_object(hs, dec.tp_handle())
        dec.tp_connect(hs)
        dist.barrier()
        if fail:
            t1 = dec.step(1, CTX)             # a joint step
            dist.barrier()
            res = None
            if rank == 0:                     # rank 1 skips this step
                try:
                    dec.step(t1, CTX + 1)
                    res = ("step returned 1",)
                except RuntimeError:
                    # the context stays usable: a plain matvec after the failed step
                    W = synth.weights(Q.Q4_K, 64, 512, seed=3)
                    dW = torch.from_numpy(W).cuda()
                    dx = torch.from_numpy(synth.activations(512, seed=3)).cuda()
                    dy = torch.empty(64, device="cuda")
                    torch.cuda.synchronize()
                    ok = kq.tb_cuda_matvec_dev(dW.data_ptr(), Q.Q4_K, 64, 512, dx.data_ptr(), dy.data_ptr(), 0)
                    torch.cuda.synchronize()
                    res = ("failed", ok, kq.tb_cuda_last_error(), bool(torch.isfinite(dy).all()))
            dist.barrier()                    # rank 1 leaves only now: nothing of rank 0 is in flight
            q.put((rank, res))
            return
        lg = np.zeros(shape.vocab // world, dtype=np.float32)
        smp = kind.endswith("_topk") or kind.endswith("_nucleus")
        u = np.random.default_rng(11).random(NTOK).astype(np.float32)   # the same variates on every rank

        def run(d, logits):
            if not smp:
                return d.generate(1, CTX, NTOK, want_tokens=True, logits=logits)[0]
            d.set_sampling(0.8, 40 if kind.endswith("_topk") else 0, 0.9)
            return d.generate_u(1, CTX, u, logits=logits)[0]

        toks = run(dec, lg)
        parts = [None] * world
        dist.all_gather_object(parts, lg)
        out = (rank, toks, np.concatenate(parts) if rank == 0 else None)
        dist.barrier()
        dec.close()
        dec = None
        if rank == 0:
            one = synthetic_model(shape, max_ctx=CTX + 2 * NTOK + 8, ctx=CTX)
            lg1 = np.zeros(shape.vocab, dtype=np.float32)
            toks1 = run(one, lg1)
            one.close()
            out = out + (toks1, lg1)
        q.put(out)
    except Exception as e:   # the parent asserts on what arrives
        q.put((rank, "error", repr(e)))
        raise
    finally:
        if dec is not None:
            dist.barrier()
            dec.close()
        dist.destroy_process_group()


def _run(world, kind, port, fail=False):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, kind, fail)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=600) for _ in range(world)], key=lambda t: t[0])
    for p in ps:
        p.join(timeout=120)
    for r in res:
        assert r[1] != "error", r
    for p in ps:
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("kind", ["dense", "moe", "dense_topk", "moe_nucleus"])
def test_parallel_decode_matches_one_gpu(world, kind):
    """Greedy, and sampled (top-k 40 / nucleus 0.9 at temperature 0.8, the same
    variates on every rank and on the single device)."""
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    res = _run(world, kind, 29700 + 10 * world + ["dense", "moe", "dense_topk", "moe_nucleus"].index(kind))
    toks = res[0][1]
    assert all(r[1] == toks for r in res)          # every rank takes the same tokens
    _, _, lg, toks1, lg1 = res[0]
    assert toks == toks1
    e = float(np.linalg.norm(lg.astype(np.float64) - lg1) / np.linalg.norm(lg1))
    assert e <= TOL, e


def test_rank_that_skips_a_step_makes_the_peer_wait_time_out():
    if _ngpu() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(2, "dense", 29790, fail=True)
    r0 = res[0][1]
    assert r0[0] == "failed", r0   # the step returned 0: a bounded wait for the missing rank ran out
    _, ok, err, finite = r0
    assert ok == 1 and err == 0 and finite
