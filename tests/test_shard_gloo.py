"""Host logic of the multi-GPU path, on CPU: world_size-2 gloo ranks.

Each rank takes its row shard of one tensor with trailblaze_b200.shard and
computes it (here with the oracle, standing in for the device call, which
needs a GPU); the gathered shards must equal the unsharded result bit for
bit, because rows are independent.  The timing reduction must return the
slowest rank's time, and the weak-scaling rate must count every rank's bytes.
"""
import os
import socket
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, qt, M, K, q):
    sys.path.insert(0, REPO)
    import torch
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from trailblaze_b200 import shard, synth
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        W = synth.weights(qt, M, K, seed=5, tensor=qt)
        x = synth.activations(K, seed=5)
        off, nbytes, rows = shard.byte_range(qt, M, K, rank, world)
        y = Oracle().matvec_f64(qt, W[off:off + nbytes], rows, K, x)
        parts = [None] * world
        dist.all_gather_object(parts, (rank, y))
        slow = shard.max_over_ranks(1.0 + rank, dist)
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            full = np.concatenate([p[1] for p in sorted(parts, key=lambda t: t[0])])
            q.put(("ok", full, slow))
    except Exception as e:  # noqa: BLE001
        q.put(("err", repr(e), None))


@pytest.mark.parametrize("qt_name,M,K", [("Q4_K", 37, 512), ("Q6_K", 64, 256), ("Q8_0", 9, 96)])
def test_row_shards_reassemble_exactly(qt_name, M, K):
    import torch.multiprocessing as mp
    from oracle.oracle import Oracle
    from trailblaze_b200 import qtypes as Q
    from trailblaze_b200 import synth
    qt = Q.BY_NAME[qt_name]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, qt, M, K, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
    status, full, slow = q.get(timeout=10)
    assert status == "ok", full
    W = synth.weights(qt, M, K, seed=5, tensor=qt)
    x = synth.activations(K, seed=5)
    want = Oracle().matvec_f64(qt, W, M, K, x)
    assert np.array_equal(full, want)
    assert slow == 2.0


def test_row_ranges_cover_and_align():
    from trailblaze_b200 import qtypes as Q
    from trailblaze_b200 import shard
    for M in (1, 7, 151936, 9728):
        for world in (1, 2, 3, 4, 8):
            cut = [shard.row_range(M, r, world) for r in range(world)]
            assert cut[0][0] == 0 and cut[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(cut, cut[1:]))
            assert max(h - l for l, h in cut) - min(h - l for l, h in cut) <= 1
    off, n, rows = shard.byte_range(Q.Q6_K, 10, 512, 1, 2)
    assert (off, n, rows) == (5 * 420, 5 * 420, 5)
    assert shard.weak_rows(1024, 3) == (3072, 4096)
    assert shard.whole_job_rate(100, 4, 2.0) == 200.0
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)
