"""Row sharding of a quantized matvec across ranks (one process per GPU).

Rows of y = dequant(W) @ x are independent, so a tensor is split into
contiguous row ranges, one per rank, and each rank runs the library's matvec
on its own range; no data crosses between ranks.  Every range starts on a row
boundary, which is a block boundary of the GGUF layout (a row is exactly
K / block_weights whole blocks), so a shard is a plain byte range of the
tensor: `W_dev + lo * row_bytes`.

This is the partition the reference's MoE expert slicing already uses for one
expert (tb_infer.c:793-827: a row offset times the row bytes into a packed
tensor); here it is applied per rank.
"""
from __future__ import annotations

from . import qtypes as Q


def row_range(M: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) rows of an M-row tensor owned by `rank` of `world` (balanced, contiguous)."""
    if world < 1 or not 0 <= rank < world or M < 0:
        raise ValueError(f"bad shard request M={M} rank={rank} world={world}")
    return (M * rank) // world, (M * (rank + 1)) // world


def byte_range(qtype: int, M: int, K: int, rank: int, world: int) -> tuple[int, int, int]:
    """(byte offset, byte length, rows) of the rank's shard of an M x K tensor."""
    lo, hi = row_range(M, rank, world)
    rb = Q.row_bytes(qtype, K)
    return lo * rb, (hi - lo) * rb, hi - lo


def weak_rows(M_per_rank: int, rank: int) -> tuple[int, int]:
    """Weak scaling: rank r owns rows [r*M, (r+1)*M) of a world*M-row tensor."""
    return rank * M_per_rank, (rank + 1) * M_per_rank


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The largest `value` across ranks (elapsed times are reported as the slowest rank's)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(bytes_per_rank: int, world: int, seconds_max: float) -> float:
    """Aggregate bytes/s of a weak-scaling job: all ranks' bytes over the slowest rank's time."""
    return world * bytes_per_rank / seconds_max


# ---------------------------------------------------------------------------
# Tensor-parallel decode shards (one rank's share of a dense layer)
# ---------------------------------------------------------------------------

def k_slice(W, qtype: int, M: int, K: int, k_lo: int, k_hi: int):
    """Columns [k_lo, k_hi) of an M x K GGUF tensor as its own M x (k_hi - k_lo)
    tensor (numpy uint8 or torch uint8, flat).  The bounds must fall on block
    boundaries; each row's blocks in that range are contiguous bytes, so the
    slice is a strided byte copy."""
    bw, bb = Q.geometry(qtype)
    if k_lo % bw or k_hi % bw or not 0 <= k_lo < k_hi <= K:
        raise ValueError(f"K slice [{k_lo}, {k_hi}) is not on {bw}-weight block boundaries of K={K}")
    rb = Q.row_bytes(qtype, K)
    rows = W.reshape(M, rb)
    return rows[:, (k_lo // bw) * bb:(k_hi // bw) * bb].reshape(-1)


def row_slice(W, qtype: int, M: int, K: int, r_lo: int, r_hi: int):
    """Rows [r_lo, r_hi) of an M x K GGUF tensor (a plain byte range)."""
    rb = Q.row_bytes(qtype, K)
    return W.reshape(M, rb)[r_lo:r_hi].reshape(-1)


def tp_layer(w: dict, H: int, NH: int, NK: int, HD: int, F: int, rank: int, world: int) -> dict:
    """Rank `rank`'s share of one dense layer for the library's tensor-parallel
    decoder (tb_cuda_dec_create_tp): q, k and v rows of its heads, o's K
    columns of its q heads, its (gate, up) row pairs, down's K columns of its
    FFN rows.  w holds the whole layer as flat uint8 GGUF bytes with the keys
    wqkv/qkv_qt, wo/o_qt, wgu/gu_qt, wd/d_qt (gate/up rows interleaved)."""
    import numpy as np
    nh, nk, f = NH // world, NK // world, F // world
    qt = w["qkv_qt"]
    qkv = np.concatenate([
        row_slice(w["wqkv"], qt, (NH + 2 * NK) * HD, H, rank * nh * HD, (rank + 1) * nh * HD),
        row_slice(w["wqkv"], qt, (NH + 2 * NK) * HD, H, (NH + rank * nk) * HD, (NH + (rank + 1) * nk) * HD),
        row_slice(w["wqkv"], qt, (NH + 2 * NK) * HD, H, (NH + NK + rank * nk) * HD, (NH + NK + (rank + 1) * nk) * HD),
    ])
    out = dict(w)
    out["wqkv"] = qkv
    out["wo"] = np.ascontiguousarray(k_slice(w["wo"], w["o_qt"], H, NH * HD, rank * nh * HD, (rank + 1) * nh * HD))
    out["wgu"] = row_slice(w["wgu"], w["gu_qt"], 2 * F, H, 2 * rank * f, 2 * (rank + 1) * f)
    out["wd"] = np.ascontiguousarray(k_slice(w["wd"], w["d_qt"], H, F, rank * f, (rank + 1) * f))
    return out
