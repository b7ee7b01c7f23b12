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
