"""Multi-GPU host logic: token sharding, column-parallel output gather, timing.

The projection path shards by token rows with no collective: per-token
scales and row statistics never leave a row, weights are replicated, so each
rank quantizes and multiplies its own contiguous block of rows.  The optional
column-parallel variant (FFN-up: each rank holds N/g output channels of W)
ends with one all-gather of the BF16 output shards.

All functions take an optional process group and work with any
torch.distributed backend (NCCL over NVLink on the GPU box, gloo in tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) rows of rank `rank`; sizes differ by at most one
    (the first m % world ranks hold one extra row), e.g. 9914 rows on 8 ranks
    -> 1240 x 2 then 1239 x 6."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if m < 0:
        raise ValueError("m must be non-negative")
    base, extra = divmod(m, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_columns(n: int, world: int, rank: int) -> tuple[int, int]:
    """Equal [start, stop) output-channel shard for the column-parallel variant."""
    if n % world:
        raise ValueError("N must be divisible by the number of ranks for column sharding")
    step = n // world
    return rank * step, (rank + 1) * step


def gather_columns(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """[M, N/g] shards of every rank -> [M, N] (rank r's shard at columns r*N/g).

    One all_gather_into_tensor into a [g, M, N/g] buffer, then a permute; the
    receive buffer is laid out so the collective writes each shard
    contiguously.
    """
    m, ns = local.shape
    recv = torch.empty((world * m, ns), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, local.contiguous(), group=group)
    return recv.view(world, m, ns).permute(1, 0, 2).reshape(m, world * ns)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Maximum of a per-rank scalar (e.g. a timed region in ms) over the group."""
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
