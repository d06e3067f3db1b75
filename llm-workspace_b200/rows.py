"""Row split of a batch over the ranks of one node (one process per GPU).

Rows of a batch are independent draws (sampling.rs:39 runs once per row), so a
batch of world * rows_per_rank rows is split into contiguous row blocks, one
per rank, with no collective on the data path: each rank samples its own
block on its own GPU.  The only collective is the timing reduction, the
maximum over ranks of each rank's device time.
"""
from __future__ import annotations


def rank_rows(rank: int, world: int, rows_per_rank: int) -> range:
    """Rows of the global batch that rank `rank` of `world` samples."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return range(rank * rows_per_rank, (rank + 1) * rows_per_rank)


def max_over_ranks(value: float, device=None) -> float:
    """The maximum of `value` over the ranks of the default process group
    (the value itself when no group is initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
