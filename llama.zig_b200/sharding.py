"""Batch sharding across ranks (one process per GPU).

Rows are independent samplers, so a batch of ``world * rows_per_rank`` rows
splits into contiguous per-rank blocks with no exchange on the data path:
rank g samples global rows ``[g * rows_per_rank, (g + 1) * rows_per_rank)``,
each row seeded by its *global* index (``seed + global_row``, as a single
process holding the whole batch would seed it), so the tokens do not depend
on the number of ranks.  The only collective is the timing reduction (the
slowest rank's device time, taken outside the timed region).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class RowShard:
    rank: int
    world: int
    rows_per_rank: int

    @property
    def row0(self) -> int:
        """First global row of this rank."""
        return self.rank * self.rows_per_rank

    @property
    def global_rows(self) -> int:
        return self.world * self.rows_per_rank

    def rows(self) -> range:
        return range(self.row0, self.row0 + self.rows_per_rank)

    def seeds(self, base_seed: int) -> np.ndarray:
        """Per-row sampler seeds keyed by the global row (seed + row)."""
        return (np.arange(self.row0, self.row0 + self.rows_per_rank, dtype=np.uint64)
                + np.uint64(base_seed)).astype(np.uint64)


def shard_for(rank: int, world: int, rows_per_rank: int) -> RowShard:
    if world < 1 or not 0 <= rank < world or rows_per_rank < 1:
        raise ValueError(f"bad shard rank={rank} world={world} rows_per_rank={rows_per_rank}")
    return RowShard(rank, world, rows_per_rank)


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The largest value over all ranks (the slowest rank's time); the value
    itself when not distributed."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_rows_per_s(shard: RowShard, steps: int, seconds: float) -> float:
    """Whole-job throughput: every rank's rows over the slowest rank's time."""
    return shard.global_rows * steps / seconds
