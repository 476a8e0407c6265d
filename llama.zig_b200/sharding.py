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


# ---------------------------------------------------------------------------
# Vocab sharding (a tensor-parallel LM head): every rank holds all B rows of
# a contiguous slice of the vocabulary.  sampler.zig's normaliser is a
# sequential f32 sum in global index order, and the exact GPU path needs a
# row's logits in that order, so the exchange is a transpose: one all-to-all
# gives rank g complete rows [g B/G, (g+1) B/G) ((G-1)/G of its shard crosses
# NVLink), rank g samples them (seeds keyed by the global row), and an
# all-gather replicates the B token ids on every rank.  A merge of per-shard
# partial sums would change the normaliser's rounding (about 1e-4 relative)
# and with it the kept-set probabilities and draws near boundaries.
@dataclass(frozen=True)
class VocabShard:
    rank: int
    world: int
    rows: int      # B, all rows (every rank holds all of them)
    vocab: int     # V, the whole vocabulary

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError(f"bad rank {self.rank} of {self.world}")
        if self.vocab % self.world or self.rows % self.world:
            raise ValueError(f"vocab {self.vocab} and rows {self.rows} must divide by {self.world} ranks")

    @property
    def cols(self) -> int:
        """Columns of each shard (V / G)."""
        return self.vocab // self.world

    @property
    def col0(self) -> int:
        return self.rank * self.cols

    @property
    def rows_per_rank(self) -> int:
        return self.rows // self.world

    @property
    def row0(self) -> int:
        """First global row this rank samples after the transpose."""
        return self.rank * self.rows_per_rank

    def seeds(self, base_seed: int) -> np.ndarray:
        return (np.arange(self.row0, self.row0 + self.rows_per_rank, dtype=np.uint64)
                + np.uint64(base_seed)).astype(np.uint64)

    def shard_of(self, full):
        """This rank's slice of a full (B, V) matrix (for tests and benchmarks)."""
        return full[:, self.col0:self.col0 + self.cols]


def rows_from_vocab_shards(lay: VocabShard, shard, dist, recv=None, out=None):
    """(B, V/G) shard on every rank -> (B/G, V) complete rows on each rank.

    The rows of rank h are contiguous in the shard, so chunk h of the send
    buffer is rank h's; chunk g of the receive buffer is shard g of this
    rank's rows, copied into columns [g V/G, (g+1) V/G)."""
    import torch
    G, R, C = lay.world, lay.rows_per_rank, lay.cols
    if tuple(shard.shape) != (lay.rows, C) or not shard.is_contiguous():
        raise ValueError(f"shard must be a contiguous ({lay.rows}, {C}) tensor")
    if G == 1:
        return shard   # the shard is the whole vocabulary
    if recv is None:
        recv = torch.empty((G, R, C), dtype=shard.dtype, device=shard.device)
    if out is None:
        out = torch.empty((R, lay.vocab), dtype=shard.dtype, device=shard.device)
    dist.all_to_all_single(recv.view(-1), shard.view(-1))
    out.view(R, G, C).copy_(recv.transpose(0, 1))
    return out


def gather_tokens(lay: VocabShard, local, dist, out=None):
    """(B/G,) token ids of this rank's rows -> (B,) on every rank."""
    import torch
    if lay.world == 1:
        return local
    if out is None:
        out = torch.empty((lay.rows,), dtype=local.dtype, device=local.device)
    dist.all_gather(list(out.view(lay.world, lay.rows_per_rank).unbind(0)), local)
    return out


class VocabShardedSampler:
    """Sampler.sample over vocab-sharded logits: every rank passes its
    (B, V/G) shard and gets the same B token ids back."""

    def __init__(self, cfg, rows: int, vocab: int, dist=None, device: int = 0, seeds_base: int | None = None):
        import torch
        from .sampler import Sampler
        world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
        rank = dist.get_rank() if world > 1 else 0
        self.lay = VocabShard(rank, world, rows, vocab)
        self.dist = dist
        base = cfg.seed if seeds_base is None else seeds_base
        self.local = Sampler(cfg, batch=self.lay.rows_per_rank, vocab=vocab, device=device,
                             seeds=self.lay.seeds(base))
        dev = torch.device("cuda", device)
        R, C, G = self.lay.rows_per_rank, self.lay.cols, world
        self._recv = torch.empty((G, R, C), dtype=torch.float32, device=dev) if G > 1 else None
        self._rows = torch.empty((R, vocab), dtype=torch.float32, device=dev) if G > 1 else None
        self._tok = torch.empty((R,), dtype=torch.int32, device=dev)
        self._all = torch.empty((rows,), dtype=torch.int32, device=dev)

    def sample(self, shard):
        rows = rows_from_vocab_shards(self.lay, shard, self.dist, self._recv, self._rows)
        self.local.sample(rows, out=self._tok)
        return gather_tokens(self.lay, self._tok, self.dist, self._all)

    def close(self):
        self.local.close()
