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
# a contiguous slice of the vocabulary, columns [g V/G, (g+1) V/G).
#
# Exact partial merge (the default, when the configuration has a top-k
# bound): sampler.zig's normaliser is one sequential f32 sum over the whole
# row in index order, reproduced as a chain over the shards in rank order.
#   1. each rank: statistics of its shard -> per-row partial (max, sum
#      relative to it, non-finite flag); one all-gather of the partials
#      (16 B per row per rank)
#   2. each rank: row reduction against the global maximum and the lower
#      shards' mass estimate; main pass over its shard
#   3. chain: rank g walks its shard's items from the exact running sum
#      rank g-1 ended with (4 B per row, point to point); the last rank's
#      result is the normaliser S, broadcast to all ranks
#   4. one all-gather of each shard's candidates (its local top-k and above)
#   5. every rank: filters and draw over the merged candidates with the
#      row's RNG state, so every rank returns the same B tokens
# Without a top-k bound (or with typical-p) a shard's candidates need not
# cover the kept set, and the sampler falls back to a transpose: one
# all-to-all gives rank g complete rows [g B/G, (g+1) B/G), it samples them
# on one GPU, and an all-gather replicates the B token ids.
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

    def all_seeds(self, base_seed: int) -> np.ndarray:
        """Seeds of all B rows (the exact merge keeps every row's RNG on every rank)."""
        return (np.arange(self.rows, dtype=np.uint64) + np.uint64(base_seed)).astype(np.uint64)

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


def history_rows(lay: VocabShard, prev_tokens):
    """This rank's rows of a (B, n_prev) previous-token history: the rows the
    transpose gives it, [row0, row0 + B/G)."""
    return prev_tokens[lay.row0:lay.row0 + lay.rows_per_rank]


def gather_tokens(lay: VocabShard, local, dist, out=None):
    """(B/G,) token ids of this rank's rows -> (B,) on every rank."""
    import torch
    if lay.world == 1:
        return local
    if out is None:
        out = torch.empty((lay.rows,), dtype=local.dtype, device=local.device)
    dist.all_gather(list(out.view(lay.world, lay.rows_per_rank).unbind(0)), local)
    return out


CAND_CAP = 512   # BS_VSHARD_CAND_CAP: candidates a shard exports per row


class _ShardState:
    """One rank's handle and buffers of the exact partial merge."""

    def __init__(self, cfg, lay: VocabShard, device: int, seeds):
        import torch
        from .sampler import Sampler
        self.lay = lay
        self.smp = Sampler(cfg, batch=lay.rows, vocab=lay.cols, device=device, seeds=seeds)
        dev = torch.device("cuda", device)
        B = lay.rows
        self.part = torch.empty((B, 2), dtype=torch.int64, device=dev)          # 16 B per row
        self.exit = torch.empty((B,), dtype=torch.float32, device=dev)
        self.cand = torch.empty((B, CAND_CAP, 2), dtype=torch.int32, device=dev)
        self.count = torch.empty((B,), dtype=torch.int32, device=dev)
        self.out = torch.empty((B,), dtype=torch.int32, device=dev)

    def _lib(self):
        from .sampler import lib, _check
        return lib(), _check

    def stats(self, shard, prev, stream, push=False):
        """push: the partials go straight to every rank's exchange words."""
        L, check = self._lib()
        pp, n_prev = (None, 0) if prev is None else (prev.data_ptr(), prev.shape[1])
        check(L.bs_vshard_stats(self.smp._h, shard.data_ptr(), shard.stride(0), self.lay.col0, self.lay.rows,
                                pp, n_prev, None if push else self.part.data_ptr(), stream), "bs_vshard_stats")
        return self.part

    def main(self, parts_all, stream):
        """parts_all None: the partials from the exchange words."""
        L, check = self._lib()
        check(L.bs_vshard_main(self.smp._h, None if parts_all is None else parts_all.data_ptr(), self.lay.world,
                               self.lay.rank, stream), "bs_vshard_main")

    def walk(self, entry, stream):
        L, check = self._lib()
        check(L.bs_vshard_walk(self.smp._h, None if entry is None else entry.data_ptr(), self.exit.data_ptr(),
                               stream), "bs_vshard_walk")
        return self.exit

    def export(self, stream, push=False):
        """push: the candidates go straight to every rank's exchange words."""
        L, check = self._lib()
        check(L.bs_vshard_export(self.smp._h, self.lay.col0, None if push else self.cand.data_ptr(),
                                 None if push else self.count.data_ptr(), stream), "bs_vshard_export")
        return self.cand, self.count

    def draw(self, cand_all, count_all, S, stream):
        """S: the normaliser per row, or None to take it from the peer-memory
        chain's exchange words."""
        L, check = self._lib()
        check(L.bs_vshard_draw(self.smp._h, None if cand_all is None else cand_all.data_ptr(),
                               None if count_all is None else count_all.data_ptr(), self.lay.world,
                               None if S is None else S.data_ptr(), self.out.data_ptr(), stream), "bs_vshard_draw")
        return self.out

    def open_peers(self, dist):
        """Exchange the CUDA IPC handles of the ranks' chain words (host
        all-gather) and map the others' (bs_vshard_ipc_handle / _open)."""
        import ctypes
        L, check = self._lib()
        h = ctypes.create_string_buffer(64)
        check(L.bs_vshard_ipc_handle(self.smp._h, self.lay.world, h), "bs_vshard_ipc_handle")
        hs = [None] * self.lay.world
        dist.all_gather_object(hs, h.raw)
        allh = b"".join(hs)
        check(L.bs_vshard_ipc_open(self.smp._h, self.lay.world, self.lay.rank, allh), "bs_vshard_ipc_open")

    def chain(self, stream):
        L, check = self._lib()
        check(L.bs_vshard_chain(self.smp._h, stream), "bs_vshard_chain")


def exact_merge_supported(cfg) -> bool:
    """The exact partial merge needs a top-k bound (0 < top_k <= 256), a
    positive temperature and typical-p off."""
    typ = 0.0 < cfg.typical_p < 1.0
    return cfg.temperature > 0 and 0 < cfg.top_k <= 256 and not typ


def sample_vocab_sharded_emulated(states, shards, prevs=None):
    """The exact partial merge with every rank in this process on one GPU:
    the collectives become copies.  `states` and `shards` are per rank.
    Returns each rank's (B,) tokens (all equal)."""
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    G = len(states)
    parts = torch.stack([st.stats(shards[g], None if prevs is None else prevs[g], stream).clone()
                         for g, st in enumerate(states)])
    for st in states:
        st.main(parts, stream)
    entry = None
    for st in states:
        entry = st.walk(entry, stream).clone()
    S = entry
    cands, counts = zip(*[(c.clone(), n.clone()) for c, n in (st.export(stream) for st in states)])
    cand_all, count_all = torch.stack(cands), torch.stack(counts)
    return [st.draw(cand_all, count_all, S, stream).clone() for st in states]


class VocabShardedSampler:
    """Sampler.sample over vocab-sharded logits: every rank passes its
    (B, V/G) shard (and, for the repetition penalty, the (B, n_prev) previous
    token ids) and gets the same B token ids back."""

    def __init__(self, cfg, rows: int, vocab: int, dist=None, device: int = 0, seeds_base: int | None = None,
                 exact: bool | None = None, transport: str = "nccl"):
        import torch
        world = dist.get_world_size() if dist is not None and dist.is_initialized() else 1
        rank = dist.get_rank() if world > 1 else 0
        self.lay = VocabShard(rank, world, rows, vocab)
        self.dist = dist
        self.device = device
        base = cfg.seed if seeds_base is None else seeds_base
        self.exact = exact_merge_supported(cfg) if exact is None else exact
        self._capturing = False
        if transport not in ("nccl", "p2p"):
            raise ValueError("transport is 'nccl' or 'p2p'")
        # p2p: the chain of walks through peer memory (exact merge, 2+ ranks)
        self.p2p = transport == "p2p" and world > 1 and self.exact
        if self.exact and not exact_merge_supported(cfg):
            raise ValueError("the exact partial merge needs 0 < top_k <= 256, temperature > 0 and typical-p off")
        dev = torch.device("cuda", device)
        R, C, G = self.lay.rows_per_rank, self.lay.cols, world
        if self.exact:
            self.st = _ShardState(cfg, self.lay, device, self.lay.all_seeds(base))
            if self.p2p:
                self.st.open_peers(dist)
            self._parts = torch.empty((G, rows, 2), dtype=torch.int64, device=dev)
            self._cand_all = torch.empty((G, rows, CAND_CAP, 2), dtype=torch.int32, device=dev)
            self._count_all = torch.empty((G, rows), dtype=torch.int32, device=dev)
            self._entry = torch.empty((rows,), dtype=torch.float32, device=dev)
            self._S = torch.empty((rows,), dtype=torch.float32, device=dev)
        else:
            from .sampler import Sampler
            self.local = Sampler(cfg, batch=R, vocab=vocab, device=device, seeds=self.lay.seeds(base))
            self._recv = torch.empty((G, R, C), dtype=torch.float32, device=dev) if G > 1 else None
            self._rows = torch.empty((R, vocab), dtype=torch.float32, device=dev) if G > 1 else None
            self._tok = torch.empty((R,), dtype=torch.int32, device=dev)
            self._all = torch.empty((rows,), dtype=torch.int32, device=dev)

    def sample(self, shard, prev_tokens=None):
        import torch
        if not self.exact:
            rows = rows_from_vocab_shards(self.lay, shard, self.dist, self._recv, self._rows)
            pv = None if prev_tokens is None else history_rows(self.lay, prev_tokens).to(torch.int32).contiguous()
            self.local.sample(rows, pv, out=self._tok)
            return gather_tokens(self.lay, self._tok, self.dist, self._all)
        lay, st, dist = self.lay, self.st, self.dist
        stream = torch.cuda.current_stream().cuda_stream
        prev = None if prev_tokens is None else prev_tokens.to(torch.int32).contiguous()
        if self.p2p:
            # the whole step through peer memory, no collective: partials and
            # candidates stored straight into every rank's exchange words,
            # each waited for by its step tag; the chain inside the walk
            # kernels; the draw from this rank's words
            st.stats(shard, prev, stream, push=True)
            st.main(None, stream)
            st.export(stream, push=True)
            st.chain(stream)
            return st.draw(None, None, None, stream)
        part = st.stats(shard, prev, stream)
        if lay.world == 1:
            self._parts[0].copy_(part)
        else:
            dist.all_gather_into_tensor(self._parts, part)
        st.main(self._parts, stream)
        # the candidates are final after the main pass: their all-gather runs
        # while the chain of walks does
        cand, count = st.export(stream)
        works = []
        if lay.world == 1:
            self._cand_all[0].copy_(cand)
            self._count_all[0].copy_(count)
        else:
            # (asynchronous when eager; a captured step keeps stream order)
            a = not self._capturing
            works.append(dist.all_gather_into_tensor(self._cand_all, cand, async_op=a))
            works.append(dist.all_gather_into_tensor(self._count_all, count, async_op=a))
        # the chain of walks in rank order: link k broadcasts rank k's exit
        # state, which is rank k + 1's entry; the last link's is the row's S.
        # Every rank takes part in every link (one collective sequence on all
        # ranks, which a CUDA graph can hold)
        if lay.world == 1:
            self._S.copy_(st.walk(None, stream))
        else:
            for k in range(lay.world):
                if lay.rank == k:
                    self._S.copy_(st.walk(self._entry if k > 0 else None, stream))
                dist.broadcast(self._S, src=k)
                if lay.rank == k + 1:
                    self._entry.copy_(self._S)
        for wk in works:
            if wk is not None:
                wk.wait()
        return st.draw(self._cand_all, self._count_all, self._S, stream)

    def graph(self, shard, prev_tokens=None):
        """One sample() step on these buffers captured into a CUDA graph,
        collectives included: ``g.replay()`` repeats the step (new logits
        copied into ``shard`` first) with no host work.  Returns (graph,
        token tensor).  Call sample() once before, so that the collectives'
        communicators exist."""
        import torch
        if not self.exact:
            raise ValueError("graph capture is built for the exact partial merge")
        self._capturing = True
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = self.sample(shard, prev_tokens)
        finally:
            self._capturing = False
        return g, out

    def last_status(self) -> int:
        return self.st.smp.last_status() if self.exact else self.local.last_status()

    def close(self):
        if self.exact:
            self.st.smp.close()
        else:
            self.local.close()
