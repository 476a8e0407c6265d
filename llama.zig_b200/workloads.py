"""Seeded synthetic logits and sampler settings for the benchmark configurations.

No public dataset is involved: every configuration is defined by the shape,
distribution and filter settings below.  Logits are generated on the host with
numpy's PCG64 / ziggurat generator (deterministic for a given seed) and are fed
byte-identically to the CUDA sampler and to the CPU checker.

Repetition penalty is off in every configuration (penalty 1.0, window 0), as
both reference callers set it (engine.zig:205-214, main.zig:508-517).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    rows: int
    vocab: int
    scale: float            # logits = scale * N(0,1)
    n_spikes: int           # distinct uniform indices that get +U(lo, hi)
    spike_lo: float
    spike_hi: float
    argmax_spike: float     # added to the row-wise argmax (0 = none)
    temperature: float
    top_k: int = 0
    top_p: float = 1.0
    min_p: float = 0.0
    typical_p: float = 1.0
    seed: int = 42          # sampler seed of row 0; row r uses seed + r
    steps: int = 1          # fresh logits per step (config 0 runs 1000)
    notes: str = ""
    sampler: dict = field(default_factory=dict)

    def config(self, **over) -> dict:
        c = dict(temperature=self.temperature, top_k=self.top_k, top_p=self.top_p,
                 min_p=self.min_p, typical_p=self.typical_p, seed=self.seed,
                 repetition_window=0, repetition_penalty=1.0)
        c.update(over)
        return c

    def seeds(self, rows: int | None = None, offset: int = 0) -> np.ndarray:
        n = self.rows if rows is None else rows
        return (np.arange(offset, offset + n, dtype=np.uint64) + np.uint64(self.seed)).astype(np.uint64)


# The benchmark configurations 0-4 of BASELINE.json plus the headline B=256 cases.
WORKLOADS = {
    # config 0: the CLI's single-row sampler, top-p only, 1000 sequential steps
    "c0": Workload("c0", 1, 128256, 3.0, 16, 5.0, 15.0, 0.0, 0.8, top_p=0.9, steps=1000),
    # config 1: combined filters, per-row seeds seed+row
    "c1": Workload("c1", 64, 128256, 3.0, 16, 5.0, 15.0, 0.0, 0.7, top_k=40, top_p=0.95, min_p=0.05),
    # config 2: typical-p at a larger vocabulary
    "c2": Workload("c2", 256, 151936, 4.0, 64, 4.0, 12.0, 0.0, 1.0, typical_p=0.9),
    # config 3: greedy (T=0) and near-greedy (top_k=1) at a very large vocabulary.
    # The top_k=1 run leaves T/top_p unstated: T=1.0, top_p=1.0, min_p=0.
    "c3_greedy": Workload("c3_greedy", 1024, 256000, 2.0, 0, 0.0, 0.0, 8.0, 0.0),
    "c3_topk1": Workload("c3_topk1", 1024, 256000, 2.0, 0, 0.0, 0.0, 8.0, 1.0, top_k=1),
    # config 4: vocabulary-sharded sampling (tensor-parallel LM head)
    "c4": Workload("c4", 512, 128256, 3.0, 16, 5.0, 15.0, 0.0, 0.8, top_k=50, top_p=0.9, min_p=0.02, seed=7),
    # headline: B=256, V=128256 with config 1's filter set ...
    "headline": Workload("headline", 256, 128256, 3.0, 16, 5.0, 15.0, 0.0, 0.7, top_k=40, top_p=0.95, min_p=0.05),
    # ... and with config 0's top-p-only set (the harder no-top-k case)
    "headline_topp": Workload("headline_topp", 256, 128256, 3.0, 16, 5.0, 15.0, 0.0, 0.8, top_p=0.9),
}


def make_logits(w: Workload, step: int = 0, rows: int | None = None, row_offset: int = 0,
                vocab: int | None = None) -> np.ndarray:
    """Logits for ``step`` of workload ``w`` as a (rows, vocab) float32 array.

    Rows are generated in blocks of 64 from PCG64 streams keyed by
    (workload, step, block), so any row range is reproducible on its own.
    """
    n_rows = w.rows if rows is None else rows
    V = w.vocab if vocab is None else vocab
    out = np.empty((n_rows, V), dtype=np.float32)
    key = sum(ord(c) * (31 ** i) for i, c in enumerate(w.name)) & 0xFFFFFFFF
    blk = 64
    r = 0
    while r < n_rows:
        g_row = row_offset + r
        b0 = (g_row // blk) * blk
        rng = np.random.default_rng([key, step, b0 // blk, V])
        nb = min(blk, (b0 + blk) - g_row, n_rows - r)
        full = rng.standard_normal((blk, V), dtype=np.float32)
        lo = g_row - b0
        block = full[lo:lo + nb]
        block *= np.float32(w.scale)
        if w.n_spikes:
            for i in range(blk):
                idx = rng.choice(V, size=w.n_spikes, replace=False)
                add = rng.uniform(w.spike_lo, w.spike_hi, size=w.n_spikes).astype(np.float32)
                if lo <= i < lo + nb:
                    block[i - lo, idx] += add
        if w.argmax_spike:
            am = np.argmax(block, axis=1)
            block[np.arange(nb), am] += np.float32(w.argmax_spike)
        out[r:r + nb] = block
        r += nb
    return out
