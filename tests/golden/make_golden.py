"""Generates the golden fixtures in this directory from the CPU checker.

The reference (llama.zig src/sampler.zig) ships no golden vectors and cannot be
built here (no Zig toolchain), so these fixtures are CHECKER-DERIVED: they pin
the C restatement (oracle/ref_sampler.c) against regressions and give the CUDA
sampler a fixed target.  The first two cases are the reference's own tests
(sampler.zig:171-193 and :195-213).

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def cfg(**kw):
    c = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, typical_p=1.0, seed=0,
             repetition_window=0, repetition_penalty=1.0)
    c.update(kw)
    return c


def gen(rng, kind, steps, rows, V):
    x = np.empty((steps, rows, V), dtype=np.float32)
    for s in range(steps):
        for r in range(rows):
            if kind == "zeros":
                v = np.zeros(V)
            elif kind == "ref_topk1":
                v = np.array([2.0, 1.9, 1.8])
            elif kind == "normal3":
                v = 3 * rng.standard_normal(V)
            elif kind == "spiky":
                v = 3 * rng.standard_normal(V)
                idx = rng.choice(V, size=min(16, V), replace=False)
                v[idx] += rng.uniform(5, 15, size=idx.size)
            elif kind == "typical":
                v = 4 * rng.standard_normal(V)
                idx = rng.choice(V, size=min(64, V), replace=False)
                v[idx] += rng.uniform(4, 12, size=idx.size)
            elif kind == "ties":
                v = np.round(2 * rng.standard_normal(V)) / 2
            elif kind == "flat":
                v = 0.05 * rng.standard_normal(V)
            elif kind == "special":
                v = rng.standard_normal(V)
                if r == 0:
                    v[V // 3] = np.nan
                elif r == 1:
                    v[V // 2] = np.inf
                elif r == 2:
                    v[:] = -np.inf
                elif r == 3:
                    v[0] = np.nan
            else:
                raise ValueError(kind)
            x[s, r] = v.astype(np.float32)
    return x


CASES = [
    # name, kind, V, rows, steps, config, penalty window tokens
    ("ref_determinism", "zeros", 4, 2, 8, cfg(temperature=1.0, seed=1234), 0),
    ("ref_topk1", "ref_topk1", 3, 1, 16, cfg(temperature=1.0, top_k=1, seed=1), 0),
    ("topp_small", "normal3", 17, 4, 4, cfg(temperature=0.8, top_p=0.9, seed=42), 0),
    ("topp_spiky", "spiky", 2000, 4, 4, cfg(temperature=0.8, top_p=0.9, seed=42), 0),
    ("combo", "spiky", 3000, 4, 3, cfg(temperature=0.7, top_k=40, top_p=0.95, min_p=0.05, seed=42), 0),
    ("topk_only", "normal3", 1000, 4, 3, cfg(temperature=1.0, top_k=20, seed=5), 0),
    ("minp_only", "spiky", 1000, 4, 3, cfg(temperature=1.0, min_p=0.1, seed=9), 0),
    ("nofilter", "normal3", 257, 4, 3, cfg(temperature=1.0, seed=3), 0),
    ("flat_nofilter", "flat", 1500, 2, 2, cfg(temperature=1.5, seed=11), 0),
    ("typical", "typical", 2000, 4, 3, cfg(temperature=1.0, typical_p=0.9, seed=42), 0),
    ("typical_combo", "spiky", 2000, 4, 3, cfg(temperature=0.8, top_p=0.95, typical_p=0.5, seed=4), 0),
    ("penalty", "normal3", 500, 4, 3, cfg(temperature=0.9, top_p=0.95, repetition_window=8,
                                            repetition_penalty=1.3, seed=21), 12),
    ("greedy", "normal3", 1000, 4, 1, cfg(temperature=0.0, seed=1), 0),
    ("ties", "ties", 64, 4, 3, cfg(temperature=1.0, top_k=10, top_p=0.9, seed=8), 0),
    ("special", "special", 64, 4, 1, cfg(temperature=1.0, top_p=0.9, seed=2), 0),
]


def make_case(name, kind, V, rows, steps, c, n_prev, rng):
    x = gen(rng, kind, steps, rows, V)
    prev = None
    if n_prev:
        prev = rng.integers(0, V, size=(steps, rows, n_prev)).astype(np.uint32)
        prev[:, :, -1] = prev[:, :, 0]  # a repeated id: penalised once
    seeds = (np.arange(rows, dtype=np.uint64) + np.uint64(c["seed"])).astype(np.uint64)
    oc = O.make_config(**c)
    states = None
    tokens = np.zeros((steps, rows), np.uint32)
    st_after = np.zeros((steps, rows, 4), np.uint64)
    tr = np.zeros((steps, rows, 5), np.float32)   # S, total, u, path, n_kept
    for s in range(steps):
        out, traces, states = O.sample_batch(oc, x[s], seeds=seeds if states is None else None,
                                             states=states, prev=None if prev is None else prev[s])
        tokens[s] = out
        st_after[s] = states
        for r in range(rows):
            t = traces[r]
            tr[s, r] = [t.sum, t.total, t.u, t.path, t.n_kept]
    arrs = dict(logits=x, seeds=seeds, tokens=tokens, states=st_after, traces=tr,
                config=np.array(json.dumps(c)))
    if prev is not None:
        arrs["prev"] = prev
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrs)
    return tokens


def main():
    O.build()
    rng = np.random.default_rng(20261201)
    for case in CASES:
        toks = make_case(*case, rng)
        print(case[0], toks.ravel()[:16].tolist())


if __name__ == "__main__":
    main()
