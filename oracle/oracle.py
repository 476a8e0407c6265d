"""ctypes front-end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline /
reference leg may import this module.  It loads ``oracle/liboracle.so`` (the C
restatement of llama.zig ``src/sampler.zig``, built by ``oracle/Makefile``)
and is the checker for the CUDA sampler, never part of the product path.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

PATH_ARGMAX_T, PATH_ARGMAX_SUM, PATH_EMPTY, PATH_DRAW, PATH_DRAW_FALLBACK = range(5)


class OrcConfig(ctypes.Structure):
    """Mirror of SamplerConfig (sampler.zig:4-13); same layout as bs_config."""

    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_uint32),
        ("top_p", ctypes.c_float),
        ("min_p", ctypes.c_float),
        ("typical_p", ctypes.c_float),
        ("_pad0", ctypes.c_uint32),
        ("seed", ctypes.c_uint64),
        ("repetition_window", ctypes.c_uint32),
        ("repetition_penalty", ctypes.c_float),
    ]


class OrcSampler(ctypes.Structure):
    _fields_ = [("cfg", OrcConfig), ("s", ctypes.c_uint64 * 4)]


class OrcTrace(ctypes.Structure):
    _fields_ = [
        ("token", ctypes.c_uint32),
        ("path", ctypes.c_uint32),
        ("n_kept", ctypes.c_uint32),
        ("draws", ctypes.c_uint32),
        ("max_logit", ctypes.c_float),
        ("sum", ctypes.c_float),
        ("entropy", ctypes.c_float),
        ("total", ctypes.c_float),
        ("u", ctypes.c_float),
        ("r0", ctypes.c_float),
        ("sum_f64", ctypes.c_double),
        ("cut_topp", ctypes.c_uint32),
        ("_pad", ctypes.c_uint32),
        ("draw_margin", ctypes.c_double),
        ("thr_margin", ctypes.c_double),
    ]


_lib = None


def build() -> str:
    """Compile liboracle.so with the oracle's Makefile (strict IEEE f32 flags)."""
    subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u64p = ctypes.POINTER(ctypes.c_uint64)
        L.orc_rng_seed.argtypes = [u64p, ctypes.c_uint64]
        L.orc_rng_next.argtypes = [u64p]
        L.orc_rng_next.restype = ctypes.c_uint64
        L.orc_rng_float.argtypes = [u64p, ctypes.POINTER(ctypes.c_uint32)]
        L.orc_rng_float.restype = ctypes.c_float
        L.orc_expf.argtypes = [ctypes.c_float]
        L.orc_expf.restype = ctypes.c_float
        L.orc_logf.argtypes = [ctypes.c_float]
        L.orc_logf.restype = ctypes.c_float
        L.orc_expm1f.argtypes = [ctypes.c_float]
        L.orc_expm1f.restype = ctypes.c_float
        L.orc_tanhf.argtypes = [ctypes.c_float]
        L.orc_tanhf.restype = ctypes.c_float
        L.orc_prologue.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_float]
        L.orc_prologue.restype = None
        L.orc_sampler_init.argtypes = [ctypes.POINTER(OrcSampler), ctypes.POINTER(OrcConfig)]
        L.orc_argmax.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
        L.orc_argmax.restype = ctypes.c_uint32
        L.orc_sample.argtypes = [ctypes.POINTER(OrcSampler), ctypes.c_void_p, ctypes.c_size_t,
                                 ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(OrcTrace)]
        L.orc_sample.restype = ctypes.c_uint32
        L.orc_sample_batch.argtypes = [ctypes.POINTER(OrcSampler), ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                       ctypes.c_size_t, ctypes.c_void_p, ctypes.POINTER(OrcTrace),
                                       ctypes.c_int]
        L.orc_sample_batch.restype = ctypes.c_int
        _lib = L
    return _lib


def make_config(temperature=0.8, top_k=0, top_p=0.9, min_p=0.0, typical_p=1.0, seed=0,
                repetition_window=32, repetition_penalty=1.1) -> OrcConfig:
    """Defaults are SamplerConfig's defaults (sampler.zig:5-12)."""
    return OrcConfig(temperature, top_k, top_p, min_p, typical_p, 0, seed,
                     repetition_window, repetition_penalty)


class Sampler:
    """One oracle sampler per row: Sampler.init / Sampler.sample (sampler.zig:19-28)."""

    def __init__(self, cfg: OrcConfig):
        self._s = OrcSampler()
        lib().orc_sampler_init(ctypes.byref(self._s), ctypes.byref(cfg))

    @property
    def state(self) -> np.ndarray:
        return np.array(list(self._s.s), dtype=np.uint64)

    @state.setter
    def state(self, st) -> None:
        for i in range(4):
            self._s.s[i] = int(st[i])

    def sample(self, logits: np.ndarray, prev=None, trace: bool = False):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        p = None if prev is None or len(prev) == 0 else np.ascontiguousarray(prev, dtype=np.uint32)
        tr = OrcTrace()
        tok = lib().orc_sample(ctypes.byref(self._s), x.ctypes.data, x.size,
                               None if p is None else p.ctypes.data, 0 if p is None else p.size,
                               ctypes.byref(tr))
        return (tok, tr) if trace else tok


def prologue(logits: np.ndarray, softcap: float, logit_scale: float) -> np.ndarray:
    """The engine's logit prologue (engine.zig:341-354) on a copy: soft-cap
    tanh(v / s) * s when s > 0, then v *= 1 / logit_scale unless it is 1 or 0."""
    x = np.array(logits, dtype=np.float32, copy=True, order="C")
    lib().orc_prologue(x.ctypes.data, x.size, softcap, logit_scale)
    return x


def argmax(logits: np.ndarray) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_argmax(x.ctypes.data, x.size))


def rng_seed(seed: int) -> np.ndarray:
    st = (ctypes.c_uint64 * 4)()
    lib().orc_rng_seed(st, seed)
    return np.array(list(st), dtype=np.uint64)


def sample_batch(cfg: OrcConfig, logits: np.ndarray, seeds=None, states=None, prev=None,
                 nthreads: int = 0):
    """Sample every row of ``logits`` (rows x n) with its own oracle sampler.

    Row r is seeded with ``seeds[r]`` (zero -> 0xDEADBEEF as Sampler.init does),
    or starts from ``states[r]`` (4 x u64).  Returns (tokens, traces, states_after).
    """
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rows, n = x.shape
    samplers = (OrcSampler * rows)()
    L = lib()
    for r in range(rows):
        c = OrcConfig.from_buffer_copy(cfg)
        if seeds is not None:
            c.seed = int(seeds[r])
        L.orc_sampler_init(ctypes.byref(samplers[r]), ctypes.byref(c))
        if states is not None:
            for i in range(4):
                samplers[r].s[i] = int(states[r][i])
    out = np.zeros(rows, dtype=np.uint32)
    traces = (OrcTrace * rows)()
    pv = None
    n_prev = 0
    if prev is not None:
        pv = np.ascontiguousarray(prev, dtype=np.uint32)
        n_prev = pv.shape[1]
    rc = L.orc_sample_batch(samplers, x.ctypes.data, rows, n, n, None if pv is None else pv.ctypes.data,
                            n_prev, out.ctypes.data, traces, nthreads)
    if rc != 0:
        raise MemoryError("oracle: allocation failed")
    st = np.array([[samplers[r].s[i] for i in range(4)] for r in range(rows)], dtype=np.uint64)
    return out, traces, st


def parity_report(got_tokens, ref_tokens, traces, draw_eps: float = 1e-6) -> dict:
    """Parity counts of one sampled batch against the checker, as the spec asks.

    A row is a draw-boundary case when the reference's uniform draw lies within
    ``draw_eps`` of a boundary of the kept tokens' CDF (``draw_margin``), and a
    threshold-boundary case when a filter decision lies closer to its
    threshold than the reference's own normaliser error (the relative error of
    its sequential f32 sum against the f64 sum of the same terms).  Mismatches
    are split by those classes; ``mismatch_other`` must be 0.
    """
    got = np.asarray(got_tokens, dtype=np.uint32).ravel()
    ref = np.asarray(ref_tokens, dtype=np.uint32).ravel()
    rows = len(ref)
    draw_b = np.zeros(rows, bool)
    thr_b = np.zeros(rows, bool)
    for r in range(rows):
        t = traces[r]
        draw_b[r] = t.draw_margin < draw_eps
        rel = abs(t.sum - t.sum_f64) / t.sum_f64 if t.sum_f64 > 0 else 0.0
        thr_b[r] = t.thr_margin < rel
    bad = got != ref
    return {
        "rows": int(rows),
        "exact": int((~bad).sum()),
        "draw_boundary_rows": int(draw_b.sum()),
        "threshold_boundary_rows": int(thr_b.sum()),
        "mismatch_draw_boundary": int((bad & draw_b).sum()),
        "mismatch_threshold_boundary": int((bad & thr_b & ~draw_b).sum()),
        "mismatch_other": int((bad & ~draw_b & ~thr_b).sum()),
        "draw_eps": draw_eps,
    }
