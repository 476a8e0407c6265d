"""Host-side mirror of llama.zig's sampler interface over the C ABI.

Mirrors ``src/sampler.zig``:

* :class:`SamplerConfig`  <- ``SamplerConfig`` (sampler.zig:4-13), same fields
  and defaults;
* :class:`Sampler`        <- ``Sampler`` (sampler.zig:15-29): ``Sampler(cfg)``
  is ``Sampler.init`` (sampler.zig:19-24) and :meth:`Sampler.sample` is
  ``Sampler.sample`` (sampler.zig:26-28); one object holds ``batch`` rows, each
  an independent Zig ``Sampler`` with its own xoshiro256++ state;
* :func:`sample_argmax`   <- ``sampleArgmax`` (sampler.zig:31-41).

Errors follow the reference: an allocation failure raises :class:`MemoryError`
(``error.OutOfMemory``); anything else raises :class:`SamplerError`.

All sampling runs in ``libb200_sampler.so`` (CUDA, sm_100a).  There is no CPU
fallback: if the library or a GPU is missing, constructing a Sampler fails.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libb200_sampler.so")

BS_OK, BS_EINVAL, BS_ENOMEM, BS_ECUDA, BS_ENCCL, BS_ETIMEOUT, BS_ENOTSUP, BS_EINTERNAL = range(8)

# Every entry point include/b200_sampler.h declares (checked by the tests).
EXPORTS = [
    "bs_config_default", "bs_create", "bs_sample", "bs_sample_host", "bs_argmax",
    "bs_get_rng_state", "bs_set_rng_state", "bs_last_device_status", "bs_destroy",
    "bs_status_string", "bs_profile_enable", "bs_profile_read", "bs_argmax_ex", "bs_set_logit_prologue",
    "bs_sample_static", "bs_seed_state",
]


class SamplerError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


class BsConfig(ctypes.Structure):
    """bs_config: SamplerConfig field for field (sampler.zig:4-13)."""

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


class RowTrace(ctypes.Structure):
    """Per-row diagnostics of the last call (S, kept mass, draw, path, and
    with typical-p the entropy H)."""

    _fields_ = [
        ("S", ctypes.c_float),
        ("total", ctypes.c_float),
        ("u", ctypes.c_float),
        ("n_kept", ctypes.c_uint32),
        ("path", ctypes.c_uint32),
        ("flags", ctypes.c_uint32),
        ("n_cand", ctypes.c_uint32),
        ("status", ctypes.c_uint32),
        ("n_items", ctypes.c_uint32),
        ("n_wc", ctypes.c_uint32),
        ("n_slow", ctypes.c_uint32),
        ("H", ctypes.c_float),
    ]


@dataclass
class SamplerConfig:
    """SamplerConfig with the reference defaults (sampler.zig:5-12)."""

    temperature: float = 0.8
    top_k: int = 0
    top_p: float = 0.9
    min_p: float = 0.0
    typical_p: float = 1.0
    seed: int = 0
    repetition_window: int = 32
    repetition_penalty: float = 1.1

    def to_c(self) -> BsConfig:
        return BsConfig(self.temperature, self.top_k, self.top_p, self.min_p, self.typical_p, 0,
                        self.seed & 0xFFFFFFFFFFFFFFFF, self.repetition_window,
                        self.repetition_penalty)


_lib = None


def lib() -> ctypes.CDLL:
    """Load libb200_sampler.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run llama.zig_b200/build.py "
                              "(the sampler has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        vp, u32, u64p = ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint64)
        L.bs_config_default.argtypes = [ctypes.POINTER(BsConfig)]
        L.bs_config_default.restype = None
        L.bs_create.argtypes = [ctypes.POINTER(BsConfig), u32, u32, ctypes.c_int, u64p, ctypes.POINTER(vp)]
        L.bs_sample.argtypes = [vp, vp, ctypes.c_size_t, u32, u32, vp, u32, vp, vp]
        L.bs_sample_host.argtypes = [vp, vp, ctypes.c_size_t, u32, u32, vp, u32, vp]
        L.bs_argmax.argtypes = [vp, ctypes.c_size_t, u32, u32, vp, vp]
        L.bs_argmax_ex.argtypes = [vp, ctypes.c_size_t, u32, u32, ctypes.c_float, ctypes.c_float, vp, vp]
        L.bs_set_logit_prologue.argtypes = [vp, ctypes.c_float, ctypes.c_float]
        L.bs_vshard_stats.argtypes = [vp, vp, ctypes.c_size_t, u32, u32, vp, u32, vp, vp]
        L.bs_vshard_main.argtypes = [vp, vp, u32, u32, vp]
        L.bs_vshard_walk.argtypes = [vp, vp, vp, vp]
        L.bs_vshard_export.argtypes = [vp, u32, vp, vp, vp]
        L.bs_vshard_draw.argtypes = [vp, vp, vp, u32, vp, vp, vp]
        L.bs_vshard_ipc_handle.argtypes = [vp, u32, vp]
        L.bs_vshard_ipc_open.argtypes = [vp, u32, u32, ctypes.c_char_p]
        L.bs_vshard_chain.argtypes = [vp, vp]
        for name in ("bs_vshard_stats", "bs_vshard_main", "bs_vshard_walk", "bs_vshard_export", "bs_vshard_draw",
                     "bs_vshard_ipc_handle", "bs_vshard_ipc_open", "bs_vshard_chain"):
            getattr(L, name).restype = ctypes.c_int
        L.bs_get_rng_state.argtypes = [vp, u64p]
        L.bs_seed_state.argtypes = [ctypes.c_uint64, u64p]
        L.bs_seed_state.restype = ctypes.c_int
        L.bs_set_rng_state.argtypes = [vp, u64p]
        L.bs_last_device_status.argtypes = [vp]
        L.bs_destroy.argtypes = [vp]
        L.bs_destroy.restype = None
        L.bs_status_string.argtypes = [ctypes.c_int]
        L.bs_status_string.restype = ctypes.c_char_p
        L.bs_debug_row_traces.argtypes = [vp, vp, ctypes.c_size_t]
        L.bs_profile_enable.argtypes = [vp, u32]
        L.bs_profile_read.argtypes = [vp, vp, u32, ctypes.POINTER(u32)]
        for name in ("bs_create", "bs_sample", "bs_sample_host", "bs_argmax", "bs_argmax_ex",
                     "bs_set_logit_prologue", "bs_get_rng_state",
                     "bs_set_rng_state", "bs_last_device_status", "bs_debug_row_traces",
                     "bs_profile_enable", "bs_profile_read"):
            getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def status_string(st: int) -> str:
    return lib().bs_status_string(st).decode()


def _check(st: int, what: str) -> None:
    if st == BS_OK:
        return
    if st == BS_ENOMEM:
        raise MemoryError(f"{what}: out of memory")
    raise SamplerError(st, what)


def _stream_ptr(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return int(getattr(stream, "cuda_stream", stream))


def seed_state(seed: int) -> np.ndarray:
    """The xoshiro256++ state Sampler.init gives ``seed`` (sampler.zig:22;
    0 -> 0xDEADBEEF), computed by the library on the host (bs_seed_state)."""
    st = np.zeros(4, dtype=np.uint64)
    _check(lib().bs_seed_state(ctypes.c_uint64(int(seed) & (2**64 - 1)),
                               st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))), "bs_seed_state")
    return st


class Sampler:
    """``batch`` independent Zig Samplers on one GPU (Sampler.init, sampler.zig:19-24).

    Row r is seeded with ``cfg.seed + r`` (0 -> 0xDEADBEEF), or ``seeds[r]``.
    """

    def __init__(self, cfg: SamplerConfig, batch: int = 1, vocab: int = 0, device: int = 0,
                 seeds=None):
        self.cfg = cfg
        self.batch = int(batch)
        self.vocab = int(vocab)
        self.device = int(device)
        self._h = ctypes.c_void_p()
        self._pending_state = None
        if self.vocab <= 0:
            # Sampler.init(cfg) exactly (sampler.zig:19-24): no vocabulary yet,
            # so the state is seeded on the host and the device handle is made
            # by the first sample, sized by that call's logits
            if self.batch != 1 or seeds is not None or vocab < 0:
                raise ValueError("vocab must be positive (only a one-row Sampler binds it lazily)")
            self._pending_state = seed_state(cfg.seed)[None, :]
            return
        self._create(seeds)

    @classmethod
    def init(cls, cfg: SamplerConfig, device: int = 0) -> "Sampler":
        """Sampler.init (sampler.zig:19-24): one row, no device work until
        the first :meth:`sample`, which takes the vocabulary from its logits."""
        return cls(cfg, batch=1, vocab=0, device=device)

    def _create(self, seeds=None) -> None:
        c = self.cfg.to_c()
        sp = None
        if seeds is not None:
            self._seeds = np.ascontiguousarray(seeds, dtype=np.uint64)
            sp = self._seeds.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
        _check(lib().bs_create(ctypes.byref(c), self.batch, self.vocab, self.device, sp,
                               ctypes.byref(self._h)), "bs_create")
        if getattr(self, "_prologue", None) is not None:
            _check(lib().bs_set_logit_prologue(self._h, *self._prologue), "bs_set_logit_prologue")

    def _bind(self, vocab: int) -> None:
        """Make (or remake, for another vocabulary) the lazily bound handle,
        carrying the xoshiro256++ state over."""
        if self._h and vocab == self.vocab:
            return
        if self._pending_state is None:
            if not self._h:
                raise ValueError("sampler is closed")
            self._pending_state = self.rng_state
            self.close()
        self.vocab = int(vocab)
        self._create()
        self.rng_state = self._pending_state
        self._pending_state = None

    def close(self) -> None:
        if self._h:
            lib().bs_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- Sampler.sample (sampler.zig:26-28) ---------------------------------
    def sample(self, logits, prev_tokens=None, out=None, row0: int = 0, stream=None):
        """Sample one token per row.

        ``logits``: a CUDA tensor (rows x vocab, float32, rows on a stride) --
        stream-ordered, returns a CUDA uint32/int32 tensor -- or a host numpy
        array / list (the engine.zig:355 compatibility path), which returns a
        numpy uint32 array (or an int for a 1-D input, like the reference).
        ``prev_tokens``: previous token ids for the repetition penalty, rows x
        n_prev (same device kind as ``logits``).
        """
        lazy = self._pending_state is not None or getattr(self, "_lazy", False)
        if isinstance(logits, np.ndarray) or isinstance(logits, (list, tuple)):
            if lazy:
                self._lazy = True
                self._bind(np.shape(logits)[-1])
            return self._sample_host(logits, prev_tokens, row0)
        import torch
        x = logits
        if x.dim() == 1:
            x = x.unsqueeze(0)
        if lazy:
            self._lazy = True
            self._bind(x.shape[1])
        if x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
            raise ValueError("logits must be a CUDA float32 tensor with unit column stride")
        rows = x.shape[0]
        if x.shape[1] != self.vocab:
            raise ValueError("logits width != vocab")
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=x.device)
        pp, n_prev = None, 0
        if prev_tokens is not None and prev_tokens.numel() > 0:
            pt = prev_tokens if prev_tokens.dim() == 2 else prev_tokens.unsqueeze(0).expand(rows, -1)
            pt = pt.to(torch.int32).contiguous()
            pp, n_prev = pt.data_ptr(), pt.shape[1]
            self._keep = pt
        _check(lib().bs_sample(self._h, x.data_ptr(), x.stride(0), row0, rows, pp, n_prev,
                               out.data_ptr(), _stream_ptr(stream)), "bs_sample")
        return out

    def _sample_host(self, logits, prev_tokens, row0):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        one = x.ndim == 1
        if one:
            x = x[None, :]
        rows = x.shape[0]
        out = np.zeros(rows, dtype=np.uint32)
        pp, n_prev = None, 0
        if prev_tokens is not None and len(prev_tokens) > 0:
            pv = np.ascontiguousarray(prev_tokens, dtype=np.uint32)
            if pv.ndim == 1:
                pv = np.broadcast_to(pv, (rows, pv.size)).copy()
            pp, n_prev = pv.ctypes.data, pv.shape[1]
        _check(lib().bs_sample_host(self._h, x.ctypes.data, x.shape[1], row0, rows, pp, n_prev,
                                    out.ctypes.data), "bs_sample_host")
        return int(out[0]) if one else out

    # -- PRNG state ------------------------------------------------------------
    @property
    def rng_state(self) -> np.ndarray:
        if self._pending_state is not None:
            return self._pending_state.copy()
        st = np.zeros((self.batch, 4), dtype=np.uint64)
        _check(lib().bs_get_rng_state(self._h, st.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))),
               "bs_get_rng_state")
        return st

    @rng_state.setter
    def rng_state(self, st) -> None:
        a = np.ascontiguousarray(st, dtype=np.uint64).reshape(self.batch, 4)
        if self._pending_state is not None and not self._h:
            self._pending_state = a.copy()
            return
        _check(lib().bs_set_rng_state(self._h, a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))),
               "bs_set_rng_state")

    def set_logit_prologue(self, final_logit_softcapping: float = 0.0, logit_scale: float = 1.0) -> None:
        """The engine's logit prologue (engine.zig:341-354) for every later
        sample(): soft-cap tanh(v / s) * s when s > 0, then v * (1 / logit_scale)
        unless it is 1 or 0; the model's ModelConfig fields (model.zig:34-35)."""
        self._prologue = (float(final_logit_softcapping), float(logit_scale))
        if self._h:
            _check(lib().bs_set_logit_prologue(self._h, *self._prologue), "bs_set_logit_prologue")

    def last_status(self) -> int:
        return lib().bs_last_device_status(self._h)

    def profile_enable(self, max_calls: int) -> None:
        """Record CUDA events around both kernels of the next max_calls calls."""
        _check(lib().bs_profile_enable(self._h, max_calls), "bs_profile_enable")

    def profile_read(self):
        """(n_calls, 3) array of per-call kernel durations in ms: statistics
        pass, main pass, walk/draw pass."""
        cap = 1 << 18
        a = np.zeros(3 * cap, np.float32)
        n = ctypes.c_uint32(0)
        _check(lib().bs_profile_read(self._h, a.ctypes.data, cap, ctypes.byref(n)), "bs_profile_read")
        return a[:3 * n.value].reshape(n.value, 3).copy()

    def traces(self):
        tr = (RowTrace * self.batch)()
        _check(lib().bs_debug_row_traces(self._h, ctypes.addressof(tr), ctypes.sizeof(tr)),
               "bs_debug_row_traces")
        return tr


def sample_argmax(logits, out=None, stream=None, final_logit_softcapping: float = 0.0, logit_scale: float = 1.0):
    """sampleArgmax (sampler.zig:31-41) on each row of a CUDA float32 tensor,
    after the engine's logit prologue when a soft-cap or scale is given."""
    import torch
    x = logits if logits.dim() == 2 else logits.unsqueeze(0)
    if x.dtype != torch.float32 or not x.is_cuda or x.stride(1) != 1:
        raise ValueError("logits must be a CUDA float32 tensor with unit column stride")
    if out is None:
        out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    _check(lib().bs_argmax_ex(x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], final_logit_softcapping,
                              logit_scale, out.data_ptr(), _stream_ptr(stream)), "bs_argmax_ex")
    return out
