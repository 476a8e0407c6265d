"""bs_sample_static (static device scratch, no allocation) against the
handle-based bs_sample on the same logits and RNG states, over two
consecutive calls so that the second runs on scratch the first left behind."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _lib(pkg):
    L = pkg.lib()
    vp, u32 = ctypes.c_void_p, ctypes.c_uint32
    L.bs_sample_static.argtypes = [ctypes.POINTER(pkg.sampler.BsConfig), vp, vp, ctypes.c_size_t, u32, u32,
                                   vp, u32, vp, vp]
    L.bs_sample_static.restype = ctypes.c_int
    return L


@pytest.mark.parametrize("name,rows,vocab", [("c1", 4, None), ("c1", 3, 40000), ("headline_topp", 2, None)])
def test_static_scratch_matches_handle_path(gpu_pkg, name, rows, vocab):
    L = _lib(gpu_pkg)
    w = gpu_pkg.workloads.WORKLOADS[name]
    V = vocab or w.vocab
    cfg = gpu_pkg.SamplerConfig(**w.config())
    seeds = w.seeds(rows)
    ref = gpu_pkg.Sampler(cfg, batch=rows, vocab=V, seeds=seeds)
    rng = torch.from_numpy(ref.rng_state.astype(np.uint64).view(np.int64).copy()).cuda()
    c = cfg.to_c()
    for step in range(2):
        x = gpu_pkg.workloads.make_logits(w, step=step, rows=rows)[:, :V]
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        want = ref.sample(xd).cpu().numpy().astype(np.uint32)
        out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        st = L.bs_sample_static(ctypes.byref(c), _ptr(rng), _ptr(xd), ctypes.c_size_t(V), rows, V,
                                None, 0, _ptr(out), None)
        assert st == 0, gpu_pkg.status_string(st)
        torch.cuda.synchronize()
        got = out.cpu().numpy().astype(np.uint32)
        assert np.array_equal(got, want), (step, got, want)
        assert np.array_equal(rng.cpu().numpy().view(np.uint64), ref.rng_state), step
    ref.close()


def test_static_scratch_rejects_oversize(gpu_pkg):
    L = _lib(gpu_pkg)
    c = gpu_pkg.SamplerConfig(temperature=1.0).to_c()
    x = torch.zeros((5, 1000), dtype=torch.float32, device="cuda")
    rng = torch.zeros((5, 4), dtype=torch.int64, device="cuda")
    out = torch.zeros(5, dtype=torch.int32, device="cuda")
    assert L.bs_sample_static(ctypes.byref(c), _ptr(rng), _ptr(x), ctypes.c_size_t(1000), 5, 1000,
                              None, 0, _ptr(out), None) == 1
    big = torch.zeros((1, 140000), dtype=torch.float32, device="cuda")
    assert L.bs_sample_static(ctypes.byref(c), _ptr(rng), _ptr(big), ctypes.c_size_t(140000), 1, 140000,
                              None, 0, _ptr(out), None) == 1


def test_static_scratch_matches_checker(gpu_pkg, orc):
    # the allocation-free entry point directly against the CPU checker, with
    # a repetition-penalty history, over two calls (RNG states carried on the
    # device by the caller)
    L = _lib(gpu_pkg)
    w = gpu_pkg.workloads.WORKLOADS["c1"]
    rows, V = 4, w.vocab
    cfgd = w.config(repetition_window=16, repetition_penalty=1.3)
    c = gpu_pkg.SamplerConfig(**cfgd).to_c()
    seeds = w.seeds(rows)
    states = np.stack([orc.rng_seed(int(sd)) for sd in seeds])
    rng = torch.from_numpy(states.astype(np.uint64).view(np.int64).copy()).cuda()
    prev = np.random.default_rng(4).integers(0, V, size=(rows, 20)).astype(np.uint32)
    pd = torch.from_numpy(prev.astype(np.int32)).cuda()
    for step in range(2):
        x = gpu_pkg.workloads.make_logits(w, step=step, rows=rows)
        xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        st = L.bs_sample_static(ctypes.byref(c), _ptr(rng), _ptr(xd), ctypes.c_size_t(V), rows, V,
                                _ptr(pd), 20, _ptr(out), None)
        assert st == 0, gpu_pkg.status_string(st)
        torch.cuda.synchronize()
        exp, _, states = orc.sample_batch(orc.make_config(**cfgd), x, states=states, prev=prev)
        assert np.array_equal(out.cpu().numpy().astype(np.uint32), exp), step
        assert np.array_equal(rng.cpu().numpy().view(np.uint64), states), step
