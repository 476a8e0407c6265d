"""GPU parity: the CUDA sampler (through the C ABI) against the CPU checker.

Token ids, the RNG state after every call and the reference's own f32
intermediates (the sequential normaliser S, the kept mass, the uniform draw)
must be bit-identical: the CUDA path reproduces sampler.zig's f32 operation
order exactly, so no tolerance is needed.
"""
import glob
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

HERE = os.path.dirname(os.path.abspath(__file__))
pytestmark = pytest.mark.gpu


def f32bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def run_gpu(gpu_pkg, c, logits_steps, seeds, prev_steps=None):
    """Sample `steps` batches on the GPU; returns tokens, states, traces."""
    steps, rows, V = logits_steps.shape
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=rows, vocab=V, seeds=seeds)
    toks, states, traces = [], [], []
    for i in range(steps):
        x = torch.from_numpy(np.ascontiguousarray(logits_steps[i])).cuda()
        pv = None if prev_steps is None else torch.from_numpy(prev_steps[i].astype(np.int32)).cuda()
        out = s.sample(x, pv)
        torch.cuda.synchronize()
        toks.append(out.cpu().numpy().astype(np.uint32))
        states.append(s.rng_state)
        traces.append([(t.S, t.total, t.u, t.path, t.status, t.flags) for t in s.traces()])
    s.close()
    return np.array(toks), np.array(states), traces


def run_oracle(orc, c, logits_steps, seeds, prev_steps=None):
    oc = orc.make_config(**c)
    states = None
    toks, sts, trs = [], [], []
    for i in range(logits_steps.shape[0]):
        out, tr, states = orc.sample_batch(oc, logits_steps[i], seeds=seeds if states is None else None,
                                           states=states, prev=None if prev_steps is None else prev_steps[i],
                                           nthreads=os.cpu_count() or 1)
        toks.append(out)
        sts.append(states)
        trs.append([(t.sum, t.total, t.u, t.path) for t in tr])
    return np.array(toks), np.array(sts), trs


def assert_same(gpu, ref, what=""):
    gt, gs, gtr = gpu
    rt, rs, rtr = ref
    bad = np.argwhere(gt != rt)
    if len(bad):
        i, r = bad[0]
        raise AssertionError(f"{what}: {len(bad)} token mismatches; first step {i} row {r}: "
                             f"gpu {gt[i, r]} ref {rt[i, r]}; gpu trace {gtr[i][r]} ref trace {rtr[i][r]}")
    assert np.array_equal(gs, rs), f"{what}: RNG states differ"
    for i in range(len(gtr)):
        for r in range(len(gtr[i])):
            g, o = gtr[i][r], rtr[i][r]
            assert g[4] == 0, f"{what}: row status {g}"
            if o[3] >= 2:   # S was computed (not the T<=0 path)
                assert f32bits(g[0]) == f32bits(o[0]) or (np.isnan(g[0]) and np.isnan(o[0])), \
                    f"{what}: S differs at step {i} row {r}: {g[0]!r} vs {o[0]!r}"


# ---------------------------------------------------------------------------
def test_reference_tests_through_c_abi(gpu_pkg):
    # sampler.zig:171-193: two samplers with the same seed agree
    c = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, typical_p=1.0, seed=1234,
             repetition_window=0, repetition_penalty=1.0)
    z = np.zeros((8, 1, 4), np.float32)
    a = run_gpu(gpu_pkg, c, z, seeds=[1234])[0].ravel().tolist()
    b = run_gpu(gpu_pkg, c, z, seeds=[1234])[0].ravel().tolist()
    assert a == b
    # sampler.zig:195-213: top_k = 1 always returns the argmax
    c.update(top_k=1, seed=1)
    x = np.tile(np.array([2.0, 1.9, 1.8], np.float32), (16, 1, 1))
    assert run_gpu(gpu_pkg, c, x, seeds=[1])[0].ravel().tolist() == [0] * 16


def test_xoshiro256pp_known_answer_on_gpu(gpu_pkg):
    # the published xoshiro256++ vector from the state {1, 2, 3, 4}: one draw
    # consumes the first output, 41943041, whose Random.float(f32) value is
    # 2^-39 (1 + 2^-23); the state then is {7, 0, 262146, 6 * 2^45}
    c = gpu_pkg.SamplerConfig(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, typical_p=1.0, seed=1,
                              repetition_window=0, repetition_penalty=1.0)
    s = gpu_pkg.Sampler(c, batch=1, vocab=4)
    s.rng_state = np.array([[1, 2, 3, 4]], np.uint64)
    tok = s.sample(torch.zeros((1, 4), dtype=torch.float32, device="cuda"))
    torch.cuda.synchronize()
    assert int(tok.cpu()[0]) == 0          # r = u * 1 <= 0.25: the first token
    tr = s.traces()[0]
    assert np.float32(tr.u) == np.float32(2.0 ** -39 * (1 + 2.0 ** -23))
    assert s.rng_state.tolist() == [[7, 0, 262146, 6 << 45]]
    s.close()


GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_golden_fixtures_on_gpu(gpu_pkg, path):
    name = os.path.basename(path)[:-4]
    f = np.load(path)
    c = json.loads(str(f["config"]))
    prev = f["prev"] if "prev" in f.files else None
    toks, states, traces = run_gpu(gpu_pkg, c, f["logits"], f["seeds"], prev)
    assert np.array_equal(toks, f["tokens"]), f"{name}: {toks.ravel()[:12]} vs {f['tokens'].ravel()[:12]}"
    if c["temperature"] > 0:
        assert np.array_equal(states, f["states"])
        for i in range(len(traces)):
            for r in range(len(traces[i])):
                g = traces[i][r]
                o = f["traces"][i, r]
                if o[3] >= 2:
                    assert f32bits(g[0]) == f32bits(o[0]) or (np.isnan(g[0]) and np.isnan(o[0])), (i, r, g, o)


@pytest.mark.parametrize("V", [1, 2, 31, 33, 1025, 16385, 40000])
def test_odd_vocab_sizes(gpu_pkg, orc, V):
    rng = np.random.default_rng(V)
    x = (3 * rng.standard_normal((2, 4, V))).astype(np.float32)
    c = dict(temperature=0.9, top_k=0, top_p=0.9, min_p=0.0, typical_p=1.0, seed=77,
             repetition_window=0, repetition_penalty=1.0)
    seeds = np.arange(4, dtype=np.uint64) + 77
    assert_same(run_gpu(gpu_pkg, c, x, seeds), run_oracle(orc, c, x, seeds), f"V={V}")


@pytest.mark.parametrize("scale,min_p", [(0.3, 0.0), (2.5, 0.0), (3.0, 0.0), (3.0, 0.002)])
def test_top_p_large_kept_sets(gpu_pkg, orc, scale, min_p):
    # flat rows: top-p keeps thousands of tokens (past the shared-memory
    # candidate sort and past the stored running sums of the kept mass), and
    # min-p may cut the top-p prefix further
    rng = np.random.default_rng(int(scale * 10) + int(min_p * 100))
    x = (scale * rng.standard_normal((1, 6, 50000))).astype(np.float32)
    c = dict(temperature=1.0, top_k=0, top_p=0.9, min_p=min_p, typical_p=1.0, seed=5,
             repetition_window=0, repetition_penalty=1.0)
    seeds = np.arange(6, dtype=np.uint64) + 5
    assert_same(run_gpu(gpu_pkg, c, x, seeds), run_oracle(orc, c, x, seeds), f"scale={scale} min_p={min_p}")


def _workload(pkg, name, rows, steps=1):
    w = pkg.workloads.WORKLOADS[name]
    x = np.stack([pkg.workloads.make_logits(w, step=s, rows=rows) for s in range(steps)])
    return w, x


# every configuration at its full batch (c4's 512 rows on one GPU here; its
# vocabulary-sharded form is tested in test_gpu_vocab_shard.py)
@pytest.mark.parametrize("name,rows,steps", [
    ("c1", 64, 2),
    ("headline", 256, 1),
    ("headline_topp", 256, 1),
    ("c2", 256, 1),
    ("c4", 512, 1),
    ("c0", 1, 40),
])
def test_benchmark_configs_match_checker(gpu_pkg, orc, name, rows, steps):
    w, x = _workload(gpu_pkg, name, rows, steps)
    c = w.config()
    seeds = w.seeds(rows)
    assert_same(run_gpu(gpu_pkg, c, x, seeds), run_oracle(orc, c, x, seeds), name)


def test_topk1_large_vocab(gpu_pkg, orc):
    # config 3's top_k = 1 run at its full size, 1024 rows x 256000
    w, x = _workload(gpu_pkg, "c3_topk1", 1024)
    c = w.config()
    seeds = w.seeds(1024)
    assert_same(run_gpu(gpu_pkg, c, x, seeds), run_oracle(orc, c, x, seeds), "c3_topk1")


def test_greedy_full_size_property(gpu_pkg):
    # config 3 (T=0) at full size: the first index of the row maximum
    w = gpu_pkg.workloads.WORKLOADS["c3_greedy"]
    x = gpu_pkg.workloads.make_logits(w, rows=w.rows)
    out = gpu_pkg.sample_argmax(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(out, np.argmax(x, axis=1))


def test_host_path_matches_device_path(gpu_pkg, orc):
    w, x = _workload(gpu_pkg, "c1", 16)
    c = w.config()
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=16, vocab=w.vocab, seeds=w.seeds(16))
    got = s.sample(x[0])           # numpy in -> bs_sample_host
    exp, _, st = orc.sample_batch(orc.make_config(**c), x[0], seeds=w.seeds(16))
    assert np.array_equal(got, exp)
    assert np.array_equal(s.rng_state, st)


def test_sampler_init_binds_lazily_like_the_reference(gpu_pkg, orc):
    # the drop-in's life cycle: Sampler.init(cfg) with no vocabulary
    # (sampler.zig:19-24), then sample(allocator, logits, prev) per token
    # (sampler.zig:26-28, engine.zig:355) with the history growing; a second
    # vocabulary rebinds the handle and keeps the xoshiro256++ stream
    cfgd = dict(temperature=0.7, top_k=40, top_p=0.95, min_p=0.05, seed=4242,
                repetition_window=16, repetition_penalty=1.3)
    s = gpu_pkg.Sampler.init(gpu_pkg.SamplerConfig(**cfgd))
    r = orc.Sampler(orc.make_config(**cfgd))
    rng = np.random.default_rng(11)
    hist = []
    for step in range(12):
        V = 3001 if step < 8 else 5003
        x = (rng.standard_normal(V) * 3).astype(np.float32)
        if step % 2:
            got = s.sample(x, prev_tokens=np.array(hist, dtype=np.uint32) if hist else None)
        else:
            pt = torch.tensor(hist, dtype=torch.int32).cuda() if hist else None
            got = int(s.sample(torch.from_numpy(x).cuda(), prev_tokens=pt).cpu()[0])
        exp = r.sample(x, np.array(hist, dtype=np.uint32) if hist else None)
        assert got == exp, step
        hist.append(got)
    assert np.array_equal(s.rng_state[0], r.state)
    s.close()


def test_rng_state_roundtrip_and_resync(gpu_pkg, orc):
    w, x = _workload(gpu_pkg, "c1", 4, steps=3)
    c = w.config()
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=4, vocab=w.vocab, seeds=w.seeds(4))
    st = s.rng_state
    ref = np.stack([orc.rng_seed(int(sd)) for sd in w.seeds(4)])
    assert np.array_equal(st, ref)
    s.sample(torch.from_numpy(x[0]).cuda())
    s.rng_state = st                      # rewind and replay
    a = s.sample(torch.from_numpy(x[1]).cuda()).cpu().numpy()
    exp, _, _ = orc.sample_batch(orc.make_config(**c), x[1], states=st)
    assert np.array_equal(a.astype(np.uint32), exp)


def test_special_values_rows(gpu_pkg, orc):
    V = 5000
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1, 6, V)).astype(np.float32)
    x[0, 0, 100] = np.nan
    x[0, 1, 200] = np.inf
    x[0, 2, :] = -np.inf
    x[0, 3, 0] = np.nan
    x[0, 4, :] = 1.0          # all equal: every token ties
    x[0, 5, 7] = 1e30
    for c in [dict(temperature=1.0, top_p=0.9), dict(temperature=1e-20, top_p=0.5),
              dict(temperature=float("inf"), top_k=3), dict(temperature=0.5, min_p=0.2)]:
        cc = dict(top_k=0, top_p=1.0, min_p=0.0, typical_p=1.0, seed=5, repetition_window=0,
                  repetition_penalty=1.0)
        cc.update(c)
        seeds = np.arange(6, dtype=np.uint64) + 5
        assert_same(run_gpu(gpu_pkg, cc, x, seeds), run_oracle(orc, cc, x, seeds), str(c))


def test_repetition_penalty(gpu_pkg, orc):
    w, x = _workload(gpu_pkg, "c1", 8, steps=2)
    rng = np.random.default_rng(1)
    prev = rng.integers(0, w.vocab, size=(2, 8, 40)).astype(np.uint32)
    top = np.argsort(-x, axis=2)[:, :, :5]          # penalise the likely tokens
    prev[:, :, -5:] = top
    prev[:, :, -6] = prev[:, :, -1]                 # a repeated id is penalised once
    c = w.config(repetition_window=16, repetition_penalty=1.5)
    seeds = w.seeds(8)
    assert_same(run_gpu(gpu_pkg, c, x, seeds, prev), run_oracle(orc, c, x, seeds, prev), "penalty")


@pytest.mark.parametrize("window,n_prev", [(300, 400), (1000, 400), (5000, 6000)])
def test_repetition_penalty_long_window(gpu_pkg, orc, window, n_prev):
    # windows of any length (sampler.zig:58: the last min(n_prev, window) ids):
    # the likely tokens sit inside the window, decoys just before it must stay
    # unpenalised, ids past the vocabulary match nothing
    w, x = _workload(gpu_pkg, "c1", 6, steps=1)
    rng = np.random.default_rng(window)
    prev = rng.integers(0, w.vocab, size=(1, 6, n_prev)).astype(np.uint32)
    order = np.argsort(-x, axis=2)
    win = min(window, n_prev)
    prev[:, :, n_prev - win:n_prev - win + 4] = order[:, :, :4]      # oldest ids inside the window
    prev[:, :, n_prev - 3] = order[:, :, 0]                          # repeated: penalised once
    prev[:, :, n_prev - 2] = w.vocab + 7                             # outside the vocabulary
    if n_prev > win:
        prev[:, :, n_prev - win - 1] = order[:, :, 4]                # just outside the window
    c = w.config(repetition_window=window, repetition_penalty=1.3)
    seeds = w.seeds(6)
    assert_same(run_gpu(gpu_pkg, c, x, seeds, prev), run_oracle(orc, c, x, seeds, prev),
                f"penalty window={window} n_prev={n_prev}")


def test_certificate_bound_holds(gpu_pkg):
    # the main pass accepts a fast-exp grid count only when it is certified;
    # every certified count must equal the exact one (cert_eps in sampler.cu)
    import ctypes
    L = gpu_pkg.lib()
    L.bs_debug_cert_check.argtypes = [ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p]
    L.bs_debug_cert_check.restype = ctypes.c_int
    out = np.zeros(3, np.uint64)
    for seed in range(4):
        assert L.bs_debug_cert_check(1 << 22, seed, out.ctypes.data) == 0
        bad, certified, total = (int(v) for v in out)
        assert total > (1 << 20)
        assert bad == 0, f"{bad} certified counts differ from the exact ones (seed {seed})"
        assert certified > total // 2


def test_window_crossing_search_exhaustive(gpu_pkg):
    # the walker's search for the tile where a WINDOW stretch leaves its
    # binade (find_crossing in sampler.cu): every stretch length up to 300
    # tiles, every crossing position, both entry parities
    import ctypes
    L = gpu_pkg.lib()
    L.bs_debug_crossing_check.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
    L.bs_debug_crossing_check.restype = ctypes.c_int
    out = np.zeros(2, np.uint64)
    assert L.bs_debug_crossing_check(300, out.ctypes.data) == 0
    bad, cases = (int(v) for v in out)
    assert cases == 2 * sum(range(1, 301))
    assert bad == 0, f"{bad} of {cases} crossing searches wrong"


def test_entropy_certificate_bound_holds(gpu_pkg):
    # the entropy pass's certificate (cert_eps_h): seeds with the top bit set
    # select the entropy-term check
    import ctypes
    L = gpu_pkg.lib()
    L.bs_debug_cert_check.argtypes = [ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p]
    L.bs_debug_cert_check.restype = ctypes.c_int
    out = np.zeros(3, np.uint64)
    for seed in range(4):
        assert L.bs_debug_cert_check(1 << 22, (1 << 63) | seed, out.ctypes.data) == 0
        bad, certified, total = (int(v) for v in out)
        assert total > (1 << 20)
        assert bad == 0, f"{bad} certified entropy counts differ from the exact ones (seed {seed})"
        assert certified > total // 4


def _typical_case(gpu_pkg, orc, c, x, seeds, what):
    """Tokens, RNG states, S and the entropy H bit for bit."""
    rows, V = x.shape
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=rows, vocab=V, seeds=seeds)
    tok = s.sample(torch.from_numpy(x).cuda()).cpu().numpy().astype(np.uint32)
    torch.cuda.synchronize()
    tr = s.traces()
    st = s.rng_state
    s.close()
    exp, otr, ost = orc.sample_batch(orc.make_config(**c), x, seeds=seeds)
    for r in range(rows):
        assert tr[r].status == 0, f"{what}: row {r} status {tr[r].status} flags {tr[r].flags}"
    bad = np.flatnonzero(tok != exp)
    assert len(bad) == 0, f"{what}: rows {bad[:8]} gpu {tok[bad[:8]]} ref {exp[bad[:8]]}"
    assert np.array_equal(st, ost), f"{what}: RNG states differ"
    for r in range(rows):
        if otr[r].path >= 2 and np.isfinite(otr[r].entropy):
            assert f32bits(tr[r].H) == f32bits(otr[r].entropy), (what, r, tr[r].H, otr[r].entropy)
            assert f32bits(tr[r].S) == f32bits(otr[r].sum), (what, r)


@pytest.mark.parametrize("rows,vocab", [(16, 151936), (8, 40000)])
def test_typical_alone_matches_checker(gpu_pkg, orc, rows, vocab):
    # config 2: typical_p = 0.9 alone (the dev band path)
    w = gpu_pkg.workloads.WORKLOADS["c2"]
    x = gpu_pkg.workloads.make_logits(w, rows=rows, vocab=vocab)
    _typical_case(gpu_pkg, orc, w.config(), x, w.seeds(rows), f"c2 V={vocab}")


@pytest.mark.parametrize("extra", [dict(top_k=40), dict(top_p=0.95), dict(min_p=0.05),
                                   dict(top_k=200, top_p=0.9, min_p=0.01)])
def test_typical_with_other_filters(gpu_pkg, orc, extra):
    # typical-p over the selected set of another filter
    w = gpu_pkg.workloads.WORKLOADS["c2"]
    x = gpu_pkg.workloads.make_logits(w, rows=8, vocab=50000)
    _typical_case(gpu_pkg, orc, w.config(**extra), x, w.seeds(8), str(extra))


def test_config0_thousand_sequential_steps(gpu_pkg, orc):
    # config 0 as the CLI runs it: B=1, 1000 steps of fresh logits, one
    # persistent RNG state; every token and the final state bit-exact
    w = gpu_pkg.workloads.WORKLOADS["c0"]
    c = w.config()
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=1, vocab=w.vocab, seeds=w.seeds(1))
    oc = orc.make_config(**c)
    states = None
    d = torch.empty((1, w.vocab), dtype=torch.float32, device="cuda")
    for step in range(w.steps):
        x = gpu_pkg.workloads.make_logits(w, step=step, rows=1)
        d.copy_(torch.from_numpy(x))
        got = int(s.sample(d).cpu().numpy()[0])
        exp, _, states = orc.sample_batch(oc, x, seeds=w.seeds(1) if states is None else None, states=states)
        assert got == int(exp[0]), f"step {step}: gpu {got} ref {int(exp[0])}"
    assert np.array_equal(s.rng_state, states)
    s.close()


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("name,rows", [("c1", 64), ("headline_topp", 256), ("c2", 64), ("c3_topk1", 64),
                                       ("headline", 256), ("c4", 512)])
def test_persistent_kernel_matches_checker(gpu_pkg, orc, name, rows, mode):
    # the persistent-kernel forms of the statistics, row reduction and main
    # pass (one launch, tasks claimed from device counters) against the
    # checker: 1 the task queue, 2 the read-once kernel (a CTA keeps its
    # segment from the statistics to the main pass)
    import ctypes
    L = gpu_pkg.sampler.lib()
    L.bs_debug_set_fused.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
    w, x = _workload(gpu_pkg, name, rows, steps=2)
    c = w.config()
    seeds = w.seeds(rows)
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=rows, vocab=w.vocab, seeds=seeds)
    assert L.bs_debug_set_fused(s._h, mode) == 0
    toks, states = [], []
    for i in range(2):
        toks.append(s.sample(torch.from_numpy(x[i]).cuda()).cpu().numpy().astype(np.uint32))
        states.append(s.rng_state)
        assert s.last_status() == 0
    s.close()
    ref = run_oracle(orc, c, x, seeds)
    assert np.array_equal(np.array(toks), ref[0]), name
    assert np.array_equal(np.array(states), ref[1]), name


@pytest.mark.parametrize("softcap,scale,fused", [(30.0, 1.0, 0), (0.0, 8.0, 0), (30.0, 0.5, 0), (30.0, 8.0, 1),
                                                 (30.0, 8.0, 2), (0.0, 1.0, 2)])
def test_logit_prologue_matches_checker(gpu_pkg, orc, softcap, scale, fused):
    # the engine's prologue (engine.zig:341-354: soft-cap, then 1 / logit_scale)
    # fused into the sampler, with a repetition penalty on top; the checker
    # samples the logits the engine would hand it
    import ctypes
    w, x = _workload(gpu_pkg, "c1", 16, steps=2)
    rng = np.random.default_rng(5)
    prev = rng.integers(0, w.vocab, size=(2, 16, 24)).astype(np.uint32)
    prev[:, :, -3:] = np.argsort(-x, axis=2)[:, :, :3]
    c = w.config(repetition_window=16, repetition_penalty=1.3)
    seeds = w.seeds(16)
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=16, vocab=w.vocab, seeds=seeds)
    s.set_logit_prologue(softcap, scale)
    L = gpu_pkg.sampler.lib()
    L.bs_debug_set_fused.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
    L.bs_debug_set_fused(s._h, fused)
    toks, states = [], []
    for i in range(2):
        pv = torch.from_numpy(prev[i].astype(np.int32)).cuda()
        toks.append(s.sample(torch.from_numpy(x[i]).cuda(), pv).cpu().numpy().astype(np.uint32))
        states.append(s.rng_state)
        assert s.last_status() == 0
    s.close()
    xp = np.stack([orc.prologue(x[i], softcap, scale) for i in range(2)])
    ref = run_oracle(orc, c, xp, seeds, prev)
    assert np.array_equal(np.array(toks), ref[0])
    assert np.array_equal(np.array(states), ref[1])


@pytest.mark.parametrize("softcap,scale", [(30.0, 1.0), (0.0, 8.0), (5.0, 0.25)])
def test_argmax_after_prologue(gpu_pkg, orc, softcap, scale):
    # T <= 0 (sampler.zig:50) on the engine's logits: the soft-cap saturates
    # large logits to equal values, so the first of them wins
    w = gpu_pkg.workloads.WORKLOADS["c3_greedy"]
    x = gpu_pkg.workloads.make_logits(w, rows=64, vocab=20000)
    x[:, 7] = 500.0
    x[:, 3000] = 400.0              # both saturate under a small soft-cap
    got = gpu_pkg.sample_argmax(torch.from_numpy(x).cuda(), final_logit_softcapping=softcap,
                                logit_scale=scale).cpu().numpy()
    ref = np.array([orc.argmax(orc.prologue(x[r], softcap, scale)) for r in range(64)])
    assert np.array_equal(got, ref)
    c = dict(temperature=0.0, top_k=0, top_p=1.0, min_p=0.0, typical_p=1.0, seed=1,
             repetition_window=0, repetition_penalty=1.0)
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=64, vocab=20000)
    s.set_logit_prologue(softcap, scale)
    assert np.array_equal(s.sample(torch.from_numpy(x).cuda()).cpu().numpy(), ref)
    s.close()


@pytest.mark.parametrize("world,rows,extras", [(2, 64, False), (4, 64, True), (8, 32, False), (2, 512, False)])
def test_vocab_sharded_exact_merge_emulated(gpu_pkg, orc, world, rows, extras):
    # config 4's exact partial merge with `world` ranks emulated on one GPU
    # (the collectives are copies): every rank's tokens and RNG states equal
    # one sampler's over the whole rows, over two steps; with extras, a
    # repetition penalty and the logit prologue on every shard
    sh = gpu_pkg.sharding
    w = gpu_pkg.workloads.WORKLOADS["c4"]
    c = w.config(repetition_window=16, repetition_penalty=1.3) if extras else w.config()
    cfg = gpu_pkg.SamplerConfig(**c)
    lays = [sh.VocabShard(g, world, rows, w.vocab) for g in range(world)]
    states = [sh._ShardState(cfg, lay, 0, lay.all_seeds(w.seed)) for lay in lays]
    if extras:
        for st in states:
            st.smp.set_logit_prologue(30.0, 2.0)
    rng = np.random.default_rng(world)
    x = np.stack([gpu_pkg.workloads.make_logits(w, step=s, rows=rows) for s in range(2)])
    prev = rng.integers(0, w.vocab, size=(2, rows, 24)).astype(np.uint32) if extras else None
    if extras:
        prev[:, :, -3:] = np.argsort(-x, axis=2)[:, :, :3]
    toks = []
    for s in range(2):
        shards = [torch.from_numpy(np.ascontiguousarray(lay.shard_of(x[s]))).cuda() for lay in lays]
        pv = None if prev is None else [torch.from_numpy(prev[s].astype(np.int32)).cuda()] * world
        out = sh.sample_vocab_sharded_emulated(states, shards, pv)
        got = [o.cpu().numpy().astype(np.uint32) for o in out]
        for g in range(1, world):
            assert np.array_equal(got[g], got[0])
        toks.append(got[0])
        for st in states:
            assert st.smp.last_status() == 0
    xr = np.stack([orc.prologue(x[s], 30.0, 2.0) for s in range(2)]) if extras else x
    ref = run_oracle(orc, c, xr, w.seeds(rows), prev)
    assert np.array_equal(np.array(toks), ref[0])
    for st in states:
        assert np.array_equal(st.smp.rng_state, ref[1][-1])
        st.smp.close()


RF_FULL = 1 << 5


@pytest.mark.parametrize("name,rows,vocab,extra", [
    ("c1", 12, 128256, {}),
    ("headline_topp", 8, 128256, {}),
    ("c3_topk1", 4, 256000, {}),
    ("c2", 8, 151936, {}),                       # typical-p alone: the band's retry
    ("c2", 6, 50000, dict(top_k=200, min_p=0.01)),   # typical-p over a selected set
    ("c1", 6, 40000, dict(top_k=0, top_p=1.0, min_p=0.0)),   # nothing filtered: every token kept
])
def test_full_vocabulary_retry_matches_checker(gpu_pkg, orc, name, rows, vocab, extra):
    # the path of rows whose candidates (or typical-p band) fail their cover
    # check: the whole vocabulary sorted by the CTA.  The test hook sends
    # every row through it, with penalised history and the logit prologue
    import ctypes
    L = gpu_pkg.sampler.lib()
    L.bs_debug_set_force_full.argtypes = [ctypes.c_void_p, ctypes.c_uint32]
    w = gpu_pkg.workloads.WORKLOADS[name]
    c = dict(w.config(), **extra)
    x = gpu_pkg.workloads.make_logits(w, rows=rows, vocab=vocab)
    seeds = w.seeds(rows)
    rng = np.random.default_rng(5)
    prev = rng.integers(0, vocab, size=(rows, 24)).astype(np.uint32)
    c = dict(c, repetition_penalty=1.2, repetition_window=20)
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=rows, vocab=vocab, seeds=seeds)
    assert L.bs_debug_set_force_full(s._h, 1) == 0
    got = s.sample(torch.from_numpy(x).cuda(), prev_tokens=torch.from_numpy(prev.astype(np.int32)).cuda())
    got = got.cpu().numpy().astype(np.uint32)
    torch.cuda.synchronize()
    tr = s.traces()
    st = s.rng_state
    s.close()
    exp, _, ost = orc.sample_batch(orc.make_config(**c), x, seeds=seeds, prev=prev)
    for r in range(rows):
        assert tr[r].status == 0, (name, r, tr[r].status, tr[r].flags)
    if c["temperature"] > 0:
        assert all(tr[r].flags & RF_FULL for r in range(rows)), [tr[r].flags for r in range(rows)]
    bad = np.flatnonzero(got != exp)
    assert len(bad) == 0, f"{name}: rows {bad[:8]} gpu {got[bad[:8]]} ref {exp[bad[:8]]}"
    assert np.array_equal(st, ost)


def test_cuda_graph_capture_matches_eager(gpu_pkg, orc):
    # the device-resident decode step: bs_sample captured into a CUDA graph
    # (static input, history and output buffers, no host synchronisation)
    # and replayed token after token gives the eager tokens and RNG states,
    # which match the checker
    w, x = _workload(gpu_pkg, "c1", 8, steps=4)
    c = w.config(repetition_window=16, repetition_penalty=1.3)
    seeds = w.seeds(8)
    rng = np.random.default_rng(3)
    prev = rng.integers(0, w.vocab, size=(4, 8, 20)).astype(np.uint32)
    s = gpu_pkg.Sampler(gpu_pkg.SamplerConfig(**c), batch=8, vocab=w.vocab, seeds=seeds)
    st0 = s.rng_state
    eager = []
    for i in range(4):
        pv = torch.from_numpy(prev[i].astype(np.int32)).cuda()
        eager.append(s.sample(torch.from_numpy(x[i]).cuda(), pv).cpu().numpy().astype(np.uint32))
    st_e = s.rng_state
    s.rng_state = st0
    xin = torch.empty((8, w.vocab), dtype=torch.float32, device="cuda")
    hin = torch.empty((8, 20), dtype=torch.int32, device="cuda")
    out = torch.empty(8, dtype=torch.int32, device="cuda")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        s.sample(xin, hin, out=out)
    graph = []
    for i in range(4):
        xin.copy_(torch.from_numpy(x[i]))
        hin.copy_(torch.from_numpy(prev[i].astype(np.int32)))
        g.replay()
        graph.append(out.cpu().numpy().astype(np.uint32))
    st_g = s.rng_state
    assert s.last_status() == 0
    del g
    s.close()
    assert np.array_equal(np.array(graph), np.array(eager))
    assert np.array_equal(st_g, st_e)
    ref = run_oracle(orc, c, x, seeds, prev)
    assert np.array_equal(np.array(graph), ref[0])
