"""CPU checks of the seeded synthetic workloads."""
import numpy as np


def test_workloads_are_deterministic_and_row_addressable(pkg):
    w = pkg.workloads.WORKLOADS["c1"]
    a = pkg.workloads.make_logits(w, rows=70)
    b = pkg.workloads.make_logits(w, rows=70)
    assert a.shape == (70, w.vocab) and a.dtype == np.float32
    assert np.array_equal(a, b)
    c = pkg.workloads.make_logits(w, rows=5, row_offset=63)
    assert np.array_equal(c, a[63:68])
    d = pkg.workloads.make_logits(w, step=1, rows=2)
    assert not np.array_equal(d, a[:2])


def test_workload_shapes_and_distributions(pkg):
    W = pkg.workloads.WORKLOADS
    x = pkg.workloads.make_logits(W["c1"], rows=4)
    # 16 spikes of +U(5,15) over 3*N(0,1)
    assert (x > 17).sum() >= 4
    assert abs(np.median(x) ) < 0.05 and 2.8 < np.std(x[:, :50000]) < 3.3
    g = pkg.workloads.make_logits(W["c3_topk1"], rows=3)
    am = g.argmax(1)
    second = np.sort(g, axis=1)[:, -2]
    assert np.all(g[np.arange(3), am] - second > 7.0)
    assert W["headline"].rows == 256 and W["headline"].vocab == 128256
    assert W["c2"].vocab == 151936 and W["c3_greedy"].temperature == 0.0


def test_seeds_are_seed_plus_row(pkg):
    w = pkg.workloads.WORKLOADS["c4"]
    s = w.seeds(4, offset=10)
    assert s.tolist() == [17, 18, 19, 20]
