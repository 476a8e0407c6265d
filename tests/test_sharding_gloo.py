"""The N>1 batch-sharding host logic on CPU: two gloo ranks each sample their
block of a batch with the checker, seeded by global row; the gathered tokens
and RNG states must equal one process sampling the whole batch, and the
timing reduction must return the slowest rank's value."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows_per_rank, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    pkg = graft.load_package()
    orc = graft.load_oracle()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = pkg.workloads.WORKLOADS["c1"]
        sh = pkg.sharding.shard_for(rank, world, rows_per_rank)
        x = pkg.workloads.make_logits(w, rows=rows_per_rank, row_offset=sh.row0, vocab=4096)
        tok, _, st = orc.sample_batch(orc.make_config(**w.config()), x, seeds=sh.seeds(w.seed))
        # gather every rank's block (test only: the data path has no collective)
        t_all = [torch.zeros(rows_per_rank, dtype=torch.int64) for _ in range(world)]
        s_all = [torch.zeros(rows_per_rank * 4, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(t_all, torch.from_numpy(tok.astype(np.int64)))
        dist.all_gather(s_all, torch.from_numpy(st.reshape(-1).view(np.int64).copy()))
        slowest = pkg.sharding.max_over_ranks(10.0 + rank, dist)
        if rank == 0:
            np.savez(os.path.join(out_dir, "shards.npz"),
                     tokens=torch.cat(t_all).numpy(), states=torch.cat(s_all).numpy().view(np.uint64),
                     slowest=np.float64(slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_match_one_process(tmp_path, pkg, orc):
    world, rpr = 2, 6
    mp.start_processes(_rank_main, args=(world, _free_port(), rpr, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    got = np.load(tmp_path / "shards.npz")
    w = pkg.workloads.WORKLOADS["c1"]
    x = pkg.workloads.make_logits(w, rows=world * rpr, vocab=4096)
    tok, _, st = orc.sample_batch(orc.make_config(**w.config()), x, seeds=w.seeds(world * rpr))
    assert np.array_equal(got["tokens"], tok.astype(np.int64))
    assert np.array_equal(got["states"].reshape(-1, 4), st)
    assert float(got["slowest"]) == 11.0


def test_shard_layout():
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    sh = graft.load_package().sharding
    blocks = [list(sh.shard_for(r, 4, 3).rows()) for r in range(4)]
    assert sum(blocks, []) == list(range(12))
    assert list(sh.shard_for(2, 4, 3).seeds(42)) == [48, 49, 50]
    assert sh.aggregate_rows_per_s(sh.shard_for(0, 4, 3), steps=10, seconds=2.0) == 60.0
    assert sh.max_over_ranks(3.5) == 3.5
    with pytest.raises(ValueError):
        sh.shard_for(4, 4, 3)


def _vocab_rank_main(rank, world, port, rows, vocab, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    pkg = graft.load_package()
    orc = graft.load_oracle()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = pkg.workloads.WORKLOADS["c4"]
        full = torch.from_numpy(pkg.workloads.make_logits(w, rows=rows, vocab=vocab))
        lay = pkg.sharding.VocabShard(rank, world, rows, vocab)
        shard = lay.shard_of(full).contiguous()
        mine = pkg.sharding.rows_from_vocab_shards(lay, shard, dist)
        assert torch.equal(mine, full[lay.row0:lay.row0 + lay.rows_per_rank])
        # with a repetition penalty: each rank takes its rows of the history
        hist = torch.from_numpy(np.random.default_rng(9).integers(0, vocab, size=(rows, 12)).astype(np.uint32))
        prev = pkg.sharding.history_rows(lay, hist).numpy()
        tok, _, st = orc.sample_batch(orc.make_config(**w.config(repetition_window=8, repetition_penalty=1.3)),
                                      mine.numpy(), seeds=lay.seeds(w.seed), prev=prev)
        allt = pkg.sharding.gather_tokens(lay, torch.from_numpy(tok.astype(np.int64)), dist)
        if rank == 0:
            np.save(os.path.join(out_dir, "vocab_tokens.npy"), allt.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_vocab_sharded_transpose_matches_one_process(tmp_path, pkg, orc, world):
    rows, vocab = 8, 4096
    mp.start_processes(_vocab_rank_main, args=(world, _free_port(), rows, vocab, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    got = np.load(tmp_path / "vocab_tokens.npy")
    w = pkg.workloads.WORKLOADS["c4"]
    x = pkg.workloads.make_logits(w, rows=rows, vocab=vocab)
    hist = np.random.default_rng(9).integers(0, vocab, size=(rows, 12)).astype(np.uint32)
    tok, _, _ = orc.sample_batch(orc.make_config(**w.config(repetition_window=8, repetition_penalty=1.3)), x,
                                 seeds=w.seeds(rows), prev=hist)
    assert np.array_equal(got, tok.astype(np.int64))


def test_vocab_shard_layout():
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    sh = graft.load_package().sharding
    lay = sh.VocabShard(2, 4, 512, 128256)
    assert (lay.cols, lay.col0, lay.rows_per_rank, lay.row0) == (32064, 64128, 128, 256)
    assert list(lay.seeds(7)[:2]) == [263, 264]
    with pytest.raises(ValueError):
        sh.VocabShard(0, 3, 512, 128256)


def test_vocab_sharded_transport_is_checked():
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    pkg = graft.load_package()
    cfg = pkg.SamplerConfig(top_k=50)
    with pytest.raises(ValueError):
        pkg.sharding.VocabShardedSampler(cfg, 8, 4096, None, transport="shm")
