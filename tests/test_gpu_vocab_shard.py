"""Vocab-sharded sampling (config 4) on two GPUs over NCCL: every rank passes
its (B, V/2) shard and must get the checker's tokens for all B rows.  Skipped
with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, rows, out_dir, transport):
    import datetime
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    pkg = graft.load_package()
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = pkg.workloads.WORKLOADS["c4"]
        vs = pkg.sharding.VocabShardedSampler(pkg.SamplerConfig(**w.config()), rows, w.vocab, dist, device=rank,
                                              transport=transport)
        assert vs.p2p == (transport == "p2p")
        toks = []
        shards = [torch.from_numpy(np.ascontiguousarray(vs.lay.shard_of(pkg.workloads.make_logits(w, step=step, rows=rows))))
                  for step in range(3)]
        # step 0 eager; steps 1 and 2 replayed from one CUDA graph of the
        # whole step (collectives included) on a static shard buffer
        buf = shards[0].cuda()
        toks.append(vs.sample(buf).cpu().numpy())
        g, out = vs.graph(buf)
        for step in (1, 2):
            buf.copy_(shards[step])
            g.replay()
            toks.append(out.cpu().numpy())
        torch.cuda.synchronize()
        del g
        vs.close()
        np.save(os.path.join(out_dir, f"tok{rank}.npy"), np.stack(toks))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_vocab_sharded_two_gpus(tmp_path, orc, transport):
    # nccl: the chain of walks as one broadcast per link; p2p: the chain
    # inside the walk kernels through peer memory (CUDA IPC over NVLink)
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__ as graft
    pkg = graft.load_package()
    rows = 32
    mp.start_processes(_rank, args=(2, _port(), rows, str(tmp_path), transport), nprocs=2, join=True,
                       start_method="spawn")
    w = pkg.workloads.WORKLOADS["c4"]
    states = None
    for step in range(3):
        x = pkg.workloads.make_logits(w, step=step, rows=rows)
        exp, _, states = orc.sample_batch(orc.make_config(**w.config()), x,
                                          seeds=w.seeds(rows) if states is None else None, states=states)
        for r in range(2):
            got = np.load(tmp_path / f"tok{r}.npy")[step]
            assert np.array_equal(got.astype(np.uint32), exp), (step, r)
