#!/usr/bin/env python
"""Benchmark of the B200 token sampler: rows sampled per second.

Metric: rows sampled/s at V=128256, B=256, fp32 logits, with
config 1's filters (T=0.7, top_k=40, top_p=0.95, min_p=0.05), and the achieved
HBM GB/s of the dominant kernel against the measured B200 peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

One step = one bs_sample call over one batch of B rows resident in HBM.  Four
distinct batches rotate (4 x 131 MB > the 126 MB L2), so no step reads logits
left in L2 by the previous one.  Under torchrun each rank samples its own B
rows (weak scaling, seeds keyed by the global row); the data path has no
collective.  `--impl reference` times the reference algorithm on the host
cores instead (the C restatement of sampler.zig, all threads).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
import __graft_entry__ as graft  # noqa: E402

ROTATE = 4
NVML_REASONS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
    0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(workload):
    """DRAM bytes of one sampling step (the three kernels) from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p))
    e = d.get(workload)
    return None if e is None else e.get("dram_bytes_per_launch")


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML while running."""

    def __init__(self, device: int):
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._nv is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for b, n in NVML_REASONS.items() if self.reasons & b]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def workload_desc(w):
    return (f"{w.name}: B={w.rows} V={w.vocab} T={w.temperature} top_k={w.top_k} top_p={w.top_p} "
            f"min_p={w.min_p} typical_p={w.typical_p}")


def cpu_baseline(pkg, w, budget_s: float, nthreads: int, x=None):
    """The checker (C restatement of sampler.zig, single-threaded per row like
    the reference) on the host cores: rows spread over all `nthreads` threads,
    and one core alone, each on a bounded sample of the workload's rows."""
    orc = graft.load_oracle()
    cfg = orc.make_config(**w.config())
    if x is None:
        x = pkg.workloads.make_logits(w, rows=min(w.rows, max(nthreads, 16)))

    def timed(threads, rows_min, budget):
        done, t0 = 0, time.perf_counter()
        while done < rows_min or time.perf_counter() - t0 < budget:
            m = min(x.shape[0], max(threads, 1))
            orc.sample_batch(cfg, x[:m], seeds=w.seeds(m), nthreads=threads)
            done += m
        return done, time.perf_counter() - t0

    n_all, t_all = timed(nthreads, 2 * nthreads, budget_s)
    n_one, t_one = timed(1, 2, budget_s / 2)
    return {"value": n_all / t_all, "unit": "rows/s", "cores": nthreads, "kind": "port",
            "sample": f"{n_all} rows of {w.name} (V={w.vocab}) on {nthreads} threads, {t_all:.1f} s",
            "value_1core": n_one / t_one,
            "sample_1core": f"{n_one} rows on 1 thread, {t_one:.1f} s"}


def parity_check(pkg, w, smp, dev_x, host_x, states):
    """One step of the benched batch against the checker: exact token matches
    and the draw-/threshold-boundary classes (the sampler is meant to match
    everywhere; boundary cases are only counted)."""
    orc = graft.load_oracle()
    smp.rng_state = states
    got = smp.sample(dev_x).cpu().numpy().astype(np.uint32)
    ref, traces, _ = orc.sample_batch(orc.make_config(**w.config()), host_x, states=states,
                                      nthreads=os.cpu_count() or 1)
    return orc.parity_report(got, ref, traces)


def graph_step_times(torch, smp, dev, out, n):
    """Per-step device time of the step replayed from CUDA graphs (one graph
    per rotating input, each one captured bs_sample call): median and p95."""
    graphs = []
    for x in dev:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            smp.sample(x, out=out)
        graphs.append(g)
    for i in range(8):
        graphs[i % len(graphs)].replay()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    stream = torch.cuda.current_stream()
    for i in range(n):
        evs[i][0].record(stream)
        graphs[i % len(graphs)].replay()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    us = sorted(a.elapsed_time(b) * 1e3 for a, b in evs)
    del graphs
    return {"median": us[len(us) // 2], "p95": us[min(len(us) - 1, int(0.95 * len(us)))], "steps": n}


def b1_token_latency(torch, pkg, local, n=500):
    """Config 0's decode step: one row of V=128256 logits already in HBM,
    with a 32-token history for the repetition penalty (window 32, 1.1, the
    SamplerConfig defaults), token id left in HBM.  Per-token device latency
    replayed from a CUDA graph (no host synchronisation between tokens) and
    with eager launches; median and p95."""
    w = pkg.workloads.WORKLOADS["c0"]
    cfg = pkg.SamplerConfig(**w.config(repetition_window=32, repetition_penalty=1.1))
    smp = pkg.Sampler(cfg, batch=1, vocab=w.vocab, device=local, seeds=w.seeds(1))
    xs = [torch.from_numpy(pkg.workloads.make_logits(w, step=s, rows=1)).cuda() for s in range(2)]
    hist = torch.randint(0, w.vocab, (1, 32), dtype=torch.int32, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    def timed(step):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            evs[i][0].record(stream)
            step(i)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
        us = sorted(a.elapsed_time(b) * 1e3 for a, b in evs)
        return {"median": us[len(us) // 2], "p95": us[min(len(us) - 1, int(0.95 * len(us)))]}

    for i in range(10):
        smp.sample(xs[i % 2], prev_tokens=hist, out=out)
    torch.cuda.synchronize()
    eager = timed(lambda i: smp.sample(xs[i % 2], prev_tokens=hist, out=out))
    graphs = []
    for x in xs:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            smp.sample(x, prev_tokens=hist, out=out)
        graphs.append(g)
    for i in range(10):
        graphs[i % 2].replay()
    graph = timed(lambda i: graphs[i % 2].replay())
    st = smp.last_status()
    del graphs
    smp.close()
    if st != 0:
        raise RuntimeError(f"sampler status {st}")
    return {"graph_us": graph, "eager_us": eager, "tokens": n,
            "config": "c0: B=1 V=128256 T=0.8 top_p=0.9, penalty 1.1 over a 32-token history"}


def run_reference(args, pkg, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    nthreads = os.cpu_count() or 1
    orc = graft.load_oracle()
    cfg = orc.make_config(**w.config())
    # the benched batch itself, unless the run's --steps/--warmup would then
    # take longer than a few minutes (about 25 ms per row on one core)
    per_row_s = 0.025 * max(1.0, w.vocab / 128256) / nthreads
    fit = int(args.ref_budget / max(1, args.steps + args.warmup) / per_row_s)
    rows = max(min(w.rows, nthreads), min(w.rows, fit))
    x = pkg.workloads.make_logits(w, rows=rows)
    seeds = w.seeds(x.shape[0])
    for _ in range(args.warmup):
        orc.sample_batch(cfg, x, seeds=seeds, nthreads=nthreads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        orc.sample_batch(cfg, x, seeds=seeds, nthreads=nthreads)
    dt = time.perf_counter() - t0
    rows = x.shape[0] * args.steps
    v = rows / dt
    line = {
        "impl": "reference", "metric": "rows sampled/sec", "value": v, "unit": "rows/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_desc(w), "rows_per_step": x.shape[0],
                   "same_batch": x.shape[0] == w.rows},
        "cpu_baseline": {"value": v, "unit": "rows/s", "cores": nthreads, "kind": "port",
                         "sample": f"{x.shape[0]} of the {w.rows} rows per step on {nthreads} threads "
                                   f"(one sampler per row), {args.steps} steps"},
        "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_vocab_sharded(args, pkg, w, torch, dist, world, rank, local):
    """Config 4: all B rows, vocab split over the ranks (a tensor-parallel LM
    head).  One step = the exact partial merge: statistics of this rank's
    shard, one all-gather of per-row partials, the main pass, the chain of
    walks over the shards in rank order, the broadcast of the normaliser, one
    all-gather of the candidates and the draw (every rank returns the same B
    token ids)."""
    B, V = w.rows, w.vocab
    cfg = pkg.SamplerConfig(**w.config())
    vs = pkg.sharding.VocabShardedSampler(cfg, B, V, dist if world > 1 else None, device=local,
                                          transport=args.vs_transport)
    lay = vs.lay
    host = [np.ascontiguousarray(lay.shard_of(pkg.workloads.make_logits(w, step=s, rows=B))) for s in range(ROTATE)]
    dev = [torch.from_numpy(h).cuda() for h in host]
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        vs.sample(dev[i % ROTATE])
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            vs.sample(dev[i % ROTATE])
        end.record(stream)
        torch.cuda.synchronize()
    eager_ms = pkg.sharding.max_over_ranks(start.elapsed_time(end), dist, device="cuda")
    if vs.last_status() != 0:
        raise RuntimeError(f"sampler status {vs.last_status()}")
    ms = eager_ms
    graphed = False
    if vs.exact:
        # the step as CUDA graphs (one per rotating input; collectives
        # inside), replayed with no host work between steps
        graphs = [vs.graph(x)[0] for x in dev]
        for i in range(args.warmup):
            graphs[i % ROTATE].replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            graphs[i % ROTATE].replay()
        end.record(stream)
        torch.cuda.synchronize()
        ms = pkg.sharding.max_over_ranks(start.elapsed_time(end), dist, device="cuda")
        del graphs
        graphed = True
        if vs.last_status() != 0:
            raise RuntimeError(f"sampler status {vs.last_status()}")
    # end to end: pinned host shard -> device, sample, B token ids -> host
    pinned = [torch.from_numpy(h).pin_memory() for h in host[:2]]
    d_in = torch.empty_like(dev[0])
    for i in range(3):
        d_in.copy_(pinned[i % 2], non_blocking=True)
        vs.sample(d_in).cpu()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        d_in.copy_(pinned[i % 2], non_blocking=True)
        vs.sample(d_in).cpu()
    e2e_s = pkg.sharding.max_over_ranks(time.perf_counter() - t0, dist, device="cuda")
    if rank == 0:
        peak, peak_kind = peaks()
        step_s = ms / args.steps / 1e3
        per_gpu_bytes = 4.0 * V * B / world
        ach = per_gpu_bytes / step_s / 1e9
        line = {
            "metric": "rows sampled/sec", "value": B / step_s, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": workload_desc(w), "rows": B, "vocab": V,
                       "parallelism": (f"vocab-sharded x{world}: exact partial merge (all-gather of per-row "
                                       "partials, all-gather of candidates, chain of shard walks "
                                       + ("through peer memory)" if vs.p2p else "by NCCL broadcasts)")
                                       if vs.exact else f"vocab-sharded x{world}: all-to-all transpose"),
                       "l2": f"{ROTATE} rotating shard batches ({ROTATE * per_gpu_bytes / 1e6:.0f} MB per GPU)"},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole step per GPU (its 4 V B / G bytes of shard over the step time)"},
            "clocks": clk.summary(),
            "e2e": {"value": B * args.e2e_steps / e2e_s, "unit": "rows/s",
                    "h2d_bytes_per_step": int(per_gpu_bytes), "d2h_bytes_per_step": 4 * B,
                    "api": "VocabShardedSampler.sample (pinned host shard)"},
            # per step: statistics and partials, row reduction and main pass,
            # export, walk, merge and draw (the peer transport adds its
            # one-thread step-tag kernel); the transpose: the single-GPU four
            "gpu_launches": ((9 if vs.p2p else 8) if vs.exact else 4) * args.steps,
            "timing": ("CUDA-graph replay of the whole step (collectives captured)" if graphed else "eager launches"),
            "eager_ms_per_step": eager_ms / args.steps,
        }
        print(json.dumps(line), flush=True)
    vs.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="headline")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--ref-budget", type=float, default=150.0,
                    help="seconds the reference arm may take in all (sizes its rows per step)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-b1", action="store_true", help="skip the B=1 per-token latency (config 0)")
    ap.add_argument("--vs-transport", default="p2p", choices=["nccl", "p2p"],
                    help="config 4's chain of walks: through peer memory (p2p) or by NCCL broadcasts")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    pkg = graft.load_package()
    w = pkg.workloads.WORKLOADS[args.workload]
    if args.impl == "reference":
        return run_reference(args, pkg, w)

    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    if w.name == "c4":
        return run_vocab_sharded(args, pkg, w, torch, dist, world, rank, local)

    B, V = w.rows, w.vocab
    # this rank's rows; seeds keyed by the global row
    shard = pkg.sharding.shard_for(rank, world, B)
    host = [pkg.workloads.make_logits(w, step=s, rows=B, row_offset=shard.row0) for s in range(ROTATE)]
    dev = [torch.from_numpy(h).cuda() for h in host]
    cfg = pkg.SamplerConfig(**w.config())
    smp = pkg.Sampler(cfg, batch=B, vocab=V, device=local, seeds=shard.seeds(w.seed))
    states0 = smp.rng_state
    out = torch.empty(B, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    for i in range(args.warmup):
        smp.sample(dev[i % ROTATE], out=out)
    torch.cuda.synchronize()
    if smp.last_status() != 0:
        raise RuntimeError(f"sampler status {smp.last_status()}")

    greedy = w.temperature <= 0.0
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            smp.sample(dev[i % ROTATE], out=out)
        end.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = pkg.sharding.max_over_ranks(start.elapsed_time(end), dist, device="cuda")
    if smp.last_status() != 0:
        raise RuntimeError(f"sampler status {smp.last_status()}")
    # per-step device times (events around every step) for the median and p95
    nper = min(args.steps, 200)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(nper)]
    for i in range(nper):
        evs[i][0].record(stream)
        smp.sample(dev[i % ROTATE], out=out)
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    per_us = sorted(a.elapsed_time(b) * 1e3 for a, b in evs)
    step_us = {"median": per_us[len(per_us) // 2], "p95": per_us[min(len(per_us) - 1, int(0.95 * len(per_us)))],
               "steps": nper}
    graph_us = graph_step_times(torch, smp, dev, out, nper)
    launches_per_step = 1 if greedy else (6 if w.typical_p < 1.0 else 4)
    kernel_ms = None
    if not greedy:
        # a separate profiled run: the events between kernel groups keep them
        # from overlapping, so it gives the breakdown, not the step time
        nprof = min(args.steps, 200)
        smp.profile_enable(nprof)
        for i in range(nprof):
            smp.sample(dev[i % ROTATE], out=out)
        prof = smp.profile_read()
        kernel_ms = [float(v) for v in prof.mean(axis=0)]
        smp.profile_enable(0)

    # end to end through the public host API: pinned host logits -> device,
    # sample, token ids -> host, every step
    pinned = [torch.from_numpy(h).pin_memory() for h in host[:2]]
    pin_np = [p.numpy() for p in pinned]
    for i in range(3):
        smp.sample(pin_np[i % 2])
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        smp.sample(pin_np[i % 2])
    e2e_s = pkg.sharding.max_over_ranks(time.perf_counter() - t0, dist, device="cuda")
    e2e_rows = pkg.sharding.aggregate_rows_per_s(shard, args.e2e_steps, e2e_s)

    # parity of one benched step against the checker, summed over the ranks
    parity = None
    if not args.no_parity and not greedy:
        parity = parity_check(pkg, w, smp, dev[0], host[0], states0)
        if dist:
            keys = [k for k, v in parity.items() if isinstance(v, int)]
            t = torch.tensor([parity[k] for k in keys], dtype=torch.int64, device="cuda")
            dist.all_reduce(t)
            parity.update({k: int(v) for k, v in zip(keys, t.tolist())})

    if rank == 0:
        rows_per_s = pkg.sharding.aggregate_rows_per_s(shard, args.steps, ms / 1e3)
        peak, peak_kind = peaks()
        alg_bytes = 4.0 * V * B
        roof = None
        if kernel_ms is None:   # greedy: one argmax kernel per step
            kernel_ms = [ms / args.steps, 0.0, 0.0]
        step_ms = ms / args.steps
        ach = alg_bytes / (step_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                "traffic": profile_traffic(args.workload),
                "kernel": "sampling step (all kernels of one call, overlapped; device time per step)",
                "peak_kind": peak_kind,
                "kernel_ms": {"stats": kernel_ms[0], "main": kernel_ms[1], "walk": kernel_ms[2],
                              "note": "separate profiled run, kernel groups serialised by the events"},
                "stats_kernel_gbs": alg_bytes / (kernel_ms[0] / 1e3) / 1e9 if kernel_ms[0] > 0 else None,
                "algorithmic_bytes_per_launch": alg_bytes}
        line = {
            "metric": "rows sampled/sec", "value": rows_per_s, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": workload_desc(w), "rows_per_gpu": B, "vocab": V,
                       "parallelism": f"batch-sharded x{world}" if world > 1 else "single GPU",
                       "l2": f"{ROTATE} rotating input batches ({ROTATE * alg_bytes / 1e6:.0f} MB) > L2"},
            "roofline": roof,
            "clocks": clk.summary(),
            "e2e": {"value": e2e_rows, "unit": "rows/s", "h2d_bytes_per_step": int(alg_bytes),
                    "d2h_bytes_per_step": 4 * B, "api": "bs_sample_host (pinned host logits)"},
            "gpu_launches": launches_per_step * args.steps,
            "step_us": step_us,
            "graph_step_us": graph_us,
        }
        if not args.no_b1:   # (rank 0 only: the other ranks wait at the closing barrier)
            line["b1_latency"] = b1_token_latency(torch, pkg, local)
        if parity is not None:
            line["parity"] = parity
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(pkg, w, args.cpu_budget, os.cpu_count() or 1)
        print(json.dumps(line), flush=True)
    smp.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
