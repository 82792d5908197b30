#!/usr/bin/env python
"""Benchmark: QPS of the B200 query engine on RAVEN's headline workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (default): gmm1m-d128-sparse — 1M x 128 integer-valued f32 vectors
(5000-centre Gaussian mixture, sigma 12, 30% zero components; stand-in for
SIFT-1M's shape), Vamana R=32/L=200/alpha=1.2/DirectionalPrune/nav_m=32 index,
SQ4 search with k=10, rerank_factor=8, batches of 10,000 queries, at the
workload's operating point: the smallest ef whose recall@10 reaches 0.95
(ef=140 on this stand-in; the reference reaches 0.95 at ef=50 on SIFT-1M, and
the ef=50 point is reported beside it).

A step = one batch of 10,000 queries through the search kernel. `value` is
whole-job QPS with queries already in HBM (sum over ranks / max-over-ranks
device time); `e2e` is the same through the public C ABI call with host
buffers (pinned), copies included. Multi-GPU (torchrun): the index is
replicated, each rank searches its own query batches, no data-path
collective (weak scaling).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "QPS at recall@10>=0.95 (SQ4, ef=50, k=10) on 1M×128, per GPU and at 1/2/4/8 B200"
UNIT = "queries/s"
FALLBACK_HBM_GBS = 6650.0
N_BATCHES = 4  # distinct 10k-query batches rotated across steps
# Operating point per workload: the smallest ef whose recall@10 (SQ4, k=10,
# rr=8, against exact kNN) reaches 0.95 on that workload, measured on B200 with
# this engine's ef sweep. On SIFT-1M the reference reaches 0.95 at ef=50; the
# Gaussian-mixture stand-in with a random 30% zero mask is harder.
OPERATING_EF = {"gmm100k-d128": 50, "gmm1m-d128-sparse": 140}
SWEEP_EFS = (40, 45, 50, 55, 65, 80, 100, 120, 140, 160, 200)
PREFETCH_OFFSET = 8  # with_prefetch_offset of the measured configurations (po=8)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="gmm1m-d128-sparse")
    ap.add_argument("--ef", type=int, default=None, help="default: the workload's operating point")
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--rr", type=int, default=8)
    ap.add_argument("--batch", type=int, default=10000)
    ap.add_argument("--quant", choices=["sq4", "sq8"], default="sq4")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle parity check (outside the timed region)")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sharded-collection record (8 shards, all-gather + GPU merge) of the default line")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the ef sweep, the AdaptiveEf points and the 64-query latency run")
    ap.add_argument("--sweep", action="store_true", help="report the ef sweep even with --no-extras")
    ap.add_argument("--hash-bits", type=int, default=0)
    ap.add_argument("--spill-bits", type=int, default=0,
                    help="log2 of the global visited-spill slots per warp (0 = automatic)")
    ap.add_argument("--shards", type=int, default=0,
                    help="split the workload into this many per-shard graphs (all-gather + merge across ranks)")
    ap.add_argument("--shard-n", type=int, default=0, help="vectors per shard (default: workload n / shards)")
    ap.add_argument("--build-device", type=int, default=None,
                    help="build a missing index with the GPU build on this device (default: this rank's GPU)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def measured_hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(workload):
    """DRAM bytes per launch of the search kernel on this workload, from the
    committed ncu summary named for it (None when there is none)."""
    name = {"gmm1m-d128-sparse": "search_sq4_gmm1m"}.get(workload)
    if name is None:
        return None
    for fn in sorted(os.listdir(os.path.join(ROOT, "profiles"))) if os.path.isdir(os.path.join(ROOT, "profiles")) else []:
        if fn.startswith(name) and fn.endswith(".md"):
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(os.path.join(ROOT, "profiles", fn)).read())
            if m:
                return float(m.group(1))
    return None


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out, _ = self.p.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def load_workload(args, rank, barrier=None, device=None):
    """Base vectors, this rank's query batches and the cached graph. A missing
    graph is built once (rank 0; the others wait at `barrier`) and saved; the
    GPU build (`device`) gives the host build's graph byte for byte, faster."""
    from raven_b200 import datasets

    base, _ = datasets.make(args.workload, nq=1)
    qs = [datasets.make_queries(args.workload, args.batch, offset=rank * N_BATCHES + b) for b in range(N_BATCHES)]
    t0 = time.time()
    dev = args.build_device if args.build_device is not None else device
    if barrier is not None and rank != 0:
        barrier()
    # the other ranks wait, so the build's host part may use every core (torchrun
    # sets OMP_NUM_THREADS=1)
    g = datasets.load_or_build(args.workload, base=base, device=dev, threads=os.cpu_count() or 1)
    if barrier is not None and rank == 0:
        barrier()
    args.load_s = time.time() - t0
    return base, np.stack(qs), g


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_baseline(args, base, g, queries, rank, budget_s=12.0, rounds=5):
    """The oracle (CPU restatement of the reference batch_search) on this
    box's host cores, on a bounded sample of the same workload: after a
    warm-up, `rounds` timed rounds with all host threads, each a pass over the
    bench's query batches (wrapping around) sized so that the rounds take about
    `budget_s` in total; the value is the median round's rate (the method of
    the reference's ef sweep, src/bin/sq4_ef_sweep.rs:102-131). A one-thread
    rate (median of 3 short rounds) is reported beside it."""
    import tempfile

    from oracle import oracle as O

    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        oi = O.OracleIndex(p)
    oi.set_vectors(base, sq4=args.quant == "sq4", sq8=args.quant == "sq8")
    threads = os.cpu_count() or 1
    q = queries.reshape(-1, queries.shape[-1])
    quant = 0 if args.quant == "sq4" else 1
    pos = [0]

    def timed(n, th):
        """Search the next n queries (wrapping around) on th threads; seconds."""
        done = 0
        t0 = time.perf_counter()
        while done < n:
            s = pos[0] % q.shape[0]
            m = min(q.shape[0] - s, n - done)
            oi.search(q[s:s + m], k=args.k, ef=args.ef, rerank_factor=args.rr, quant=quant, threads=th,
                      prefetch_offset=PREFETCH_OFFSET)
            done += m
            pos[0] += m
        return time.perf_counter() - t0

    timed(256, threads)  # warm-up
    probe = timed(1024, threads)
    per_round = int(max(1024, 1024 * budget_s / rounds / max(probe, 1e-3)))
    rates = sorted(per_round / timed(per_round, threads) for _ in range(rounds))
    one = sorted(128 / timed(128, 1) for _ in range(3))
    return {"value": rates[len(rates) // 2], "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"median of {rounds} rounds of {per_round} queries of {args.workload} (wrapping over its "
                      f"{q.shape[0]} bench queries), ef={args.ef}, k={args.k}, rr={args.rr}, {threads} host threads",
            "rounds_qps": [round(r, 1) for r in rates], "single_thread_qps": round(one[1], 1),
            "cpu_model": cpu_model(), "nproc": threads}


def workload_desc(args, n, dim):
    """The `config.workload` string both arms print for the same workload."""
    return (f"{args.workload}: {n} x {dim} seeded Gaussian mixture (SIFT-1M shape stand-in), Vamana R=32 L=200 "
            f"alpha=1.2 DirectionalPrune nav_m=32; {args.quant.upper()} ef={args.ef} k={args.k} rr={args.rr}; "
            f"batch {args.batch} queries per step")


def run_reference(args):
    """The reference arm: the oracle port of GraphSearcher::batch_search (the
    Rust reference cannot be built here) on this box's host cores, on the same
    workload, index, query batches and search parameters as the engine's arm;
    one step = one batch, the batches rotating as in the engine's arm. The
    index is read with the oracle's own ANNX reader; if it is not cached, it is
    built with the host build (oracle/_build/libhostbuild.so) and saved. The
    engine's CUDA library is not loaded."""
    if args.ef is None:
        args.ef = OPERATING_EF.get(args.workload, 50)
    rank, world, local = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O

    from raven_b200 import datasets

    base, _ = datasets.make(args.workload, nq=1)
    qb = np.stack([datasets.make_queries(args.workload, args.batch, offset=b) for b in range(N_BATCHES)])
    path = datasets.index_path(args.workload)
    t0 = time.time()
    if not os.path.exists(path):
        os.makedirs(os.path.dirname(path), exist_ok=True)
        O.build_index_file(base, path + ".tmp")
        os.replace(path + ".tmp", path)
    oi = O.OracleIndex(path)
    oi.set_vectors(base, sq4=args.quant == "sq4", sq8=args.quant == "sq8")
    load_s = time.time() - t0
    threads = os.cpu_count() or 1
    quant = 0 if args.quant == "sq4" else 1

    def step(i):
        oi.search(qb[i % N_BATCHES], k=args.k, ef=args.ef, rerank_factor=args.rr, quant=quant, threads=threads,
                  prefetch_offset=PREFETCH_OFFSET)

    for w in range(args.warmup):
        step(w)
    t0 = time.perf_counter()
    for st in range(args.steps):
        step(st)
    dt = time.perf_counter() - t0
    qps = args.steps * args.batch / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "sq4-int32+f32" if quant == 0 else "sq8-int32+f32",
        "data": "synthetic (seeded Gaussian mixture with the SIFT-1M shape; no dataset download)",
        "config": {"workload": workload_desc(args, base.shape[0], base.shape[1]), "ef": args.ef,
                   "index": f"host-built or cached graph (oracle ANNX reader), loaded/built in {load_s:.1f} s"},
        "cpu_baseline": {"value": qps, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{args.batch} queries per step x {args.steps} steps ({N_BATCHES} batches "
                                   f"rotating), {threads} host threads (C++ restatement of "
                                   "GraphSearcher::batch_search; the Rust reference cannot be built here)",
                         "cpu_model": cpu_model()},
        "e2e": {"value": qps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def parity_check(args, g, base, dev, qbatches, n_check=1000):
    """Checker, outside the timed region: the engine (raven_search_batch, the
    public C ABI with host buffers) against the oracle on the first `n_check`
    queries of batch 0, at the bench's ef and at ef=50, on every output:
    top-k ids, result counts, visited counts, visited order, ef used,
    navigation evaluations, expansions and the f32 rerank distances (exact
    visited set), and every one of these but the visited count and order for
    the timed mode, which runs without the visited set."""
    import tempfile

    from oracle import oracle as O
    from raven_b200 import _lib as L

    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        oi = O.OracleIndex(p)
    oi.set_vectors(base, sq4=args.quant == "sq4", sq8=args.quant == "sq8")
    quant = 0 if args.quant == "sq4" else 1
    q = np.ascontiguousarray(qbatches[0][:n_check])
    hist = 16384
    res = {"queries": int(q.shape[0]), "efs": [], "ids_equal": True, "counts_equal": True, "visited_equal": True,
           "history_equal": True, "stats_equal": True, "max_rel_dist_err": 0.0,
           "oracle": "C++ restatement of the reference search (oracle/), pinned by the reference's known answers"}
    for ef in sorted({args.ef, 50}):
        params = L.SearchParams(ef=ef, k=args.k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=0,
                                gamma=0.0, min_ef=0, max_ef=0)
        got = dev.search(q, params, history_cap=hist)
        # the timed path: no visited counts requested, pool membership decides
        fast = dev.search(q, params, visited=False)
        exp = oi.search(q, k=args.k, ef=ef, rerank_factor=args.rr, quant=quant, history_cap=hist,
                        threads=os.cpu_count() or 1)
        res["efs"].append(ef)
        res["pool_membership_mode_equal"] = res.get("pool_membership_mode_equal", True) and bool(
            all(np.array_equal(fast[k], exp[k]) for k in ("ids", "dists", "counts", "ef_used", "n_nav", "expansions")))
        res["ids_equal"] &= bool(np.array_equal(got["ids"], exp["ids"]))
        res["counts_equal"] &= bool(np.array_equal(got["counts"], exp["counts"]))
        res["visited_equal"] &= bool(np.array_equal(got["visited"], exp["visited"]))
        res["stats_equal"] &= bool(all(np.array_equal(got[k], exp[k]) for k in ("ef_used", "n_nav", "expansions")))
        h_ok = bool(np.array_equal(got["history_len"], exp["history_len"]))
        if h_ok:
            for i in range(q.shape[0]):
                h = min(int(got["history_len"][i]), hist)
                if not np.array_equal(got["history"][i, :h], exp["history"][i, :h]):
                    h_ok = False
                    break
        res["history_equal"] &= h_ok
        den = np.maximum(np.abs(exp["dists"]), 1e-30)
        res["max_rel_dist_err"] = max(res["max_rel_dist_err"], float(np.max(np.abs(got["dists"] - exp["dists"]) / den)))
        res["bad_status"] = int(np.sum(got["status"] != 0))
    return res


SHARDED_N = 8  # shards of the sharded-collection record in the default line


def _shard_graph(args, part, s, S, shard_n, world, local):
    """The cached graph of shard s, or a GPU build of it (saved for later runs)."""
    from raven_b200 import datasets
    from raven_b200.index import Graph

    path = datasets.shard_index_path(args.workload, s, S, shard_n)
    if os.path.exists(path):
        return Graph.load(path), path
    # torchrun sets OMP_NUM_THREADS=1: give each rank's host part of the build
    # its share of the cores explicitly
    g = Graph.build(part, r=32, l=200, alpha=1.2, nav_m=32, directional=True, seed=42 + s,
                    threads=max(1, (os.cpu_count() or 1) // world), device=local)
    os.makedirs(os.path.dirname(path), exist_ok=True)
    g.save(path + f".tmp{os.getpid()}")
    os.replace(path + f".tmp{os.getpid()}", path)
    return g, path


def sharded_record(args, base, world, rank, local, steps, n_shards=SHARDED_N, n_check=200):
    """The sharded-collection layout at this N (every rank takes part): the
    workload's base vectors split into `n_shards` contiguous shards, each with
    its own Vamana graph (GPU build, f32 candidate search) and SQ4 codes,
    shard s on rank s % N; a step = one batch searched on every shard (SQ4,
    ef=50, k, rr), the per-shard lists all-gathered over NCCL and merged on
    the GPU. Device-timed (max over ranks) with the step's split into search,
    exchange and merge; e2e through the same call with the batch copied from
    pinned host memory and the merged ids copied back every step; recall
    against the exact top-k of the whole collection (exact kNN per shard,
    merged the same way); and a check that the merged lists equal the
    reference's per-shard searches (the oracle) merged on the host."""
    import torch
    import torch.distributed as tdist

    from oracle import oracle as O
    from raven_b200 import _lib as L
    from raven_b200 import datasets
    from raven_b200 import multigpu as M
    from raven_b200.index import DeviceIndex

    dist_on = world > 1
    S, n, k, B = n_shards, base.shape[0], args.k, args.batch
    shard_n = n // S
    mine = M.shards_of_rank(S, world, rank)
    t0 = time.time()
    shards, paths, parts = {}, {}, {}
    for s in mine:
        parts[s] = np.ascontiguousarray(base[s * shard_n:(s + 1) * shard_n])
        g, paths[s] = _shard_graph(args, parts[s], s, S, shard_n, world, local)
        shards[s] = DeviceIndex(g, parts[s], device=local, sq4=True)
    build_s = time.time() - t0
    coll = M.ShardedCollection(shards, S, shard_n)
    qb = np.stack([datasets.make_queries(args.workload, B, offset=b) for b in range(N_BATCHES)])
    d_q = torch.from_numpy(qb).cuda()
    params = L.SearchParams(ef=50, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=L.RAVEN_QUANT_SQ4,
                            adaptive=0, gamma=0.0, min_ef=0, max_ef=0)
    stream = torch.cuda.Stream()
    truth = []
    for b in range(N_BATCHES):
        ti, _, _ = coll.exact(d_q[b], k, stream)
        stream.synchronize()
        truth.append(ti.cpu().numpy().view(np.uint32))
    for i in range(max(3, N_BATCHES)):
        coll.search(d_q[i % N_BATCHES], params, stream)
    stream.synchronize()
    rec = []
    for b in range(N_BATCHES):
        ids, _, _ = coll.search(d_q[b], params, stream)
        stream.synchronize()
        got = ids.cpu().numpy().view(np.uint32)
        rec += [len(set(got[i]) & set(truth[b][i])) / k for i in range(B)]
    # timed region: `steps` steps, events around each phase
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    if dist_on:
        tdist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        ev[i][0].record(stream)
        coll.search(d_q[i % N_BATCHES], params, stream, marks=(ev[i][1], ev[i][2]))
        ev[i][3].record(stream)
    torch.cuda.synchronize()
    tot = sum(e[0].elapsed_time(e[3]) for e in ev)
    t_search = sum(e[0].elapsed_time(e[1]) for e in ev)
    t_xchg = sum(e[1].elapsed_time(e[2]) for e in ev)
    t_merge = sum(e[2].elapsed_time(e[3]) for e in ev)
    ms = M.max_over_ranks(tot, device=torch.device("cuda", local))
    xchg_max = M.max_over_ranks(t_xchg, device=torch.device("cuda", local))
    # e2e: batch from pinned host memory, merged ids back to the host, every step
    hq = torch.from_numpy(qb).pin_memory()
    h_ids = torch.zeros((B, k), dtype=torch.int32).pin_memory()
    e2e_steps = max(5, steps // 4)
    if dist_on:
        tdist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(e2e_steps):
        with torch.cuda.stream(stream):
            dq = hq[i % N_BATCHES].to("cuda", non_blocking=True)
        ids, _, _ = coll.search(dq, params, stream)
        with torch.cuda.stream(stream):
            h_ids.copy_(ids, non_blocking=True)
        stream.synchronize()
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = M.max_over_ranks(f0.elapsed_time(f1), device=torch.device("cuda", local))
    # parity: this rank's shard lists against the oracle's search of each shard;
    # rank 0: the merge of the gathered lists against the host merge rule
    ok = True
    q = np.ascontiguousarray(qb[0][:n_check])
    for s in mine:
        oi = O.OracleIndex(paths[s])
        oi.set_vectors(parts[s], sq4=True)
        exp = oi.search(q, k=k, ef=50, rerank_factor=args.rr, threads=max(1, (os.cpu_count() or 1) // world))
        got = shards[s].search(q, params, visited=True)
        ok &= all(np.array_equal(got[f], exp[f]) for f in ("ids", "dists", "counts", "visited"))
        fast = shards[s].search(q, params, visited=False)  # the mode the collection's search runs in
        ok &= all(np.array_equal(fast[f], exp[f]) for f in ("ids", "dists", "counts", "expansions"))
    ids, _, cnt = coll.search(d_q[0], params, stream)
    stream.synchronize()
    gi, gd, gc = M.read_gathered(coll.gathered(B, k, d_q.device), S, world, B, k)
    if rank == 0:
        wi, wd, wc = O.merge_shard_lists(gi[:, :n_check], gd[:, :n_check], gc[:, :n_check], shard_n, k)
        ok &= bool(np.array_equal(ids.cpu().numpy().view(np.uint32)[:n_check], wi) and
                   np.array_equal(cnt.cpu().numpy().view(np.uint32)[:n_check], wc))
    ok_all = M.max_over_ranks(0.0 if ok else 1.0, device=torch.device("cuda", local)) == 0.0
    rec_mean = float(np.mean(rec))
    del coll, shards
    return {
        "layout": f"{args.workload} split into {S} contiguous shards of {shard_n}, each its own Vamana graph "
                  f"(R=32 L=200 alpha=1.2 DirectionalPrune nav_m=32, GPU build) and SQ4 codes; shard s on rank "
                  f"s % {world}; SQ4 ef=50 k={k} rr={args.rr}; every query of a {B}-query batch on every shard",
        "qps": steps * B / (ms / 1e3), "ms_per_step": ms / steps,
        "e2e_qps": e2e_steps * B / (e2e_ms / 1e3),
        "step_split_ms": {"search": t_search / steps, "all_gather": t_xchg / steps, "merge": t_merge / steps},
        "all_gather_share": xchg_max / ms if ms > 0 else None,
        "exchange_bytes_per_rank_per_step": M.per_rank(S, world) * M.block_words(B, k) * 4,
        "recall_at_10": round(rec_mean, 4), "queries_scored": len(rec),
        "merged_equal": bool(ok_all),
        "merged_check": f"{n_check} queries: every rank's per-shard lists equal the oracle's search of that shard "
                        f"(ids, distances, counts, visited); the GPU merge of the gathered lists equals the host "
                        f"merge rule (distance, shard, rank)",
        "shards_per_rank": len(mine), "build_or_load_s": round(build_s, 1),
        "gpu_launches_per_step": len(mine) + 1,
    }


def run_sharded(args):
    """Collection split into `args.shards` contiguous per-shard graphs (shard s
    on rank s % world): every query is searched on every shard, the per-shard
    top-k lists are all-gathered and merged on the GPU (raven_b200.multigpu).
    A step = one batch through ShardedCollection.search; recall against the
    exact kNN of the whole collection (exact per shard, merged the same way)."""
    import datetime

    import torch
    import torch.distributed as tdist

    from raven_b200 import _lib as L
    from raven_b200 import datasets
    from raven_b200 import multigpu as M
    from raven_b200.index import DeviceIndex, Graph

    rank, world, local = dist_env()
    dist = world > 1
    torch.cuda.set_device(local)
    if dist:
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800),
                                 device_id=torch.device("cuda", local))
    S = args.shards
    shard_n = args.shard_n or datasets.WORKLOADS[args.workload]["n"] // S
    mine = M.shards_of_rank(S, world, rank)
    t0 = time.time()
    shards = {}
    for sh in mine:
        base = datasets.make_shard(args.workload, sh, S, shard_n)
        path = datasets.shard_index_path(args.workload, sh, S, shard_n)
        if os.path.exists(path):
            g = Graph.load(path)
        else:
            # torchrun sets OMP_NUM_THREADS=1: give each rank's host part of the
            # build its share of the cores explicitly
            g = Graph.build(base, r=32, l=200, alpha=1.2, nav_m=32, directional=True, seed=42 + sh,
                            threads=max(1, (os.cpu_count() or 1) // world),
                            device=local if args.build_device is not None else None)
            os.makedirs(os.path.dirname(path), exist_ok=True)
            g.save(path + ".tmp")
            os.replace(path + ".tmp", path)
        shards[sh] = DeviceIndex(g, base, device=local, sq4=True)
        del base
    build_s = time.time() - t0
    lib = L.load()
    coll = M.ShardedCollection(shards, S, shard_n)
    B, k = args.batch, args.k
    qb = np.stack([datasets.make_queries(args.workload, B, offset=b) for b in range(N_BATCHES)])
    d_q = torch.from_numpy(qb).cuda()
    params = L.SearchParams(ef=args.ef, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=L.RAVEN_QUANT_SQ4,
                            adaptive=0, gamma=0.0, min_ef=0, max_ef=0)
    stream = torch.cuda.Stream()
    # exact kNN of the whole collection: exact per local shard, exchanged and merged
    truth = []
    for b in range(N_BATCHES):
        ti, _, _ = coll.exact(d_q[b], k, stream)
        stream.synchronize()
        truth.append(ti.cpu().numpy().view(np.uint32))
    for i in range(max(args.warmup, N_BATCHES)):
        coll.search(d_q[i % N_BATCHES], params, stream)
    torch.cuda.synchronize()
    rec = []
    for b in range(N_BATCHES):
        ids, _, _ = coll.search(d_q[b], params, stream)
        torch.cuda.synchronize()
        got = ids.cpu().numpy().view(np.uint32)
        rec += [len(set(got[i]) & set(truth[b][i])) / k for i in range(B)]
    recall = float(np.mean(rec))
    clocks = ClockSampler(local)
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        coll.search(d_q[i % N_BATCHES], params, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    if dist:
        tdist.barrier()
    clk = clocks.stop()
    ms = M.max_over_ranks(e0.elapsed_time(e1), device=torch.device("cuda", local))
    value = args.steps * B / (ms / 1e3)
    # e2e: queries from pinned host memory, ids back to the host, every step
    hq = torch.from_numpy(qb).pin_memory()
    h_ids = torch.zeros((B, k), dtype=torch.int32).pin_memory()
    e2e_steps = max(5, args.steps // 4)
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    for i in range(e2e_steps):
        with torch.cuda.stream(stream):
            dq = hq[i % N_BATCHES].to("cuda", non_blocking=True)
        ids, _, _ = coll.search(dq, params, stream)
        with torch.cuda.stream(stream):
            h_ids.copy_(ids, non_blocking=True)
        stream.synchronize()
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = M.max_over_ranks(f0.elapsed_time(f1), device=torch.device("cuda", local))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "sq4-int32+f32",
        "data": "synthetic (seeded Gaussian mixture, per-shard seeds around shared centres)",
        "config": {
            "workload": f"{args.workload}: {S} contiguous shards of {shard_n} x "
                        f"{datasets.WORKLOADS[args.workload]['dim']}, each its own Vamana graph "
                        f"(R=32 L=200 alpha=1.2 DirectionalPrune nav_m=32) and SQ4 codes; every query on every "
                        f"shard; SQ4 ef={args.ef} k={k} rr={args.rr}; batch {B} queries per step",
            "parallelism": f"sharded collection: shard s on rank s % {world}; all-gather of per-shard top-k + "
                           f"GPU merge (ties by distance, shard, rank)",
            "shards_per_rank": len(mine), "recall_at_10": round(recall, 4), "queries_scored": len(rec),
            "index": f"{'GPU-built' if args.build_device is not None else 'host-built or cached'} shard graphs, "
                     f"rank-0 load/build {build_s:.1f} s",
            "l2": "not flushed: each rank's shard working set is larger than the 126 MB L2",
        },
        "e2e": {"value": e2e_steps * B / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": B * qb.shape[2] * 4,
                "d2h_bytes_per_step": B * k * 4},
        "gpu_launches": args.steps * (len(mine) + 1),
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del coll, shards
    if dist:
        tdist.barrier()
        tdist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.shards:
        if args.ef is None:
            args.ef = 50
        return run_sharded(args)
    if args.ef is None:
        args.ef = OPERATING_EF.get(args.workload, 50)
    import torch

    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex
    from raven_b200.multigpu import max_over_ranks

    rank, world, local = dist_env()
    dist = world > 1
    if dist:
        import datetime

        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev_id = torch.cuda.current_device()

    base, qbatches, g = load_workload(args, rank, barrier=tdist.barrier if dist else None, device=dev_id)
    quant = L.RAVEN_QUANT_SQ4 if args.quant == "sq4" else L.RAVEN_QUANT_SQ8
    dev = DeviceIndex(g, base, device=dev_id, sq4=quant == 0, sq8=quant == 1, adaptive=True)
    if args.hash_bits or args.spill_bits:
        dev.set_tuning(hash_bits=args.hash_bits, spill_bits=args.spill_bits)
    if args.no_extras:
        # the timed batch kernel gathers codes: the copies stored beside the
        # rows serve only the small-batch latency runs, which are skipped
        dev.set_fat_rows(False)
    lib = L.load()
    nb, B, dim = qbatches.shape
    k = args.k
    d_q = torch.from_numpy(qbatches).cuda()
    d_ids = torch.zeros((nb, B, k), dtype=torch.int32, device="cuda")
    d_d = torch.zeros((nb, B, k), dtype=torch.float32, device="cuda")
    stats = {n: torch.zeros((nb, B), dtype=torch.int32, device="cuda")
             for n in ("counts", "visited", "ef_used", "status", "n_nav", "expansions")}
    params = L.SearchParams(ef=args.ef, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=0,
                            gamma=0.0, min_ef=0, max_ef=0)
    stream = torch.cuda.Stream()

    def outs(b, with_stats=True, with_visited=False):
        def p(t, ty):
            return C.cast(t[b].data_ptr(), ty)

        return L.SearchOutputs(
            ids=p(d_ids, L.u32p), dists=p(d_d, L.f32p),
            counts=p(stats["counts"], L.u32p) if with_stats else None,
            visited=p(stats["visited"], L.u32p) if with_visited else None,
            ef_used=p(stats["ef_used"], L.u32p) if with_stats else None,
            status=p(stats["status"], L.i32p) if with_stats else None,
            n_nav=p(stats["n_nav"], L.u32p) if with_stats else None,
            expansions=p(stats["expansions"], L.u32p) if with_stats else None,
            history=None, history_cap=0, history_len=None)

    # the timed steps ask for no visited counts: the search decides new
    # neighbours by pool membership (same results, no visited tables)
    out_objs = [outs(b) for b in range(nb)]

    def step(i, objs=out_objs):
        b = i % nb
        L.check(lib.raven_search_batch_device(dev._h, d_q[b].data_ptr(), B, C.byref(params), C.byref(objs[b]),
                                              stream.cuda_stream))

    # untimed pass with the exact visited set: the visited counts that the
    # algorithmic bytes are counted from, and the results both modes must share
    vis_objs = [outs(b, with_visited=True) for b in range(nb)]
    for b in range(nb):
        step(b, vis_objs)
    torch.cuda.synchronize()
    exact_ids, exact_d = d_ids.clone(), d_d.clone()
    exact_exp = stats["expansions"].clone()
    # warm-up (also fills stats and results for every batch)
    for i in range(max(args.warmup, nb)):
        step(i)
    torch.cuda.synchronize()
    modes_equal = bool(torch.equal(exact_ids, d_ids) and torch.equal(exact_d, d_d)
                       and torch.equal(exact_exp, stats["expansions"]))

    # recall@10 against the exact kNN kernel on all batches
    gt = torch.zeros((nb, B, k), dtype=torch.int32, device="cuda")
    gtd = torch.zeros((nb, B, k), dtype=torch.float32, device="cuda")
    for b in range(nb):
        L.check(lib.raven_knn_exact_device(dev._h, d_q[b].data_ptr(), B, k, gt[b].data_ptr(), gtd[b].data_ptr(),
                                           stream.cuda_stream))
    torch.cuda.synchronize()
    got = d_ids.cpu().numpy().reshape(-1, k)
    truth = gt.cpu().numpy().reshape(-1, k)
    recall = float(np.mean([len(set(got[i]) & set(truth[i])) / k for i in range(got.shape[0])]))
    st = {n: t.cpu().numpy().astype(np.int64) for n, t in stats.items()}
    bad_status = int((st["status"] != 0).sum())

    # algorithmic bytes per query (counted from the kernel's own per-query stats)
    R = 32 * ((g.info().r_max + 31) // 32)
    code_bytes = 64 if quant == 0 else 128
    rerank_n = np.minimum(np.maximum(k * args.rr, k), np.minimum(st["ef_used"], st["visited"]))
    bq = (4 * dim + st["n_nav"] * 4 * dim + st["expansions"] * 4 * R + st["visited"] * code_bytes
          + rerank_n * 4 * dim + k * 8)
    bytes_per_batch = float(bq.sum()) / nb

    # timed region
    clocks = ClockSampler(dev_id)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    t0 = time.perf_counter()
    for i in range(args.steps):
        ev[i][0].record(stream)
        step(i)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if dist:
        tdist.barrier()
    clk = clocks.stop()
    per = [a.elapsed_time(b) for a, b in ev]  # ms, launch-stream device time
    dev_ms = float(sum(per))
    dev_ms_max = max_over_ranks(dev_ms, device=torch.device("cuda", dev_id))
    total_q = args.steps * B * world
    value = total_q / (dev_ms_max / 1e3)
    ms_per_step = dev_ms_max / args.steps

    # e2e through the public C ABI with pinned host buffers
    hq = torch.from_numpy(qbatches).pin_memory()
    h_ids = torch.zeros((B, k), dtype=torch.int32).pin_memory()
    h_d = torch.zeros((B, k), dtype=torch.float32).pin_memory()
    hout = L.SearchOutputs(ids=C.cast(h_ids.data_ptr(), L.u32p), dists=C.cast(h_d.data_ptr(), L.f32p))
    e2e_steps = max(20, args.steps // 4)
    for i in range(3):
        L.check(lib.raven_search_batch(dev._h, C.cast(hq[i % nb].data_ptr(), L.f32p), B, C.byref(params),
                                       C.byref(hout), stream.cuda_stream))
    if dist:
        tdist.barrier()
    torch.cuda.synchronize()
    # device time on the launch stream: each call's H2D copy, kernel, D2H copy
    # and the host gaps between calls (the call returns with results on the
    # host); five runs of e2e_steps calls, the median run (host-side noise
    # moves single runs by several per cent)
    runs = []
    for _ in range(5):
        e2e_ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        e2e_ev[0].record(stream)
        for i in range(e2e_steps):
            L.check(lib.raven_search_batch(dev._h, C.cast(hq[i % nb].data_ptr(), L.f32p), B, C.byref(params),
                                           C.byref(hout), stream.cuda_stream))
        e2e_ev[1].record(stream)
        torch.cuda.synchronize()
        runs.append(e2e_ev[0].elapsed_time(e2e_ev[1]) / 1e3)
    e2e_s = max_over_ranks(sorted(runs)[len(runs) // 2], device=torch.device("cuda", dev_id))
    e2e_value = e2e_steps * B * world / e2e_s

    # the sharded-collection layout at this N (all ranks take part)
    sharded = None
    if not args.no_sharded:
        sharded = sharded_record(args, base, world, rank, dev_id, steps=args.steps)

    sweep = None
    if (args.sweep or not args.no_extras) and rank == 0:
        sweep = {}
        for ef in SWEEP_EFS:
            p2 = L.SearchParams(ef=ef, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=0,
                                gamma=0.0, min_ef=0, max_ef=0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            o0 = outs(0, with_stats=False)
            L.check(lib.raven_search_batch_device(dev._h, d_q[0].data_ptr(), B, C.byref(p2), C.byref(o0),
                                                  stream.cuda_stream))
            e0.record(stream)
            for r in range(5):
                L.check(lib.raven_search_batch_device(dev._h, d_q[r % nb].data_ptr(), B, C.byref(p2),
                                                      C.byref(outs(r % nb, with_stats=False)), stream.cuda_stream))
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 5
            g2 = d_ids.cpu().numpy().reshape(-1, k)
            rec = float(np.mean([len(set(g2[i]) & set(truth[i])) / k for i in range(g2.shape[0])]))
            sweep[str(ef)] = {"qps": B / (ms / 1e3), "recall_at_10": round(rec, 4)}

    # the reference's published working point (ef=50), for comparison
    ef50 = None
    if rank == 0 and args.ef != 50:
        p50 = L.SearchParams(ef=50, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=0,
                             gamma=0.0, min_ef=0, max_ef=0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        L.check(lib.raven_search_batch_device(dev._h, d_q[0].data_ptr(), B, C.byref(p50),
                                              C.byref(outs(0, with_stats=False)), stream.cuda_stream))
        e0.record(stream)
        for r in range(nb):
            L.check(lib.raven_search_batch_device(dev._h, d_q[r].data_ptr(), B, C.byref(p50),
                                                  C.byref(outs(r, with_stats=False)), stream.cuda_stream))
        e1.record(stream)
        torch.cuda.synchronize()
        g50 = d_ids.cpu().numpy().reshape(-1, k)
        r50 = float(np.mean([len(set(g50[i]) & set(truth[i])) / k for i in range(g50.shape[0])]))
        ef50 = {"qps": nb * B / (e0.elapsed_time(e1) / 1e3), "recall_at_10": round(r50, 4)}

    # AdaptiveEf Pareto points (gamma x (min_ef, max_ef)) on the same batches,
    # and the small-batch latency run: 64-query launches, p50/p99 per launch
    adaptive = latency = None
    if rank == 0 and not args.no_extras:
        adaptive = []
        for gamma in (2.0, 2.4, 3.5):
            for mn, mx in ((35, 65), (35, 75), (35, 85)):
                pa = L.SearchParams(ef=mx, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=1,
                                    gamma=gamma, min_ef=mn, max_ef=mx)
                L.check(lib.raven_search_batch_device(dev._h, d_q[0].data_ptr(), B, C.byref(pa),
                                                      C.byref(outs(0, with_stats=False)), stream.cuda_stream))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for r in range(nb):
                    L.check(lib.raven_search_batch_device(dev._h, d_q[r].data_ptr(), B, C.byref(pa),
                                                          C.byref(outs(r)), stream.cuda_stream))
                e1.record(stream)
                torch.cuda.synchronize()
                ga = d_ids.cpu().numpy().reshape(-1, k)
                ra = float(np.mean([len(set(ga[i]) & set(truth[i])) / k for i in range(ga.shape[0])]))
                adaptive.append({"gamma": gamma, "min_ef": mn, "max_ef": mx,
                                 "qps": nb * B / (e0.elapsed_time(e1) / 1e3), "recall_at_10": round(ra, 4),
                                 "mean_ef": float(stats["ef_used"].float().mean().item())})
        lat_q, lat_n = 64, 300
        ql = d_q[0][:lat_q]
        lat = {}
        ad24 = L.SearchParams(ef=75, k=k, rerank_factor=args.rr, prefetch_offset=8, quant=quant, adaptive=1,
                              gamma=2.4, min_ef=35, max_ef=75)
        # small batches run one CTA per query (by default up to one wave of
        # CTAs); the persistent one-warp-per-query kernel is timed beside it
        runs = (("ef%d" % args.ef, params, lat_q, None), ("adaptive gamma=2.4 (35,75)", ad24, lat_q, None),
                ("ef%d, 1 query" % args.ef, params, 1, None),
                ("ef%d, persistent kernel" % args.ef, params, lat_q, 0))
        for name, pl, nql, sb in runs:
            if sb is not None:
                dev.set_small_batch(sb)
            ol = outs(0, with_stats=False)
            for _ in range(20):
                L.check(lib.raven_search_batch_device(dev._h, ql.data_ptr(), nql, C.byref(pl), C.byref(ol),
                                                      stream.cuda_stream))
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(lat_n)]
            for a_, b_ in evs:
                a_.record(stream)
                L.check(lib.raven_search_batch_device(dev._h, ql.data_ptr(), nql, C.byref(pl), C.byref(ol),
                                                      stream.cuda_stream))
                b_.record(stream)
            torch.cuda.synchronize()
            if sb is not None:
                from raven_b200.index import SMALL_BATCH_AUTO

                dev.set_small_batch(SMALL_BATCH_AUTO)
            ts = sorted(a_.elapsed_time(b_) * 1e3 for a_, b_ in evs)
            lat[name] = {"queries": nql, "p50_us": round(ts[len(ts) // 2], 1), "p99_us": round(ts[int(len(ts) * 0.99)], 1)}
        latency = {"queries_per_launch": lat_q, "launches": lat_n, "device_time_per_launch": lat}

    parity = None
    if rank == 0 and not args.no_parity:
        try:
            parity = parity_check(args, g, base, dev, qbatches)
        except Exception as e:  # reported in the line, never silently dropped
            parity = {"error": f"{type(e).__name__}: {e}"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu = cpu_baseline(args, base, g, qbatches, rank)
        except Exception as e:  # the baseline is reported, not required
            cpu = {"value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}

    peak, peak_kind = measured_hbm_peak()
    achieved = bytes_per_batch / (ms_per_step / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "sq4-int32+f32" if quant == 0 else "sq8-int32+f32",
        "data": "synthetic (seeded Gaussian mixture with the SIFT-1M shape; no dataset download)",
        "config": {
            "workload": workload_desc(args, base.shape[0], dim),
            "ef": args.ef, "ef_choice": "smallest ef with recall@10 >= 0.95 on this workload "
                                        "(the reference reaches 0.95 at ef=50 on SIFT-1M)",
            "ef50_point": ef50,
            "parity": parity,
            "sharded": sharded,
            "recall_at_10": round(recall, 4), "queries_scored": int(got.shape[0]),
            "bad_status_queries": bad_status,
            "visited_mode": "timed steps request no visited counts: new neighbours are decided by pool membership "
                            "(same results); the visited counts come from an untimed pass with the exact visited set",
            "visited_modes_equal": modes_equal,
            "avg_visited": float(st["visited"].mean()), "avg_expansions": float(st["expansions"].mean()),
            "avg_nav_evals": float(st["n_nav"].mean()),
            "l2": f"not flushed: index working set ~{(base.nbytes + base.shape[0] * (code_bytes + 4 * R)) / 2**20:.0f} "
                  f"MiB > 126 MB L2; {nb} distinct query batches rotate per step",
            "parallelism": f"replicated index, query-batch partition x{world}",
            "index": f"cached graph or a GPU build (the host build's graph, byte for byte), "
                     f"loaded/built in {args.load_s:.1f} s",
            "wall_s_timed": wall,
        },
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": profiled_traffic(args.workload),
                     "peak_source": peak_kind,
                     "algorithmic_bytes_per_query": bytes_per_batch / B},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": B * dim * 4,
                "d2h_bytes_per_step": B * k * 8},
        "gpu_launches": args.steps,
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    if sweep is not None:
        line["config"]["ef_sweep"] = sweep
    if adaptive is not None:
        line["config"]["adaptive_ef"] = adaptive
        line["config"]["latency_64q"] = latency
    if rank == 0:
        print(json.dumps(line), flush=True)
    del dev
    if dist:
        tdist.barrier()
        tdist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
