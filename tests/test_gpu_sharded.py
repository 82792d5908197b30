"""Sharded collection on the GPU: every query searched on every shard's own
graph, per-shard top-k lists written into per-rank send blocks, exchanged
(all-gather) and merged in place by raven_merge_topk_gathered_device. Checked
against the oracle's search of each shard,
merged on the host by the (distance, shard, rank) rule: ids, distances and
counts bit-exact.

One GPU: all shards on cuda:0, no process group. Two GPUs (when visible): two
NCCL ranks, shard s on rank s % 2, both ranks must return the same merged lists.
"""
import datetime
import os
import socket
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N_SHARDS, SHARD_SIZE, NQ, K = 4, 1500, 200, 10


def _params():
    from raven_b200 import _lib as L

    return L.SearchParams(ef=50, k=K, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=0, gamma=0.0, min_ef=0,
                          max_ef=0)


@pytest.fixture(scope="module")
def shard_data(raven_lib, oracle):
    from raven_b200 import datasets
    from raven_b200.index import Graph

    base, q = datasets.make("gmm100k-d128", n=N_SHARDS * SHARD_SIZE, nq=NQ)
    d = tempfile.mkdtemp(prefix="raven_shards_")
    ids = np.zeros((N_SHARDS, NQ, K), np.uint32)
    ds = np.zeros((N_SHARDS, NQ, K), np.float32)
    cs = np.zeros((N_SHARDS, NQ), np.uint32)
    for s in range(N_SHARDS):
        part = np.ascontiguousarray(base[s * SHARD_SIZE:(s + 1) * SHARD_SIZE])
        g = Graph.build(part, r=32, l=64, alpha=1.2, nav_m=8, directional=True, seed=21 + s)
        g.save(os.path.join(d, f"shard{s}.annx"))
        oi = oracle.OracleIndex(os.path.join(d, f"shard{s}.annx"))
        oi.set_vectors(part, sq4=True)
        r = oi.search(q, k=K, ef=50, rerank_factor=8)
        ids[s], ds[s], cs[s] = r["ids"], r["dists"], r["counts"]
    want = oracle.merge_shard_lists(ids, ds, cs, SHARD_SIZE, K)
    np.save(os.path.join(d, "base.npy"), base)
    np.save(os.path.join(d, "q.npy"), q)
    return d, base, q, want


def _search_rank(d, rank, world, device):
    """Load this rank's shards on `device`, run one sharded search, return host arrays."""
    import torch

    from raven_b200 import multigpu as M
    from raven_b200.index import DeviceIndex, Graph

    base = np.load(os.path.join(d, "base.npy"))
    q = np.load(os.path.join(d, "q.npy"))
    shards = {}
    for s in M.shards_of_rank(N_SHARDS, world, rank):
        g = Graph.load(os.path.join(d, f"shard{s}.annx"))
        shards[s] = DeviceIndex(g, np.ascontiguousarray(base[s * SHARD_SIZE:(s + 1) * SHARD_SIZE]), device=device,
                                sq4=True)
    coll = M.ShardedCollection(shards, N_SHARDS, SHARD_SIZE)
    stream = torch.cuda.Stream(device)
    dq = torch.from_numpy(q).to(f"cuda:{device}")
    torch.cuda.synchronize(device)
    i, dd, c = coll.search(dq, _params(), stream)
    torch.cuda.synchronize(device)
    return i.cpu().numpy().view(np.uint32), dd.cpu().numpy(), c.cpu().numpy().view(np.uint32)


def test_sharded_one_gpu_matches_host_merge(shard_data):
    d, base, q, (wi, wd, wc) = shard_data
    i, dd, c = _search_rank(d, 0, 1, 0)
    np.testing.assert_array_equal(c, wc)
    np.testing.assert_array_equal(i, wi)
    np.testing.assert_array_equal(dd, wd)


def _nccl_rank(rank, world, port, d):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        i, dd, c = _search_rank(d, rank, world, rank)
        np.savez(os.path.join(d, f"out{rank}.npz"), i=i, d=dd, c=c)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_sharded_two_gpus_nccl(shard_data):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    d, base, q, (wi, wd, wc) = shard_data
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_nccl_rank, args=(2, port, d), nprocs=2, join=True)
    for r in range(2):
        got = np.load(os.path.join(d, f"out{r}.npz"))
        np.testing.assert_array_equal(got["c"], wc)
        np.testing.assert_array_equal(got["i"], wi)
        np.testing.assert_array_equal(got["d"], wd)


def test_gathered_merge_layout_three_ranks(shard_data, oracle):
    """raven_merge_topk_gathered_device on the buffer three ranks' all-gather
    would leave (4 shards, two blocks per rank, the last block unused), built
    on one GPU from the oracle's per-shard lists: equal to the host merge."""

    import torch

    from raven_b200 import _lib as L
    from raven_b200 import multigpu as M

    d, base, q, (wi, wd, wc) = shard_data
    ids = np.zeros((N_SHARDS, NQ, K), np.uint32)
    ds = np.zeros((N_SHARDS, NQ, K), np.float32)
    cs = np.zeros((N_SHARDS, NQ), np.uint32)
    for s in range(N_SHARDS):
        oi = oracle.OracleIndex(os.path.join(d, f"shard{s}.annx"))
        oi.set_vectors(np.ascontiguousarray(base[s * SHARD_SIZE:(s + 1) * SHARD_SIZE]), sq4=True)
        r = oi.search(q, k=K, ef=50, rerank_factor=8)
        ids[s], ds[s], cs[s] = r["ids"], r["dists"], r["counts"]
    world = 3
    per = M.per_rank(N_SHARDS, world)
    buf = torch.full((world * per * M.block_words(NQ, K),), -1, dtype=torch.int32)
    for s in range(N_SHARDS):
        bi, bd, bc = M.block_views(buf, M.gathered_block(s, world, per), NQ, K)
        bi.copy_(torch.from_numpy(ids[s].view(np.int32)))
        bd.copy_(torch.from_numpy(ds[s]))
        bc.copy_(torch.from_numpy(cs[s].view(np.int32)))
    g = buf.cuda()
    oi_ = torch.zeros((NQ, K), dtype=torch.int32, device="cuda")
    od = torch.zeros((NQ, K), dtype=torch.float32, device="cuda")
    oc = torch.zeros(NQ, dtype=torch.int32, device="cuda")
    lib = L.load()
    L.check(lib.raven_merge_topk_gathered_device(g.data_ptr(), N_SHARDS, world, per, NQ, K, SHARD_SIZE,
                                                 oi_.data_ptr(), od.data_ptr(), oc.data_ptr(), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oi_.cpu().numpy().view(np.uint32), wi)
    np.testing.assert_array_equal(od.cpu().numpy(), wd)
    np.testing.assert_array_equal(oc.cpu().numpy().view(np.uint32), wc)
    with pytest.raises(L.RavenError):  # per_rank must be ceil(n_shards / world)
        L.check(lib.raven_merge_topk_gathered_device(g.data_ptr(), N_SHARDS, world, per + 1, NQ, K, SHARD_SIZE,
                                                     oi_.data_ptr(), od.data_ptr(), oc.data_ptr(), None))


@pytest.mark.parametrize("n_shards,k", [(8, 10), (5, 7), (40, 10)])
def test_merge_kernel_ties_and_short_lists(oracle, n_shards, k):
    """raven_merge_topk_device against the host merge rule (distance, shard,
    rank) on lists with many equal distances and shards that return fewer
    than k results; 8 x 10 and 5 x 7 candidates per query are staged in shared
    memory, 40 x 10 (above 256) take the unstaged path."""
    import torch
    from raven_b200 import _lib as L

    rng = np.random.default_rng(n_shards * 100 + k)
    nq, size = 300, 1000
    d = np.sort(rng.integers(0, 12, size=(n_shards, nq, k)).astype(np.float32), axis=2)  # many ties
    ids = rng.integers(0, size, size=(n_shards, nq, k)).astype(np.uint32)
    c = rng.integers(0, k + 1, size=(n_shards, nq)).astype(np.uint32)
    wi, wd, wc = oracle.merge_shard_lists(ids, d, c, size, k)

    def dev(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a).view(dt)).cuda()

    di, dd, dc = dev(ids, np.int32), dev(d, np.float32), dev(c, np.int32)
    oi_ = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
    od = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    oc = torch.zeros(nq, dtype=torch.int32, device="cuda")
    lib = L.load()
    L.check(lib.raven_merge_topk_device(di.data_ptr(), dd.data_ptr(), dc.data_ptr(), n_shards, nq, k, size,
                                        oi_.data_ptr(), od.data_ptr(), oc.data_ptr(), None))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oc.cpu().numpy().view(np.uint32), wc)
    np.testing.assert_array_equal(oi_.cpu().numpy().view(np.uint32), wi)
    np.testing.assert_array_equal(od.cpu().numpy(), wd)
