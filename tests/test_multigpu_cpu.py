"""Host logic of the multi-GPU layouts (raven_b200/multigpu.py), run on CPU:
query partition, shard placement, the exchange block layout, and — with two gloo
ranks — the max-over-ranks timing reduction and the all-gather that brings
every shard's top-k lists to every rank, followed by the (distance, shard,
rank) merge, checked against a single-process merge of the same lists.

The per-shard lists come from the oracle's search of three small shard
graphs (standing in for the per-shard device searches, which need a GPU).
"""
import os
import socket

import numpy as np
import pytest
import torch

from raven_b200 import multigpu as M


def test_query_slice_partitions_exactly():
    for nq in (0, 1, 7, 10000, 10001):
        for world in (1, 2, 3, 8):
            parts = [M.query_slice(nq, world, r) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == nq
            assert all(parts[r][1] == parts[r + 1][0] for r in range(world - 1))
            sizes = [hi - lo for lo, hi in parts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        M.query_slice(10, 2, 2)


def test_shards_of_rank():
    assert M.shards_of_rank(8, 2, 0) == [0, 2, 4, 6]
    assert M.shards_of_rank(8, 8, 7) == [7]
    assert M.shards_of_rank(5, 2, 1) == [1, 3]
    for world in (1, 2, 3, 4, 8):
        got = sorted(s for r in range(world) for s in M.shards_of_rank(8, world, r))
        assert got == list(range(8))


def test_block_layout_keeps_bit_patterns():
    """A shard's lists written into a block of the exchange buffer and read
    back in shard order through the gathered-buffer indexing (here three
    ranks' buffers laid end to end, as an all-gather leaves them)."""
    rng = np.random.default_rng(3)
    S, world, nq, k = 5, 3, 4, 10
    ids = rng.integers(0, 2**32, size=(S, nq, k), dtype=np.uint64).astype(np.uint32)
    d = rng.standard_normal((S, nq, k)).astype(np.float32)
    d[0, 0, :3] = [-0.0, np.inf, 1e-45]
    c = rng.integers(0, 11, size=(S, nq)).astype(np.uint32)
    per = M.per_rank(S, world)
    bufs = []
    for r in range(world):
        send = torch.zeros(per * M.block_words(nq, k), dtype=torch.int32)
        for j, s in enumerate(M.shards_of_rank(S, world, r)):
            bi, bd, bc = M.block_views(send, j, nq, k)
            bi.copy_(torch.from_numpy(ids[s].view(np.int32)))
            bd.copy_(torch.from_numpy(d[s]))
            bc.copy_(torch.from_numpy(c[s].view(np.int32)))
        bufs.append(send)
    i2, d2, c2 = M.read_gathered(torch.cat(bufs), S, world, nq, k)
    assert np.array_equal(i2, ids) and np.array_equal(c2, c)
    assert np.array_equal(d2.view(np.uint32), d.view(np.uint32))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, tmp, n_shards, k):
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # max-over-ranks timing reduction
        tmax = M.max_over_ranks(10.0 + rank)
        # this rank's shards written into its send blocks, exchanged, merged
        lists = np.load(os.path.join(tmp, "lists.npz"))
        mine = M.shards_of_rank(n_shards, world, rank)
        nq = lists["ids"].shape[1]
        send = torch.zeros(M.per_rank(n_shards, world) * M.block_words(nq, k), dtype=torch.int32)
        for j, s in enumerate(mine):
            bi, bd, bc = M.block_views(send, j, nq, k)
            bi.copy_(torch.from_numpy(lists["ids"][s].view(np.int32)))
            bd.copy_(torch.from_numpy(lists["d"][s]))
            bc.copy_(torch.from_numpy(lists["c"][s].view(np.int32)))
        i, d, c = M.read_gathered(M.exchange_blocks(send), n_shards, world, nq, k)
        mi, md, mc = O.merge_shard_lists(i, d, c, int(lists["size"]), k)
        np.savez(os.path.join(tmp, f"rank{rank}.npz"), tmax=tmax, i=mi, d=md, c=mc,
                 slice=np.array(M.query_slice(1001, world, rank)))
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope="module")
def shard_lists(oracle, tmp_path_factory):
    """Three shards of a small integer mixture, each with its own graph,
    searched by the oracle: [S][nq][k] lists in the device layout."""
    from raven_b200 import datasets
    from raven_b200.index import Graph

    n_shards, size, k = 3, 1200, 10
    base, q = datasets.make("gmm100k-d128", n=n_shards * size, nq=64)
    ids = np.zeros((n_shards, q.shape[0], k), np.uint32)
    d = np.zeros((n_shards, q.shape[0], k), np.float32)
    c = np.zeros((n_shards, q.shape[0]), np.uint32)
    tmp = tmp_path_factory.mktemp("shards")
    for s in range(n_shards):
        part = base[s * size:(s + 1) * size]
        g = Graph.build(part, r=32, l=64, alpha=1.2, nav_m=8, directional=True, seed=11 + s)
        path = str(tmp / f"shard{s}.annx")
        g.save(path)
        oi = oracle.OracleIndex(path)
        oi.set_vectors(part, sq4=True)
        r = oi.search(q, k=k, ef=50, rerank_factor=8)
        ids[s], d[s], c[s] = r["ids"], r["dists"], r["counts"]
    np.savez(tmp / "lists.npz", ids=ids, d=d, c=c, size=size)
    return tmp, n_shards, size, k, base, q, (ids, d, c)


def test_two_gloo_ranks_exchange_and_merge(oracle, shard_lists):
    import torch.multiprocessing as mp

    tmp, n_shards, size, k, base, q, (ids, d, c) = shard_lists
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp), n_shards, k), nprocs=world, join=True)
    want_i, want_d, want_c = oracle.merge_shard_lists(ids, d, c, size, k)
    slices = []
    for r in range(world):
        got = np.load(tmp / f"rank{r}.npz")
        assert float(got["tmax"]) == 10.0 + world - 1
        np.testing.assert_array_equal(got["i"], want_i)
        np.testing.assert_array_equal(got["d"], want_d)
        np.testing.assert_array_equal(got["c"], want_c)
        slices.append(tuple(got["slice"]))
    assert slices == [(0, 501), (501, 1001)]
    # the merged lists are the exact top-k of the union when every shard's list is exact
    gi, gd = oracle.bruteforce(base, q, k)
    assert np.mean([len(set(want_i[j]) & set(gi[j])) / k for j in range(q.shape[0])]) >= 0.9


def test_merge_rule_ties(oracle):
    # equal distances: lower shard first, then earlier rank in the shard's list
    ids = np.array([[[5, 6]], [[7, 8]]], np.uint32)
    d = np.array([[[1.0, 2.0]], [[1.0, 1.5]]], np.float32)
    c = np.array([[2], [2]], np.uint32)
    i, dd, cc = oracle.merge_shard_lists(ids, d, c, 100, 3)
    assert i.tolist() == [[5, 107, 108]] and dd.tolist() == [[1.0, 1.0, 1.5]] and cc.tolist() == [3]


def test_make_shard_deterministic_and_distinct():
    from raven_b200 import datasets

    a = datasets.make_shard("gmm40m-d128", 3, 8, shard_n=500)
    b = datasets.make_shard("gmm40m-d128", 3, 8, shard_n=500)
    c = datasets.make_shard("gmm40m-d128", 4, 8, shard_n=500)
    assert a.shape == (500, 128) and a.dtype == np.float32
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert np.all(a == np.rint(a)) and a.min() >= 0 and a.max() <= 255
    assert datasets.shard_index_path("gmm40m-d128", 3, 8, 500).endswith("gmm40m-d128-shard3of8-n500.annx")
