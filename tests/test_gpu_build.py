"""Vamana build with the per-batch search + DirectionalPrune on the GPU
(raven_graph_build_gpu): a valid graph (degrees within r_max, no self loops,
no repeated neighbours, ids in range, navigation built), deterministic (two
builds serialise to the same bytes), and the same graph as the host build
(raven_graph_build), byte for byte, on integer and on float data: the GPU's
candidate search is the f32 beam of greedy_search_vec_build and its prune
takes the same decisions with the same distances.
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def data(raven_lib):
    from raven_b200 import datasets

    base = datasets.clustered_int(20000, 128, 200, 12.0, seed=11, centre_seed=12)
    q = datasets.clustered_int(500, 128, 200, 12.0, seed=13, centre_seed=12)
    return base, q


def _build(base, device):
    from raven_b200.index import Graph

    return Graph.build(base, r=32, l=100, alpha=1.2, nav_m=16, directional=True, seed=5, device=device)


def _bytes(g):
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        return open(p, "rb").read()


def test_gpu_build_structure_and_determinism(data):
    base, _ = data
    g1 = _build(base, 0)
    n = base.shape[0]
    info = g1.info()
    assert info.n == n and info.r_max == 32 and info.has_nav
    for v in range(0, n, 97):
        nb = g1.neighbors(v)
        assert len(nb) <= 32
        assert v not in set(nb.tolist())
        assert len(set(nb.tolist())) == len(nb)
        assert np.all(nb < n)
    assert _bytes(g1) == _bytes(_build(base, 0))


def test_gpu_build_equals_host_build(data, oracle):
    from raven_b200 import _lib as L
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex, Graph

    base, q = data
    gpu = _build(base, 0)
    assert _bytes(gpu) == _bytes(_build(base, None))
    # float data: the AVX-512 summation order decides both builds' comparisons
    fb = datasets.clustered_unit(8000, 96, 80, 0.3, seed=21, centre_seed=22)
    kw = dict(r=32, l=100, alpha=1.2, nav_m=16, directional=True, seed=9)
    assert _bytes(Graph.build(fb, device=0, **kw)) == _bytes(Graph.build(fb, **kw))
    # and the graph searches with oracle parity
    dev = DeviceIndex(gpu, base, sq4=True)
    p = L.SearchParams(ef=50, k=10, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=0, gamma=0.0, min_ef=0,
                       max_ef=0)
    got = dev.search(q, p, visited=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "g.annx")
        gpu.save(path)
        oi = oracle.OracleIndex(path)
    oi.set_vectors(base, sq4=True)
    exp = oi.search(q, k=10, ef=50, rerank_factor=8)
    np.testing.assert_array_equal(got["ids"], exp["ids"])
    np.testing.assert_array_equal(got["visited"], exp["visited"])


def test_saved_index_serves_without_vectors(tmp_path, raven_lib):
    """Index.save -> Index.load(path, dim) -> searcher(): the vectors come from
    the file saved beside the graph; results equal the original searcher's."""
    from raven_b200 import datasets
    from raven_b200.index import Index

    base, q = datasets.make("gmm100k-d128", n=3000, nq=100)
    ix = Index("L2", 128, r=16, l=32, nav_m=8, quantization="sq4", rerank_factor=8)
    ix.build(base)
    path = str(tmp_path / "ix.annx")
    ix.save(path)
    s1 = ix.searcher()
    s1.set_ef(50)
    want = s1.batch_search(q, 10)
    s2 = Index.load(path, 128, quantization="sq4", rerank_factor=8).searcher()
    s2.set_ef(50)
    np.testing.assert_array_equal(s2.batch_search(q, 10), want)
