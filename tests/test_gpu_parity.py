"""GPU engine vs the oracle (CPU restatement of the reference) on the same
index file and queries, through the C ABI.

Bar: top-k ids, result counts, visited counts, visited order (history),
ef_used, navigation evaluation counts and expansion counts are bit-exact;
f32 rerank distances within 1e-5 relative (RTOL below) — and bit-exact for
integer-valued data, where every partial sum is an exact integer.
"""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

from annx_util import annx_bytes, nav_bytes
from search_check import search_both

pytestmark = pytest.mark.gpu
RTOL = 1e-5
# Batches up to one wave of CTAs run the small-batch kernel (one CTA per
# query), larger ones the persistent one-warp-per-query kernel; the cases
# below run on both by switching the index's small-batch limit.
KERNELS = ["persistent", "cta"]


def _use(dev, path):
    from raven_b200.index import SMALL_BATCH_AUTO

    dev.set_small_batch(0 if path == "persistent" else SMALL_BATCH_AUTO)


def _oracle_for(oracle, graph, base, sq8=True, adaptive=True):
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        graph.save(p)
        oi = oracle.OracleIndex(p)
    oi.set_vectors(base, sq4=True, sq8=sq8, adaptive=adaptive)
    return oi


def _params(**kw):
    from raven_b200 import _lib as L

    p = dict(ef=50, k=10, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=0, gamma=2.0, min_ef=30, max_ef=100)
    p.update(kw)
    return L.SearchParams(**p)


def _compare(g, o, exact_dists=True, history=True):
    np.testing.assert_array_equal(g["counts"], o["counts"])
    np.testing.assert_array_equal(g["ids"], o["ids"])
    np.testing.assert_array_equal(g["visited"], o["visited"])
    np.testing.assert_array_equal(g["ef_used"], o["ef_used"])
    np.testing.assert_array_equal(g["n_nav"], o["n_nav"])
    np.testing.assert_array_equal(g["expansions"], o["expansions"])
    assert np.all(g["status"] == 0)
    np.testing.assert_allclose(g["dists"], o["dists"], rtol=RTOL, atol=0)
    if exact_dists:
        np.testing.assert_array_equal(g["dists"], o["dists"])
    if history:
        np.testing.assert_array_equal(g["history_len"], o["history_len"])
        cap = g["history"].shape[1]
        for i in range(g["history"].shape[0]):
            h = min(int(g["history_len"][i]), cap)
            np.testing.assert_array_equal(g["history"][i, :h], o["history"][i, :h])


@pytest.fixture(scope="module", params=KERNELS)
def small(request, small_case, oracle):
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, sq8=True, adaptive=True)
    _use(dev, request.param)
    oi = _oracle_for(oracle, g, base)
    return base, q, g, dev, oi


def test_device_codes_and_params_match_oracle(small):
    base, q, g, dev, oi = small
    for quant in (0, 1):
        np.testing.assert_array_equal(dev.sq_params(quant), oi.sq_params(quant))
        np.testing.assert_array_equal(dev.codes(quant), oi.codes(quant))


def test_adaptive_samples_match_oracle(small):
    base, q, g, dev, oi = small
    np.testing.assert_array_equal(dev.adaptive_samples(), oi.adaptive_samples())


@pytest.mark.parametrize("ef,k,rr", [(50, 10, 8), (10, 10, 5), (1, 1, 1), (100, 10, 3), (64, 32, 2), (5, 10, 8),
                                     (200, 10, 8)])
def test_search_sq4_parity(small, ef, k, rr):
    base, q, g, dev, oi = small
    got = search_both(dev, q, _params(ef=ef, k=k, rerank_factor=rr), history_cap=4096)
    exp = oi.search(q, k=k, ef=ef, rerank_factor=rr, quant=0, history_cap=4096)
    _compare(got, exp)


@pytest.mark.parametrize("ef,k", [(50, 10), (10, 10), (1, 1), (200, 10), (64, 32)])
def test_search_f32_parity(small, ef, k):
    """GraphSearcher::search: the beam over f32 distances, results = the first
    k of the pool (no rerank)."""
    from raven_b200 import _lib as L

    base, q, g, dev, oi = small
    got = search_both(dev, q, _params(ef=ef, k=k, quant=L.RAVEN_QUANT_F32), history_cap=4096)
    exp = oi.search(q, k=k, ef=ef, quant=2, history_cap=4096)
    _compare(got, exp)


@pytest.mark.parametrize("ef", [40, 50, 100])
def test_search_sq8_parity(small, ef):
    base, q, g, dev, oi = small
    got = search_both(dev, q, _params(ef=ef, quant=1), history_cap=4096)
    exp = oi.search(q, k=10, ef=ef, rerank_factor=8, quant=1, history_cap=4096)
    _compare(got, exp)


@pytest.mark.parametrize("gamma,lo,hi", [(2.0, 35, 65), (2.4, 35, 75), (3.5, 35, 85), (1.0, 10, 10)])
def test_adaptive_ef_parity(small, gamma, lo, hi):
    base, q, g, dev, oi = small
    got = search_both(dev, q, _params(adaptive=1, gamma=gamma, min_ef=lo, max_ef=hi), history_cap=4096)
    exp = oi.search(q, k=10, rerank_factor=8, adaptive=True, gamma=gamma, min_ef=lo, max_ef=hi, history_cap=4096)
    _compare(got, exp)
    assert got["ef_used"].min() >= max(lo, 10) or lo < 10


def test_base_vectors_find_themselves(small):
    # src/graph/vamana.rs:2169-2191: the query itself ranks first.
    base, q, g, dev, oi = small
    idx = np.arange(0, base.shape[0], 97)
    got = search_both(dev, base[idx], _params(ef=50, k=5))
    np.testing.assert_array_equal(got["ids"][:, 0], idx)
    assert np.all(got["dists"][:, 0] == 0.0)


@pytest.mark.parametrize("path", KERNELS)
def test_float_data_parity_dim96(oracle, raven_lib, path):
    """Unit-normalised floats: nav entry points and rerank depend on the
    AVX-512 summation order, which the device reproduces."""
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex, Graph

    base, q = datasets.make("gmm10m-d96-unit", n=5000, nq=300)
    g = Graph.build(base, r=32, l=64, nav_m=8, seed=3)
    dev = DeviceIndex(g, base, sq4=True, sq8=True, adaptive=True)
    _use(dev, path)
    oi = _oracle_for(oracle, g, base)
    np.testing.assert_array_equal(dev.adaptive_samples(), oi.adaptive_samples())
    for quant in (0, 1, 2):
        got = search_both(dev, q, _params(ef=50, quant=quant), history_cap=4096)
        exp = oi.search(q, k=10, ef=50, rerank_factor=8, quant=quant, history_cap=4096)
        _compare(got, exp, exact_dists=True)
    got = search_both(dev, q, _params(adaptive=1, gamma=2.0, min_ef=35, max_ef=75), history_cap=4096)
    exp = oi.search(q, k=10, rerank_factor=8, adaptive=True, gamma=2.0, min_ef=35, max_ef=75, history_cap=4096)
    _compare(got, exp)


def _handmade(oracle, n, dim, r_max, rows, nav=None, seed=0, path="persistent"):
    from raven_b200.index import DeviceIndex, Graph

    rng = np.random.default_rng(seed)
    base = rng.integers(0, 256, size=(n, dim)).astype(np.float32)
    b = annx_bytes(n, dim, 0, r_max, rows, nav=nav)
    g = Graph.from_bytes(b)
    dev = DeviceIndex(g, base, sq4=True, sq8=True, adaptive=nav is not None)
    _use(dev, path)
    oi = oracle.OracleIndex(data=b)
    oi.set_vectors(base, sq4=True, sq8=True, adaptive=nav is not None)
    q = rng.integers(0, 256, size=(64, dim)).astype(np.float32)
    return base, q, dev, oi


@pytest.mark.parametrize("path", KERNELS)
@pytest.mark.parametrize("r_max", [20, 32, 64, 96])
def test_degree_padding_and_wide_rows(oracle, raven_lib, r_max, path):
    rng = np.random.default_rng(r_max)
    n, dim = 700, 32
    rows = []
    for i in range(n):
        deg = int(rng.integers(0, r_max + 1))
        rows.append([int(x) for x in rng.choice(n, size=deg, replace=False)])
    base, q, dev, oi = _handmade(oracle, n, dim, r_max, rows, path=path)
    for quant in (0, 1, 2):
        got = search_both(dev, q, _params(ef=40, quant=quant), history_cap=2048)
        exp = oi.search(q, k=10, ef=40, rerank_factor=8, quant=quant, history_cap=2048)
        _compare(got, exp)


@pytest.mark.parametrize("path", KERNELS)
def test_duplicate_ids_in_a_row(oracle, raven_lib, path):
    # The reference's visited tracker counts the first occurrence only.
    rng = np.random.default_rng(9)
    n, dim = 300, 16
    rows = []
    for i in range(n):
        r = [int(x) for x in rng.integers(0, n, size=24)]  # with repeats
        rows.append(r)
    base, q, dev, oi = _handmade(oracle, n, dim, 32, rows, path=path)
    got = search_both(dev, q, _params(ef=30), history_cap=1024)
    exp = oi.search(q, k=10, ef=30, rerank_factor=8, history_cap=1024)
    _compare(got, exp)


@pytest.mark.parametrize("path", KERNELS)
def test_graph_without_nav_uses_medoid(oracle, raven_lib, path):
    rng = np.random.default_rng(4)
    n = 500
    rows = [[int(x) for x in rng.choice(n, size=16, replace=False)] for _ in range(n)]
    base, q, dev, oi = _handmade(oracle, n, 24, 16, rows, path=path)
    got = search_both(dev, q, _params(ef=20), history_cap=1024)
    exp = oi.search(q, k=10, ef=20, rerank_factor=8, history_cap=1024)
    _compare(got, exp)
    assert np.all(got["n_nav"] == 0)


@pytest.mark.parametrize("path", KERNELS)
def test_handmade_nav_with_self_padding(oracle, raven_lib, path):
    rng = np.random.default_rng(8)
    n, dim, k = 400, 16, 4
    rows = [[int(x) for x in rng.choice(n, size=12, replace=False)] for _ in range(n)]
    levels = [0] * n
    upper = [[] for _ in range(n)]
    l1 = list(range(0, n, 7))
    l2 = list(range(0, n, 49))
    for u in l1:
        levels[u] = 1
    for u in l2:
        levels[u] = 2
    for u in l1:
        e1 = [int(x) for x in rng.choice(l1, size=3, replace=False)] + [u]  # padded with self
        upper[u] = e1
    for u in l2:
        e2 = [int(x) for x in rng.choice(l2, size=2, replace=False)] + [u, u]
        upper[u] = upper[u] + e2
    nav = nav_bytes(0, 2, k, levels, upper, [0])
    base, q, dev, oi = _handmade(oracle, n, dim, 12, rows, nav=nav, path=path)
    got = search_both(dev, q, _params(ef=16), history_cap=1024)
    exp = oi.search(q, k=10, ef=16, rerank_factor=8, history_cap=1024)
    _compare(got, exp)
    got = search_both(dev, q, _params(adaptive=1, gamma=2.0, min_ef=8, max_ef=30), history_cap=1024)
    exp = oi.search(q, k=10, rerank_factor=8, adaptive=True, gamma=2.0, min_ef=8, max_ef=30, history_cap=1024)
    _compare(got, exp)


def test_empty_batch_and_padding(small):
    base, q, g, dev, oi = small
    r = search_both(dev, q[:0], _params())
    assert r["ids"].shape == (0, 10)
    # k larger than the pool: fewer results, zero padding (src/python.rs:344-349)
    got = search_both(dev, q[:20], _params(ef=4, k=10, rerank_factor=1))
    exp = oi.search(q[:20], k=10, ef=4, rerank_factor=1)
    np.testing.assert_array_equal(got["counts"], exp["counts"])
    assert np.all(got["counts"] == 4)
    assert np.all(got["ids"][:, 4:] == 0) and np.all(got["dists"][:, 4:] == 0)
    np.testing.assert_array_equal(got["ids"], exp["ids"])


def test_nan_and_extreme_queries(small):
    base, q, g, dev, oi = small
    qq = q[:8].copy()
    qq[0, 5] = np.nan
    qq[1, :] = 1e30
    qq[2, :] = -1e30
    qq[3, :] = 0.0
    got = search_both(dev, qq, _params(), history_cap=4096)
    exp = oi.search(qq, k=10, ef=50, rerank_factor=8, history_cap=4096)
    np.testing.assert_array_equal(got["ids"], exp["ids"])
    np.testing.assert_array_equal(got["visited"], exp["visited"])
    np.testing.assert_array_equal(got["history_len"], exp["history_len"])
    for i in range(qq.shape[0]):
        h = int(got["history_len"][i])
        np.testing.assert_array_equal(got["history"][i, :h], exp["history"][i, :h])


def test_errors_are_status_codes(small):
    from raven_b200 import _lib as L

    base, q, g, dev, oi = small
    with pytest.raises(L.RavenError) as e:
        search_both(dev, q[:2], _params(ef=0))
    assert e.value.code == L.RAVEN_EINVAL
    with pytest.raises(L.RavenError) as e:
        search_both(dev, q[:2], _params(ef=300))
    assert e.value.code == L.RAVEN_ELIMIT
    with pytest.raises(L.RavenError) as e:
        search_both(dev, q[:2], _params(k=0))
    assert e.value.code == L.RAVEN_EINVAL
    with pytest.raises(L.RavenError) as e:
        search_both(dev, q[:2], _params(adaptive=1, min_ef=50, max_ef=10))
    assert e.value.code == L.RAVEN_EINVAL


def test_quantiser_not_uploaded_is_state_error(small_case, raven_lib):
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, sq8=False)
    with pytest.raises(L.RavenError) as e:
        search_both(dev, q[:2], _params(quant=1))
    assert e.value.code == L.RAVEN_ESTATE


@pytest.mark.parametrize("hash_bits,spill_bits,ef", [(8, 0, 100), (8, 10, 200)])
def test_small_visited_table_spills_exactly(small, hash_bits, spill_bits, ef):
    """Force the shared-memory visited table over into the global spill levels
    (256 shared slots; with 1024-slot level A, level B takes the rest); results
    stay exact."""
    base, q, g, dev, oi = small
    dev.set_tuning(hash_bits=hash_bits, spill_bits=spill_bits)
    try:
        got = search_both(dev, q, _params(ef=ef), history_cap=8192)
        exp = oi.search(q, k=10, ef=ef, rerank_factor=8, history_cap=8192)
        _compare(got, exp)
        if spill_bits:
            assert got["visited"].max() > 192 + 768  # some queries reached level B
    finally:
        dev.set_tuning(hash_bits=0, spill_bits=0)


def test_device_entry_point_matches_host_entry(small):
    import torch

    from raven_b200 import _lib as L

    base, q, g, dev, oi = small
    qt = torch.from_numpy(q).cuda()
    nq, k = q.shape[0], 10
    ids = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
    ds = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    out = L.SearchOutputs(ids=C.cast(ids.data_ptr(), L.u32p), dists=C.cast(ds.data_ptr(), L.f32p))
    st = torch.cuda.current_stream()
    L.check(L.load().raven_search_batch_device(dev._h, qt.data_ptr(), nq, C.byref(_params()), C.byref(out),
                                               st.cuda_stream))
    torch.cuda.synchronize()
    host = search_both(dev, q, _params())
    np.testing.assert_array_equal(ids.cpu().numpy().view(np.uint32), host["ids"])
    np.testing.assert_array_equal(ds.cpu().numpy(), host["dists"])


def test_exact_knn_kernel(small, oracle):
    import torch

    from raven_b200 import _lib as L

    base, q, g, dev, oi = small
    k = 10
    qt = torch.from_numpy(q).cuda()
    ids = torch.zeros((q.shape[0], k), dtype=torch.int32, device="cuda")
    ds = torch.zeros((q.shape[0], k), dtype=torch.float32, device="cuda")
    L.check(L.load().raven_knn_exact_device(dev._h, qt.data_ptr(), q.shape[0], k, ids.data_ptr(), ds.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    gi, gd = oracle.bruteforce(base, q, k)
    np.testing.assert_array_equal(ds.cpu().numpy(), gd)
    np.testing.assert_array_equal(ids.cpu().numpy().view(np.uint32), gi)


def test_shard_merge_kernel():
    import torch

    from raven_b200 import _lib as L

    rng = np.random.default_rng(1)
    S, nq, k, shard = 4, 300, 10, 1000
    d = np.sort(rng.integers(0, 50, size=(S, nq, k)).astype(np.float32), axis=2)  # many ties
    i = rng.integers(0, shard, size=(S, nq, k)).astype(np.uint32)
    cnt = rng.integers(5, k + 1, size=(S, nq)).astype(np.uint32)
    exp_i = np.zeros((nq, k), np.uint32)
    exp_d = np.zeros((nq, k), np.float32)
    for qi in range(nq):
        c = [(d[s, qi, r], s, r, s * shard + int(i[s, qi, r])) for s in range(S) for r in range(cnt[s, qi])]
        c.sort(key=lambda t: (t[0], t[1], t[2]))
        for r, t in enumerate(c[:k]):
            exp_d[qi, r], exp_i[qi, r] = t[0], t[3]
    td, ti, tc = (torch.from_numpy(x).cuda() for x in (d, i.view(np.int32), cnt.view(np.int32)))
    oi_ = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
    od = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    oc = torch.zeros(nq, dtype=torch.int32, device="cuda")
    L.check(L.load().raven_merge_topk_device(ti.data_ptr(), td.data_ptr(), tc.data_ptr(), S, nq, k, shard,
                                             oi_.data_ptr(), od.data_ptr(), oc.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(oi_.cpu().numpy().view(np.uint32), exp_i)
    np.testing.assert_array_equal(od.cpu().numpy(), exp_d)
    assert np.all(oc.cpu().numpy() == k)


def test_gmm100k_full_parity(oracle, raven_lib):
    """The CPU-runnable reference configuration: 100k x 128, 10k queries,
    ef=50, k=10, rr=8 — every output compared."""
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex

    base, q = datasets.make("gmm100k-d128")
    g = datasets.load_or_build("gmm100k-d128", base=base)
    dev = DeviceIndex(g, base, sq4=True, sq8=False, adaptive=True)
    oi = _oracle_for(oracle, g, base, sq8=False)
    got = search_both(dev, q, _params(ef=50, k=10, rerank_factor=8), history_cap=4096)
    exp = oi.search(q, k=10, ef=50, rerank_factor=8, history_cap=4096)
    _compare(got, exp)
    gi, _ = oracle.bruteforce(base, q[:1000], 10)
    rec = np.mean([len(set(got["ids"][j]) & set(gi[j])) / 10 for j in range(1000)])
    assert rec >= 0.95


def test_gmm1m_headline_parity(oracle, raven_lib):
    """The headline 1M x 128 workload (SQ4, k=10, rr=8) at ef=50 and at its
    recall>=0.95 operating point ef=140: 2,000 queries compared with the oracle
    on every output, and no query of a 10,000 batch hits a capacity limit.
    Without a cached index file the graph is built here with the GPU build
    (about a minute) and cached; parity holds on whichever graph is searched."""
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex

    wl = "gmm1m-d128-sparse"
    base, _ = datasets.make(wl, nq=1)
    q = datasets.make_queries(wl, 10000)
    g = datasets.load_or_build(wl, base=base, device=0)
    dev = DeviceIndex(g, base, sq4=True)
    oi = _oracle_for(oracle, g, base, sq8=False, adaptive=False)
    for ef in (50, 140):
        full = search_both(dev, q, _params(ef=ef))
        assert np.all(full["status"] == 0)
        got = search_both(dev, q[:2000], _params(ef=ef), history_cap=8192)
        exp = oi.search(q[:2000], k=10, ef=ef, rerank_factor=8, history_cap=8192)
        _compare(got, exp)


@pytest.mark.parametrize("path", KERNELS)
@pytest.mark.parametrize("dim", [70, 131])
def test_odd_dim_parity(oracle, raven_lib, dim, path):
    """Dims whose 16-lane chains are a multiple of 4 long but whose rows are not
    a multiple of 4 floats: staged rows are then not 16-byte aligned (scalar
    loads), descent, search and rerank must still match the oracle."""
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex, Graph

    base = datasets.clustered_int(3000, dim, 30, 12.0, seed=dim, centre_seed=dim + 1)
    q = datasets.clustered_int(200, dim, 30, 12.0, seed=dim + 2, centre_seed=dim + 1)
    g = Graph.build(base, r=32, l=64, alpha=1.2, nav_m=8, directional=True, seed=3)
    dev = DeviceIndex(g, base, sq4=True, sq8=dim <= 128, adaptive=True)
    _use(dev, path)
    oi = _oracle_for(oracle, g, base, sq8=dim <= 128)
    for quant in ([0, 1] if dim <= 128 else [0]):
        got = search_both(dev, q, _params(ef=50, k=10, rerank_factor=8, quant=quant), history_cap=4096)
        exp = oi.search(q, k=10, ef=50, rerank_factor=8, quant=quant, history_cap=4096)
        _compare(got, exp)


@pytest.mark.parametrize("dim", [128, 70, 75])
def test_f16_rerank_parity(oracle, raven_lib, dim):
    """GraphSearcher::with_f16: rerank on the f16 vectors (F16Dataset) with
    l2_f16_mixed's order, on float data so the conversion rounds; 16-byte,
    4-byte and plain-load staging of the f16 rows."""
    from raven_b200 import datasets
    from raven_b200.index import DeviceIndex, Graph

    base = datasets.clustered_unit(3000, dim, 30, 0.3, seed=dim, centre_seed=dim + 1) * 3.0
    q = datasets.clustered_unit(200, dim, 30, 0.3, seed=dim + 2, centre_seed=dim + 1) * 3.0
    g = Graph.build(base, r=32, l=64, alpha=1.2, nav_m=8, directional=True, seed=3)
    dev = DeviceIndex(g, base, sq4=True, f16=True)
    oi = _oracle_for(oracle, g, base, sq8=False, adaptive=False)
    oi.set_vectors(base, sq4=True, f16=True)
    got = search_both(dev, q, _params(ef=50, k=10, rerank_factor=8, rerank_f16=1), history_cap=4096)
    exp = oi.search(q, k=10, ef=50, rerank_factor=8, history_cap=4096, rerank_f16=True)
    _compare(got, exp)
    f32 = oi.search(q, k=10, ef=50, rerank_factor=8)
    assert not np.array_equal(exp["dists"], f32["dists"])  # the f16 path really differs from the f32 one
