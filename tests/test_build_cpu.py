"""Host-side index build / ANNX I/O / Python API (CPU only)."""
import os
import tempfile

import numpy as np
import pytest

from annx_util import annx_bytes


def _data(n=3000, nq=200, name="gmm100k-d128"):
    from raven_b200 import datasets

    return datasets.make(name, n=n, nq=nq)


def test_build_is_deterministic_and_thread_count_independent(raven_lib):
    from raven_b200.index import Graph

    base, _ = _data(2500)
    with tempfile.TemporaryDirectory() as d:
        paths = []
        for threads in (1, 3, 8):
            g = Graph.build(base, r=16, l=40, nav_m=8, threads=threads, seed=5)
            p = os.path.join(d, f"g{threads}.annx")
            g.save(p)
            paths.append(p)
        blobs = [open(p, "rb").read() for p in paths]
    assert blobs[0] == blobs[1] == blobs[2]


def test_saved_file_is_standard_annx(raven_lib, oracle):
    """A file written by the engine's builder parses with the oracle's reader
    (independent code) into the same graph, and zlib's CRC-32 agrees."""
    import struct
    import zlib

    from raven_b200.index import Graph

    base, _ = _data(1500)
    g = Graph.build(base, r=16, l=40, nav_m=8, seed=1)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        b = open(p, "rb").read()
        oi = oracle.OracleIndex(p)
    magic, ver, flags, crc = struct.unpack("<IIII", b[:16])
    assert magic == 0x414E4E58 and ver == 1 and flags == 3
    assert crc == zlib.crc32(b[16:]) & 0xFFFFFFFF
    gi = g.info()
    assert oi.n == gi.n and oi.dim == gi.dim and oi.r_max == gi.r_max and oi.entry == gi.entry_point
    assert oi.nav_present and oi.nav_max_level == gi.nav_max_level and oi.nav_k == gi.nav_k == 8
    for node in range(0, 1500, 37):
        assert oi.neighbors(node).tolist() == g.neighbors(node).tolist()


def test_graph_roundtrip_and_reference_invariants(raven_lib):
    from raven_b200.index import Graph

    base, _ = _data(2000)
    g = Graph.build(base, r=32, l=60, nav_m=16, seed=2)
    gi = g.info()
    n = int(gi.n)
    for node in range(0, n, 13):
        nb = g.neighbors(node)
        assert len(nb) <= 32 and node not in nb.tolist() and len(set(nb.tolist())) == len(nb)
        assert np.all(nb < n)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        g2 = Graph.load(p)
        assert all(g.neighbors(i).tolist() == g2.neighbors(i).tolist() for i in range(0, n, 7))


def test_built_graph_recall_with_oracle_search(raven_lib, oracle):
    """Build quality gate: SQ4 ef=50 rr=8 recall@10 >= 0.95 on a 5k mixture."""
    from raven_b200.index import Graph

    base, q = _data(5000, 300)
    g = Graph.build(base, nav_m=16, seed=9)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        oi = oracle.OracleIndex(p)
    oi.set_vectors(base)
    r = oi.search(q, k=10, ef=50, rerank_factor=8)
    gt, _ = oracle.bruteforce(base, q, 10)
    rec = np.mean([len(set(r["ids"][i]) & set(gt[i])) / 10 for i in range(len(q))])
    assert rec >= 0.95


def test_pyo3_surface_errors(raven_lib):
    from raven_b200 import Index

    with pytest.raises(ValueError):
        Index("L2", 8, quantization="pq4")
    ix = Index("L2", 8, quantization="SQ4")  # case-insensitive like the reference
    with pytest.raises(ValueError):
        ix.build(np.zeros((10, 9), np.float32))
    with pytest.raises(RuntimeError):
        ix.searcher()
    with pytest.raises(RuntimeError):
        ix.save("/tmp/x.annx")
    with pytest.raises(IOError):
        Index.load("/nonexistent.annx", 8)


def test_index_load_without_vectors_raises_instead_of_aborting(raven_lib):
    from raven_b200 import Index

    b = annx_bytes(3, 4, 0, 2, [[1, 2], [0], [0, 1]])
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        open(p, "wb").write(b)
        ix = Index.load(p, 4)
        with pytest.raises(RuntimeError):
            ix.searcher()


def test_datasets_are_seeded():
    from raven_b200 import datasets

    a, qa = datasets.make("gmm1m-d128-sparse", n=2000, nq=50)
    b, qb = datasets.make("gmm1m-d128-sparse", n=2000, nq=50)
    assert np.array_equal(a, b) and np.array_equal(qa, qb)
    assert a.min() >= 0 and a.max() <= 255 and np.all(a == np.rint(a))
    frac0 = float((a == 0).mean())
    assert 0.28 < frac0 < 0.40
    u, _ = datasets.make("gmm10m-d96-unit", n=1000, nq=10)
    assert np.allclose(np.linalg.norm(u, axis=1), 1.0, atol=1e-5)
    _, q1 = datasets.make("gmm1m-d128-sparse", n=10, nq=50, query_offset=1)
    assert not np.array_equal(qa, q1)


def test_index_save_load_restores_vectors(tmp_path, raven_lib):
    """Index.save writes the base vectors beside the ANNX file; Index.load
    restores them, so searcher() works without re-supplying them. A damaged
    vector file is an IOError."""
    from raven_b200 import datasets
    from raven_b200.index import Index, load_vectors, vectors_path

    base, _ = datasets.make("gmm100k-d128", n=1500, nq=1)
    ix = Index("L2", 128, r=16, l=32, nav_m=8, quantization="sq4")
    ix.build(base)
    path = str(tmp_path / "ix.annx")
    ix.save(path)
    np.testing.assert_array_equal(load_vectors(vectors_path(path)), base)
    ix2 = Index.load(path, 128, quantization="sq4")
    np.testing.assert_array_equal(ix2._vectors, base)
    raw = bytearray(open(vectors_path(path), "rb").read())
    raw[100] ^= 0x55
    open(vectors_path(path), "wb").write(bytes(raw))
    with pytest.raises(IOError):
        Index.load(path, 128)
