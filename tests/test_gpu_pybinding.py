"""The reference's end-to-end binding scenario (test_pybinding.py: 1000 x 64
Gaussian base vectors, 10 queries, Index("L2", 64, r=16, l=100, alpha=1.2,
nav_m=16, directional=True) with the default quantization, SQ8, and rerank
factor 5; single-query and batch search; ef switched over 20/50/100; recall
against brute force) through the `raven` package. Beyond the
reference's printed recall: single and batch results are equal, both equal
the oracle's search of the same index at every ef, and recall does not drop
as ef grows.
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_pybinding_scenario(raven_lib, oracle):
    import raven

    rng = np.random.default_rng(42)
    data = rng.standard_normal((1000, 64)).astype(np.float32)
    queries = rng.standard_normal((10, 64)).astype(np.float32)
    k = 10
    index = raven.Index("L2", 64, r=16, l=100, alpha=1.2, nav_m=16, directional=True)
    index.build(data)
    with tempfile.TemporaryDirectory() as d:  # keep the graph for the oracle before searcher() moves it
        path = os.path.join(d, "g.annx")
        index.save(path)
        oi = oracle.OracleIndex(path)
    oi.set_vectors(data, sq4=False, sq8=True)
    gt, _ = oracle.bruteforce(data, queries, k)
    searcher = index.searcher()
    recalls = []
    for ef in (20, 50, 100):
        searcher.set_ef(ef)
        one = np.stack([searcher.search(v, k) for v in queries])
        assert searcher.last_ef_used == ef
        batch = searcher.batch_search(queries, k).reshape(-1, k)
        np.testing.assert_array_equal(one, batch)
        exp = oi.search(queries, k=k, ef=ef, rerank_factor=5, quant=1)
        np.testing.assert_array_equal(batch, exp["ids"].astype(batch.dtype))
        recalls.append(np.mean([len(set(batch[i].tolist()) & set(gt[i].tolist())) / k for i in range(len(queries))]))
    assert recalls == sorted(recalls) and recalls[1] >= 0.9
