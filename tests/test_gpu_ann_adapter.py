"""The call sequence of the ann-benchmarks adapter
(ann_benchmarks/algorithms/raven/module.py:47-91) against the `raven`
package: Index(..., adaptive_ef=True) -> build -> searcher(); fixed ef via
set_ef and AdaptiveEf via set_adaptive_ef; per-query search() and
batch_search().reshape(-1, n). Single-query results equal the batch results,
and both equal the oracle's search of the same index.
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_ann_benchmarks_call_sequence(raven_lib, oracle):
    import raven
    from raven_b200 import datasets

    base, q = datasets.make("gmm100k-d128", n=4000, nq=40)
    index = raven.Index("L2", 128, r=32, l=64, alpha=1.2, nav_m=8, directional=True, quantization="sq4",
                        rerank_factor=8, threads=0, adaptive_ef=True)
    index.build(base)
    with tempfile.TemporaryDirectory() as d:  # keep the graph for the oracle before searcher() moves it
        path = os.path.join(d, "g.annx")
        index.save(path)
        oi = oracle.OracleIndex(path)
    oi.set_vectors(base, sq4=True, adaptive=True)
    searcher = index.searcher()
    n = 10
    # fixed ef (set_query_arguments with one argument)
    searcher.set_ef(50)
    one = np.stack([searcher.search(v, n) for v in q])
    batch = searcher.batch_search(q, n).reshape(-1, n)
    np.testing.assert_array_equal(one, batch)
    exp = oi.search(q, k=n, ef=50, rerank_factor=8)
    np.testing.assert_array_equal(batch, exp["ids"].astype(batch.dtype))
    # AdaptiveEf (three arguments)
    searcher.set_adaptive_ef(2.4, 35, 75)
    batch = searcher.batch_search(q, n).reshape(-1, n)
    exp = oi.search(q, k=n, adaptive=True, gamma=2.4, min_ef=35, max_ef=75, rerank_factor=8)
    np.testing.assert_array_equal(batch, exp["ids"].astype(batch.dtype))
    np.testing.assert_array_equal(searcher.search(q[0], n), batch[0])
