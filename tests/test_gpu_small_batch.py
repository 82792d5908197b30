"""The small-batch path (one CTA of four warps per query, search_cta.cuh),
taken by searches of at most `small_batch_max` queries (default: one wave of
CTAs, three per SM at dim 128),
against the oracle on every output — ids, distances, counts, visited counts
and order, ef used, navigation evaluations, expansions — and against the
persistent one-warp-per-query kernel on the same queries.
"""
import os
import tempfile

import numpy as np
import pytest
from search_check import search_both

from test_gpu_parity import _compare, _params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def case(small_case, oracle):
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, sq8=True, adaptive=True)
    with tempfile.TemporaryDirectory() as d:
        p = os.path.join(d, "g.annx")
        g.save(p)
        oi = oracle.OracleIndex(p)
    oi.set_vectors(base, sq4=True, sq8=True, adaptive=True)
    return base, q, dev, oi


@pytest.mark.parametrize("nq", [1, 8, 64])
@pytest.mark.parametrize("ef,k,rr", [(50, 10, 8), (140, 10, 8), (1, 1, 1), (200, 32, 2)])
def test_small_batch_sq4_parity(case, nq, ef, k, rr):
    base, q, dev, oi = case
    got = search_both(dev, q[:nq], _params(ef=ef, k=k, rerank_factor=rr), history_cap=8192)
    exp = oi.search(q[:nq], k=k, ef=ef, rerank_factor=rr, history_cap=8192)
    _compare(got, exp)


def test_small_batch_sq8_and_adaptive_parity(case):
    base, q, dev, oi = case
    got = search_both(dev, q[:64], _params(ef=60, quant=1), history_cap=8192)
    exp = oi.search(q[:64], k=10, ef=60, rerank_factor=8, quant=1, history_cap=8192)
    _compare(got, exp)
    got = search_both(dev, q[:64], _params(adaptive=1, gamma=2.4, min_ef=35, max_ef=75), history_cap=8192)
    exp = oi.search(q[:64], k=10, rerank_factor=8, adaptive=True, gamma=2.4, min_ef=35, max_ef=75, history_cap=8192)
    _compare(got, exp)


def test_small_batch_spill_levels_exact(case):
    """A 256-slot shared table and 1024-slot level A (tuning hook) send the
    queries through both global spill levels of the small-batch kernel."""
    base, q, dev, oi = case
    dev.set_tuning(hash_bits=8, spill_bits=10)
    try:
        got = search_both(dev, q[:64], _params(ef=200), history_cap=8192)
    finally:
        dev.set_tuning(hash_bits=0, spill_bits=0)
    exp = oi.search(q[:64], k=10, ef=200, rerank_factor=8, history_cap=8192)
    assert np.mean(exp["visited"] > 224 + 768) > 0.5  # past level A (3/4 of 1024 slots) into level B
    _compare(got, exp)


def test_small_batch_equals_persistent_kernel(case):
    base, q, dev, oi = case
    p = _params(ef=100)
    small = search_both(dev, q[:400], p, history_cap=8192)
    dev.set_small_batch(0)
    try:
        batch = search_both(dev, q[:400], p, history_cap=8192)
    finally:
        from raven_b200.index import SMALL_BATCH_AUTO

        dev.set_small_batch(SMALL_BATCH_AUTO)
    for key in small:
        np.testing.assert_array_equal(small[key], batch[key], err_msg=key)
