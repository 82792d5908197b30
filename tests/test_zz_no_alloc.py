"""raven_search_batch_device_noalloc: the device search for callers that may
not allocate GPU memory while serving (their memory is reserved up front by
another allocator, or a fixed memory budget is set at start-up). Its scratch
comes from a fixed device array inside the library instead of the allocator.

Checked through the C ABI against raven_search_batch_device on the same index,
queries and parameters, for calls in a row (the fixed array keeps the previous
call's contents, so later calls show that leftover state does not leak into
results): every output, the visited order included. The second test shrinks the
shared-memory visited table so that queries continue in both global spill
levels, and runs enough queries that the fixed array's block cap applies and
warp slots are reused within a call. This file is collected last so that a
failure here does not stop the rest of the GPU suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
RTOL = 1e-5  # the f32 rerank tolerance used by the parity tests
HIST = 8192


def _run(lib, L, fn, dev, q, params, visited=True):
    import torch

    nq, k = q.shape[0], params.k
    qt = torch.from_numpy(q).cuda()
    ids = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
    ds = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    stats = {n: torch.zeros(nq, dtype=torch.int32, device="cuda")
             for n in ("counts", "visited", "status", "ef_used", "history_len")}
    hist = torch.zeros((nq, HIST), dtype=torch.int32, device="cuda")
    out = L.SearchOutputs(ids=C.cast(ids.data_ptr(), L.u32p), dists=C.cast(ds.data_ptr(), L.f32p),
                          counts=C.cast(stats["counts"].data_ptr(), L.u32p),
                          ef_used=C.cast(stats["ef_used"].data_ptr(), L.u32p),
                          status=C.cast(stats["status"].data_ptr(), L.i32p))
    if visited:  # the visited count and order: the search keeps the exact visited set
        out.visited = C.cast(stats["visited"].data_ptr(), L.u32p)
        out.history = C.cast(hist.data_ptr(), L.u32p)
        out.history_cap = HIST
        out.history_len = C.cast(stats["history_len"].data_ptr(), L.u32p)
    stream = torch.cuda.Stream()
    L.check(fn(dev._h, qt.data_ptr(), nq, C.byref(params), C.byref(out), stream.cuda_stream))
    torch.cuda.synchronize()
    res = {"ids": ids.cpu().numpy().view(np.uint32), "dists": ds.cpu().numpy(),
           "history": hist.cpu().numpy().view(np.uint32)}
    res.update({n: t.cpu().numpy() for n, t in stats.items()})
    return res


def _same(got, want):
    assert np.all(got["status"] == 0)
    for key in ("ids", "counts", "visited", "ef_used", "history_len"):
        np.testing.assert_array_equal(got[key], want[key], err_msg=key)
    for i in range(got["history"].shape[0]):
        h = min(int(got["history_len"][i]), HIST)
        np.testing.assert_array_equal(got["history"][i, :h], want["history"][i, :h])
    np.testing.assert_allclose(got["dists"], want["dists"], rtol=RTOL, atol=0)


def _params(L, **kw):
    p = dict(ef=50, k=10, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=0, gamma=0.0, min_ef=0, max_ef=0)
    p.update(kw)
    return L.SearchParams(**p)


def test_noalloc_search_matches_allocating_search_twice(small_case, raven_lib):
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, adaptive=True)
    calls = [_params(L, ef=50), _params(L, ef=100, adaptive=1, gamma=2.0, min_ef=35, max_ef=120)]
    for params in calls:  # two calls in a row on the shared fixed array
        want = _run(raven_lib, L, raven_lib.raven_search_batch_device, dev, q, params)
        got = _run(raven_lib, L, raven_lib.raven_search_batch_device_noalloc, dev, q, params)
        _same(got, want)


def test_noalloc_spilling_queries_reuse_slots(small_case, raven_lib):
    """A 256-slot shared table (tuning hook) sends every query into spill level
    A, and at ef=200 most into level B too; 4,000 queries need more warp slots
    than the fixed array holds, so slots (and their spill tables) are reused
    inside the call. Run twice in a row, against the allocating search."""
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True)
    dev.set_tuning(hash_bits=8)
    qq = np.ascontiguousarray(np.tile(q, (10, 1)))  # 4,000 queries
    params = _params(L, ef=200)
    want = _run(raven_lib, L, raven_lib.raven_search_batch_device, dev, qq, params)
    assert np.mean(want["visited"] > 256 + 1536) > 0.5  # most queries reach level B of the fixed array's tables
    for _ in range(2):
        got = _run(raven_lib, L, raven_lib.raven_search_batch_device_noalloc, dev, qq, params)
        _same(got, want)


def test_noalloc_without_visited_counts(small_case, raven_lib):
    """Without the visited count and order the search keeps no visited tables
    (pool membership decides new neighbours) and the fixed array holds only
    the work counter and the ef table: 4,000 queries at ef=200 in one grid,
    twice in a row, against the allocating search in the same mode and in the
    exact-visited mode."""
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, adaptive=True)
    qq = np.ascontiguousarray(np.tile(q, (10, 1)))
    for params in (_params(L, ef=200), _params(L, ef=100, adaptive=1, gamma=2.0, min_ef=35, max_ef=120)):
        exact = _run(raven_lib, L, raven_lib.raven_search_batch_device, dev, qq, params)
        want = _run(raven_lib, L, raven_lib.raven_search_batch_device, dev, qq, params, visited=False)
        for _ in range(2):
            got = _run(raven_lib, L, raven_lib.raven_search_batch_device_noalloc, dev, qq, params, visited=False)
            assert np.all(got["status"] == 0)
            for key in ("ids", "dists", "counts", "ef_used"):
                np.testing.assert_array_equal(got[key], want[key], err_msg=key)
                np.testing.assert_array_equal(got[key], exact[key], err_msg=key)
