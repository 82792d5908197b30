"""raven_search_batch_device_noalloc: the device search for callers that may
not allocate GPU memory while serving (their memory is reserved up front by
another allocator, or a fixed memory budget is set at start-up). Its scratch
comes from a fixed device array inside the library instead of the allocator.

Checked through the C ABI against raven_search_batch_device on the same index,
queries and parameters, for two calls in a row (the fixed array keeps the
previous call's contents, so the second call shows that leftover state does not
leak into results). This file is collected last so that a failure here does not
stop the rest of the GPU suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
RTOL = 1e-5  # the f32 rerank tolerance used by the parity tests


def _run(lib, L, fn, dev, q, params):
    import torch

    nq, k = q.shape[0], params.k
    qt = torch.from_numpy(q).cuda()
    ids = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
    ds = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
    stats = {n: torch.zeros(nq, dtype=torch.int32, device="cuda") for n in ("counts", "visited", "status")}
    out = L.SearchOutputs(ids=C.cast(ids.data_ptr(), L.u32p), dists=C.cast(ds.data_ptr(), L.f32p),
                          counts=C.cast(stats["counts"].data_ptr(), L.u32p),
                          visited=C.cast(stats["visited"].data_ptr(), L.u32p),
                          status=C.cast(stats["status"].data_ptr(), L.i32p))
    stream = torch.cuda.Stream()
    L.check(fn(dev._h, qt.data_ptr(), nq, C.byref(params), C.byref(out), stream.cuda_stream))
    torch.cuda.synchronize()
    res = {"ids": ids.cpu().numpy().view(np.uint32), "dists": ds.cpu().numpy()}
    res.update({n: t.cpu().numpy() for n, t in stats.items()})
    return res


def test_noalloc_search_matches_allocating_search_twice(small_case, raven_lib):
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex

    base, q, g = small_case
    dev = DeviceIndex(g, base, sq4=True, adaptive=True)
    calls = [
        L.SearchParams(ef=50, k=10, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=0, gamma=0.0, min_ef=0,
                       max_ef=0),
        L.SearchParams(ef=100, k=10, rerank_factor=8, prefetch_offset=8, quant=0, adaptive=1, gamma=2.0,
                       min_ef=35, max_ef=120),
    ]
    for params in calls:  # two calls in a row on the shared fixed array
        want = _run(raven_lib, L, raven_lib.raven_search_batch_device, dev, q, params)
        got = _run(raven_lib, L, raven_lib.raven_search_batch_device_noalloc, dev, q, params)
        assert np.all(got["status"] == 0)
        np.testing.assert_array_equal(got["ids"], want["ids"])
        np.testing.assert_array_equal(got["counts"], want["counts"])
        np.testing.assert_array_equal(got["visited"], want["visited"])
        np.testing.assert_allclose(got["dists"], want["dists"], rtol=RTOL, atol=0)
