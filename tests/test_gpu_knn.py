"""Exact kNN (recall ground truth) through raven_knn_exact_device against the
oracle's brute force.

Integer-valued data takes the one-pass tensor-core path (TF32-exact inputs,
exact f32 sums): distances and ids (ties by id) must be bit-identical to the
oracle's direct sum of squared differences. Non-integer data takes the
three-pass hi/lo split: distances to f32 accuracy (the |q|^2 + |x|^2 - 2q.x
form rounds differently from a direct sum, so near-ties may swap), checked
with tolerances. A dim that is not a multiple of 4 takes the CUDA-core
kernel. Shapes cover 2, 3 and 4 K blocks, k in {1, 10, 32}, and base and
query counts that are not multiples of the 128-row tiles.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _index(base, seed=3):
    from raven_b200.index import DeviceIndex, Graph

    g = Graph.build(base, r=16, l=32, alpha=1.2, nav_m=8, directional=True, seed=seed)
    return DeviceIndex(g, base, sq4=True)


def _knn(dev, q, k):
    import torch

    from raven_b200 import _lib as L

    qt = torch.from_numpy(np.ascontiguousarray(q, np.float32)).cuda()
    ids = torch.zeros((q.shape[0], k), dtype=torch.int32, device="cuda")
    ds = torch.zeros((q.shape[0], k), dtype=torch.float32, device="cuda")
    L.check(L.load().raven_knn_exact_device(dev._h, qt.data_ptr(), q.shape[0], k, ids.data_ptr(), ds.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return ids.cpu().numpy().view(np.uint32), ds.cpu().numpy()


def _int_data(n, nq, dim, seed):
    from raven_b200 import datasets

    base = datasets.clustered_int(n, dim, 40, 12.0, seed=seed, centre_seed=seed + 100)
    q = datasets.clustered_int(nq, dim, 40, 12.0, seed=seed + 1, centre_seed=seed + 100)
    return base, q


@pytest.mark.parametrize("n,nq,dim,k", [(6000, 400, 128, 10), (6000, 400, 128, 32), (6000, 400, 128, 1),
                                        (5003, 301, 96, 10), (3001, 130, 64, 16), (2000, 77, 30, 10)])
def test_knn_integer_data_exact(raven_lib, oracle, n, nq, dim, k):
    base, q = _int_data(n, nq, dim, seed=n + dim)
    dev = _index(base)
    gi, gd = _knn(dev, q, k)
    oi, od = oracle.bruteforce(base, q, k)
    np.testing.assert_array_equal(gd, od)
    np.testing.assert_array_equal(gi, oi)


def test_knn_float_data_three_pass(raven_lib, oracle):
    from raven_b200 import datasets

    base = datasets.clustered_unit(4000, 96, 30, 0.3, seed=5, centre_seed=6)
    q = datasets.clustered_unit(257, 96, 30, 0.3, seed=7, centre_seed=6)
    assert not np.all(base == np.rint(base))  # the three-pass path
    dev = _index(base)
    k = 10
    gi, gd = _knn(dev, q, k)
    oi, od = oracle.bruteforce(base, q, k)
    np.testing.assert_allclose(gd, od, rtol=1e-4, atol=2e-6)
    agree = np.mean([len(set(gi[i]) & set(oi[i])) / k for i in range(q.shape[0])])
    assert agree >= 0.995
    # whatever the order of near-ties, each returned id's true distance is within tolerance of its slot
    true_d = np.array([[np.sum((q[i] - base[j]) ** 2, dtype=np.float64) for j in gi[i]] for i in range(q.shape[0])])
    np.testing.assert_allclose(true_d, od, rtol=1e-4, atol=2e-6)
