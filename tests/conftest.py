import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _has_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def raven_lib():
    from raven_b200 import build

    build.build()
    from raven_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def small_case(raven_lib):
    """A 6000 x 128 integer mixture, its graph (built once) and 400 queries."""
    from raven_b200 import datasets
    from raven_b200.index import Graph

    base, q = datasets.make("gmm100k-d128", n=6000, nq=400)
    g = Graph.build(base, r=32, l=64, alpha=1.2, nav_m=8, directional=True, seed=7)
    return base, q, g
