"""raven_b200 — B200-native batched query engine for RAVEN's Vamana graph search.

The engine itself is libraven_gpu.so (hand-written CUDA for sm_100a behind the
C ABI in include/raven_gpu.h). This package is its host side: a ctypes binding
and the `Index` / `Searcher` / `GraphSearcher` surface of the reference.
"""
from .index import AdaptiveEfConfig, DeviceIndex, Graph, GraphSearcher, Index, Searcher  # noqa: F401
from ._lib import RavenError, SearchParams  # noqa: F401

__all__ = ["Index", "Searcher", "Graph", "GraphSearcher", "DeviceIndex", "AdaptiveEfConfig", "RavenError",
           "SearchParams"]
