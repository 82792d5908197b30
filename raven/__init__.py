"""`raven` — the import name of RAVEN's Python module (src/python.rs:355-360
registers `Index` and `Searcher` as module `raven`), served by the B200
engine.

    import raven
    index = raven.Index("L2", 128, quantization="sq4", rerank_factor=8)
    index.build(X)
    searcher = index.searcher()
    ids = searcher.batch_search(Q, 10)

The classes are those of `raven_b200.index`, with the reference's
signatures, defaults, errors and result layout; searching runs in
libraven_gpu.so on a GPU.
"""
from raven_b200.index import Index, Searcher

__all__ = ["Index", "Searcher"]
