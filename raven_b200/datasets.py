"""Seeded synthetic workloads with the shapes of the reference's benchmark.

The reference measures on SIFT-1M (1M x 128, integer-valued descriptors,
src/bin/sq4_ef_sweep.rs:59-63), which is not available here. These
Gaussian-mixture stand-ins have the same shapes and value ranges:

  clustered_int(n, dim, n_centres, sigma, seed, ...)
      centres ~ U[0,128)^dim drawn from `centre_seed`, points = centre +
      N(0, sigma^2) per component, clamped to [0,255], rounded, stored f32;
      optionally a Bernoulli(zero_frac) mask sets components to 0 (sparse
      non-negative descriptors).
  clustered_unit(n, dim, n_centres, sigma, seed, ...)
      centres ~ N(0,1)^dim, points = centre + N(0, sigma^2), L2-normalised.

Generation is chunked so 1M-40M rows fit in host memory as f32 only.
"""
from __future__ import annotations

import numpy as np

_CHUNK = 131072


def _centres_int(n_centres: int, dim: int, centre_seed: int) -> np.ndarray:
    rng = np.random.default_rng(centre_seed)
    return rng.uniform(0.0, 128.0, size=(n_centres, dim)).astype(np.float32)


def clustered_int(n: int, dim: int, n_centres: int, sigma: float, seed: int, centre_seed: int,
                  zero_frac: float = 0.0) -> np.ndarray:
    centres = _centres_int(n_centres, dim, centre_seed)
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), dtype=np.float32)
    for s in range(0, n, _CHUNK):
        e = min(n, s + _CHUNK)
        assign = rng.integers(0, n_centres, size=e - s)
        x = centres[assign].astype(np.float64) + rng.normal(0.0, sigma, size=(e - s, dim))
        np.clip(x, 0.0, 255.0, out=x)
        np.rint(x, out=x)
        if zero_frac > 0.0:
            x[rng.random(size=(e - s, dim)) < zero_frac] = 0.0
        out[s:e] = x.astype(np.float32)
    return out


def clustered_unit(n: int, dim: int, n_centres: int, sigma: float, seed: int, centre_seed: int) -> np.ndarray:
    rng_c = np.random.default_rng(centre_seed)
    centres = rng_c.normal(0.0, 1.0, size=(n_centres, dim))
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), dtype=np.float32)
    for s in range(0, n, _CHUNK):
        e = min(n, s + _CHUNK)
        assign = rng.integers(0, n_centres, size=e - s)
        x = centres[assign] + rng.normal(0.0, sigma, size=(e - s, dim))
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        out[s:e] = x.astype(np.float32)
    return out


# The five workloads (base, queries). Names say what they are.
WORKLOADS = {
    # 100k x 128 integer mixture, 1000 centres, sigma 12 (CPU-runnable case)
    "gmm100k-d128": dict(kind="int", n=100_000, nq=10_000, dim=128, centres=1000, sigma=12.0, seed=42, qseed=43,
                         zero=0.0),
    # 1M x 128 integer mixture, 5000 centres, sigma 12, 30% zeros (the headline workload)
    "gmm1m-d128-sparse": dict(kind="int", n=1_000_000, nq=10_000, dim=128, centres=5000, sigma=12.0, seed=1001,
                              qseed=1002, zero=0.3),
    # 10M x 96 unit-normalised mixture, 10k centres, sigma 0.3
    "gmm10m-d96-unit": dict(kind="unit", n=10_000_000, nq=10_000, dim=96, centres=10_000, sigma=0.3, seed=2001,
                            qseed=2002, zero=0.0),
    # 40M x 128 integer mixture, 40k centres, sigma 12 (8 shards of 5M)
    "gmm40m-d128": dict(kind="int", n=40_000_000, nq=10_000, dim=128, centres=40_000, sigma=12.0, seed=7, qseed=8,
                        zero=0.0),
}


def make(name: str, n: int | None = None, nq: int | None = None, query_offset: int = 0):
    """Return (base, queries) for a named workload; `n`/`nq` override the
    sizes (smaller parity cases); `query_offset` selects another query slice
    (extra seed) for multi-rank runs."""
    w = WORKLOADS[name]
    n = w["n"] if n is None else n
    nq = w["nq"] if nq is None else nq
    if w["kind"] == "int":
        base = clustered_int(n, w["dim"], w["centres"], w["sigma"], w["seed"], centre_seed=w["seed"] + 500,
                             zero_frac=w["zero"])
        q = clustered_int(nq, w["dim"], w["centres"], w["sigma"], w["qseed"] + 7919 * query_offset,
                          centre_seed=w["seed"] + 500, zero_frac=w["zero"])
    else:
        base = clustered_unit(n, w["dim"], w["centres"], w["sigma"], w["seed"], centre_seed=w["seed"] + 500)
        q = clustered_unit(nq, w["dim"], w["centres"], w["sigma"], w["qseed"] + 7919 * query_offset,
                           centre_seed=w["seed"] + 500)
    return base, q


def make_queries(name: str, nq: int, offset: int = 0) -> np.ndarray:
    """Queries only (same generator as `make`, query slice `offset`)."""
    w = WORKLOADS[name]
    if w["kind"] == "int":
        return clustered_int(nq, w["dim"], w["centres"], w["sigma"], w["qseed"] + 7919 * offset,
                             centre_seed=w["seed"] + 500, zero_frac=w["zero"])
    return clustered_unit(nq, w["dim"], w["centres"], w["sigma"], w["qseed"] + 7919 * offset,
                          centre_seed=w["seed"] + 500)


def make_shard(name: str, shard: int, n_shards: int, shard_n: int | None = None) -> np.ndarray:
    """Base vectors of one contiguous shard of a workload: shard s holds global
    ids [s * shard_n, (s + 1) * shard_n) (shard_n = n / n_shards by default),
    drawn from its own seed around the workload's shared centres, so each rank
    generates only the shards it holds. The collection is the concatenation of
    the shards in order; queries come from `make_queries`."""
    w = WORKLOADS[name]
    size = w["n"] // n_shards if shard_n is None else shard_n
    seed = w["seed"] * 1000 + 17 * shard
    if w["kind"] == "int":
        return clustered_int(size, w["dim"], w["centres"], w["sigma"], seed, centre_seed=w["seed"] + 500,
                             zero_frac=w["zero"])
    return clustered_unit(size, w["dim"], w["centres"], w["sigma"], seed, centre_seed=w["seed"] + 500)


def shard_index_path(name: str, shard: int, n_shards: int, shard_n: int) -> str:
    return _os.path.join(DATA_DIR, f"{name}-shard{shard}of{n_shards}-n{shard_n}.annx")


# ---------------------------------------------------------------------------
# Cached index files (ANNX v1) for the workloads, built with the reference's
# PyO3 build parameters: R=32, L=200, alpha=1.2, DirectionalPrune, nav_m=32,
# R_soft=48, 2 iterations (src/python.rs:109-123).
# ---------------------------------------------------------------------------
import os as _os

DATA_DIR = _os.environ.get("RAVEN_DATA_DIR",
                           _os.path.join(_os.path.dirname(_os.path.dirname(_os.path.abspath(__file__))), "data"))


def index_path(name: str, n: int | None = None) -> str:
    n = WORKLOADS[name]["n"] if n is None else n
    return _os.path.join(DATA_DIR, f"{name}-n{n}.annx")


def load_or_build(name: str, base=None, n: int | None = None, threads: int = 0, verbose: bool = False,
                  device: int | None = None):
    """Load the cached graph for a workload or build and save it (on the host,
    or with the GPU build on `device`, which makes the same graph)."""
    from .index import Graph

    path = index_path(name, n)
    if _os.path.exists(path):
        return Graph.load(path)
    if base is None:
        base, _ = make(name, n=n, nq=1)
    g = Graph.build(base, r=32, l=200, alpha=1.2, nav_m=32, directional=True, threads=threads, verbose=verbose,
                    device=device)
    _os.makedirs(DATA_DIR, exist_ok=True)
    tmp = f"{path}.tmp{_os.getpid()}"
    g.save(tmp)
    _os.replace(tmp, path)
    return g
