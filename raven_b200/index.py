"""Host-side API mirroring RAVEN's interfaces over the CUDA engine.

* `Graph`          — VamanaGraph (src/graph/vamana.rs:85): build / load / save.
* `GraphSearcher`  — the Rust query builder (src/graph/vamana.rs:1428-2110):
                     new / with_sq4 / with_sq8 / with_rerank_factor /
                     with_prefetch_offset / with_adaptive_ef / search (f32) /
                     search_sq4 / search_sq8 / batch_search / last_visited_count /
                     last_ef_used.
* `Index`, `Searcher` — the PyO3 module `raven` (src/python.rs:27-361) with the
                     same signatures, defaults, errors and result layout.

All search work runs in libraven_gpu.so on a B200; nothing here computes
distances.
"""
from __future__ import annotations

import ctypes as C
import os
import struct
import zlib
from dataclasses import dataclass
from typing import List, Optional, Tuple

import numpy as np

from . import _lib as L

SENTINEL = 0xFFFFFFFF
SMALL_BATCH_AUTO = (1 << 64) - 1  # RAVEN_SMALL_BATCH_AUTO

# Base vectors saved beside an ANNX file (`<path>.vec`), so that a saved index
# can be loaded and searched without the caller supplying the vectors (the
# ANNX format holds only the graph). Layout, little endian: magic "RVEC" u32,
# version u32 (1), n u64, dim u32, CRC-32/IEEE of the payload u32, then n*dim
# f32. SQ parameters, codes and AdaptiveEf samples are recomputed from the
# vectors on upload (deterministically), so they are not stored.
_VEC_MAGIC = 0x43455652
_VEC_HEADER = struct.Struct("<IIQII")


def vectors_path(path: str) -> str:
    return path + ".vec"


def save_vectors(path: str, vectors) -> None:
    v = _f32c(vectors)
    payload = v.astype("<f4", copy=False).tobytes()
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(_VEC_HEADER.pack(_VEC_MAGIC, 1, v.shape[0], v.shape[1], zlib.crc32(payload) & 0xFFFFFFFF))
        f.write(payload)
    os.replace(tmp, path)


def load_vectors(path: str) -> np.ndarray:
    """Read a `.vec` file; IOError on a bad magic, version, size or checksum."""
    with open(path, "rb") as f:
        head = f.read(_VEC_HEADER.size)
        if len(head) != _VEC_HEADER.size:
            raise IOError(f"{path}: truncated header")
        magic, version, n, dim, crc = _VEC_HEADER.unpack(head)
        if magic != _VEC_MAGIC:
            raise IOError(f"{path}: not a vector file")
        if version != 1:
            raise IOError(f"{path}: unsupported version {version}")
        payload = f.read()
    if len(payload) != n * dim * 4:
        raise IOError(f"{path}: expected {n * dim * 4} payload bytes, found {len(payload)}")
    if zlib.crc32(payload) & 0xFFFFFFFF != crc:
        raise IOError(f"{path}: checksum mismatch")
    return np.frombuffer(payload, dtype="<f4").reshape(n, dim).astype(np.float32)


def _f32c(x, name="array") -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return a


class Graph:
    """Host VamanaGraph handle (owned by the C library)."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)

    @classmethod
    def build(cls, vectors, r: int = 32, l: int = 200, alpha: float = 1.2, nav_m: int = 32,
              directional: bool = True, r_soft: Optional[int] = None, max_iterations: int = 2,
              seed: int = 42, threads: int = 0, layered_nav: bool = True, verbose: bool = False,
              device: Optional[int] = None) -> "Graph":
        """VamanaGraph::build with the PyO3 configuration (src/python.rs:109-126).

        `device`: run each batch's search + DirectionalPrune on that GPU
        (raven_graph_build_gpu); None builds on the host."""
        lib = L.load()
        v = _f32c(vectors)
        if v.ndim != 2:
            raise ValueError("vectors must be a 2-D float32 array")
        cfg = L.BuildConfig(
            alpha=alpha, l_build=l, r_max=r,
            r_soft=int(r * 1.5) if r_soft is None else r_soft,
            max_iterations=max_iterations, saturate=0 if directional else 1, layered_nav=1 if layered_nav else 0,
            nav_m=nav_m, directional=1 if directional else 0, seed=seed, threads=threads, verbose=1 if verbose else 0,
        )
        h = C.c_void_p()
        if device is None:
            L.check(lib.raven_graph_build(L.ptr(v, C.c_float), v.shape[0], v.shape[1], C.byref(cfg), C.byref(h)))
        else:
            L.check(lib.raven_graph_build_gpu(L.ptr(v, C.c_float), v.shape[0], v.shape[1], C.byref(cfg), int(device),
                                              C.byref(h)))
        return cls(h.value)

    @classmethod
    def load(cls, path: str) -> "Graph":
        lib = L.load()
        h = C.c_void_p()
        L.check(lib.raven_graph_load(os.fsencode(path), C.byref(h)))
        return cls(h.value)

    @classmethod
    def from_bytes(cls, data: bytes) -> "Graph":
        lib = L.load()
        h = C.c_void_p()
        L.check(lib.raven_graph_load_bytes(data, len(data), C.byref(h)))
        return cls(h.value)

    def save(self, path: str) -> None:
        L.check(L.load().raven_graph_save(self._h, os.fsencode(path)))

    def info(self) -> L.GraphInfo:
        gi = L.GraphInfo()
        L.check(L.load().raven_graph_info(self._h, C.byref(gi)))
        return gi

    def __len__(self) -> int:
        return int(self.info().n)

    @property
    def dim(self) -> int:
        return int(self.info().dim)

    def entry_point(self) -> int:
        return int(self.info().entry_point)

    def neighbors(self, node: int) -> np.ndarray:
        gi = self.info()
        out = np.zeros(int(gi.r_max), dtype=np.uint32)
        deg = C.c_uint32()
        L.check(L.load().raven_graph_neighbors(self._h, node, L.ptr(out, C.c_uint32), out.size, C.byref(deg)))
        return out[: deg.value].copy()

    def close(self) -> None:
        if self._h and self._h.value:
            L.load().raven_graph_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceIndex:
    """Graph + vectors + quantised codes resident in one GPU's HBM."""

    def __init__(self, graph: Graph, vectors, device: int = 0, sq4: bool = True, sq8: bool = False,
                 adaptive: bool = False, f16: bool = False):
        lib = L.load()
        v = _f32c(vectors)
        if v.ndim != 2:
            raise ValueError("vectors must be a 2-D float32 array")
        opt = L.UploadOptions(device=device, build_sq4=int(sq4), build_sq8=int(sq8), build_adaptive=int(adaptive),
                              build_f16=int(f16))
        h = C.c_void_p()
        L.check(lib.raven_index_upload(graph._h, L.ptr(v, C.c_float), v.shape[0], v.shape[1], C.byref(opt),
                                       C.byref(h)))
        self._h = h
        self.n, self.dim = v.shape
        self.device = device
        self.has_sq4, self.has_sq8, self.has_adaptive, self.has_f16 = sq4, sq8, adaptive, f16

    def adaptive_samples(self) -> np.ndarray:
        n = C.c_uint32()
        L.check(L.load().raven_index_adaptive_samples(self._h, None, 0, C.byref(n)))
        out = np.zeros(n.value, dtype=np.float32)
        L.check(L.load().raven_index_adaptive_samples(self._h, L.ptr(out, C.c_float), n.value, C.byref(n)))
        return out

    def sq_params(self, quant: int) -> np.ndarray:
        out = np.zeros((5, self.dim), dtype=np.float32)
        L.check(L.load().raven_index_sq_params(self._h, quant, L.ptr(out, C.c_float)))
        return out

    def codes(self, quant: int) -> np.ndarray:
        nb = (self.dim + 1) // 2 if quant == L.RAVEN_QUANT_SQ4 else self.dim
        out = np.zeros((self.n, nb), dtype=np.uint8)
        L.check(L.load().raven_index_codes(self._h, quant, L.ptr(out, C.c_uint8), out.size))
        return out

    def set_tuning(self, hash_bits: int = 0, spill_bits: int = 0) -> None:
        L.check(L.load().raven_index_set_tuning(self._h, hash_bits, spill_bits))

    def set_small_batch(self, max_nq: int) -> None:
        """Batches of at most `max_nq` queries run one CTA per query (0: never;
        SMALL_BATCH_AUTO, the default: one wave of CTAs, at most four per SM)."""
        L.check(L.load().raven_index_set_small_batch(self._h, max_nq))

    def set_fat_rows(self, enable: bool) -> None:
        """Neighbour codes stored beside each row (default: built at upload when
        they fit); False frees them and the search gathers codes instead."""
        L.check(L.load().raven_index_set_fat_rows(self._h, int(bool(enable))))

    def search(self, queries, params: L.SearchParams, history_cap: int = 0, stats: bool = True,
               visited: Optional[bool] = None) -> dict:
        """Host-buffer batch search (raven_search_batch). Returns a dict of arrays.

        `stats` adds ef_used, status, n_nav and expansions; `visited` (default:
        with the history) adds the per-query visited count, which runs the
        search with the exact visited set; results are the same either way."""
        q = _f32c(queries)
        if q.ndim == 1:
            q = q[None, :]
        if q.shape[1] != self.dim:
            raise ValueError(f"dim mismatch: expected {self.dim}, got {q.shape[1]}")
        nq, k = q.shape[0], params.k
        res = {
            "ids": np.zeros((nq, k), dtype=np.uint32),
            "dists": np.zeros((nq, k), dtype=np.float32),
            "counts": np.zeros(nq, dtype=np.uint32),
        }
        if stats:
            for name, dt in (("ef_used", np.uint32), ("status", np.int32), ("n_nav", np.uint32),
                             ("expansions", np.uint32)):
                res[name] = np.zeros(nq, dtype=dt)
        if visited or (visited is None and history_cap):
            res["visited"] = np.zeros(nq, dtype=np.uint32)
        if history_cap:
            res["history"] = np.zeros((nq, history_cap), dtype=np.uint32)
            res["history_len"] = np.zeros(nq, dtype=np.uint32)
        out = L.SearchOutputs(
            ids=L.ptr(res["ids"], C.c_uint32), dists=L.ptr(res["dists"], C.c_float),
            counts=L.ptr(res["counts"], C.c_uint32),
            visited=L.ptr(res.get("visited"), C.c_uint32), ef_used=L.ptr(res.get("ef_used"), C.c_uint32),
            status=L.ptr(res.get("status"), C.c_int32), n_nav=L.ptr(res.get("n_nav"), C.c_uint32),
            expansions=L.ptr(res.get("expansions"), C.c_uint32),
            history=L.ptr(res.get("history"), C.c_uint32), history_cap=history_cap,
            history_len=L.ptr(res.get("history_len"), C.c_uint32),
        )
        L.check(L.load().raven_search_batch(self._h, L.ptr(q, C.c_float), nq, C.byref(params), C.byref(out), None))
        return res

    def close(self) -> None:
        if self._h and self._h.value:
            L.load().raven_index_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class AdaptiveEfConfig:
    """AdaptiveEfConfig parameters (src/graph/adaptive_ef.rs:209-246); the
    sorted sample distances live with the device index."""

    min_ef: int = 30
    max_ef: int = 100
    gamma: float = 2.0

    def with_params(self, min_ef: int, max_ef: int, gamma: float) -> "AdaptiveEfConfig":
        return AdaptiveEfConfig(min_ef, max_ef, gamma)


class GraphSearcher:
    """Mirror of the Rust `GraphSearcher` builder (src/graph/vamana.rs:1428-2110)."""

    def __init__(self, vectors, graph: Graph, ef_search: int, device: int = 0):
        self._vectors = _f32c(vectors)
        self._graph = graph
        self.ef_search = int(ef_search)
        self.prefetch_offset = 16          # vamana.rs:1490
        self.rerank_factor = 5             # vamana.rs:1498
        self._quant: Optional[int] = None  # None: with_sq4/with_sq8 not called
        self._want = {"sq4": False, "sq8": False}
        self._adaptive: Optional[AdaptiveEfConfig] = None
        self._f16 = False  # with_f16: rerank with f16 vectors
        self._device = device
        self._dev: Optional[DeviceIndex] = None
        self._last_visited = 0
        self._last_ef = self.ef_search

    def with_prefetch_offset(self, po: int) -> "GraphSearcher":
        self.prefetch_offset = int(po)  # accepted; no effect on the GPU
        return self

    def with_rerank_factor(self, factor: int) -> "GraphSearcher":
        self.rerank_factor = max(int(factor), 1)  # vamana.rs:1547-1550
        return self

    def with_sq4(self, sq4=None) -> "GraphSearcher":
        self._want["sq4"] = True
        self._dev = None
        return self

    def with_sq8(self, sq8=None) -> "GraphSearcher":
        self._want["sq8"] = True
        self._dev = None
        return self

    def with_f16(self, f16=None) -> "GraphSearcher":
        """GraphSearcher::with_f16 (src/graph/vamana.rs:1559): rerank with the
        vectors converted to f16 (F16Dataset::build), as rerank_f16 does."""
        self._f16 = True
        if self._dev is not None and not self._dev.has_f16:
            self._dev = None
        return self

    def with_adaptive_ef(self, config: AdaptiveEfConfig) -> "GraphSearcher":
        self._adaptive = config
        if self._dev is not None and not self._dev.has_adaptive:
            self._dev = None
        return self

    def _device_index(self) -> DeviceIndex:
        if self._dev is None:
            self._dev = DeviceIndex(self._graph, self._vectors, device=self._device, sq4=self._want["sq4"],
                                    sq8=self._want["sq8"], adaptive=self._adaptive is not None, f16=self._f16)
        return self._dev

    def _params(self, k: int, quant: int) -> L.SearchParams:
        p = L.SearchParams(ef=self.ef_search, k=k, rerank_factor=self.rerank_factor,
                           prefetch_offset=self.prefetch_offset, quant=quant, adaptive=0, gamma=0.0, min_ef=0,
                           max_ef=0, rerank_f16=int(self._f16))
        if self._adaptive is not None:
            p.adaptive = 1
            p.gamma = self._adaptive.gamma
            p.min_ef = self._adaptive.min_ef
            p.max_ef = self._adaptive.max_ef
        return p

    def _search(self, queries, k: int, quant: int, visited: bool = True):
        if quant != L.RAVEN_QUANT_F32 and not self._want["sq4" if quant == L.RAVEN_QUANT_SQ4 else "sq8"]:
            name = "sq4" if quant == L.RAVEN_QUANT_SQ4 else "sq8"
            raise RuntimeError(f"search_{name} requires with_{name}() first")
        # single-query calls keep last_visited_count (the exact visited set);
        # batch_search has no such diagnostic and runs without it
        return self._device_index().search(queries, self._params(k, quant), visited=visited)

    def search(self, query, k: int) -> List[Tuple[int, float]]:
        """GraphSearcher::search (src/graph/vamana.rs:1627-1672): the beam over
        f32 distances (greedy_search_vec_reuse), no rerank; the first k of the
        pool."""
        r = self._search(np.asarray(query, dtype=np.float32)[None, :], k, L.RAVEN_QUANT_F32)
        self._last_visited = int(r["visited"][0])
        self._last_ef = int(r["ef_used"][0])
        c = int(r["counts"][0])
        return [(int(i), float(d)) for i, d in zip(r["ids"][0, :c], r["dists"][0, :c])]

    def search_sq4(self, query, k: int) -> List[Tuple[int, float]]:
        r = self._search(np.asarray(query, dtype=np.float32)[None, :], k, L.RAVEN_QUANT_SQ4)
        self._last_visited = int(r["visited"][0])
        self._last_ef = int(r["ef_used"][0])
        c = int(r["counts"][0])
        return [(int(i), float(d)) for i, d in zip(r["ids"][0, :c], r["dists"][0, :c])]

    def search_sq8(self, query, k: int) -> List[Tuple[int, float]]:
        r = self._search(np.asarray(query, dtype=np.float32)[None, :], k, L.RAVEN_QUANT_SQ8)
        self._last_visited = int(r["visited"][0])
        self._last_ef = int(r["ef_used"][0])
        c = int(r["counts"][0])
        return [(int(i), float(d)) for i, d in zip(r["ids"][0, :c], r["dists"][0, :c])]

    def batch_search(self, queries, k: int) -> List[List[Tuple[int, float]]]:
        """Branch order SQ8 > SQ4 > f32 traversal (vamana.rs:2063-2091)."""
        quant = (L.RAVEN_QUANT_SQ8 if self._want["sq8"] else
                 L.RAVEN_QUANT_SQ4 if self._want["sq4"] else L.RAVEN_QUANT_F32)
        q = _f32c(queries)
        r = self._search(q, k, quant, visited=False)
        return [[(int(i), float(d)) for i, d in zip(r["ids"][j, : r["counts"][j]], r["dists"][j, : r["counts"][j]])]
                for j in range(q.shape[0])]

    def batch_search_ids(self, queries, k: int) -> List[List[int]]:
        return [[i for i, _ in row] for row in self.batch_search(queries, k)]

    def last_visited_count(self) -> int:
        return self._last_visited

    def last_ef_used(self) -> int:
        return self._last_ef


class Searcher:
    """PyO3 `raven.Searcher` (src/python.rs:222-353)."""

    def __init__(self, graph: Graph, vectors: np.ndarray, dim: int, quant: str, rerank: int, threads: int,
                 adaptive: bool, device: int = 0):
        self._graph = graph
        self._vectors = vectors
        self.dim = dim
        self._quant = L.RAVEN_QUANT_SQ8 if quant == "sq8" else L.RAVEN_QUANT_SQ4
        self.ef = 50                      # src/python.rs:171
        self.po = 16                      # src/python.rs:172
        self.rerank = rerank
        self.threads = threads
        self._has_adaptive = adaptive
        self.use_adaptive = False
        self.cur_gamma, self.cur_min_ef, self.cur_max_ef = 2.0, 30, 100
        self._dev = DeviceIndex(graph, vectors, device=device, sq4=self._quant == L.RAVEN_QUANT_SQ4,
                                sq8=self._quant == L.RAVEN_QUANT_SQ8, adaptive=adaptive)
        self.last_ef_used = self.ef

    @property
    def device_index(self) -> DeviceIndex:
        return self._dev

    def set_ef(self, ef: int) -> None:
        self.ef = int(ef)
        self.use_adaptive = False

    def set_adaptive_ef(self, gamma: float, min_ef: int, max_ef: int) -> None:
        self.cur_gamma, self.cur_min_ef, self.cur_max_ef = float(gamma), int(min_ef), int(max_ef)
        self.ef = int(max_ef)
        self.use_adaptive = self._has_adaptive

    def set_po(self, po: int) -> None:
        self.po = int(po)

    def params(self, k: int) -> L.SearchParams:
        p = L.SearchParams(ef=self.ef, k=k, rerank_factor=max(self.rerank, 1), prefetch_offset=self.po,
                           quant=self._quant, adaptive=0, gamma=0.0, min_ef=0, max_ef=0)
        if self.use_adaptive:
            p.adaptive, p.gamma, p.min_ef, p.max_ef = 1, self.cur_gamma, self.cur_min_ef, self.cur_max_ef
        return p

    def search(self, q, k: int) -> np.ndarray:
        """One query -> up to k ids (no padding), numpy uintp like PyO3's Vec<usize>."""
        q = _f32c(q).reshape(-1)
        if q.shape[0] != self.dim:
            raise ValueError(f"dim mismatch: expected {self.dim}, got {q.shape[0]}")
        r = self._dev.search(q[None, :], self.params(k))
        self.last_ef_used = int(r["ef_used"][0])
        return r["ids"][0, : r["counts"][0]].astype(np.uintp)

    def batch_search(self, queries, k: int) -> np.ndarray:
        """(nq, dim) -> flat nq*k ids, zero padded (src/python.rs:313-352)."""
        q = _f32c(queries)
        if q.ndim != 2 or q.shape[1] != self.dim:
            got = q.shape[1] if q.ndim == 2 else q.shape
            raise ValueError(f"dim mismatch: expected {self.dim}, got {got}")
        r = self._dev.search(q, self.params(k))
        return r["ids"].reshape(-1).astype(np.uintp)


class Index:
    """PyO3 `raven.Index` (src/python.rs:27-215)."""

    def __init__(self, metric: str, dim: int, r: int = 32, l: int = 200, alpha: float = 1.2, nav_m: int = 32,
                 directional: bool = True, quantization: str = "sq8", rerank_factor: int = 5, threads: int = 0,
                 adaptive_ef: bool = False, *, device: int = 0):
        q = quantization.lower()
        if q not in ("sq8", "sq4"):
            raise ValueError(f"unknown quantization '{quantization}', expected 'sq8' or 'sq4'")
        self.metric = metric  # L2 only
        self.dim = int(dim)
        self.r, self.l, self.alpha, self.nav_m, self.directional = r, l, alpha, nav_m, directional
        self.quant = q
        self.rerank = rerank_factor
        self.threads = threads
        self.adaptive_ef = adaptive_ef
        self.device = device
        self._graph: Optional[Graph] = None
        self._vectors: Optional[np.ndarray] = None

    def build(self, X) -> None:
        x = _f32c(X)
        if x.ndim != 2 or x.shape[1] != self.dim:
            got = x.shape[1] if x.ndim == 2 else x.shape
            raise ValueError(f"dim mismatch: expected {self.dim}, got {got}")
        self._vectors = x
        self._graph = Graph.build(x, r=self.r, l=self.l, alpha=self.alpha, nav_m=self.nav_m,
                                  directional=self.directional)

    def searcher(self) -> Searcher:
        if self._graph is None:
            raise RuntimeError("Index not built yet, call build() first")
        if self._vectors is None or self._vectors.shape[0] != len(self._graph):
            raise RuntimeError("index has no base vectors: pass vectors= to Index.load (the ANNX file does not "
                               "store them)")
        graph, vectors = self._graph, self._vectors
        self._graph, self._vectors = None, None  # moved into the searcher (src/python.rs:135-139)
        return Searcher(graph, vectors, self.dim, self.quant, self.rerank, self.threads, self.adaptive_ef,
                        device=self.device)

    def save(self, path: str) -> None:
        """The graph as an ANNX file at `path` and, when the index holds its
        base vectors, `<path>.vec` beside it."""
        if self._graph is None:
            raise RuntimeError("Index not built yet")
        try:
            self._graph.save(path)
        except L.RavenError as e:
            raise IOError(str(e)) from e
        if self._vectors is not None:
            save_vectors(vectors_path(path), self._vectors)

    @staticmethod
    def load(path: str, dim: int, *, vectors=None, quantization: str = "sq8", rerank_factor: int = 3,
             adaptive_ef: bool = False, device: int = 0) -> "Index":
        """Index.load (src/python.rs:196-214): sq8, rerank 3. The base vectors
        come from `vectors`, else from `<path>.vec` when it exists (written by
        `save`); without either, `searcher()` raises instead of aborting."""
        try:
            g = Graph.load(path)
        except L.RavenError as e:
            raise IOError(str(e)) from e
        ix = Index("L2", dim, quantization=quantization, rerank_factor=rerank_factor, adaptive_ef=adaptive_ef,
                   device=device)
        ix._graph = g
        if vectors is None and os.path.exists(vectors_path(path)):
            vectors = load_vectors(vectors_path(path))
            if vectors.shape != (len(g), dim):
                raise IOError(f"{vectors_path(path)}: holds {vectors.shape}, expected ({len(g)}, {dim})")
        if vectors is not None:
            v = _f32c(vectors)
            if v.ndim != 2 or v.shape[1] != dim:
                raise ValueError("vectors shape does not match dim")
            ix._vectors = v
        return ix
