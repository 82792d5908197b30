"""ctypes wrapper of oracle/_build/liboracle.so — the CPU restatement of the
reference query path. TEST INFRASTRUCTURE ONLY: imported by tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference leg, never by
the raven_b200 package.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")

u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)


class OracleParams(C.Structure):
    _fields_ = [("ef", C.c_uint32), ("k", C.c_uint32), ("rerank_factor", C.c_uint32), ("quant", C.c_uint32),
                ("adaptive", C.c_uint32), ("gamma", C.c_float), ("min_ef", C.c_uint32), ("max_ef", C.c_uint32),
                ("rerank_f16", C.c_uint32), ("prefetch_offset", C.c_uint32)]


_SIG = {
    "oracle_last_error": (C.c_char_p, []),
    "oracle_crc32": (C.c_uint32, [C.c_void_p, C.c_size_t]),
    "oracle_l2_avx512": (C.c_float, [f32p, f32p, C.c_size_t]),
    "oracle_f16_from_f32": (C.c_uint16, [C.c_float]),
    "oracle_f16_to_f32": (C.c_float, [C.c_uint16]),
    "oracle_l2_f16_mixed": (C.c_float, [f32p, C.POINTER(C.c_uint16), C.c_size_t]),
    "oracle_index_build_f16": (C.c_int, [C.c_void_p]),
    "oracle_l2_avx2": (C.c_float, [f32p, f32p, C.c_size_t]),
    "oracle_l2_sq4_raw": (C.c_float, [u8p, u8p, C.c_size_t]),
    "oracle_l2_sq8_raw": (C.c_float, [u8p, u8p, C.c_size_t]),
    "oracle_sq_fit": (None, [f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p]),
    "oracle_sq4_encode": (None, [f32p, C.c_uint32, f32p, C.c_uint64, u8p]),
    "oracle_sq8_encode": (None, [f32p, C.c_uint32, f32p, C.c_uint64, u8p]),
    "oracle_pool_new": (C.c_void_p, [C.c_size_t]),
    "oracle_pool_free": (None, [C.c_void_p]),
    "oracle_pool_insert": (C.c_int, [C.c_void_p, C.c_uint32, C.c_float]),
    "oracle_pool_pop": (C.c_int, [C.c_void_p, u32p, f32p]),
    "oracle_pool_has_next": (C.c_int, [C.c_void_p]),
    "oracle_pool_len": (C.c_size_t, [C.c_void_p]),
    "oracle_pool_cursor": (C.c_size_t, [C.c_void_p]),
    "oracle_pool_worst": (C.c_float, [C.c_void_p]),
    "oracle_pool_clear": (None, [C.c_void_p]),
    "oracle_pool_reset_for": (None, [C.c_void_p, C.c_size_t]),
    "oracle_pool_sorted": (C.c_size_t, [C.c_void_p, u32p, f32p]),
    "oracle_estimate_ef": (C.c_size_t, [f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float, C.c_float]),
    "oracle_index_load": (C.c_void_p, [C.c_char_p]),
    "oracle_index_from_bytes": (C.c_void_p, [C.c_void_p, C.c_size_t, C.POINTER(C.c_int)]),
    "oracle_index_free": (None, [C.c_void_p]),
    "oracle_index_info": (None, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "oracle_index_main_block": (u32p, [C.c_void_p]),
    "oracle_index_degree": (C.c_uint32, [C.c_void_p, C.c_uint32]),
    "oracle_index_nav_list": (C.c_size_t, [C.c_void_p, C.c_uint32, C.POINTER(u32p)]),
    "oracle_index_nav_level": (C.c_uint32, [C.c_void_p, C.c_uint32]),
    "oracle_index_nav_candidates": (C.c_size_t, [C.c_void_p, C.POINTER(u32p)]),
    "oracle_index_set_vectors": (C.c_int, [C.c_void_p, f32p, C.c_uint64, C.c_uint32, C.c_int, C.c_int, C.c_int]),
    "oracle_index_adaptive_samples": (C.c_size_t, [C.c_void_p, C.POINTER(f32p)]),
    "oracle_index_sq4_codes": (u8p, [C.c_void_p]),
    "oracle_index_sq8_codes": (u8p, [C.c_void_p]),
    "oracle_index_sq_params": (None, [C.c_void_p, C.c_int, f32p]),
    "oracle_nav_initialize": (None, [C.c_void_p, f32p, u32p, f32p, u32p]),
    "oracle_search_batch": (C.c_int, [C.c_void_p, f32p, C.c_uint64, C.POINTER(OracleParams), C.c_int, u32p, f32p,
                                      u32p, u32p, u32p, u32p, u32p, u32p, C.c_uint32, u32p]),
    "oracle_bruteforce": (None, [f32p, C.c_uint64, f32p, C.c_uint64, C.c_uint32, C.c_uint32, C.c_int, u32p, f32p]),
}

_lib = None


def build() -> str:
    """Compile liboracle.so with its Makefile (g++ only)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        l = C.CDLL(LIB)
        for name, (res, args) in _SIG.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def _p(a, t):
    return None if a is None else a.ctypes.data_as(C.POINTER(t))


def crc32(data: bytes) -> int:
    return int(lib().oracle_crc32(data, len(data)))


def l2_avx512(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().oracle_l2_avx512(_p(a, C.c_float), _p(b, C.c_float), a.size))


def f16_from_f32(x: float) -> int:
    return int(lib().oracle_f16_from_f32(float(x)))


def f16_to_f32(h: int) -> float:
    return float(lib().oracle_f16_to_f32(int(h)))


def l2_f16_mixed(q, db_f16) -> float:
    q = np.ascontiguousarray(q, np.float32)
    d = np.ascontiguousarray(db_f16, np.uint16)
    return float(lib().oracle_l2_f16_mixed(_p(q, C.c_float), d.ctypes.data_as(C.POINTER(C.c_uint16)), q.size))


def l2_avx2(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return float(lib().oracle_l2_avx2(_p(a, C.c_float), _p(b, C.c_float), a.size))


def sq_fit(data, levels: int) -> np.ndarray:
    d = np.ascontiguousarray(data, np.float32)
    out = np.zeros((5, d.shape[1]), np.float32)
    lib().oracle_sq_fit(_p(d, C.c_float), d.shape[0], d.shape[1], levels, _p(out, C.c_float))
    return out


def sq4_encode(params, v) -> np.ndarray:
    v = np.ascontiguousarray(np.atleast_2d(v), np.float32)
    p = np.ascontiguousarray(params, np.float32)
    dim = v.shape[1]
    out = np.zeros((v.shape[0], (dim + 1) // 2), np.uint8)
    lib().oracle_sq4_encode(_p(p, C.c_float), dim, _p(v, C.c_float), v.shape[0], _p(out, C.c_uint8))
    return out


def sq8_encode(params, v) -> np.ndarray:
    v = np.ascontiguousarray(np.atleast_2d(v), np.float32)
    p = np.ascontiguousarray(params, np.float32)
    dim = v.shape[1]
    out = np.zeros((v.shape[0], dim), np.uint8)
    lib().oracle_sq8_encode(_p(p, C.c_float), dim, _p(v, C.c_float), v.shape[0], _p(out, C.c_uint8))
    return out


def l2_sq4_raw(a, b) -> float:
    a = np.ascontiguousarray(a, np.uint8)
    b = np.ascontiguousarray(b, np.uint8)
    return float(lib().oracle_l2_sq4_raw(_p(a, C.c_uint8), _p(b, C.c_uint8), a.size))


def l2_sq8_raw(a, b) -> float:
    a = np.ascontiguousarray(a, np.uint8)
    b = np.ascontiguousarray(b, np.uint8)
    return float(lib().oracle_l2_sq8_raw(_p(a, C.c_uint8), _p(b, C.c_uint8), a.size))


def estimate_ef(sorted_samples, min_ef, max_ef, gamma, d) -> int:
    s = np.ascontiguousarray(sorted_samples, np.float32)
    return int(lib().oracle_estimate_ef(_p(s, C.c_float), s.size, min_ef, max_ef, gamma, d))


class Pool:
    """LinearPool handle (src/graph/linear_pool.rs)."""

    def __init__(self, ef):
        self.h = lib().oracle_pool_new(ef)

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_pool_free(self.h)

    def insert(self, node, d) -> bool:
        return bool(lib().oracle_pool_insert(self.h, node, d))

    def pop(self):
        i, d = C.c_uint32(), C.c_float()
        if lib().oracle_pool_pop(self.h, C.byref(i), C.byref(d)):
            return int(i.value), float(d.value)
        return None

    def has_next(self):
        return bool(lib().oracle_pool_has_next(self.h))

    def __len__(self):
        return int(lib().oracle_pool_len(self.h))

    @property
    def cursor(self):
        return int(lib().oracle_pool_cursor(self.h))

    def worst_distance(self):
        return float(lib().oracle_pool_worst(self.h))

    def clear(self):
        lib().oracle_pool_clear(self.h)

    def reset_for(self, ef):
        lib().oracle_pool_reset_for(self.h, ef)

    def to_sorted_vec(self):
        n = len(self)
        ids = np.zeros(max(n, 1), np.uint32)
        ds = np.zeros(max(n, 1), np.float32)
        lib().oracle_pool_sorted(self.h, _p(ids, C.c_uint32), _p(ds, C.c_float))
        return [(int(i), float(d)) for i, d in zip(ids[:n], ds[:n])]


class OracleIndex:
    """An ANNX index file + base vectors, searched by the CPU restatement."""

    def __init__(self, path: str | None = None, data: bytes | None = None):
        if path is not None:
            self.h = lib().oracle_index_load(os.fsencode(path))
            if not self.h:
                raise IOError(lib().oracle_last_error().decode())
        else:
            st = C.c_int()
            self.h = lib().oracle_index_from_bytes(data, len(data), C.byref(st))
            if not self.h:
                raise IOError(f"[{st.value}] " + lib().oracle_last_error().decode())
            self.status = st.value
        info = (C.c_uint64 * 8)()
        lib().oracle_index_info(self.h, info)
        (self.n, self.dim, self.r_max, self.entry, self.nav_present, self.nav_max_level, self.nav_k,
         self.flags) = [int(x) for x in info]

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_index_free(self.h)

    def neighbors(self, node) -> np.ndarray:
        deg = lib().oracle_index_degree(self.h, node)
        mb = lib().oracle_index_main_block(self.h)
        return np.ctypeslib.as_array(mb, shape=(self.n * self.r_max,))[node * self.r_max: node * self.r_max + deg].copy()

    def nav_list(self, node) -> np.ndarray:
        p = u32p()
        n = lib().oracle_index_nav_list(self.h, node, C.byref(p))
        return np.ctypeslib.as_array(p, shape=(n,)).copy() if n else np.zeros(0, np.uint32)

    def nav_level(self, node) -> int:
        return int(lib().oracle_index_nav_level(self.h, node))

    def entry_candidates(self) -> np.ndarray:
        p = u32p()
        n = lib().oracle_index_nav_candidates(self.h, C.byref(p))
        return np.ctypeslib.as_array(p, shape=(n,)).copy() if n else np.zeros(0, np.uint32)

    def set_vectors(self, vectors, sq4=True, sq8=False, adaptive=False, f16=False):
        v = np.ascontiguousarray(vectors, np.float32)
        self._vectors = v
        rc = lib().oracle_index_set_vectors(self.h, _p(v, C.c_float), v.shape[0], v.shape[1], int(sq4), int(sq8),
                                            int(adaptive))
        if rc == 0 and f16:
            rc = lib().oracle_index_build_f16(self.h)
        if rc != 0:
            raise RuntimeError(lib().oracle_last_error().decode())

    def adaptive_samples(self) -> np.ndarray:
        p = f32p()
        n = lib().oracle_index_adaptive_samples(self.h, C.byref(p))
        return np.ctypeslib.as_array(p, shape=(n,)).copy() if n else np.zeros(0, np.float32)

    def codes(self, quant: int) -> np.ndarray:
        nb = (self.dim + 1) // 2 if quant == 0 else self.dim
        p = lib().oracle_index_sq4_codes(self.h) if quant == 0 else lib().oracle_index_sq8_codes(self.h)
        return np.ctypeslib.as_array(p, shape=(self.n * nb,)).reshape(self.n, nb).copy()

    def sq_params(self, quant: int) -> np.ndarray:
        out = np.zeros((5, self.dim), np.float32)
        lib().oracle_index_sq_params(self.h, quant, _p(out, C.c_float))
        return out

    def nav_initialize(self, q):
        q = np.ascontiguousarray(q, np.float32)
        e, d, n = C.c_uint32(), C.c_float(), C.c_uint32()
        lib().oracle_nav_initialize(self.h, _p(q, C.c_float), C.byref(e), C.byref(d), C.byref(n))
        return int(e.value), float(d.value), int(n.value)

    def search(self, queries, k=10, ef=50, rerank_factor=5, quant=0, adaptive=False, gamma=2.0, min_ef=30,
               max_ef=100, threads=0, history_cap=0, rerank_f16=False, prefetch_offset=16) -> dict:
        q = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
        nq = q.shape[0]
        p = OracleParams(ef=ef, k=k, rerank_factor=rerank_factor, quant=quant, adaptive=int(adaptive), gamma=gamma,
                         min_ef=min_ef, max_ef=max_ef, rerank_f16=int(rerank_f16),
                         prefetch_offset=prefetch_offset)
        r = {"ids": np.zeros((nq, k), np.uint32), "dists": np.zeros((nq, k), np.float32),
             "counts": np.zeros(nq, np.uint32), "visited": np.zeros(nq, np.uint32),
             "ef_used": np.zeros(nq, np.uint32), "n_nav": np.zeros(nq, np.uint32),
             "expansions": np.zeros(nq, np.uint32)}
        hist = np.zeros((nq, history_cap), np.uint32) if history_cap else None
        hl = np.zeros(nq, np.uint32) if history_cap else None
        rc = lib().oracle_search_batch(self.h, _p(q, C.c_float), nq, C.byref(p), threads, _p(r["ids"], C.c_uint32),
                                       _p(r["dists"], C.c_float), _p(r["counts"], C.c_uint32),
                                       _p(r["visited"], C.c_uint32), _p(r["ef_used"], C.c_uint32),
                                       _p(r["n_nav"], C.c_uint32), _p(r["expansions"], C.c_uint32),
                                       _p(hist, C.c_uint32), history_cap, _p(hl, C.c_uint32))
        if rc != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        if history_cap:
            r["history"], r["history_len"] = hist, hl
        return r


def bruteforce(base, queries, k=10, threads=0):
    b = np.ascontiguousarray(base, np.float32)
    q = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
    ids = np.zeros((q.shape[0], k), np.uint32)
    ds = np.zeros((q.shape[0], k), np.float32)
    lib().oracle_bruteforce(_p(b, C.c_float), b.shape[0], _p(q, C.c_float), q.shape[0], b.shape[1], k, threads,
                            _p(ids, C.c_uint32), _p(ds, C.c_float))
    return ids, ds


def merge_shard_lists(ids, dists, counts, shard_size, k):
    """Host merge of per-shard top-k lists (shard-major [S][nq][k], ids local
    to each shard) into global top-k per query, the rule a host-side combiner
    of per-shard reference searches follows: sort the valid entries by
    (distance, shard, rank in the shard's list), keep k; global id =
    shard * shard_size + local id. Missing entries are 0 / 0.0."""
    ids = np.asarray(ids, np.uint32)
    dists = np.asarray(dists, np.float32)
    counts = np.asarray(counts, np.int64)
    S, nq, kk = ids.shape
    out_i = np.zeros((nq, k), np.uint32)
    out_d = np.zeros((nq, k), np.float32)
    out_c = np.zeros(nq, np.uint32)
    for qi in range(nq):
        c = [(float(dists[s, qi, r]), s, r) for s in range(S) for r in range(min(int(counts[s, qi]), kk))]
        c.sort()
        for r, (d, s, rr) in enumerate(c[:k]):
            out_d[qi, r] = d
            out_i[qi, r] = s * shard_size + int(ids[s, qi, rr])
        out_c[qi] = min(len(c), k)
    return out_i, out_d, out_c


HOSTBUILD_LIB = os.path.join(HERE, "_build", "libhostbuild.so")


def build_index_file(vectors, path, r=32, l=200, alpha=1.2, nav_m=32, directional=True, r_soft=None,
                     max_iterations=2, seed=42, threads=0) -> None:
    """Build the Vamana index of `vectors` on the host (the C++ restatement of
    the reference's offline pipeline, PyO3 build parameters by default) and
    write it to `path` as an ANNX v1 file, through oracle/_build/libhostbuild.so
    (the engine's CUDA library is not loaded)."""
    if not os.path.exists(HOSTBUILD_LIB):
        build()
    hb = C.CDLL(HOSTBUILD_LIB)
    f = hb.hostbuild_build_save
    f.restype = C.c_int
    f.argtypes = [f32p, C.c_ulonglong, C.c_uint, C.c_float, C.c_uint, C.c_uint, C.c_uint, C.c_uint, C.c_int,
                  C.c_uint, C.c_ulonglong, C.c_int, C.c_char_p, C.c_char_p, C.c_size_t]
    v = np.ascontiguousarray(vectors, np.float32)
    err = C.create_string_buffer(512)
    rc = f(_p(v, C.c_float), v.shape[0], v.shape[1], alpha, l, r, int(r * 1.5) if r_soft is None else r_soft,
           max_iterations, int(directional), nav_m, seed, threads, os.fsencode(path), err, len(err))
    if rc != 0:
        raise RuntimeError(f"host build failed ({rc}): {err.value.decode()}")
