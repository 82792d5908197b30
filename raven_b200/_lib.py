"""ctypes binding of the C ABI in include/raven_gpu.h (libraven_gpu.so).

The library is the only implementation of the engine: there is no CPU or
Python fallback. Loading fails loudly when the shared library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libraven_gpu.so")

RAVEN_OK = 0
RAVEN_EINVAL = -1
RAVEN_EIO = -2
RAVEN_EMAGIC = -3
RAVEN_EVERSION = -4
RAVEN_ECRC = -5
RAVEN_EFORMAT = -6
RAVEN_ESTATE = -7
RAVEN_ECUDA = -8
RAVEN_ENOMEM = -9
RAVEN_ELIMIT = -10

RAVEN_QUANT_SQ4 = 0
RAVEN_QUANT_SQ8 = 1
RAVEN_QUANT_F32 = 2

u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)


class BuildConfig(C.Structure):
    _fields_ = [
        ("alpha", C.c_float),
        ("l_build", C.c_uint32),
        ("r_max", C.c_uint32),
        ("r_soft", C.c_uint32),
        ("max_iterations", C.c_uint32),
        ("saturate", C.c_int32),
        ("layered_nav", C.c_int32),
        ("nav_m", C.c_uint32),
        ("directional", C.c_int32),
        ("seed", C.c_uint64),
        ("threads", C.c_int32),
        ("verbose", C.c_int32),
    ]


class GraphInfo(C.Structure):
    _fields_ = [
        ("n", C.c_uint64),
        ("dim", C.c_uint64),
        ("r_max", C.c_uint64),
        ("entry_point", C.c_uint32),
        ("has_nav", C.c_int32),
        ("nav_entry", C.c_uint32),
        ("nav_max_level", C.c_uint32),
        ("nav_k", C.c_uint32),
        ("nav_upper_nodes", C.c_uint64),
    ]


class UploadOptions(C.Structure):
    _fields_ = [
        ("device", C.c_int32),
        ("build_sq4", C.c_int32),
        ("build_sq8", C.c_int32),
        ("build_adaptive", C.c_int32),
        ("build_f16", C.c_int32),
    ]


class SearchParams(C.Structure):
    _fields_ = [
        ("ef", C.c_uint32),
        ("k", C.c_uint32),
        ("rerank_factor", C.c_uint32),
        ("prefetch_offset", C.c_uint32),
        ("quant", C.c_int32),
        ("adaptive", C.c_int32),
        ("gamma", C.c_float),
        ("min_ef", C.c_uint32),
        ("max_ef", C.c_uint32),
        ("rerank_f16", C.c_int32),
    ]


class SearchOutputs(C.Structure):
    _fields_ = [
        ("ids", u32p),
        ("dists", f32p),
        ("counts", u32p),
        ("visited", u32p),
        ("ef_used", u32p),
        ("status", i32p),
        ("n_nav", u32p),
        ("expansions", u32p),
        ("history", u32p),
        ("history_cap", C.c_uint32),
        ("history_len", u32p),
    ]


class Limits(C.Structure):
    _fields_ = [("max_ef", C.c_uint32), ("max_dim", C.c_uint32), ("max_r", C.c_uint32), ("max_nav_k", C.c_uint32)]


# name -> (restype, argtypes); every symbol declared in include/raven_gpu.h
SIGNATURES = {
    "raven_graph_build": (C.c_int, [f32p, C.c_uint64, C.c_uint32, C.POINTER(BuildConfig), C.POINTER(C.c_void_p)]),
    "raven_graph_build_gpu": (C.c_int, [f32p, C.c_uint64, C.c_uint32, C.POINTER(BuildConfig), C.c_int,
                                        C.POINTER(C.c_void_p)]),
    "raven_graph_load": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "raven_graph_load_bytes": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p)]),
    "raven_graph_save": (C.c_int, [C.c_void_p, C.c_char_p]),
    "raven_graph_free": (None, [C.c_void_p]),
    "raven_graph_info": (C.c_int, [C.c_void_p, C.POINTER(GraphInfo)]),
    "raven_graph_neighbors": (C.c_int, [C.c_void_p, C.c_uint32, u32p, C.c_uint32, u32p]),
    "raven_index_upload": (C.c_int, [C.c_void_p, f32p, C.c_uint64, C.c_uint32, C.POINTER(UploadOptions),
                                     C.POINTER(C.c_void_p)]),
    "raven_index_free": (C.c_int, [C.c_void_p]),
    "raven_index_adaptive_samples": (C.c_int, [C.c_void_p, f32p, C.c_uint32, u32p]),
    "raven_index_sq_params": (C.c_int, [C.c_void_p, C.c_int32, f32p]),
    "raven_index_codes": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_uint8), C.c_uint64]),
    "raven_search_batch": (C.c_int, [C.c_void_p, f32p, C.c_uint64, C.POINTER(SearchParams),
                                     C.POINTER(SearchOutputs), C.c_void_p]),
    "raven_search_batch_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.POINTER(SearchParams),
                                            C.POINTER(SearchOutputs), C.c_void_p]),
    "raven_search_batch_device_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.POINTER(SearchParams),
                                                    C.POINTER(SearchOutputs), C.c_void_p]),
    "raven_knn_exact_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint32, C.c_void_p, C.c_void_p,
                                         C.c_void_p]),
    "raven_merge_topk_device": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint64, C.c_uint32,
                                          C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "raven_merge_topk_gathered_device": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint64,
                                                   C.c_uint32, C.c_uint64, C.c_void_p, C.c_void_p, C.c_void_p,
                                                   C.c_void_p]),
    "raven_limits": (None, [C.POINTER(Limits)]),
    "raven_index_set_tuning": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32]),
    "raven_index_set_small_batch": (C.c_int, [C.c_void_p, C.c_uint64]),
    "raven_index_set_fat_rows": (C.c_int, [C.c_void_p, C.c_int32]),
    "raven_last_error": (C.c_char_p, []),
    "raven_version": (C.c_char_p, []),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load libraven_gpu.so (built by `python -m raven_b200.build`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build the CUDA engine with `python -m raven_b200.build` "
            "(there is no CPU fallback)"
        )
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class RavenError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def check(rc: int) -> None:
    if rc != RAVEN_OK:
        msg = load().raven_last_error()
        raise RavenError(rc, msg.decode() if msg else "")


def ptr(a, ctype):
    """ctypes pointer to a numpy array's data (None for None)."""
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(ctype))
