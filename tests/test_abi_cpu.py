"""CPU-side checks of the C ABI library: it loads, exports every symbol the
header declares, and reports errors as status codes (no GPU needed)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from annx_util import annx_bytes

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    txt = open(os.path.join(ROOT, "include", "raven_gpu.h")).read()
    return sorted(set(re.findall(r"RAVEN_API\s+(?:const\s+)?\w+\*?\s+(raven_\w+)\(", txt)))


def test_header_declares_the_api():
    names = _declared()
    for must in ("raven_index_upload", "raven_search_batch", "raven_search_batch_device", "raven_last_error",
                 "raven_graph_load", "raven_graph_build", "raven_index_free"):
        assert must in names


def test_library_exports_every_declared_symbol(raven_lib):
    for name in _declared():
        assert hasattr(raven_lib, name), name


def test_binding_covers_every_declared_symbol():
    from raven_b200 import _lib as L

    assert set(_declared()) == set(L.SIGNATURES)


def test_version_and_limits(raven_lib):
    from raven_b200 import _lib as L

    assert b"sm_100a" in raven_lib.raven_version()
    lim = L.Limits()
    raven_lib.raven_limits(C.byref(lim))
    assert lim.max_ef >= 100 and lim.max_dim >= 128 and lim.max_r >= 32 and lim.max_nav_k >= 16


def test_graph_load_errors_are_codes(raven_lib):
    from raven_b200 import _lib as L
    from raven_b200.index import Graph

    good = annx_bytes(3, 4, 0, 2, [[1, 2], [0], [0, 1]])
    g = Graph.from_bytes(good)
    assert len(g) == 3 and g.neighbors(0).tolist() == [1, 2] and g.neighbors(1).tolist() == [0]
    for mutate, code in (("magic", L.RAVEN_EMAGIC), ("version", L.RAVEN_EVERSION), ("crc", L.RAVEN_ECRC),
                         ("trunc", L.RAVEN_EFORMAT)):
        b = bytearray(good)
        if mutate == "magic":
            b[0] = 0
        elif mutate == "version":
            b[4] = 2
        elif mutate == "crc":
            b[-1] ^= 1
        else:
            b = b[:24]
        with pytest.raises(L.RavenError) as e:
            Graph.from_bytes(bytes(b))
        assert e.value.code == code
    with pytest.raises(L.RavenError) as e:
        Graph.load("/nonexistent/file.annx")
    assert e.value.code == L.RAVEN_EIO


def test_upload_without_gpu_fails_loudly(raven_lib):
    """On a machine without a GPU the engine refuses with a CUDA status (no
    silent CPU fallback)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex, Graph

    g = Graph.from_bytes(annx_bytes(3, 4, 0, 2, [[1, 2], [0], [0, 1]]))
    with pytest.raises(L.RavenError) as e:
        DeviceIndex(g, np.zeros((3, 4), np.float32))
    assert e.value.code == L.RAVEN_ECUDA


def test_upload_validates_ids_before_device_work(raven_lib):
    from raven_b200 import _lib as L
    from raven_b200.index import DeviceIndex, Graph

    g = Graph.from_bytes(annx_bytes(3, 4, 0, 2, [[1, 7], [0], [0, 1]]))  # id 7 >= n
    with pytest.raises(L.RavenError) as e:
        DeviceIndex(g, np.zeros((3, 4), np.float32))
    assert e.value.code == L.RAVEN_EFORMAT
    g2 = Graph.from_bytes(annx_bytes(3, 4, 0, 2, [[1, 2], [0], [0, 1]]))
    with pytest.raises(L.RavenError) as e:
        DeviceIndex(g2, np.zeros((3, 5), np.float32))
    assert e.value.code == L.RAVEN_EINVAL


# ctypes mirror -> C typedef in include/raven_gpu.h
_STRUCTS = {"BuildConfig": "raven_build_config", "GraphInfo": "raven_graph_info_t",
            "UploadOptions": "raven_upload_options", "SearchParams": "raven_search_params",
            "SearchOutputs": "raven_search_outputs", "Limits": "raven_limits_t"}


def test_binding_structs_match_header_layout(tmp_path):
    """Every ctypes struct has the C struct's size and each field's offset, as
    compiled by gcc from the header (the layout a Rust #[repr(C)] mirror must
    also have)."""
    import shutil
    import subprocess

    from raven_b200 import _lib as L

    if shutil.which("gcc") is None:
        pytest.skip("gcc not available")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "raven_gpu.h"', "int main(void) {"]
    for py, c in _STRUCTS.items():
        lines.append(f'  printf("{py} size %zu\\n", sizeof({c}));')
        for f, _ in getattr(L, py)._fields_:
            lines.append(f'  printf("{py} {f} %zu\\n", offsetof({c}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {tuple(ln.split()[:2]): int(ln.split()[2]) for ln in out if ln.strip()}
    for py in _STRUCTS:
        cls = getattr(L, py)
        assert got[(py, "size")] == C.sizeof(cls), py
        for f, _ in cls._fields_:
            assert got[(py, f)] == getattr(cls, f).offset, (py, f)


def test_raven_import_name():
    """`import raven` gives the PyO3 module's two classes (src/python.rs:355-360)
    with the reference's constructor defaults and errors."""
    import raven

    assert set(raven.__all__) == {"Index", "Searcher"}
    ix = raven.Index("L2", 64)
    assert (ix.r, ix.l, ix.alpha, ix.nav_m, ix.quant, ix.rerank) == (32, 200, 1.2, 32, "sq8", 5)
    with pytest.raises(ValueError):
        raven.Index("L2", 64, quantization="pq")
    with pytest.raises(RuntimeError):
        ix.searcher()
