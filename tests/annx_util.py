"""Pure-Python ANNX v1 writer for hand-made test graphs.

Layout (all little-endian) as written by the reference:
  header  magic u32 0x414E4E58, version u32 1, flags u32, crc32(body) u32
          (src/memory/serialize.rs:58-89)
  body    n u64, dim u64, entry u32                      (src/graph/vamana.rs:1280-1282)
          [flag 0x1] meta_len u32, TOML bytes, pad to 4  (:1286-1291)
          [flag 0x2] nav_len u32, nav bytes, pad to 4    (:1294-1300)
          csr: n u64, r_max u64, mb_len u64, u32[mb_len],
               ov_count u64, {node u32, len u64, u32[len]} (src/memory/graph.rs:322-345)
  nav     entry u32, max_level u8, 3 pad, k u32, n u32, node_levels u8[n],
          count u32, {node u32, len u32, u32[len]}, ec_len u32, u32[ec_len]
          (src/graph/navigation.rs:670-706)
"""
from __future__ import annotations

import struct
import zlib

SENTINEL = 0xFFFFFFFF


def nav_bytes(entry, max_level, k, node_levels, upper, entry_candidates=None) -> bytes:
    b = bytearray()
    b += struct.pack("<I", entry)
    b += bytes([max_level, 0, 0, 0])
    b += struct.pack("<II", k, len(node_levels))
    b += bytes(node_levels)
    nonempty = [(i, l) for i, l in enumerate(upper) if len(l)]
    b += struct.pack("<I", len(nonempty))
    for i, l in nonempty:
        b += struct.pack("<II", i, len(l))
        b += struct.pack(f"<{len(l)}I", *l)
    if entry_candidates is not None:
        b += struct.pack("<I", len(entry_candidates))
        b += struct.pack(f"<{len(entry_candidates)}I", *entry_candidates)
    return bytes(b)


def annx_bytes(n, dim, entry, r_max, rows, overflow=None, nav: bytes | None = None, meta: str | None = None,
               version=1, magic=0x414E4E58) -> bytes:
    """rows: list of neighbour lists (each <= r_max, SENTINEL padded here)."""
    body = bytearray()
    body += struct.pack("<QQI", n, dim, entry)
    flags = 0
    if meta:
        mb = meta.encode()
        flags |= 1
        body += struct.pack("<I", len(mb)) + mb + b"\0" * ((4 - len(mb) % 4) % 4)
    if nav is not None:
        flags |= 2
        body += struct.pack("<I", len(nav)) + nav + b"\0" * ((4 - len(nav) % 4) % 4)
    body += struct.pack("<QQQ", n, r_max, n * r_max)
    for r in rows:
        full = list(r) + [SENTINEL] * (r_max - len(r))
        body += struct.pack(f"<{r_max}I", *full)
    ov = overflow or {}
    body += struct.pack("<Q", len(ov))
    for node, l in ov.items():
        body += struct.pack("<IQ", node, len(l)) + struct.pack(f"<{len(l)}I", *l)
    crc = zlib.crc32(bytes(body)) & 0xFFFFFFFF
    return struct.pack("<IIII", magic, version, flags, crc) + bytes(body)
