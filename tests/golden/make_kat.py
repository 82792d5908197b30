"""Check tests/golden/reference_kat.json against the reference's test sources.

The known answers in reference_kat.json were transcribed from the reference's
#[test] functions (it is Rust and cannot be built here). When the reference
tree is available this script re-reads each cited test and asserts that the
constants in the JSON occur in it, so a transcription error is caught. The
tree's location is required, as the first argument or the REF_ROOT variable:

    python tests/golden/make_kat.py <reference source tree>
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

# tokens that must appear in the cited line range of each case
TOKENS = {
    "crc32": ["hello world", "0x0D4A1185"],
    "header_le": ["0x12345678", "0x58, 0x4E, 0x4E, 0x41", "0x78, 0x56, 0x34, 0x12"],
    "linear_pool.insert_and_pop_basic": ["LinearPool::new(5)", "pool.insert(1, 3.0)", "pool.insert(2, 1.0)",
                                         "pool.insert(3, 2.0)"],
    "linear_pool.capacity_rejects_worst": ["LinearPool::new(3)", "pool.insert(4, 4.0)", "pool.insert(5, 2.5)"],
    "linear_pool.has_next_terminates_at_ef": ["LinearPool::new(3)"],
    "linear_pool.insert_before_cursor_adjusts_cursor": ["LinearPool::new(10)", "pool.insert(1, 5.0)",
                                                        "pool.insert(3, 3.0)", "assert_eq!(pool.cursor, 0)"],
    "linear_pool.sorted_order_maintained": ["[5.0, 1.0, 3.0, 2.0, 4.0, 0.5, 2.5]"],
    "linear_pool.large_capacity_stress": ["LinearPool::new(100)", "0..200", "0.5"],
    "adaptive_ef.estimate_ef_basic": ["20, 80, 1.0", "estimate_ef(-1.0), 20", "estimate_ef(200.0), 80"],
    "adaptive_ef.estimate_ef_power_law": ["20, 80, 3.0", "mid_ef >= 26 && mid_ef <= 30"],
    "adaptive_ef.estimate_ef_monotonic": ["10, 100, 2.0", "0..2000"],
    "adaptive_ef.estimate_ef_respects_bounds": ["vec![1.0, 2.0, 3.0, 4.0, 5.0]", "30, 70, 3.0"],
    "adaptive_ef.empty_samples_returns_average": ["20, 80, 3.0", "estimate_ef(42.0), 50"],
    "adaptive_ef.build_f32_simple": ["10, 50, 2.0", "sample_count(), 10", "assert_eq!(ef, 10)"],
    "sq4.sq4_params_fit_basic": ["[0.0, 0.0, 1.0, 2.0, 0.5, 1.0]", "1.0 / 15.0"],
    "sq4.sq4_encode_decode_roundtrip": ["0..256", "let dim = 128", "0.01"],
    "sq4.sq4_memory_compression": ["let n = 1000", "8.0"],
    "sq4.sq4_distance_correlation_with_f32": ["overlap >= 7"],
    "layered_nav_roundtrip": ["entry_point: 42", "max_level: 3", "k: 16", "vec![0, 0, 1, 2, 3, 1, 0, 2]",
                              "vec![4, 7, 2, 5, 1, 6, 0, 3]", "vec![42, 4]"],
    "layered_nav_backward_compat": ["entry_point: 7", "vec![0, 0, 1, 2]", "vec![7]"],
}


def cases(d, prefix=""):
    for k, v in d.items():
        if k.startswith("_"):
            continue
        if isinstance(v, dict) and "source" in v:
            yield prefix + k, v
        elif isinstance(v, dict):
            yield from cases(v, prefix + k + ".")


def main(argv) -> int:
    REF = argv[1] if len(argv) > 1 else os.environ.get("REF_ROOT")
    if not REF:
        print("usage: make_kat.py <reference source tree>  (or set REF_ROOT)")
        return 2
    kat = json.load(open(os.path.join(HERE, "reference_kat.json")))
    if not os.path.isdir(REF):
        print(f"reference tree not found at {REF}")
        return 2
    bad = 0
    for name, c in cases(kat):
        m = re.match(r"(.+):(\d+)-(\d+)", c["source"])
        path, a, b = m.group(1), int(m.group(2)), int(m.group(3))
        lines = open(os.path.join(REF, path), encoding="utf-8").read().split("\n")[a - 1:b]
        text = "\n".join(lines)
        for tok in TOKENS.get(name, []):
            if tok not in text:
                print(f"MISSING {name}: {tok!r} not in {c['source']}")
                bad += 1
    print("ok" if not bad else f"{bad} problems")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
