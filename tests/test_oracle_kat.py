"""Pin the oracle with the reference's own known-answer tests (golden file
tests/golden/reference_kat.json, transcribed from the reference's #[test]s)."""
import json
import os
import struct

import numpy as np
import pytest

from annx_util import annx_bytes, nav_bytes

KAT = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kat.json")))


def test_crc32_known_answer(oracle):
    c = KAT["crc32"]
    assert oracle.crc32(c["input"].encode()) == c["crc"]


def test_linear_pool_insert_and_pop_basic(oracle):
    c = KAT["linear_pool"]["insert_and_pop_basic"]
    p = oracle.Pool(c["ef"])
    assert len(p) == 0
    for i, d in c["inserts"]:
        p.insert(i, d)
    assert len(p) == c["len"]
    for i, d in c["pops"]:
        got = p.pop()
        assert got[0] == i and abs(got[1] - d) < 1e-6
    assert p.pop() is None


def test_linear_pool_capacity_rejects_worst(oracle):
    c = KAT["linear_pool"]["capacity_rejects_worst"]
    p = oracle.Pool(c["ef"])
    for i, d in c["inserts"]:
        p.insert(i, d)
    assert not p.insert(*c["rejected"])
    assert len(p) == c["ef"]
    assert p.insert(*c["accepted"])
    assert len(p) == c["ef"]
    assert abs(p.worst_distance() - c["worst_after"]) < 1e-6


def test_linear_pool_equal_distance_is_rejected_when_full(oracle):
    # dist >= worst is rejected (src/graph/linear_pool.rs:102-108)
    p = oracle.Pool(2)
    p.insert(1, 1.0)
    p.insert(2, 2.0)
    assert not p.insert(3, 2.0)


def test_linear_pool_ties_go_after_existing(oracle):
    # find_insert_pos returns the slot after every d <= dist (:252-263)
    p = oracle.Pool(5)
    for i in (1, 2, 3):
        p.insert(i, 1.0)
    assert [i for i, _ in p.to_sorted_vec()] == [1, 2, 3]


def test_linear_pool_has_next_terminates_at_ef(oracle):
    c = KAT["linear_pool"]["has_next_terminates_at_ef"]
    p = oracle.Pool(c["ef"])
    for i, d in c["inserts"]:
        p.insert(i, d)
    for _ in range(c["pops"]):
        assert p.has_next()
        p.pop()
    assert not p.has_next()


def test_linear_pool_insert_before_cursor_adjusts_cursor(oracle):
    c = KAT["linear_pool"]["insert_before_cursor_adjusts_cursor"]
    p = oracle.Pool(c["ef"])
    for i, d in c["inserts"]:
        p.insert(i, d)
    p.pop()
    assert p.cursor == c["cursor_after_pop"]
    p.insert(*c["insert"])
    assert p.cursor == c["cursor_after_insert"]
    assert p.pop()[0] == c["next_pop"]


def test_linear_pool_sorted_order(oracle):
    c = KAT["linear_pool"]["sorted_order_maintained"]
    p = oracle.Pool(c["ef"])
    for i, d in enumerate(c["distances"]):
        p.insert(i, d)
    r = [d for _, d in p.to_sorted_vec()]
    assert r == sorted(r)


def test_linear_pool_empty_and_clear(oracle):
    p = oracle.Pool(5)
    assert p.pop() is None and not p.has_next()
    assert p.worst_distance() == np.finfo(np.float32).max
    p.insert(1, 1.0)
    p.insert(2, 2.0)
    p.pop()
    p.clear()
    assert len(p) == 0 and not p.has_next()


def test_linear_pool_large_capacity_stress(oracle):
    c = KAT["linear_pool"]["large_capacity_stress"]
    p = oracle.Pool(c["ef"])
    for i in range(c["n"]):
        p.insert(i, i * c["step"])
    assert len(p) == c["len"]
    prev = -1e30
    while True:
        r = p.pop()
        if r is None:
            break
        assert r[1] >= prev
        prev = r[1]


def _samples(spec):
    if spec == "range(100)":
        return np.arange(100, dtype=np.float32)
    if spec == "range(2000)*0.1":
        return (np.arange(2000, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    return np.asarray(spec, np.float32)


def test_adaptive_ef_basic(oracle):
    c = KAT["adaptive_ef"]["estimate_ef_basic"]
    s = _samples(c["samples"])
    for d, ef in c["exact"]:
        assert oracle.estimate_ef(s, c["min_ef"], c["max_ef"], c["gamma"], d) == ef
    d, lo, hi = c["mid"]
    assert lo <= oracle.estimate_ef(s, c["min_ef"], c["max_ef"], c["gamma"], d) <= hi


def test_adaptive_ef_power_law(oracle):
    c = KAT["adaptive_ef"]["estimate_ef_power_law"]
    d, lo, hi = c["mid"]
    assert lo <= oracle.estimate_ef(_samples(c["samples"]), c["min_ef"], c["max_ef"], c["gamma"], d) <= hi


def test_adaptive_ef_monotonic(oracle):
    c = KAT["adaptive_ef"]["estimate_ef_monotonic"]
    s = _samples(c["samples"])
    efs = [oracle.estimate_ef(s, c["min_ef"], c["max_ef"], c["gamma"], d) for d in c["distances"]]
    assert efs == sorted(efs)


def test_adaptive_ef_bounds(oracle):
    c = KAT["adaptive_ef"]["estimate_ef_respects_bounds"]
    s = _samples(c["samples"])
    for d in c["distances"]:
        assert c["min_ef"] <= oracle.estimate_ef(s, c["min_ef"], c["max_ef"], c["gamma"], d) <= c["max_ef"]


def test_adaptive_ef_empty_samples_midpoint(oracle):
    c = KAT["adaptive_ef"]["empty_samples_returns_average"]
    assert oracle.estimate_ef(np.zeros(0, np.float32), c["min_ef"], c["max_ef"], c["gamma"], c["d"]) == c["ef"]


def test_adaptive_ef_build_f32_simple(oracle):
    c = KAT["adaptive_ef"]["build_f32_simple"]
    v = np.arange(20, dtype=np.float32).reshape(10, 2)
    s = np.sort(np.array([oracle.l2_avx512(v[c["entry"]], v[i]) for i in range(10)], np.float32))
    assert s.size == c["sample_count"]
    assert oracle.estimate_ef(s, c["min_ef"], c["max_ef"], c["gamma"], c["d"]) == c["ef"]


def test_sq4_params_fit_basic(oracle):
    c = KAT["sq4"]["sq4_params_fit_basic"]
    p = oracle.sq_fit(np.asarray(c["data"], np.float32).reshape(-1, c["dim"]), 15)
    assert np.allclose(p[0], c["min"], atol=1e-6) and np.allclose(p[1], c["max"], atol=1e-6)
    assert abs(p[2][0] - c["scale0"]) < 1e-6


def _sq4_decode(p, code, dim):
    out = np.zeros(dim, np.float32)
    for d in range(dim):
        raw = code[d // 2] & 0x0F if d % 2 == 0 else (code[d // 2] >> 4) & 0x0F
        out[d] = np.float32(np.fma(np.float32(raw), p[2][d], p[0][d])) if hasattr(np, "fma") else \
            np.float32(raw) * p[2][d] + p[0][d]
    return out


def test_sq4_encode_decode_roundtrip(oracle):
    c = KAT["sq4"]["sq4_encode_decode_roundtrip"]
    dim = c["dim"]
    data = (np.arange(c["n"] * dim, dtype=np.float64) * c["scale"]).astype(np.float32).reshape(c["n"], dim)
    p = oracle.sq_fit(data, 15)
    code = oracle.sq4_encode(p, data[0])[0]
    assert code.size == (dim + 1) // 2
    dec = _sq4_decode(p, code, dim)
    assert np.all(np.abs(dec - data[0]) <= p[2] + 1e-6)


def test_sq4_distance_matches_scalar_formula(oracle):
    dim = 128
    data = (np.arange(256 * dim, dtype=np.float64) * 0.01).astype(np.float32).reshape(256, dim)
    p = oracle.sq_fit(data, 15)
    codes = oracle.sq4_encode(p, data)
    q = np.sin(np.arange(dim) * 0.02).astype(np.float32)
    qc = oracle.sq4_encode(p, q)[0]
    for idx in (0, 1, 50, 100, 255):
        a = np.concatenate([qc & 15, qc >> 4]).astype(np.int64)
        b = np.concatenate([codes[idx] & 15, codes[idx] >> 4]).astype(np.int64)
        assert oracle.l2_sq4_raw(qc, codes[idx]) == float(((a - b) ** 2).sum())


def test_sq4_memory_compression(oracle):
    c = KAT["sq4"]["sq4_memory_compression"]
    data = (np.arange(c["n"] * c["dim"], dtype=np.float64) * 0.001).astype(np.float32).reshape(c["n"], c["dim"])
    codes = oracle.sq4_encode(oracle.sq_fit(data, 15), data)
    assert codes.size == c["bytes"]
    assert abs(data.nbytes / codes.size - c["ratio"]) < 0.1


def test_sq4_distance_correlation_with_f32(oracle):
    c = KAT["sq4"]["sq4_distance_correlation_with_f32"]
    n, dim = c["n"], c["dim"]
    data = (np.sin(np.arange(n * dim, dtype=np.float32) * np.float32(0.1)) * 0.5 + 0.5).astype(np.float32)
    data = data.reshape(n, dim)
    p = oracle.sq_fit(data, 15)
    codes = oracle.sq4_encode(p, data)
    q = (np.cos(np.arange(dim, dtype=np.float32) * np.float32(0.1)) * 0.5 + 0.5).astype(np.float32)
    qc = oracle.sq4_encode(p, q)[0]
    d4 = [(oracle.l2_sq4_raw(qc, codes[i]), i) for i in range(200)]
    df = [(float(((data[i] - q) ** 2).sum()), i) for i in range(200)]
    top4 = {i for _, i in sorted(d4)[:10]}
    topf = {i for _, i in sorted(df)[:10]}
    assert len(top4 & topf) >= c["min_overlap"]


def test_sq8_encode_range_and_distance(oracle):
    rng = np.random.default_rng(3)
    data = rng.normal(size=(500, 64)).astype(np.float32)
    p = oracle.sq_fit(data, 255)
    codes = oracle.sq8_encode(p, data)
    assert codes.min() == 0 and codes.max() == 255
    d = oracle.l2_sq8_raw(codes[0], codes[1])
    assert d == float(((codes[0].astype(np.int64) - codes[1]) ** 2).sum())


def test_l2_orders_agree_on_integers(oracle):
    rng = np.random.default_rng(5)
    for dim in (4, 16, 96, 100, 128):
        a = rng.integers(0, 256, dim).astype(np.float32)
        b = rng.integers(0, 256, dim).astype(np.float32)
        exact = float(((a.astype(np.int64) - b) ** 2).sum())
        assert oracle.l2_avx512(a, b) == exact
        assert oracle.l2_avx2(a, b) == exact


def test_l2_avx512_order_is_the_lane_tree(oracle):
    # dim 37: 2 full 16-lane chunks + a 5-element masked tail.
    rng = np.random.default_rng(11)
    a = rng.normal(size=37).astype(np.float32)
    b = rng.normal(size=37).astype(np.float32)
    d = (a - b).astype(np.float32)
    acc = np.zeros(16, np.float32)
    for c in range(2):
        for j in range(16):
            x = d[16 * c + j]
            acc[j] = np.float32(np.float64(x) * np.float64(x) + np.float64(acc[j]))  # exact fma then round

    def tree(v):
        v8 = (v[:8] + v[8:]).astype(np.float32)
        v4 = (v8[:4] + v8[4:]).astype(np.float32)
        v2 = (v4[:2] + v4[2:]).astype(np.float32)
        return np.float32(v2[0] + v2[1])

    t = np.zeros(16, np.float32)
    t[:5] = (d[32:] * d[32:]).astype(np.float32)
    expect = np.float32(tree(t) + tree(acc))
    assert oracle.l2_avx512(a, b) == float(expect)


def _nav_annx(case, n_graph=8):
    nav = nav_bytes(case["entry_point"], case["max_level"], case["k"], case["node_levels"], case["upper_lists"],
                    case.get("entry_candidates"))
    rows = [[(i + 1) % n_graph] for i in range(n_graph)]
    return annx_bytes(n_graph, 4, 0, 4, rows, nav=nav, meta="n = 8\n")


def test_layered_nav_serialization_roundtrip(oracle):
    c = KAT["layered_nav_roundtrip"]
    oi = oracle.OracleIndex(data=_nav_annx(c, n_graph=len(c["node_levels"])))
    assert oi.nav_present and oi.nav_max_level == c["max_level"] and oi.nav_k == c["k"]
    for i, l in enumerate(c["upper_lists"]):
        assert oi.nav_list(i).tolist() == l
        assert oi.nav_level(i) == c["node_levels"][i]
    assert oi.entry_candidates().tolist() == c["entry_candidates"]


def test_layered_nav_backward_compat(oracle):
    c = dict(KAT["layered_nav_backward_compat"])
    cand = c.pop("entry_candidates")
    c_nocand = dict(c, entry_candidates=None)
    oi = oracle.OracleIndex(data=_nav_annx(c_nocand, n_graph=len(c["node_levels"])))
    assert oi.entry_candidates().tolist() == cand


def test_header_little_endian(oracle):
    c = KAT["header_le"]
    b = annx_bytes(2, 4, 0, 2, [[1], [0]])
    assert list(b[0:4]) == c["magic_bytes"]
    hdr = struct.pack("<IIII", 0x414E4E58, 1, 0, c["crc"])
    assert list(hdr[12:16]) == c["crc_bytes"]
    oi = oracle.OracleIndex(data=b)
    assert oi.n == 2 and oi.dim == 4


@pytest.mark.parametrize("mutate,code", [("magic", -3), ("version", -4), ("crc", -5), ("truncate", -2)])
def test_oracle_rejects_corrupt_files(oracle, mutate, code):
    b = bytearray(annx_bytes(3, 4, 0, 2, [[1, 2], [0], [0, 1]]))
    if mutate == "magic":
        b[0] = 0
    elif mutate == "version":
        b[4] = 9
    elif mutate == "crc":
        b[-1] ^= 0xFF
    else:
        b = b[:30]
    with pytest.raises(IOError) as e:
        oracle.OracleIndex(data=bytes(b))
    assert f"[{code}]" in str(e.value)


def test_degree_is_first_sentinel(oracle):
    # from_parts: degree = position of the first SENTINEL (src/memory/graph.rs:234-240)
    rows = [[1, 2, 0xFFFFFFFF, 3], [0], [0, 1, 3], [2]]
    b = annx_bytes(4, 4, 0, 4, rows)
    oi = oracle.OracleIndex(data=b)
    assert oi.neighbors(0).tolist() == [1, 2]
    assert oi.neighbors(2).tolist() == [0, 1, 3]


# F16::from_f32 / to_f32 / l2_f16_mixed known answers (src/distance/f16.rs:380-470 tests)
def test_f16_conversion_kat(oracle):
    assert oracle.f16_from_f32(0.0) == 0
    assert oracle.f16_from_f32(-0.0) == 0x8000
    assert oracle.f16_from_f32(float("inf")) == 0x7C00
    assert oracle.f16_from_f32(float("-inf")) == 0xFC00
    assert oracle.f16_from_f32(70000.0) & 0x7C00 == 0x7C00  # above 65504: Inf
    for v in (1.0, 2.0, 3.0, 0.5, -1.5, 100.0, 0.001):
        r = oracle.f16_to_f32(oracle.f16_from_f32(v))
        assert abs(r - v) / max(v, 1e-6) < 0.01
    vals = [i / 100.0 for i in range(100)]
    assert max(abs(oracle.f16_to_f32(oracle.f16_from_f32(v)) - v) for v in vals) < 0.001
    # integers up to 2048 are exact
    for i in range(0, 2049, 7):
        assert oracle.f16_to_f32(oracle.f16_from_f32(float(i))) == float(i)


def test_f16_rounding_follows_reference(oracle):
    # the reference ORs the round bit into the truncated mantissa: an even
    # mantissa rounds up past half, an odd one never does
    one_plus = np.float32(1.0) + np.float32(2.0 ** -10)  # mantissa ...01 (odd), exact in f16
    assert oracle.f16_from_f32(float(one_plus)) == 0x3C01
    above_even = np.float32(1.0) + np.float32(2.0 ** -11) * 1.5  # even mantissa, remainder above half
    assert oracle.f16_from_f32(float(above_even)) == 0x3C01
    above_odd = np.float32(1.0) + np.float32(2.0 ** -10) + np.float32(2.0 ** -11) * 1.5  # odd, above half
    assert oracle.f16_from_f32(float(above_odd)) == 0x3C01  # IEEE would give 0x3C02


def test_l2_f16_mixed_kat(oracle):
    q = np.array([1.0, 2.0, 3.0], np.float32)
    db = np.array([oracle.f16_from_f32(x) for x in (4.0, 5.0, 6.0)], np.uint16)
    assert abs(oracle.l2_f16_mixed(q, db) - 27.0) < 0.5
    q = (np.arange(128) / 128.0).astype(np.float32)
    dbf = (np.arange(128) / 128.0 * 0.9).astype(np.float32)
    db = np.array([oracle.f16_from_f32(float(x)) for x in dbf], np.uint16)
    exact = float(np.sum((q.astype(np.float64) - dbf) ** 2))
    assert abs(oracle.l2_f16_mixed(q, db) - exact) / exact < 0.01
