// ORACLE — test infrastructure, not product code.
//
// A plain C++17 restatement of RAVEN's CPU query path (Juwan-Hwang/RAVEN, Rust,
// CPU-only), used ONLY as the checker for the CUDA engine in raven_b200/: by
// tests/, by __graft_entry__.smoke() and by bench.py's cpu_baseline leg.
// Nothing in the product links, imports or calls this file.
//
// Parity status: the reference cannot be compiled here (Rust, no cargo/rustc),
// so this restatement is pinned by the reference's own known-answer unit tests,
// ported as tests/test_oracle_kat.py (LinearPool, SQ4, AdaptiveEf, CRC32,
// header layout, nav serialisation) — component-level pins. End-to-end search
// output has no golden vectors in the reference; it follows the cited lines.
//
// Every function cites the reference file:line it restates. Floating point:
// compiled with -ffp-contract=off; every FMA the reference performs is an
// explicit std::fma here, every plain multiply/add stays separate.

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

#include <xmmintrin.h>

namespace {

constexpr uint32_t kSentinel = 0xFFFFFFFFu;             // src/lib.rs:37
constexpr uint32_t kIndexMagic = 0x414E4E58u;           // src/memory/serialize.rs:19
constexpr uint32_t kIndexVersion = 1;                   // src/memory/serialize.rs:23
constexpr uint32_t kFlagHasMetadata = 0x1;              // src/memory/serialize.rs:26
constexpr uint32_t kFlagHasLayeredNav = 0x2;            // src/memory/serialize.rs:29
constexpr size_t kHeaderSize = 16;                      // src/memory/serialize.rs:32

thread_local std::string g_err;

// ---------------------------------------------------------------------------
// CRC-32/IEEE (crc32fast 1.5.0 computes the standard reflected CRC-32,
// polynomial 0xEDB88320, init/xorout 0xFFFFFFFF). Pinned by
// src/memory/serialize.rs:196-202 (crc32("hello world") == 0x0D4A1185).
// ---------------------------------------------------------------------------
uint32_t crc_table[256];
bool crc_ready = false;
void crc_init() {
  for (uint32_t i = 0; i < 256; ++i) {
    uint32_t c = i;
    for (int b = 0; b < 8; ++b) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
    crc_table[i] = c;
  }
  crc_ready = true;
}
uint32_t crc32_bytes(const uint8_t* p, size_t n) {
  if (!crc_ready) crc_init();
  uint32_t c = 0xFFFFFFFFu;
  for (size_t i = 0; i < n; ++i) c = crc_table[(c ^ p[i]) & 0xFF] ^ (c >> 8);
  return c ^ 0xFFFFFFFFu;
}

template <class T>
T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}

// ---------------------------------------------------------------------------
// f32 squared-L2 in the reference's summation orders.
// ---------------------------------------------------------------------------

// src/distance/avx512.rs:31-62 — 16 lane accumulators, lane j sums
// fma(d, d, acc) over chunks c (element 16c+j) in order; a masked tail vector
// gets its own fma(d,d,0) lanes; each 16-lane vector is reduced by
// _mm512_reduce_add_ps as a halving tree (16->8: l+l+8, 8->4: l+l+4,
// 4->2: l+l+2, 2->1: l0+l1); result = tail_sum + main_sum.
float tree16(const float* v) {
  float a8[8], a4[4], a2[2];
  for (int i = 0; i < 8; ++i) a8[i] = v[i] + v[i + 8];
  for (int i = 0; i < 4; ++i) a4[i] = a8[i] + a8[i + 4];
  for (int i = 0; i < 2; ++i) a2[i] = a4[i] + a4[i + 2];
  return a2[0] + a2[1];
}
float l2_avx512_order(const float* a, const float* b, size_t n) {
  size_t chunks = n / 16, rem = n % 16;
  float acc[16];
  for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 16; ++j) {
      float d = a[c * 16 + j] - b[c * 16 + j];
      acc[j] = std::fma(d, d, acc[j]);
    }
  float result = 0.0f;
  if (rem > 0) {
    float t[16];
    for (int j = 0; j < 16; ++j) {
      float d = (size_t)j < rem ? a[chunks * 16 + j] - b[chunks * 16 + j] : 0.0f;
      t[j] = std::fma(d, d, 0.0f);
    }
    result = tree16(t);
  }
  return result + tree16(acc);
}

// ---------------------------------------------------------------------------
// f16 rerank arithmetic (src/distance/f16.rs).
// ---------------------------------------------------------------------------

// F16::from_f32 (f16.rs:26-76) with its exact behaviour: normal results OR the
// round bit into the truncated mantissa (an odd mantissa is never rounded
// up), denormal results are truncated, overflow gives Inf, NaN gives 0x7E00.
uint16_t f16_from_f32(float f) {
  uint32_t bits;
  std::memcpy(&bits, &f, 4);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const int32_t exp = (int32_t)((bits >> 23) & 0xFFu);
  const uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | (mant ? 0x7E00u : 0x7C00u));
  const int32_t new_exp = exp - 127 + 15;
  if (new_exp >= 0x1F) return (uint16_t)(sign | 0x7C00u);
  if (new_exp <= 0) {
    if (new_exp < -10) return sign;
    const uint32_t m = mant | 0x800000u;
    const int32_t shift = 14 - new_exp;
    const uint32_t half = 1u << (shift - 1);
    // the reference's round-up test compares (m & (half-1)) with half: never true
    const uint32_t up = ((m & (half - 1)) > half || ((m & half) > 0 && (m & (half - 1)) >= half)) ? 1u : 0u;
    return (uint16_t)(sign | (uint16_t)((m >> shift) + up));
  }
  const uint16_t mant_f16 = (uint16_t)(mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  const uint16_t round = (rem > 0x1000u || (rem == 0x1000u && (mant_f16 & 1u))) ? 1 : 0;
  uint16_t result = (uint16_t)(sign | ((uint16_t)new_exp << 10) | mant_f16 | round);
  if ((result & 0x7C00u) == 0x7C00u) result = (uint16_t)(sign | 0x7C00u);
  return result;
}
static float from_bits(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}
// F16::to_f32 (f16.rs:86-115), software: exact for normal numbers, a denormal
// comes out at half its value (the reference's exponent for them is one low).
float f16_to_f32_soft(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int32_t exp = (h >> 10) & 0x1F;
  const uint32_t mant = h & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return from_bits(sign);
    int32_t e = -1;
    uint32_t m = mant;
    while ((m & 0x400u) == 0) {
      m <<= 1;
      e -= 1;
    }
    m &= 0x3FFu;
    return from_bits(sign | ((uint32_t)(127 + e - 14) << 23) | (m << 13));
  }
  if (exp == 0x1F) return from_bits(sign | 0x7F800000u | (mant << 13));
  return from_bits(sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13));
}
// _mm256_cvtph_ps: IEEE f16 -> f32, exact for every value.
float f16_to_f32_ieee(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int32_t exp = (h >> 10) & 0x1F;
  const uint32_t mant = h & 0x3FFu;
  if (exp == 0) return from_bits(sign) + (sign ? -1.0f : 1.0f) * std::ldexp((float)mant, -24);
  if (exp == 0x1F) return from_bits(sign | 0x7F800000u | (mant << 13));
  return from_bits(sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13));
}
// l2_f16_mixed_avx512 (f16.rs:213-262): 16 lane accumulators over chunks with
// hardware conversion, fma(d, d, acc); the tail element by element with the
// software conversion and a separate multiply and add; result = tail + tree.
float l2_f16_mixed_avx512_order(const float* q, const uint16_t* db, size_t n) {
  const size_t chunks = n / 16, rem = n % 16;
  float acc[16];
  for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 16; ++j) {
      const float d = q[c * 16 + j] - f16_to_f32_ieee(db[c * 16 + j]);
      acc[j] = std::fma(d, d, acc[j]);
    }
  float result = 0.0f;
  for (size_t i = 0; i < rem; ++i) {
    const float d = q[chunks * 16 + i] - f16_to_f32_soft(db[chunks * 16 + i]);
    result += d * d;  // built with -ffp-contract=off: a multiply then an add
  }
  return result + tree16(acc);
}

// src/distance/avx2.rs:26-54,86-98 — 8 lanes, horizontal_sum_ps
// ((hi+lo) 4 lanes, then movehdup/movehl adds), then a sequential fma tail.
float l2_avx2_order(const float* a, const float* b, size_t n) {
  size_t chunks = n / 8, rem = n % 8;
  float acc[8];
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  for (size_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      float d = a[c * 8 + j] - b[c * 8 + j];
      acc[j] = std::fma(d, d, acc[j]);
    }
  // _mm_add_ps(hi, lo): s[j] = acc[j+4] + acc[j]
  float s[4];
  for (int j = 0; j < 4; ++j) s[j] = acc[j + 4] + acc[j];
  // movehdup + add: sums = [s0+s1, ., s2+s3, .]; movehl(sum128, sums) puts
  // sums[2] in lane 0; add_ss: (s0+s1) + (s2+s3).
  float sums0 = s[0] + s[1], sums2 = s[2] + s[3];
  float result = sums0 + sums2;
  for (size_t i = 0; i < rem; ++i) {
    float d = a[chunks * 8 + i] - b[chunks * 8 + i];
    result = std::fma(d, d, result);
  }
  return result;
}

// ---------------------------------------------------------------------------
// SQ4 / SQ8 quantisers.
// ---------------------------------------------------------------------------
struct SQParams {
  uint32_t dim = 0;
  uint32_t levels = 15;  // 15 for SQ4 (16 levels), 255 for SQ8
  std::vector<float> min, max, scale, inv_scale, neg_min_div;
};

// src/quant/sq4.rs:46-77 (levels 15) and src/quant/sq8.rs:41-75 (levels 255):
// per-dimension min/max, max<=min -> min+1, scale=(max-min)/levels,
// inv=1/scale, neg=-min*inv.
SQParams sq_fit(const float* data, uint64_t n, uint32_t dim, uint32_t levels) {
  SQParams p;
  p.dim = dim;
  p.levels = levels;
  p.min.assign(dim, 3.40282347e+38f);
  p.max.assign(dim, -3.40282347e+38f);
  for (uint64_t i = 0; i < n; ++i) {
    const float* row = data + i * dim;
    for (uint32_t d = 0; d < dim; ++d) {
      if (row[d] < p.min[d]) p.min[d] = row[d];
      if (row[d] > p.max[d]) p.max[d] = row[d];
    }
  }
  for (uint32_t d = 0; d < dim; ++d)
    if (p.max[d] <= p.min[d]) p.max[d] = p.min[d] + 1.0f;
  p.scale.resize(dim);
  p.inv_scale.resize(dim);
  p.neg_min_div.resize(dim);
  for (uint32_t d = 0; d < dim; ++d) p.scale[d] = (p.max[d] - p.min[d]) / (float)levels;
  for (uint32_t d = 0; d < dim; ++d) p.inv_scale[d] = 1.0f / p.scale[d];
  for (uint32_t d = 0; d < dim; ++d) p.neg_min_div[d] = -p.min[d] * p.inv_scale[d];
  return p;
}

// Rust `f32::round` (half away from zero) then `clamp(0, L)` then `as u8`
// (saturating; NaN -> 0).
inline uint8_t quantize(float v, float inv, float neg, float levels) {
  float q = std::round(std::fma(v, inv, neg));
  if (std::isnan(q)) return 0;
  if (q < 0.0f) q = 0.0f;
  if (q > levels) q = levels;
  return (uint8_t)q;
}

// src/quant/sq4.rs:93-105 — even dim -> low nibble (byte overwritten),
// odd dim -> high nibble (or'ed).
void sq4_encode(const SQParams& p, const float* v, uint8_t* buf) {
  for (uint32_t d = 0; d < p.dim; ++d) {
    uint8_t code = quantize(v[d], p.inv_scale[d], p.neg_min_div[d], 15.0f);
    if (d % 2 == 0) buf[d / 2] = code;
    else buf[d / 2] |= (uint8_t)(code << 4);
  }
}
// src/quant/sq8.rs:89-97
void sq8_encode(const SQParams& p, const float* v, uint8_t* buf) {
  for (uint32_t d = 0; d < p.dim; ++d)
    buf[d] = quantize(v[d], p.inv_scale[d], p.neg_min_div[d], 255.0f);
}

// src/quant/sq4.rs:248-261 (scalar; the AVX2 kernel :168-221 is the same exact
// integer sum).
float l2_sq4_raw(const uint8_t* qa, const uint8_t* qb, size_t nbytes) {
  int32_t sum = 0;
  for (size_t i = 0; i < nbytes; ++i) {
    int32_t alo = qa[i] & 0x0F, ahi = (qa[i] >> 4) & 0x0F;
    int32_t blo = qb[i] & 0x0F, bhi = (qb[i] >> 4) & 0x0F;
    int32_t dlo = alo - blo, dhi = ahi - bhi;
    sum += dlo * dlo + dhi * dhi;
  }
  return (float)sum;
}
// src/quant/sq8.rs:267-307 (exact i32 sum).
float l2_sq8_raw(const uint8_t* qa, const uint8_t* qb, size_t n) {
  int64_t sum = 0;
  for (size_t i = 0; i < n; ++i) {
    int32_t d = (int32_t)qa[i] - (int32_t)qb[i];
    sum += d * d;
  }
  return (float)sum;
}

// ---------------------------------------------------------------------------
// VisitedTracker — src/memory/visited.rs:20-134 (byte array + ordered history).
// ---------------------------------------------------------------------------
struct Visited {
  std::vector<uint8_t> mark;
  std::vector<uint32_t> history;
  explicit Visited(size_t n = 0) : mark(n, 0) {}
  bool visit(uint32_t i) {  // :47-55
    if (mark[i]) return false;
    mark[i] = 1;
    history.push_back(i);
    return true;
  }
  void reset() {  // :115-120
    for (uint32_t i : history) mark[i] = 0;
    history.clear();
  }
};

// ---------------------------------------------------------------------------
// LinearPool — src/graph/linear_pool.rs:32-264, restated line for line.
// ---------------------------------------------------------------------------
constexpr uint32_t kChecked = 1u << 31;  // :47
struct LinearPool {
  std::vector<std::pair<uint32_t, float>> data;
  size_t size = 0, cursor = 0, capacity = 0, ef = 0;
  explicit LinearPool(size_t e = 0) : data(e + 1, {0, 0.0f}), capacity(e), ef(e) {}  // :63-71
  void clear() { size = 0; cursor = 0; }                                          // :75-78
  void reset_for(size_t e) {                                                      // :85-93
    if (e + 1 > data.size()) data.resize(e + 1, {0, 0.0f});
    capacity = e;
    ef = e;
    size = 0;
    cursor = 0;
  }
  size_t find_insert_pos(float dist) const {  // :252-263 (scan from the tail)
    long i = (long)size - 1;
    while (i >= 0) {
      if (data[(size_t)i].second <= dist) return (size_t)(i + 1);
      --i;
    }
    return 0;
  }
  bool insert(uint32_t node, float dist) {  // :100-143
    if (size == capacity) {
      if (capacity == 0) return false;  // reference underflows here; never reached with ef>=1
      if (dist >= data[size - 1].second) return false;
    }
    size_t lo = find_insert_pos(dist);
    size_t move = size - lo;
    if (move > 0) std::copy_backward(data.begin() + lo, data.begin() + lo + move, data.begin() + lo + move + 1);
    data[lo] = {node, dist};
    if (size < capacity) ++size;
    if (lo < cursor) cursor = lo;
    return true;
  }
  bool has_next() const { return cursor < size && cursor < ef; }  // :177-179
  bool pop(uint32_t* id, float* dist) {                           // :150-171
    if (!has_next()) return false;
    size_t idx = cursor;
    data[idx].first |= kChecked;
    ++cursor;
    while (cursor < size && (data[cursor].first & kChecked)) ++cursor;
    *id = data[idx].first & ~kChecked;
    *dist = data[idx].second;
    return true;
  }
  float worst_distance() const { return size == 0 ? 3.40282347e+38f : data[size - 1].second; }  // :198-205
};

// ---------------------------------------------------------------------------
// Loaded index (ANNX v1) — src/graph/vamana.rs:1326-1424,
// src/memory/graph.rs:347-399, src/graph/navigation.rs:712-769.
// ---------------------------------------------------------------------------
struct Nav {
  bool present = false;
  uint32_t entry = 0;
  uint8_t max_level = 0;
  uint32_t k = 0;
  std::vector<uint8_t> node_levels;
  std::vector<std::vector<uint32_t>> upper;
  std::vector<uint32_t> entry_candidates;
};

struct Index {
  uint64_t n = 0, dim = 0, r_max = 0;
  uint32_t entry = 0;
  uint32_t flags = 0;
  std::vector<uint32_t> main_block;
  std::vector<uint16_t> degrees;
  std::vector<std::vector<uint32_t>> overflow;
  Nav nav;
  // searcher-side data (set by oracle_index_set_vectors)
  std::vector<float> vectors;
  SQParams sq4, sq8;
  std::vector<uint8_t> sq4_codes, sq8_codes;
  size_t sq4_bytes = 0;
  std::vector<uint16_t> f16;  // F16Dataset::build (src/distance/f16.rs:344-349), for with_f16
  // AdaptiveEf samples (sorted) — src/graph/adaptive_ef.rs:307-327
  std::vector<float> adaptive_samples;
};

// src/graph/navigation.rs:712-769 (returns false for None).
bool nav_deserialize(const uint8_t* buf, size_t len, Nav* nav) {
  if (len < 16) return false;
  nav->entry = rd<uint32_t>(buf);
  nav->max_level = buf[4];
  nav->k = rd<uint32_t>(buf + 8);
  uint32_t n = rd<uint32_t>(buf + 12);
  if (len < 16 + (size_t)n) return false;
  nav->node_levels.assign(buf + 16, buf + 16 + n);
  size_t off = 16 + n;
  if (len < off + 4) return false;
  uint32_t count = rd<uint32_t>(buf + off);
  off += 4;
  nav->upper.assign(n, {});
  for (uint32_t c = 0; c < count; ++c) {
    if (len < off + 8) return false;
    uint32_t node = rd<uint32_t>(buf + off);
    uint32_t ll = rd<uint32_t>(buf + off + 4);
    off += 8;
    if (len < off + (size_t)ll * 4 || node >= n) return false;
    nav->upper[node].resize(ll);
    if (ll) std::memcpy(nav->upper[node].data(), buf + off, (size_t)ll * 4);
    off += (size_t)ll * 4;
  }
  if (len >= off + 4) {
    uint32_t ec = rd<uint32_t>(buf + off);
    off += 4;
    if (len >= off + (size_t)ec * 4) {
      nav->entry_candidates.resize(ec);
      if (ec) std::memcpy(nav->entry_candidates.data(), buf + off, (size_t)ec * 4);
    } else {
      nav->entry_candidates = {nav->entry};
    }
  } else {
    nav->entry_candidates = {nav->entry};
  }
  nav->present = true;
  return true;
}

int load_index(const uint8_t* bytes, size_t len, Index* ix) {
  if (len < kHeaderSize + 20) { g_err = "file too short for VamanaGraph header"; return -2; }
  uint32_t magic = rd<uint32_t>(bytes), version = rd<uint32_t>(bytes + 4);
  uint32_t flags = rd<uint32_t>(bytes + 8), crc = rd<uint32_t>(bytes + 12);
  if (magic != kIndexMagic) { g_err = "magic mismatch"; return -3; }       // serialize.rs:112-117
  if (version != kIndexVersion) { g_err = "version mismatch"; return -4; } // serialize.rs:118-123
  const uint8_t* body = bytes + kHeaderSize;
  size_t blen = len - kHeaderSize;
  if (crc32_bytes(body, blen) != crc) { g_err = "crc32 mismatch"; return -5; }  // vamana.rs:1343-1350
  ix->flags = flags;
  ix->n = rd<uint64_t>(body);
  ix->dim = rd<uint64_t>(body + 8);
  ix->entry = rd<uint32_t>(body + 16);
  size_t off = 20;
  if (flags & kFlagHasMetadata) {  // vamana.rs:1360-1385
    if (blen < off + 4) { g_err = "body too short for metadata trailer header"; return -2; }
    uint32_t ml = rd<uint32_t>(body + off);
    off += 4;
    if (blen < off + ml) { g_err = "body too short for metadata trailer"; return -2; }
    off += ml + (4 - ml % 4) % 4;
  }
  if (flags & kFlagHasLayeredNav) {  // vamana.rs:1388-1410
    if (blen < off + 4) { g_err = "body too short for layered nav trailer header"; return -2; }
    uint32_t nl = rd<uint32_t>(body + off);
    off += 4;
    if (blen < off + nl) { g_err = "body too short for layered nav trailer"; return -2; }
    Nav nav;
    if (nav_deserialize(body + off, nl, &nav)) ix->nav = std::move(nav);
    off += nl + (4 - nl % 4) % 4;
  }
  // HybridBlockedCsr::deserialize — graph.rs:347-399
  if (off > blen || blen - off < 24) { g_err = "HybridBlockedCsr body too short"; return -2; }
  const uint8_t* c = body + off;
  size_t clen = blen - off;
  uint64_t n = rd<uint64_t>(c), r_max = rd<uint64_t>(c + 8), mb_len = rd<uint64_t>(c + 16);
  if (mb_len > (clen - 24) / 4 || clen < 24 + mb_len * 4 + 8) { g_err = "main_block truncated"; return -2; }
  if (r_max == 0 || mb_len != n * r_max) { g_err = "main_block size mismatch"; return -6; }
  ix->r_max = r_max;
  ix->main_block.resize(mb_len);
  std::memcpy(ix->main_block.data(), c + 24, mb_len * 4);
  size_t o = 24 + mb_len * 4;
  uint64_t ov = rd<uint64_t>(c + o);
  o += 8;
  ix->overflow.assign(n, {});
  for (uint64_t i = 0; i < ov; ++i) {
    if (o + 12 > clen) { g_err = "overflow entry header truncated"; return -2; }
    uint32_t node = rd<uint32_t>(c + o);
    uint64_t vl = rd<uint64_t>(c + o + 4);
    o += 12;
    if (vl > (clen - o) / 4) { g_err = "overflow entry data truncated"; return -2; }
    if (node < n) {
      ix->overflow[node].resize(vl);
      if (vl) std::memcpy(ix->overflow[node].data(), c + o, vl * 4);
    }
    o += vl * 4;
  }
  // from_parts degree rule — graph.rs:234-240
  ix->degrees.resize(n);
  for (uint64_t i = 0; i < n; ++i) {
    const uint32_t* row = ix->main_block.data() + i * r_max;
    uint64_t d = 0;
    while (d < r_max && row[d] != kSentinel) ++d;
    ix->degrees[i] = (uint16_t)d;
  }
  if (n != ix->n) { g_err = "n mismatch"; return -6; }  // vamana.rs:1416-1421
  return 0;
}

// ---------------------------------------------------------------------------
// LayeredNavigation::initialize — src/graph/navigation.rs:609-653.
// Returns (entry, f32 distance); counts distance evaluations.
// ---------------------------------------------------------------------------
std::pair<uint32_t, float> nav_initialize(const Index& ix, const float* q, uint32_t* n_evals) {
  const size_t dim = ix.dim;
  const float* V = ix.vectors.data();
  const Nav& nv = ix.nav;
  uint32_t evals = 0;
  if (nv.max_level == 0) {
    ++evals;
    if (n_evals) *n_evals = evals;
    return {nv.entry, l2_avx512_order(q, V + (size_t)nv.entry * dim, dim)};
  }
  uint32_t u = nv.entry;
  float cur = l2_avx512_order(q, V + (size_t)u * dim, dim);
  ++evals;
  for (int level = nv.max_level; level >= 1; --level) {
    bool changed = true;
    while (changed) {
      changed = false;
      const std::vector<uint32_t>& edges = nv.upper[u];
      size_t start = (size_t)(level - 1) * nv.k;
      if (start >= edges.size()) break;
      size_t end = std::min(start + (size_t)nv.k, edges.size());
      for (size_t e = start; e < end; ++e) {
        uint32_t v = edges[e];
        if (v == u) continue;
        float d = l2_avx512_order(q, V + (size_t)v * dim, dim);
        ++evals;
        if (d < cur) {
          cur = d;
          u = v;
          changed = true;
        }
      }
    }
  }
  if (n_evals) *n_evals = evals;
  return {u, cur};
}

// AdaptiveEfConfig::estimate_ef — src/graph/adaptive_ef.rs:340-359
// (default build: libm powf, no fast_powf).
size_t estimate_ef(const std::vector<float>& s, size_t min_ef, size_t max_ef, float gamma, float distance) {
  if (s.size() <= 1) return min_ef + (max_ef - min_ef) / 2;  // usize::midpoint
  size_t rank = (size_t)(std::lower_bound(s.begin(), s.end(), distance,
                                          [](float a, float d) { return a < d; }) - s.begin());
  float pct = (float)rank / (float)s.size();
  float shaped = powf(pct, gamma);
  float ef = std::fma(shaped, (float)(max_ef - min_ef), (float)min_ef);
  float r = std::round(ef);
  if (!(r > 0.0f)) return 0;  // `as usize` saturates (NaN -> 0)
  return (size_t)r;
}

// ---------------------------------------------------------------------------
// greedy_search_sq4 / greedy_search_sq8::<true> — src/graph/vamana.rs:786-861
// and :683-773, with the reference's software prefetches (no effect on
// results; kept so that the timed CPU baseline has the reference's memory
// behaviour): the next unexpanded node's adjacency lines after each pop
// (:808-819), the codes of the first `po` new neighbours (:834-842), and the
// code `po` ahead of each distance (:846-853). `code_lines` code lines are
// prefetched per neighbour (SQ4 1, SQ8 2), all with the NTA hint
// (`_mm_prefetch::<0>`).
// ---------------------------------------------------------------------------
struct SearchStats {
  uint32_t expansions = 0;
};
template <class DistFn, class CodeFn>
std::vector<std::pair<uint32_t, float>> greedy_search_q(const Index& ix, uint32_t entry, size_t l,
                                                        Visited& visited, LinearPool& pool,
                                                        DistFn dist, CodeFn code_ptr, int code_lines, size_t po,
                                                        SearchStats* st) {
  auto prefetch_code = [&](uint32_t v) {
    const char* c = (const char*)code_ptr(v);
    for (int li = 0; li < code_lines; ++li) _mm_prefetch(c + 64 * li, _MM_HINT_NTA);
  };
  const size_t graph_lines = ((size_t)ix.r_max * 4 + 63) / 64;
  visited.reset();
  pool.reset_for(l);
  float ed = dist(entry);
  visited.visit(entry);
  pool.insert(entry, ed);
  uint32_t edge_buf[128];
  uint32_t node;
  float nd;
  while (pool.pop(&node, &nd)) {
    if (st) st->expansions++;
    if (pool.has_next()) {  // peek_unchecked
      const uint32_t next = pool.data[pool.cursor].first & ~kChecked;
      const char* g = (const char*)(ix.main_block.data() + (size_t)next * ix.r_max);
      for (size_t li = 0; li < graph_lines; ++li) _mm_prefetch(g + 64 * li, _MM_HINT_NTA);
    }
    const uint32_t* nb = ix.main_block.data() + (size_t)node * ix.r_max;
    size_t deg = ix.degrees[node];
    size_t edge_size = 0;
    for (size_t i = 0; i < deg; ++i) {  // :824-832
      if (edge_size >= 128) break;
      uint32_t v = nb[i];
      bool is_new = visited.visit(v);
      edge_buf[edge_size] = v;
      edge_size += is_new ? 1 : 0;
    }
    for (size_t i = 0; i < std::min(po, edge_size); ++i) prefetch_code(edge_buf[i]);
    for (size_t i = 0; i < edge_size; ++i) {  // :846-857
      if (i + po < edge_size) prefetch_code(edge_buf[i + po]);
      pool.insert(edge_buf[i], dist(edge_buf[i]));
    }
  }
  std::vector<std::pair<uint32_t, float>> out(pool.size);
  for (size_t i = 0; i < pool.size; ++i) out[i] = {pool.data[i].first & ~kChecked, pool.data[i].second};
  return out;
}

// f32 total order key (Rust f32::total_cmp).
inline int32_t total_key(float f) {
  int32_t b;
  std::memcpy(&b, &f, 4);
  return b ^ (int32_t)(((uint32_t)(b >> 31)) >> 1);
}

// rerank_f32 — src/graph/refiner.rs:45-61,110-119. The reference sorts with
// sort_unstable_by(total_cmp), whose order among equal distances is
// unspecified; this restatement (and the CUDA engine) breaks ties by the
// candidate's position in the SQ search result (stable by pool order).
// With `f16` set: rerank_f16 / F16Refiner::rerank (src/graph/refiner.rs:87-104,
// 132-end), the same rule with l2_f16_mixed_simd on the f16 vectors.
std::vector<std::pair<uint32_t, float>> rerank_f32(const Index& ix, const float* q,
                                                   const std::vector<std::pair<uint32_t, float>>& cands,
                                                   size_t k, size_t rr, bool f16 = false) {
  size_t rerank_n = std::min(std::max(k * rr, k), cands.size());
  std::vector<std::pair<uint32_t, float>> res(rerank_n);
  for (size_t i = 0; i < rerank_n; ++i) {
    uint32_t id = cands[i].first;
    res[i] = {id, f16 ? l2_f16_mixed_avx512_order(q, ix.f16.data() + (size_t)id * ix.dim, ix.dim)
                      : l2_avx512_order(q, ix.vectors.data() + (size_t)id * ix.dim, ix.dim)};
  }
  std::stable_sort(res.begin(), res.end(), [](const std::pair<uint32_t, float>& a,
                                              const std::pair<uint32_t, float>& b) {
    return total_key(a.second) < total_key(b.second);
  });
  if (res.size() > k) res.resize(k);
  return res;
}

struct OracleParams {
  uint32_t ef;
  uint32_t k;
  uint32_t rerank_factor;
  uint32_t quant;  // 0 = SQ4, 1 = SQ8, 2 = f32 traversal (GraphSearcher::search)
  uint32_t adaptive;
  float gamma;
  uint32_t min_ef, max_ef;
  uint32_t rerank_f16;  // 1: GraphSearcher::with_f16 (src/graph/vamana.rs:1559, 1824-1828)
  uint32_t prefetch_offset;  // with_prefetch_offset (:1541); GraphSearcher::new sets 16 (:1490)
};

struct QueryOut {
  std::vector<std::pair<uint32_t, float>> results;
  uint32_t visited = 0, ef_used = 0, n_nav = 0, expansions = 0;
  std::vector<uint32_t> history;
};

// GraphSearcher::search_sq4 / search_sq8 — src/graph/vamana.rs:1772-1829 and
// :1752 -> :1700-1750 (entry via layered nav when present, else the medoid),
// adaptive ef .max(k) (:1803), rerank.
struct Worker {
  Visited visited;
  LinearPool pool;
  std::vector<uint8_t> code;
};

// GraphSearcher::search (the f32 traversal) — src/graph/vamana.rs:1627-1672:
// the same entry and adaptive ef, greedy_search_vec_reuse (:588-666: the
// loop above with l2_simd distances and one prefetched line per vector), then
// the pool sorted by total_cmp and truncated to k (the pool is already in
// ascending order; equal distances keep pool order, the tie rule used
// throughout).
int search_one(const Index& ix, const float* q, const OracleParams& p, Worker& w, QueryOut* out,
               bool want_history) {
  const size_t dim = ix.dim;
  if (p.quant == 2) {
    // no query code
  } else if (p.quant == 0) {
    w.code.assign(ix.sq4_bytes, 0);
    sq4_encode(ix.sq4, q, w.code.data());
  } else {
    w.code.assign(dim, 0);
    sq8_encode(ix.sq8, q, w.code.data());
  }
  uint32_t entry;
  float nav_dist;
  bool have_nav_dist = false;
  uint32_t n_nav = 0;
  if (ix.nav.present) {
    auto r = nav_initialize(ix, q, &n_nav);
    entry = r.first;
    nav_dist = r.second;
    have_nav_dist = true;
  } else {
    entry = ix.entry;
  }
  size_t ef = p.ef;
  if (p.adaptive) {
    float d = have_nav_dist ? nav_dist : l2_avx512_order(q, ix.vectors.data() + (size_t)entry * dim, dim);
    if (!have_nav_dist) n_nav++;
    ef = std::max(estimate_ef(ix.adaptive_samples, p.min_ef, p.max_ef, p.gamma, d), (size_t)p.k);
  }
  if (ef == 0) { g_err = "ef must be >= 1"; return -7; }
  SearchStats st;
  std::vector<std::pair<uint32_t, float>> cands;
  const uint8_t* qc = w.code.data();
  if (p.quant == 2) {
    cands = greedy_search_q(
        ix, entry, ef, w.visited, w.pool,
        [&](uint32_t id) { return l2_avx512_order(q, ix.vectors.data() + (size_t)id * dim, dim); },
        [&](uint32_t id) { return (const uint8_t*)(ix.vectors.data() + (size_t)id * dim); }, 1, p.prefetch_offset,
        &st);
  } else if (p.quant == 0) {
    const size_t cb = ix.sq4_bytes;
    cands = greedy_search_q(
        ix, entry, ef, w.visited, w.pool,
        [&](uint32_t id) { return l2_sq4_raw(qc, ix.sq4_codes.data() + (size_t)id * cb, cb); },
        [&](uint32_t id) { return ix.sq4_codes.data() + (size_t)id * cb; }, 1, p.prefetch_offset, &st);
  } else {
    cands = greedy_search_q(
        ix, entry, ef, w.visited, w.pool,
        [&](uint32_t id) { return l2_sq8_raw(qc, ix.sq8_codes.data() + (size_t)id * dim, dim); },
        [&](uint32_t id) { return ix.sq8_codes.data() + (size_t)id * dim; }, 2, p.prefetch_offset, &st);
  }
  out->visited = (uint32_t)w.visited.history.size();
  out->ef_used = (uint32_t)ef;
  out->n_nav = n_nav;
  out->expansions = st.expansions;
  if (want_history) out->history = w.visited.history;
  if (p.quant == 2) {
    if (cands.size() > p.k) cands.resize(p.k);
    out->results = cands;
    return 0;
  }
  size_t rr = std::max<uint32_t>(p.rerank_factor, 1);  // with_rerank_factor clamps >= 1 (:1547-1550)
  out->results = rerank_f32(ix, q, cands, p.k, rr, p.rerank_f16 != 0);
  return 0;
}

}  // namespace

// ===========================================================================
// C interface for ctypes (tests / smoke / bench cpu_baseline only).
// ===========================================================================
extern "C" {

const char* oracle_last_error() { return g_err.c_str(); }

uint32_t oracle_crc32(const uint8_t* p, size_t n) { return crc32_bytes(p, n); }

float oracle_l2_avx512(const float* a, const float* b, size_t n) { return l2_avx512_order(a, b, n); }
float oracle_l2_avx2(const float* a, const float* b, size_t n) { return l2_avx2_order(a, b, n); }
float oracle_l2_sq4_raw(const uint8_t* a, const uint8_t* b, size_t nbytes) { return l2_sq4_raw(a, b, nbytes); }
float oracle_l2_sq8_raw(const uint8_t* a, const uint8_t* b, size_t n) { return l2_sq8_raw(a, b, n); }

// Fit + encode a dataset. levels: 15 (SQ4) or 255 (SQ8). out_params: 5*dim
// floats (min, max, scale, inv_scale, neg_min_div). codes: n*code_bytes.
void oracle_sq_fit(const float* data, uint64_t n, uint32_t dim, uint32_t levels, float* out_params) {
  SQParams p = sq_fit(data, n, dim, levels);
  for (uint32_t d = 0; d < dim; ++d) {
    out_params[d] = p.min[d];
    out_params[dim + d] = p.max[d];
    out_params[2 * dim + d] = p.scale[d];
    out_params[3 * dim + d] = p.inv_scale[d];
    out_params[4 * dim + d] = p.neg_min_div[d];
  }
}
static SQParams params_from(const float* pp, uint32_t dim, uint32_t levels) {
  SQParams p;
  p.dim = dim;
  p.levels = levels;
  p.min.assign(pp, pp + dim);
  p.max.assign(pp + dim, pp + 2 * dim);
  p.scale.assign(pp + 2 * dim, pp + 3 * dim);
  p.inv_scale.assign(pp + 3 * dim, pp + 4 * dim);
  p.neg_min_div.assign(pp + 4 * dim, pp + 5 * dim);
  return p;
}
void oracle_sq4_encode(const float* params, uint32_t dim, const float* v, uint64_t n, uint8_t* codes) {
  SQParams p = params_from(params, dim, 15);
  size_t cb = (dim + 1) / 2;
  for (uint64_t i = 0; i < n; ++i) {
    std::memset(codes + i * cb, 0, cb);
    sq4_encode(p, v + i * dim, codes + i * cb);
  }
}
void oracle_sq8_encode(const float* params, uint32_t dim, const float* v, uint64_t n, uint8_t* codes) {
  SQParams p = params_from(params, dim, 255);
  for (uint64_t i = 0; i < n; ++i) sq8_encode(p, v + i * dim, codes + i * dim);
}

// LinearPool handle API (for the ported linear_pool.rs unit tests).
void* oracle_pool_new(size_t ef) { return new LinearPool(ef); }
void oracle_pool_free(void* h) { delete (LinearPool*)h; }
int oracle_pool_insert(void* h, uint32_t node, float d) { return ((LinearPool*)h)->insert(node, d) ? 1 : 0; }
int oracle_pool_pop(void* h, uint32_t* id, float* d) { return ((LinearPool*)h)->pop(id, d) ? 1 : 0; }
int oracle_pool_has_next(void* h) { return ((LinearPool*)h)->has_next() ? 1 : 0; }
size_t oracle_pool_len(void* h) { return ((LinearPool*)h)->size; }
size_t oracle_pool_cursor(void* h) { return ((LinearPool*)h)->cursor; }
float oracle_pool_worst(void* h) { return ((LinearPool*)h)->worst_distance(); }
void oracle_pool_clear(void* h) { ((LinearPool*)h)->clear(); }
void oracle_pool_reset_for(void* h, size_t ef) { ((LinearPool*)h)->reset_for(ef); }
size_t oracle_pool_sorted(void* h, uint32_t* ids, float* ds) {
  LinearPool* p = (LinearPool*)h;
  for (size_t i = 0; i < p->size; ++i) {
    ids[i] = p->data[i].first & ~kChecked;
    ds[i] = p->data[i].second;
  }
  return p->size;
}

// AdaptiveEf estimate on an explicit sorted sample array.
size_t oracle_estimate_ef(const float* sorted, size_t n, size_t min_ef, size_t max_ef, float gamma, float d) {
  std::vector<float> s(sorted, sorted + n);
  return estimate_ef(s, min_ef, max_ef, gamma, d);
}

// Index handle.
void* oracle_index_load(const char* path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) { g_err = std::string("cannot open ") + path; return nullptr; }
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  Index* ix = new Index();
  if (load_index(bytes.data(), bytes.size(), ix) != 0) { delete ix; return nullptr; }
  return ix;
}
void* oracle_index_from_bytes(const uint8_t* bytes, size_t len, int* status) {
  Index* ix = new Index();
  int rc = load_index(bytes, len, ix);
  if (status) *status = rc;
  if (rc != 0) { delete ix; return nullptr; }
  return ix;
}
void oracle_index_free(void* h) { delete (Index*)h; }
void oracle_index_info(void* h, uint64_t* out /*n, dim, r_max, entry, nav_present, nav_max_level, nav_k, flags*/) {
  Index* ix = (Index*)h;
  out[0] = ix->n;
  out[1] = ix->dim;
  out[2] = ix->r_max;
  out[3] = ix->entry;
  out[4] = ix->nav.present;
  out[5] = ix->nav.max_level;
  out[6] = ix->nav.k;
  out[7] = ix->flags;
}
const uint32_t* oracle_index_main_block(void* h) { return ((Index*)h)->main_block.data(); }
uint32_t oracle_index_degree(void* h, uint32_t node) { return ((Index*)h)->degrees[node]; }
size_t oracle_index_nav_list(void* h, uint32_t node, const uint32_t** out) {
  Index* ix = (Index*)h;
  if (!ix->nav.present || node >= ix->nav.upper.size()) { *out = nullptr; return 0; }
  *out = ix->nav.upper[node].data();
  return ix->nav.upper[node].size();
}
uint32_t oracle_index_nav_level(void* h, uint32_t node) {
  Index* ix = (Index*)h;
  if (!ix->nav.present || node >= ix->nav.node_levels.size()) return 0;
  return ix->nav.node_levels[node];
}
size_t oracle_index_nav_candidates(void* h, const uint32_t** out) {
  Index* ix = (Index*)h;
  *out = ix->nav.entry_candidates.data();
  return ix->nav.entry_candidates.size();
}

// Searcher creation — src/python.rs:134-163: SQ4Dataset/SQ8Dataset::build and
// (optionally) AdaptiveEfConfig::build_with_layered_nav samples
// (src/graph/adaptive_ef.rs:307-327: nav.initialize of base vectors
// 0..min(n,2000), sorted ascending).
int oracle_index_set_vectors(void* h, const float* vectors, uint64_t n, uint32_t dim, int build_sq4,
                             int build_sq8, int build_adaptive) {
  Index* ix = (Index*)h;
  if (n != ix->n || dim != ix->dim) { g_err = "vectors shape mismatch"; return -6; }
  ix->vectors.assign(vectors, vectors + n * dim);
  if (build_sq4) {
    ix->sq4 = sq_fit(vectors, n, dim, 15);
    ix->sq4_bytes = (dim + 1) / 2;
    ix->sq4_codes.assign(n * ix->sq4_bytes, 0);
    for (uint64_t i = 0; i < n; ++i) sq4_encode(ix->sq4, vectors + i * dim, ix->sq4_codes.data() + i * ix->sq4_bytes);
  }
  if (build_sq8) {
    ix->sq8 = sq_fit(vectors, n, dim, 255);
    ix->sq8_codes.assign(n * dim, 0);
    for (uint64_t i = 0; i < n; ++i) sq8_encode(ix->sq8, vectors + i * dim, ix->sq8_codes.data() + i * dim);
  }
  if (build_adaptive) {
    if (!ix->nav.present) { g_err = "AdaptiveEf requires layered nav"; return -8; }
    size_t s = std::min<uint64_t>(n, 2000);
    ix->adaptive_samples.resize(s);
    for (size_t i = 0; i < s; ++i) ix->adaptive_samples[i] = nav_initialize(*ix, vectors + i * dim, nullptr).second;
    // sort_by(partial_cmp) — distances are never NaN for finite inputs.
    std::sort(ix->adaptive_samples.begin(), ix->adaptive_samples.end());
  }
  return 0;
}
// F16Dataset::build for with_f16 reranks.
int oracle_index_build_f16(void* h) {
  Index* ix = (Index*)h;
  if (ix->vectors.empty()) { g_err = "set_vectors first"; return -7; }
  ix->f16.resize(ix->vectors.size());
  for (size_t i = 0; i < ix->vectors.size(); ++i) ix->f16[i] = f16_from_f32(ix->vectors[i]);
  return 0;
}
uint16_t oracle_f16_from_f32(float f) { return f16_from_f32(f); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32_soft(h); }
float oracle_l2_f16_mixed(const float* q, const uint16_t* db, size_t n) { return l2_f16_mixed_avx512_order(q, db, n); }
size_t oracle_index_adaptive_samples(void* h, const float** out) {
  Index* ix = (Index*)h;
  *out = ix->adaptive_samples.data();
  return ix->adaptive_samples.size();
}
const uint8_t* oracle_index_sq4_codes(void* h) { return ((Index*)h)->sq4_codes.data(); }
const uint8_t* oracle_index_sq8_codes(void* h) { return ((Index*)h)->sq8_codes.data(); }
void oracle_index_sq_params(void* h, int quant, float* out5dim) {
  Index* ix = (Index*)h;
  const SQParams& p = quant == 0 ? ix->sq4 : ix->sq8;
  uint32_t dim = (uint32_t)ix->dim;
  for (uint32_t d = 0; d < dim; ++d) {
    out5dim[d] = p.min[d];
    out5dim[dim + d] = p.max[d];
    out5dim[2 * dim + d] = p.scale[d];
    out5dim[3 * dim + d] = p.inv_scale[d];
    out5dim[4 * dim + d] = p.neg_min_div[d];
  }
}

// Nav initialize for an arbitrary query (entry, dist, evals).
void oracle_nav_initialize(void* h, const float* q, uint32_t* entry, float* dist, uint32_t* evals) {
  auto r = nav_initialize(*(Index*)h, q, evals);
  *entry = r.first;
  *dist = r.second;
}

// Batch search — GraphSearcher::batch_search (src/graph/vamana.rs:1983-2095):
// per-query independent work; `threads` workers each with their own
// VisitedTracker / LinearPool. Outputs: ids/dists nq*k (unfilled: id 0,
// dist 0), counts, visited, ef_used, n_nav, expansions; history optional
// (nq*hist_cap, with hist_len per query, truncated at hist_cap).
int oracle_search_batch(void* h, const float* queries, uint64_t nq, const OracleParams* p, int threads,
                        uint32_t* ids, float* dists, uint32_t* counts, uint32_t* visited, uint32_t* ef_used,
                        uint32_t* n_nav, uint32_t* expansions, uint32_t* history, uint32_t hist_cap,
                        uint32_t* hist_len) {
  Index* ix = (Index*)h;
  if (ix->vectors.empty()) { g_err = "vectors not set"; return -8; }
  if (p->quant == 0 && ix->sq4_codes.empty()) { g_err = "sq4 not built"; return -8; }
  if (p->quant == 1 && ix->sq8_codes.empty()) { g_err = "sq8 not built"; return -8; }
  if (p->rerank_f16 && ix->f16.empty()) { g_err = "f16 vectors not built"; return -8; }
  if (threads <= 0) threads = (int)std::thread::hardware_concurrency();
  if (threads <= 0) threads = 1;
  std::atomic<uint64_t> next(0);
  std::atomic<int> rc(0);
  auto work = [&]() {
    Worker w;
    size_t cap = p->adaptive ? std::max(p->max_ef, p->k) : p->ef;
    w.visited = Visited(ix->n);
    w.pool = LinearPool(cap);
    QueryOut out;
    while (true) {
      uint64_t i = next.fetch_add(1);
      if (i >= nq) break;
      int r = search_one(*ix, queries + i * ix->dim, *p, w, &out, history != nullptr);
      if (r != 0) { rc = r; continue; }
      uint32_t k = p->k;
      for (uint32_t j = 0; j < k; ++j) {
        ids[i * k + j] = j < out.results.size() ? out.results[j].first : 0;
        dists[i * k + j] = j < out.results.size() ? out.results[j].second : 0.0f;
      }
      if (counts) counts[i] = (uint32_t)out.results.size();
      if (visited) visited[i] = out.visited;
      if (ef_used) ef_used[i] = out.ef_used;
      if (n_nav) n_nav[i] = out.n_nav;
      if (expansions) expansions[i] = out.expansions;
      if (history) {
        uint32_t hl = (uint32_t)std::min<size_t>(out.history.size(), hist_cap);
        std::memcpy(history + i * hist_cap, out.history.data(), (size_t)hl * 4);
        hist_len[i] = (uint32_t)out.history.size();
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
  return rc.load();
}

// Exact brute-force top-k (ground truth for small cases): squared L2 in the
// AVX-512 order, ties broken by id.
void oracle_bruteforce(const float* base, uint64_t n, const float* queries, uint64_t nq, uint32_t dim,
                       uint32_t k, int threads, uint32_t* out_ids, float* out_d) {
  if (threads <= 0) threads = (int)std::thread::hardware_concurrency();
  std::atomic<uint64_t> next(0);
  auto work = [&]() {
    std::vector<std::pair<float, uint32_t>> best;
    while (true) {
      uint64_t qi = next.fetch_add(1);
      if (qi >= nq) break;
      best.clear();
      const float* q = queries + qi * dim;
      for (uint64_t i = 0; i < n; ++i) {
        float d = l2_avx512_order(q, base + i * dim, dim);
        std::pair<float, uint32_t> c{d, (uint32_t)i};
        if (best.size() < k) {
          best.push_back(c);
          std::push_heap(best.begin(), best.end());
        } else if (c < best.front()) {
          std::pop_heap(best.begin(), best.end());
          best.back() = c;
          std::push_heap(best.begin(), best.end());
        }
      }
      std::sort(best.begin(), best.end());
      for (uint32_t j = 0; j < k; ++j) {
        out_ids[qi * k + j] = j < best.size() ? best[j].second : 0;
        out_d[qi * k + j] = j < best.size() ? best[j].first : 0.0f;
      }
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
}

}  // extern "C"
