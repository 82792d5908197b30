// ANNX v1 reader/writer and the CPU Vamana build (host side of the engine).
//
// The build restates RAVEN's offline pipeline (src/graph/vamana.rs:106-201,
// src/graph/robust_prune.rs, src/graph/navigation.rs:244-595) so that an index
// file can exist without a Rust toolchain. Its random stream is this file's own
// xoshiro256** (the reference draws from rand_chacha's ChaCha8), so graphs are
// not bit-identical to a Rust build; search parity is defined on a shared file.
// The per-batch edge-connection step runs in parallel grouped by target node,
// which applies the same operations in the same order per node as the
// reference's sequential loop (vamana.rs:171-175), so the result is
// deterministic and independent of the thread count.
#include "host_index.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <unordered_set>

namespace raven {

// ---------------------------------------------------------------------------
// CRC-32/IEEE, slice-by-8 (same function as crc32fast: reflected 0xEDB88320).
// ---------------------------------------------------------------------------
static uint32_t g_crc[8][256];
static bool g_crc_init = false;
static void crc_init() {
  for (uint32_t i = 0; i < 256; ++i) {
    uint32_t c = i;
    for (int b = 0; b < 8; ++b) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
    g_crc[0][i] = c;
  }
  for (uint32_t i = 0; i < 256; ++i)
    for (int t = 1; t < 8; ++t) g_crc[t][i] = (g_crc[t - 1][i] >> 8) ^ g_crc[0][g_crc[t - 1][i] & 0xFF];
  g_crc_init = true;
}
uint32_t crc32_ieee(const uint8_t* p, size_t n, uint32_t crc) {
  if (!g_crc_init) crc_init();
  uint32_t c = ~crc;
  while (n >= 8) {
    uint32_t lo, hi;
    std::memcpy(&lo, p, 4);
    std::memcpy(&hi, p + 4, 4);
    lo ^= c;
    c = g_crc[7][lo & 0xFF] ^ g_crc[6][(lo >> 8) & 0xFF] ^ g_crc[5][(lo >> 16) & 0xFF] ^ g_crc[4][lo >> 24] ^
        g_crc[3][hi & 0xFF] ^ g_crc[2][(hi >> 8) & 0xFF] ^ g_crc[1][(hi >> 16) & 0xFF] ^ g_crc[0][hi >> 24];
    p += 8;
    n -= 8;
  }
  while (n--) c = g_crc[0][(c ^ *p++) & 0xFF] ^ (c >> 8);
  return ~c;
}

template <class T>
static T rd(const uint8_t* p) {
  T v;
  std::memcpy(&v, p, sizeof(T));
  return v;
}
template <class T>
static void wr(std::vector<uint8_t>& b, T v) {
  size_t o = b.size();
  b.resize(o + sizeof(T));
  std::memcpy(b.data() + o, &v, sizeof(T));
}

// ---------------------------------------------------------------------------
// Reader: VamanaGraph::deserialize (src/graph/vamana.rs:1326-1424),
// LayeredNavigation::deserialize_binary (src/graph/navigation.rs:712-769),
// HybridBlockedCsr::deserialize (src/memory/graph.rs:347-399).
// Error codes match include/raven_gpu.h.
// ---------------------------------------------------------------------------
static bool parse_nav(const uint8_t* buf, size_t len, LayeredNav* nav) {
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
    uint32_t node = rd<uint32_t>(buf + off), ll = rd<uint32_t>(buf + off + 4);
    off += 8;
    if (len < off + (size_t)ll * 4 || node >= n) return false;
    nav->upper[node].resize(ll);
    if (ll) std::memcpy(nav->upper[node].data(), buf + off, (size_t)ll * 4);
    off += (size_t)ll * 4;
  }
  nav->entry_candidates.clear();
  if (len >= off + 4) {
    uint32_t ec = rd<uint32_t>(buf + off);
    off += 4;
    if (len >= off + (size_t)ec * 4) {
      nav->entry_candidates.resize(ec);
      if (ec) std::memcpy(nav->entry_candidates.data(), buf + off, (size_t)ec * 4);
    } else {
      nav->entry_candidates.push_back(nav->entry);
    }
  } else {
    nav->entry_candidates.push_back(nav->entry);
  }
  nav->present = true;
  return true;
}

int parse_annx(const uint8_t* bytes, size_t len, HostGraph* g, std::string* err) {
  auto fail = [&](int code, const char* msg) {
    if (err) *err = msg;
    return code;
  };
  if (len < 16 + 20) return fail(-6, "file too short for VamanaGraph header");
  uint32_t magic = rd<uint32_t>(bytes), version = rd<uint32_t>(bytes + 4);
  uint32_t flags = rd<uint32_t>(bytes + 8), crc = rd<uint32_t>(bytes + 12);
  if (magic != kIndexMagic) return fail(-3, "magic mismatch: not a RAVEN index file");
  if (version != kIndexVersion) return fail(-4, "version mismatch: please rebuild the index");
  const uint8_t* body = bytes + 16;
  size_t blen = len - 16;
  if (crc32_ieee(body, blen) != crc) return fail(-5, "crc32 mismatch: index file corrupted");
  g->n = rd<uint64_t>(body);
  g->dim = rd<uint64_t>(body + 8);
  g->entry = rd<uint32_t>(body + 16);
  size_t off = 20;
  g->metadata_toml.clear();
  g->nav = LayeredNav();
  if (flags & kFlagHasMetadata) {
    if (blen < off + 4) return fail(-6, "body too short for metadata trailer header");
    uint32_t ml = rd<uint32_t>(body + off);
    off += 4;
    if (blen < off + ml) return fail(-6, "body too short for metadata trailer");
    g->metadata_toml.assign((const char*)body + off, ml);
    off += ml + (4 - ml % 4) % 4;
  }
  if (flags & kFlagHasLayeredNav) {
    if (blen < off + 4) return fail(-6, "body too short for layered nav trailer header");
    uint32_t nl = rd<uint32_t>(body + off);
    off += 4;
    if (blen < off + nl) return fail(-6, "body too short for layered nav trailer");
    LayeredNav nav;
    if (parse_nav(body + off, nl, &nav)) g->nav = std::move(nav);  // malformed nav -> None
    off += nl + (4 - nl % 4) % 4;
  }
  if (off > blen || blen - off < 24) return fail(-6, "HybridBlockedCsr body too short");
  const uint8_t* c = body + off;
  size_t clen = blen - off;
  uint64_t n = rd<uint64_t>(c), r_max = rd<uint64_t>(c + 8), mb_len = rd<uint64_t>(c + 16);
  if (mb_len > (clen - 24) / 4 || clen - 24 - mb_len * 4 < 8) return fail(-6, "main_block truncated");
  if (r_max == 0 || r_max > 65535 || mb_len != n * r_max) return fail(-6, "main_block size mismatch");
  g->r_max = r_max;
  g->main_block.resize(mb_len);
  std::memcpy(g->main_block.data(), c + 24, mb_len * 4);
  size_t o = 24 + mb_len * 4;
  uint64_t ov = rd<uint64_t>(c + o);
  o += 8;
  g->overflow.assign(n, {});
  for (uint64_t i = 0; i < ov; ++i) {
    if (o + 12 > clen) return fail(-6, "overflow entry header truncated");
    uint32_t node = rd<uint32_t>(c + o);
    uint64_t vl = rd<uint64_t>(c + o + 4);
    o += 12;
    if (vl > (clen - o) / 4) return fail(-6, "overflow entry data truncated");
    if (node < n) {
      g->overflow[node].resize(vl);
      if (vl) std::memcpy(g->overflow[node].data(), c + o, vl * 4);
    }
    o += vl * 4;
  }
  g->degrees.resize(n);
  for (uint64_t i = 0; i < n; ++i) {  // from_parts: degree = first SENTINEL (graph.rs:234-240)
    const uint32_t* row = g->main_block.data() + i * r_max;
    uint64_t d = 0;
    while (d < r_max && row[d] != kSentinel) ++d;
    g->degrees[i] = (uint16_t)d;
  }
  if (n != g->n) return fail(-6, "n mismatch between header and storage");
  return 0;
}

// Writer: VamanaGraph::serialize (src/graph/vamana.rs:1265-1324).
std::vector<uint8_t> serialize_annx(const HostGraph& g) {
  std::vector<uint8_t> body;
  body.reserve(64 + g.main_block.size() * 4);
  wr<uint64_t>(body, g.n);
  wr<uint64_t>(body, g.dim);
  wr<uint32_t>(body, g.entry);
  uint32_t flags = 0;
  if (!g.metadata_toml.empty()) {
    flags |= kFlagHasMetadata;
    wr<uint32_t>(body, (uint32_t)g.metadata_toml.size());
    body.insert(body.end(), g.metadata_toml.begin(), g.metadata_toml.end());
    body.resize(body.size() + (4 - g.metadata_toml.size() % 4) % 4, 0);
  }
  if (g.nav.present) {  // LayeredNavigation::serialize_binary (navigation.rs:670-706)
    std::vector<uint8_t> nb;
    const LayeredNav& nv = g.nav;
    wr<uint32_t>(nb, nv.entry);
    nb.push_back(nv.max_level);
    nb.push_back(0);
    nb.push_back(0);
    nb.push_back(0);
    wr<uint32_t>(nb, nv.k);
    wr<uint32_t>(nb, (uint32_t)nv.node_levels.size());
    nb.insert(nb.end(), nv.node_levels.begin(), nv.node_levels.end());
    uint32_t nonempty = 0;
    for (auto& l : nv.upper) nonempty += !l.empty();
    wr<uint32_t>(nb, nonempty);
    for (size_t i = 0; i < nv.upper.size(); ++i) {
      if (nv.upper[i].empty()) continue;
      wr<uint32_t>(nb, (uint32_t)i);
      wr<uint32_t>(nb, (uint32_t)nv.upper[i].size());
      for (uint32_t v : nv.upper[i]) wr<uint32_t>(nb, v);
    }
    wr<uint32_t>(nb, (uint32_t)nv.entry_candidates.size());
    for (uint32_t v : nv.entry_candidates) wr<uint32_t>(nb, v);
    if (!nb.empty()) {
      flags |= kFlagHasLayeredNav;
      wr<uint32_t>(body, (uint32_t)nb.size());
      body.insert(body.end(), nb.begin(), nb.end());
      body.resize(body.size() + (4 - nb.size() % 4) % 4, 0);
    }
  }
  // HybridBlockedCsr::serialize (src/memory/graph.rs:322-345)
  wr<uint64_t>(body, g.n);
  wr<uint64_t>(body, g.r_max);
  wr<uint64_t>(body, (uint64_t)g.main_block.size());
  size_t o = body.size();
  body.resize(o + g.main_block.size() * 4);
  if (!g.main_block.empty()) std::memcpy(body.data() + o, g.main_block.data(), g.main_block.size() * 4);
  uint64_t ov = 0;
  for (auto& l : g.overflow) ov += !l.empty();
  wr<uint64_t>(body, ov);
  for (size_t i = 0; i < g.overflow.size(); ++i) {
    if (g.overflow[i].empty()) continue;
    wr<uint32_t>(body, (uint32_t)i);
    wr<uint64_t>(body, (uint64_t)g.overflow[i].size());
    for (uint32_t v : g.overflow[i]) wr<uint32_t>(body, v);
  }
  std::vector<uint8_t> out;
  out.reserve(16 + body.size());
  wr<uint32_t>(out, kIndexMagic);
  wr<uint32_t>(out, kIndexVersion);
  wr<uint32_t>(out, flags);
  wr<uint32_t>(out, crc32_ieee(body.data(), body.size()));
  out.insert(out.end(), body.begin(), body.end());
  return out;
}

// ===========================================================================
// Vamana build
// ===========================================================================
namespace {

// xoshiro256** seeded through splitmix64.
struct Rng {
  uint64_t s[4];
  explicit Rng(uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; ++i) {
      x += 0x9E3779B97F4A7C15ull;
      uint64_t z = x;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      s[i] = z ^ (z >> 31);
    }
  }
  static uint64_t rotl(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }
  uint64_t next() {
    uint64_t r = rotl(s[1] * 5, 7) * 9, t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }
  uint32_t below(uint32_t n) {  // Lemire's unbiased bounded draw
    uint64_t m = (uint64_t)(uint32_t)next() * n;
    uint32_t l = (uint32_t)m;
    if (l < n) {
      uint32_t t = (0u - n) % n;
      while (l < t) {
        m = (uint64_t)(uint32_t)next() * n;
        l = (uint32_t)m;
      }
    }
    return (uint32_t)(m >> 32);
  }
  double uniform() { return (double)(next() >> 11) * (1.0 / 9007199254740992.0); }
};

// l2_simd as the reference computes it on AVX-512 hardware
// (src/distance/avx512.rs:31-62): 16 lane chains of fused multiply-adds over
// the full 16-element blocks, each halving-tree reduced (_mm512_reduce_add_ps:
// lanes j and j+8, then +4, +2, +1), the masked tail as its own vector reduced
// the same way, result = tail + main. The same order as the GPU kernels'
// distances, so host and GPU builds take the same decisions on float data.
inline float tree16(float (&v)[16]) {
  for (int w = 8; w >= 1; w >>= 1)
    for (int j = 0; j < w; ++j) v[j] = v[j] + v[j + w];
  return v[0];
}
inline float l2(const float* a, const float* b, size_t d) {
  float acc[16] = {0};
  size_t i = 0;
  for (; i + 16 <= d; i += 16)
    for (int j = 0; j < 16; ++j) {
      const float t = a[i + j] - b[i + j];
      acc[j] = std::fma(t, t, acc[j]);
    }
  float result = 0.0f;
  if (i < d) {
    float tail[16] = {0};
    for (size_t j = 0; i + j < d; ++j) {
      const float t = a[i + j] - b[i + j];
      tail[j] = std::fma(t, t, 0.0f);
    }
    result = tree16(tail);
  }
  return result + tree16(acc);
}

// HybridBlockedCsr mutators (src/memory/graph.rs:114-170).
struct Csr {
  uint64_t n, r;
  std::vector<uint32_t> mb;
  std::vector<uint16_t> deg;
  std::vector<std::vector<uint32_t>> ov;
  Csr(uint64_t n_, uint64_t r_) : n(n_), r(r_), mb(n_ * r_, kSentinel), deg(n_, 0), ov(n_) {}
  const uint32_t* row(uint32_t v) const { return mb.data() + (size_t)v * r; }
  size_t degree(uint32_t v) const { return deg[v] + ov[v].size(); }
  void add_edge(uint32_t from, uint32_t to) {
    uint32_t* rw = mb.data() + (size_t)from * r;
    size_t d = deg[from];
    for (size_t i = 0; i < d; ++i)
      if (rw[i] == to) return;
    if (d < r) {
      rw[d] = to;
      deg[from]++;
      return;
    }
    for (uint32_t x : ov[from])
      if (x == to) return;
    ov[from].push_back(to);
  }
  void set_neighbors(uint32_t v, const std::vector<uint32_t>& nb) {
    uint32_t* rw = mb.data() + (size_t)v * r;
    for (size_t i = 0; i < deg[v]; ++i) rw[i] = kSentinel;
    ov[v].clear();
    size_t m = std::min<size_t>(nb.size(), r);
    std::copy(nb.begin(), nb.begin() + m, rw);
    if (nb.size() > r) ov[v].assign(nb.begin() + r, nb.end());
    deg[v] = (uint16_t)m;
  }
  std::vector<uint32_t> full(uint32_t v) const {
    std::vector<uint32_t> a(row(v), row(v) + deg[v]);
    a.insert(a.end(), ov[v].begin(), ov[v].end());
    return a;
  }
};

// Fixed-capacity sorted candidate pool with the LinearPool rules
// (src/graph/linear_pool.rs:100-171).
struct Pool {
  std::vector<std::pair<uint32_t, float>> d;
  size_t sz = 0, cur = 0, cap = 0;
  void reset(size_t c) {
    cap = c;
    if (d.size() < c + 1) d.resize(c + 1);
    sz = cur = 0;
  }
  void insert(uint32_t id, float dist) {
    if (sz == cap && dist >= d[sz - 1].second) return;
    size_t lo = sz;
    while (lo > 0 && d[lo - 1].second > dist) --lo;
    std::copy_backward(d.begin() + lo, d.begin() + sz, d.begin() + sz + 1);
    d[lo] = {id, dist};
    if (sz < cap) ++sz;
    if (lo < cur) cur = lo;
  }
  bool pop(uint32_t* id) {
    if (!(cur < sz && cur < cap)) return false;
    size_t i = cur;
    d[i].first |= 0x80000000u;
    ++cur;
    while (cur < sz && (d[cur].first & 0x80000000u)) ++cur;
    *id = d[i].first & 0x7FFFFFFFu;
    return true;
  }
};

struct Visit {
  std::vector<uint8_t> m;
  std::vector<uint32_t> hist;
  explicit Visit(size_t n) : m(n, 0) {}
  bool visit(uint32_t v) {
    if (m[v]) return false;
    m[v] = 1;
    hist.push_back(v);
    return true;
  }
  void reset() {
    for (uint32_t v : hist) m[v] = 0;
    hist.clear();
  }
};

struct Ctx {
  const float* V;
  size_t dim;
  const float* vec(uint32_t i) const { return V + (size_t)i * dim; }
};

// prepare_candidates (src/graph/robust_prune.rs:22-47): drop self, distance,
// dedup by id, stable sort by distance (== sort by (distance, id)).
std::vector<std::pair<float, uint32_t>> prepare(const Ctx& c, const std::vector<uint32_t>& cands, uint32_t q) {
  std::vector<std::pair<float, uint32_t>> s;
  s.reserve(cands.size());
  std::vector<uint32_t> ids(cands);
  std::sort(ids.begin(), ids.end());
  ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
  const float* qv = c.vec(q);
  for (uint32_t id : ids)
    if (id != q) s.push_back({l2(qv, c.vec(id), c.dim), id});
  std::sort(s.begin(), s.end());
  return s;
}

// RobustPrune (src/graph/robust_prune.rs:92-185).
std::vector<uint32_t> robust_prune(const Ctx& c, const std::vector<uint32_t>& cands, uint32_t q, float alpha,
                                   size_t r_max, bool saturate) {
  std::vector<uint32_t> result;
  if (cands.empty()) return result;
  auto s = prepare(c, cands, q);
  if (s.empty()) return result;
  size_t n = s.size();
  const float FMAX = 3.40282347e+38f;
  std::vector<float> occ(n, 0.0f);
  std::vector<size_t> ridx;
  float cur_alpha = 1.0f, inc = std::min(alpha, 1.2f);
  while (result.size() < r_max) {
    for (size_t i = 0; i < n; ++i) {
      if (result.size() >= r_max) break;
      if (occ[i] == FMAX || occ[i] > cur_alpha) continue;
      const float* cv = c.vec(s[i].second);
      float diq = s[i].first;
      for (size_t j : ridx) {
        if (j >= i) continue;
        float dji = l2(c.vec(s[j].second), cv, c.dim);
        if (dji == 0.0f) {
          occ[i] = FMAX;
          break;
        }
        float ratio = diq / dji;
        if (ratio > occ[i]) occ[i] = ratio;
        if (occ[i] > cur_alpha) break;
      }
      if (occ[i] > cur_alpha) continue;
      occ[i] = FMAX;
      ridx.push_back(i);
      result.push_back(s[i].second);
    }
    if (cur_alpha >= alpha) break;
    cur_alpha = std::min(cur_alpha * inc, alpha);
  }
  if (saturate)
    for (size_t i = 0; i < n && result.size() < r_max; ++i)
      if (occ[i] != FMAX) result.push_back(s[i].second);
  return result;
}

// DirectionalPrune (src/graph/robust_prune.rs:280-385).
std::vector<uint32_t> directional_prune(const Ctx& c, const std::vector<uint32_t>& cands, uint32_t q,
                                        size_t r_max, size_t r_min, float backfill_alpha) {
  std::vector<uint32_t> result;
  if (cands.empty()) return result;
  auto s = prepare(c, cands, q);
  if (s.empty()) return result;
  for (size_t i = 0; i < s.size() && result.size() < r_max; ++i) {
    const float* cv = c.vec(s[i].second);
    bool good = true;
    for (uint32_t a : result)
      if (l2(c.vec(a), cv, c.dim) < s[i].first) {
        good = false;
        break;
      }
    if (good) result.push_back(s[i].second);
  }
  if (result.size() < r_min) {
    std::unordered_set<uint32_t> acc(result.begin(), result.end());
    for (size_t i = 0; i < s.size() && result.size() < r_min; ++i) {
      uint32_t id = s[i].second;
      if (acc.count(id)) continue;
      const float* cv = c.vec(id);
      bool good = true;
      for (uint32_t a : result) {
        float dji = l2(c.vec(a), cv, c.dim);
        if (dji == 0.0f || s[i].first / dji > backfill_alpha) {
          good = false;
          break;
        }
      }
      if (good) result.push_back(id);
    }
  }
  return result;
}

std::vector<uint32_t> prune_dispatch(const Ctx& c, const BuildConfig& cfg, const std::vector<uint32_t>& cands,
                                     uint32_t q, float alpha, size_t r_max, bool saturate) {
  if (cfg.directional) {
    size_t div = cfg.rmin_divisor ? cfg.rmin_divisor : 4;
    return directional_prune(c, cands, q, r_max, std::max<size_t>(r_max / div, 1), std::max(alpha, 1.0f));
  }
  return robust_prune(c, cands, q, alpha, r_max, saturate);
}

// greedy_search_vec_build (src/graph/vamana.rs:530-567): returns with the
// visit history filled. A row's neighbours are all marked before their
// distances are taken (the same visits in the same order, and the same inserts
// in the same order, as marking and inserting one by one), so that the vectors
// of the next few can be prefetched while a distance is computed; the next
// expansion's row is prefetched after each pop, as the reference does
// (storage.prefetch_neighbors). Prefetches do not change results.
void greedy_build(const Ctx& c, const Csr& g, uint32_t entry, const float* q, size_t l, Visit& vis, Pool& pool) {
  constexpr size_t kAhead = 4;  // vectors requested ahead of the distance loop
  const size_t vec_lines = (c.dim * 4 + 63) / 64, row_lines = (g.r * 4 + 63) / 64;
  auto prefetch_vec = [&](uint32_t v) {
    const char* p = (const char*)c.vec(v);
    for (size_t li = 0; li < vec_lines; ++li) __builtin_prefetch(p + 64 * li, 0, 3);
  };
  vis.reset();
  pool.reset(l);
  vis.visit(entry);
  pool.insert(entry, l2(q, c.vec(entry), c.dim));
  std::vector<uint32_t> fresh;
  fresh.reserve(g.r);
  uint32_t node;
  while (pool.pop(&node)) {
    if (pool.cur < pool.sz && pool.cur < pool.cap) {  // peek_unchecked
      const char* rp = (const char*)g.row(pool.d[pool.cur].first & 0x7FFFFFFFu);
      for (size_t li = 0; li < row_lines; ++li) __builtin_prefetch(rp + 64 * li, 0, 3);
    }
    const uint32_t* rw = g.row(node);
    fresh.clear();
    for (size_t i = 0; i < g.deg[node]; ++i)
      if (vis.visit(rw[i])) fresh.push_back(rw[i]);
    for (size_t i = 0; i < std::min(kAhead, fresh.size()); ++i) prefetch_vec(fresh[i]);
    for (size_t i = 0; i < fresh.size(); ++i) {
      if (i + kAhead < fresh.size()) prefetch_vec(fresh[i + kAhead]);
      pool.insert(fresh[i], l2(q, c.vec(fresh[i]), c.dim));
    }
  }
}

// compute_medoid (src/graph/vamana.rs:366-429).
uint32_t medoid(const Ctx& c, uint64_t n) {
  if (n == 0) return 0;
  std::vector<uint32_t> sample;
  if (n <= 10000) {
    sample.resize(n);
    std::iota(sample.begin(), sample.end(), 0u);
  } else {
    Rng r(42);  // independent stream, like the reference's seed-42 side RNG
    std::vector<uint32_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0u);
    for (size_t i = 0; i < 1000; ++i) std::swap(idx[i], idx[i + r.below((uint32_t)(n - i))]);
    sample.assign(idx.begin(), idx.begin() + 1000);
  }
  std::vector<float> cen(c.dim, 0.0f);
  for (uint32_t s : sample)
    for (size_t d = 0; d < c.dim; ++d) cen[d] += c.vec(s)[d];
  for (size_t d = 0; d < c.dim; ++d) cen[d] /= (float)sample.size();
  uint32_t best = sample[0];
  float bd = 3.40282347e+38f;
  for (uint32_t s : sample) {
    float d = l2(cen.data(), c.vec(s), c.dim);
    if (d < bd) {
      bd = d;
      best = s;
    }
  }
  return best;
}

// ---------------------------------------------------------------------------
// LayeredNavigation::build (src/graph/navigation.rs:244-595).
// ---------------------------------------------------------------------------
void nav_add_bidirectional(const Ctx& c, std::vector<std::vector<uint32_t>>& adj, uint32_t node, uint32_t nn,
                           size_t k) {  // :471-494
  auto& nb = adj[node];
  for (uint32_t x : nb)
    if (x == nn) return;
  nb.push_back(nn);
  if (nb.size() > k) {
    std::vector<uint32_t> all = nb;
    nb = robust_prune(c, all, node, 1.0f, k, false);
  }
}

void nav_brute(const Ctx& c, const std::vector<uint32_t>& layer, std::vector<std::vector<uint32_t>>& adj,
               size_t k) {  // :380-407
  for (size_t i = 0; i < layer.size(); ++i) {
    uint32_t u = layer[i];
    std::vector<uint32_t> cands;
    cands.reserve(layer.size());
    for (size_t j = 0; j < layer.size(); ++j)
      if (j != i) cands.push_back(layer[j]);
    auto nbrs = robust_prune(c, cands, u, 1.0f, k, false);
    adj[u] = nbrs;
    for (uint32_t v : nbrs) nav_add_bidirectional(c, adj, v, u, k);
  }
}

void nav_graph_guided(const Ctx& c, const std::vector<uint32_t>& layer, std::vector<std::vector<uint32_t>>& adj,
                      size_t k, uint64_t n) {  // :416-465
  size_t seed_count = std::min<size_t>(layer.size(), 2000);
  std::vector<uint32_t> seed(layer.begin(), layer.begin() + seed_count);
  nav_brute(c, seed, adj, k);
  if (layer.size() <= seed_count) return;
  size_t ef = k * 4;
  Visit vis(n);
  Pool pool;
  uint32_t entry = layer[0];
  for (size_t t = seed_count; t < layer.size(); ++t) {
    uint32_t u = layer[t];
    const float* q = c.vec(u);
    // search_upper_layer (:501-535)
    vis.reset();
    pool.reset(ef);
    vis.visit(entry);
    pool.insert(entry, l2(q, c.vec(entry), c.dim));
    uint32_t node;
    while (pool.pop(&node)) {
      for (uint32_t nb : adj[node]) {
        if (nb == node) continue;
        if (vis.visit(nb)) pool.insert(nb, l2(q, c.vec(nb), c.dim));
      }
    }
    std::vector<uint32_t> cands;
    for (size_t i = 0; i < pool.sz; ++i) cands.push_back(pool.d[i].first & 0x7FFFFFFFu);
    auto nbrs = robust_prune(c, cands, u, 1.0f, k, false);
    adj[u] = nbrs;
    for (uint32_t v : nbrs) nav_add_bidirectional(c, adj, v, u, k);
  }
}

LayeredNav build_nav(const Ctx& c, uint64_t n, uint32_t entry, uint32_t m, uint32_t k, int verbose) {
  LayeredNav nav;
  nav.k = k;
  if (n == 0 || k == 0) {
    nav.present = true;
    return nav;
  }
  Rng rng(42);
  double ml = 1.0 / std::log((double)m);
  nav.node_levels.assign(n, 0);
  uint8_t max_level = 0;
  for (uint64_t i = 0; i < n; ++i) {
    double u = rng.uniform();
    double lv = std::floor(-std::log(std::max(u, 1e-10)) * ml);
    uint8_t l = lv >= 255.0 ? 255 : (uint8_t)lv;
    nav.node_levels[i] = l;
    max_level = std::max(max_level, l);
  }
  nav.node_levels[entry] = max_level;
  nav.max_level = max_level;
  nav.entry = entry;
  nav.upper.assign(n, {});
  for (uint8_t level = 1; level <= max_level && max_level > 0; ++level) {
    std::vector<uint32_t> layer;
    for (uint64_t i = 0; i < n; ++i)
      if (nav.node_levels[i] >= level) layer.push_back((uint32_t)i);
    if (layer.size() <= 1) continue;
    if (verbose) fprintf(stderr, "[nav] level %d: %zu nodes\n", level, layer.size());
    std::vector<std::vector<uint32_t>> adj(n);
    if (layer.size() <= 2000) nav_brute(c, layer, adj, k);
    else nav_graph_guided(c, layer, adj, k, n);
    for (uint32_t u : layer) {
      std::vector<uint32_t> e = std::move(adj[u]);
      while (e.size() < k) e.push_back(u);
      nav.upper[u].insert(nav.upper[u].end(), e.begin(), e.end());
    }
  }
  // select_entry_candidates (:545-595)
  std::vector<uint32_t> top;
  for (uint64_t i = 0; i < n; ++i)
    if (nav.node_levels[i] >= max_level) top.push_back((uint32_t)i);
  if (top.size() <= 50) {
    nav.entry_candidates = top;
  } else {
    std::vector<uint32_t> sel{entry};
    std::vector<float> md(top.size());
    for (size_t i = 0; i < top.size(); ++i) md[i] = l2(c.vec(entry), c.vec(top[i]), c.dim);
    while (sel.size() < 50) {
      size_t bi = 0;
      for (size_t i = 1; i < md.size(); ++i)
        if (md[i] >= md[bi]) bi = i;  // Iterator::max_by keeps the last maximum
      uint32_t nn = top[bi];
      sel.push_back(nn);
      for (size_t i = 0; i < top.size(); ++i) {
        float d = l2(c.vec(nn), c.vec(top[i]), c.dim);
        if (d < md[i]) md[i] = d;
      }
    }
    nav.entry_candidates = sel;
  }
  nav.present = true;
  return nav;
}

}  // namespace

int build_vamana(const float* V, uint64_t n, uint32_t dim, const BuildConfig& cfg, HostGraph* out, std::string* err,
                 BuildAccelerator* acc) {
  if (dim == 0 || cfg.r_max == 0 || cfg.l_build == 0 || cfg.r_max > 65535) {
    if (err) *err = "invalid build configuration";
    return -1;
  }
  if (n >= 0x7FFFFFFFull) {
    if (err) *err = "too many vectors (node ids must fit in 31 bits)";
    return -1;
  }
  int threads = cfg.threads > 0 ? cfg.threads : omp_get_max_threads();
  Ctx c{V, dim};
  Csr g(n, cfg.r_max);
  Rng rng(cfg.seed);
  // init_random_graph (src/graph/vamana.rs:324-356)
  if (n > 0) {
    (void)rng.below((uint32_t)n);  // the reference draws an (unused) random entry first
    size_t cnt = std::min<uint64_t>(cfg.r_max, n - 1);
    std::vector<uint32_t> nb;
    for (uint64_t node = 0; node < n; ++node) {
      nb.clear();
      while (nb.size() < cnt) {
        uint32_t j = rng.below((uint32_t)n);
        if (j == node || std::find(nb.begin(), nb.end(), j) != nb.end()) continue;
        nb.push_back(j);
      }
      for (uint32_t j : nb) {
        g.add_edge((uint32_t)node, j);
        g.add_edge(j, (uint32_t)node);
      }
    }
  }
  uint32_t entry = medoid(c, n);
  const size_t kBatch = 10000;
  if (acc && n > 0 && acc->begin(g.mb.data(), n, g.r, entry, err) != 0) return -1;
  std::vector<Visit*> visits(threads, nullptr);
  std::vector<Pool> pools(threads);
  for (uint32_t iter = 0; iter < cfg.max_iterations && n > 0; ++iter) {
    std::vector<uint32_t> order(n);
    std::iota(order.begin(), order.end(), 0u);
    for (size_t i = n - 1; i > 0; --i) std::swap(order[i], order[rng.below((uint32_t)(i + 1))]);
    float alpha = iter == 0 ? 1.0f : cfg.alpha;
    if (cfg.verbose) fprintf(stderr, "[build] iter %u/%u alpha=%.2f\n", iter + 1, cfg.max_iterations, alpha);
    for (size_t b0 = 0; b0 < n; b0 += kBatch) {
      size_t b1 = std::min<size_t>(n, b0 + kBatch);
      std::vector<std::vector<uint32_t>> pruned(b1 - b0);
      if (acc) {
        if (acc->search_prune(order.data() + b0, b1 - b0, alpha, &pruned, err) != 0) {
          for (Visit* v : visits) delete v;
          return -1;
        }
      } else {
#pragma omp parallel for schedule(dynamic, 16) num_threads(threads)
        for (size_t p = b0; p < b1; ++p) {
          int t = omp_get_thread_num();
          if (!visits[t]) visits[t] = new Visit(n);
          uint32_t node = order[p];
          greedy_build(c, g, entry, c.vec(node), cfg.l_build, *visits[t], pools[t]);
          pruned[p - b0] =
              prune_dispatch(c, cfg, visits[t]->hist, node, alpha, cfg.r_max, cfg.saturate && alpha > 1.0f);
        }
      }
      // connect_bidirectional (vamana.rs:1117-1145), grouped by target node.
      struct Op {
        uint32_t target, pos, value;  // value == kSentinel -> SET from pruned[pos]
      };
      std::vector<Op> ops;
      for (size_t p = 0; p < pruned.size(); ++p) {
        uint32_t node = order[b0 + p];
        ops.push_back({node, (uint32_t)p, kSentinel});
        for (uint32_t nb : pruned[p]) ops.push_back({nb, (uint32_t)p, node});
      }
      std::stable_sort(ops.begin(), ops.end(), [](const Op& a, const Op& b) { return a.target < b.target; });
      std::vector<size_t> seg;
      for (size_t i = 0; i < ops.size(); ++i)
        if (i == 0 || ops[i].target != ops[i - 1].target) seg.push_back(i);
      seg.push_back(ops.size());
      const size_t n_seg = seg.size() - 1;
#pragma omp parallel for schedule(dynamic, 64) num_threads(threads)
      for (size_t s = 0; s < n_seg; ++s) {
        for (size_t i = seg[s]; i < seg[s + 1]; ++i) {
          const Op& op = ops[i];
          if (op.value == kSentinel) {
            g.set_neighbors(op.target, pruned[op.pos]);
          } else {
            g.add_edge(op.target, op.value);
            if (g.degree(op.target) > cfg.r_soft) {
              auto all = g.full(op.target);
              g.set_neighbors(op.target, prune_dispatch(c, cfg, all, op.target, alpha, cfg.r_max,
                                                        cfg.saturate && alpha > 1.0f));
            }
          }
        }
      }
      if (acc) {
        // every target of this batch's operations may have a new main block
        std::vector<uint32_t> changed;
        changed.reserve(n_seg);
        for (size_t s2 = 0; s2 < n_seg; ++s2) changed.push_back(ops[seg[s2]].target);
        if (acc->update_rows(changed.data(), changed.size(), g.mb.data(), err) != 0) {
          for (Visit* v : visits) delete v;
          return -1;
        }
      }
      if (cfg.verbose && (b0 / kBatch) % 10 == 0)
        fprintf(stderr, "[build] iter %u: %zu/%llu\n", iter + 1, b1, (unsigned long long)n);
    }
  }
  for (Visit* v : visits) delete v;
  // final_prune (vamana.rs:1150-1169)
#pragma omp parallel for schedule(dynamic, 256) num_threads(threads)
  for (uint64_t v = 0; v < n; ++v) {
    if (g.degree((uint32_t)v) <= cfg.r_max) continue;
    auto all = g.full((uint32_t)v);
    g.set_neighbors((uint32_t)v, prune_dispatch(c, cfg, all, (uint32_t)v, cfg.alpha, cfg.r_max, cfg.saturate));
  }
  out->n = n;
  out->dim = dim;
  out->r_max = cfg.r_max;
  out->entry = entry;
  out->main_block = std::move(g.mb);
  out->degrees = std::move(g.deg);
  out->overflow = std::move(g.ov);
  char meta[512];
  snprintf(meta, sizeof(meta),
           "rng_algorithm = \"xoshiro256ss\"\nrng_seed = %llu\nshard_strategy = \"static_range\"\n"
           "build_version = \"raven-b200-0.1\"\nbuild_timestamp = 0\nn = %llu\ndim = %u\nalpha = %g\n"
           "l_build = %u\nr_max = %u\nr_soft = %u\n",
           (unsigned long long)cfg.seed, (unsigned long long)n, dim, (double)cfg.alpha, cfg.l_build, cfg.r_max,
           cfg.r_soft);
  out->metadata_toml = meta;
  if (cfg.enable_layered_nav && n > 0) {
    const double t_nav = omp_get_wtime();
    out->nav = build_nav(c, n, entry, cfg.nav_m, cfg.r_max / 2, cfg.verbose);
    if (cfg.verbose) fprintf(stderr, "[nav] built in %.1f s\n", omp_get_wtime() - t_nav);
  } else {
    out->nav = LayeredNav();
  }
  return 0;
}

void sq_fit_host(const float* data, uint64_t n, uint32_t dim, float levels, float* out, int threads) {
  if (threads <= 0) threads = omp_get_max_threads();
  const uint64_t kRows = 16384;
  uint64_t nb = (n + kRows - 1) / kRows;
  std::vector<float> bmin(nb * dim), bmax(nb * dim);
#pragma omp parallel for schedule(static) num_threads(threads)
  for (uint64_t b = 0; b < nb; ++b) {
    float* mn = bmin.data() + b * dim;
    float* mx = bmax.data() + b * dim;
    for (uint32_t d = 0; d < dim; ++d) {
      mn[d] = 3.40282347e+38f;
      mx[d] = -3.40282347e+38f;
    }
    uint64_t r1 = std::min(n, (b + 1) * kRows);
    for (uint64_t i = b * kRows; i < r1; ++i) {
      const float* row = data + i * dim;
      for (uint32_t d = 0; d < dim; ++d) {
        if (row[d] < mn[d]) mn[d] = row[d];
        if (row[d] > mx[d]) mx[d] = row[d];
      }
    }
  }
  float* mn = out;
  float* mx = out + dim;
  for (uint32_t d = 0; d < dim; ++d) {
    mn[d] = 3.40282347e+38f;
    mx[d] = -3.40282347e+38f;
  }
  for (uint64_t b = 0; b < nb; ++b)
    for (uint32_t d = 0; d < dim; ++d) {
      if (bmin[b * dim + d] < mn[d]) mn[d] = bmin[b * dim + d];
      if (bmax[b * dim + d] > mx[d]) mx[d] = bmax[b * dim + d];
    }
  for (uint32_t d = 0; d < dim; ++d)
    if (mx[d] <= mn[d]) mx[d] = mn[d] + 1.0f;
  float* scale = out + 2 * dim;
  float* inv = out + 3 * dim;
  float* neg = out + 4 * dim;
  for (uint32_t d = 0; d < dim; ++d) scale[d] = (mx[d] - mn[d]) / levels;
  for (uint32_t d = 0; d < dim; ++d) inv[d] = 1.0f / scale[d];
  for (uint32_t d = 0; d < dim; ++d) neg[d] = -mn[d] * inv[d];
}

}  // namespace raven
