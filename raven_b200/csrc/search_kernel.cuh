// Device side of the query engine: one warp per query, persistent grid.
//
// Per query (all inside one warp, warp-synchronous, no block barriers):
//   1. query -> shared memory, SQ4/SQ8 encode          (src/quant/sq4.rs:93-105, sq8.rs:89-97)
//   2. layered-navigation greedy descent, f32 L2 in    (src/graph/navigation.rs:609-653,
//      the reference's AVX-512 lane/tree order          src/distance/avx512.rs:31-62)
//   3. AdaptiveEf rank -> ef table lookup, .max(k)      (src/graph/adaptive_ef.rs:340-359,
//                                                        src/graph/vamana.rs:1803)
//   4. beam search over the fixed-degree adjacency      (src/graph/vamana.rs:786-861 / 683-773,
//      with an exact visited set and the LinearPool     src/graph/linear_pool.rs:100-171,
//      ordering                                         src/memory/visited.rs:88-103)
//   5. f32 rerank of min(k*rr, |pool|) survivors        (src/graph/refiner.rs:45-61)
//
// LinearPool equivalence used by the batch merge: the pool always holds the
// first `ef` of all inserted candidates ordered by (distance, insertion order)
// and the cursor is the first unexpanded entry. A new candidate therefore loses
// every distance tie against an entry already in the pool, and candidates of
// one expansion tie-break by adjacency order, so merging one expansion's
// candidates at once gives the same pool as inserting them one by one.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace raven_dev {

constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kSent = 0xffffffffu;
constexpr uint32_t kChecked = 0x80000000u;
constexpr uint32_t kEmpty = 0xffffffffu;
constexpr int kWarpsPerBlock = 4;
constexpr uint32_t kNavStepLimit = 1u << 16;

struct SearchArgs {
  // index
  const float* __restrict__ vec;
  uint32_t dim;
  uint32_t dim_pad;  // dim rounded up to 16
  const uint32_t* __restrict__ adj;
  uint32_t r_pad;  // row stride in ids (multiple of 32)
  const uint8_t* __restrict__ codes;
  uint32_t code_stride;  // bytes per code row (power of two, >= 16)
  const float* __restrict__ q_inv;
  const float* __restrict__ q_neg;
  float levels;  // 15 (SQ4) or 255 (SQ8)
  uint32_t entry;
  int nav;
  uint32_t nav_entry, nav_max_level, nav_k;
  const uint32_t* __restrict__ nav_slot;
  const uint32_t* __restrict__ nav_off;
  const uint32_t* __restrict__ nav_edges;
  int adaptive;
  const float* __restrict__ samples;
  uint32_t n_samples;
  const uint32_t* __restrict__ ef_table;  // n_samples + 1 entries
  uint32_t ef_mid;
  uint32_t ef_fixed, k, rr;
  uint32_t hash_bits;   // shared-memory visited table: 1 << hash_bits slots
  uint32_t spill_bits;  // global spill table per warp slot: 1 << spill_bits slots
  uint32_t* spill;
  uint32_t smem_per_warp;
  // queries
  const float* __restrict__ queries;
  uint64_t nq;
  // outputs
  uint32_t* ids;
  float* dists;
  uint32_t* counts;
  uint32_t* visited;
  uint32_t* ef_used;
  int32_t* status;
  uint32_t* n_nav;
  uint32_t* expansions;
  uint32_t* history;
  uint32_t hist_cap;
  uint32_t* hist_len;
  unsigned long long* counter;
  int nav_only;  // 1: only run the descent; write entry to ids[q], distance to dists[q]
};

// Per-warp shared-memory carve-up (byte offsets; every piece 16-byte aligned).
struct WarpSmem {
  float* qf;         // dim_pad floats
  uint8_t* qcode;    // code_stride bytes
  uint32_t* pool_d;  // 32*PT
  uint32_t* pool_id; // 32*PT
  uint32_t* cand_id; // 32
  uint32_t* cand_d;  // 32
  float* nd;         // 32 (navigation distances)
  uint32_t* ht;      // 1 << hash_bits (reused as float[] by the rerank)
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline uint32_t warp_smem_bytes(uint32_t dim_pad, uint32_t code_stride, uint32_t pt,
                                                    uint32_t hash_bits) {
  return align16(dim_pad * 4) + align16(code_stride) + 2 * align16(32 * pt * 4) + 3 * 128 +
         align16((1u << hash_bits) * 4);
}

__device__ inline WarpSmem carve(uint8_t* base, const SearchArgs& a, int pt) {
  WarpSmem s;
  uint32_t o = 0;
  s.qf = (float*)(base + o);
  o += align16(a.dim_pad * 4);
  s.qcode = base + o;
  o += align16(a.code_stride);
  s.pool_d = (uint32_t*)(base + o);
  o += align16(32 * pt * 4);
  s.pool_id = (uint32_t*)(base + o);
  o += align16(32 * pt * 4);
  s.cand_id = (uint32_t*)(base + o);
  o += 128;
  s.cand_d = (uint32_t*)(base + o);
  o += 128;
  s.nd = (float*)(base + o);
  o += 128;
  s.ht = (uint32_t*)(base + o);
  return s;
}

__device__ inline uint32_t lanemask_lt(int lane) { return (1u << lane) - 1u; }

// ---------------------------------------------------------------------------
// f32 squared L2 of the query (shared memory) against one row, computed by a
// half-warp in the order of _mm512 code: lane j accumulates fma(d,d,acc) over
// elements 16c+j, then the 16 lanes are reduced by the halving tree
// (xor 8, 4, 2, 1), a masked tail is reduced the same way, result = tail+main.
// Both half-warps run this for their own row; every lane returns the value.
// ---------------------------------------------------------------------------
__device__ inline float tree16(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 8));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 1));
  return v;
}

// Two rows per half-warp (loads of both issued together). row_a/row_b may be
// null (then that result is garbage but all lanes still join the shuffles).
__device__ inline void hw_l2_pair(const float* __restrict__ qf, const float* __restrict__ row_a,
                                  const float* __restrict__ row_b, uint32_t dim, int j, float* out_a,
                                  float* out_b) {
  const uint32_t chunks = dim >> 4, rem = dim & 15;
  float acc_a = 0.0f, acc_b = 0.0f;
  uint32_t c = 0;
  for (; c + 4 <= chunks; c += 4) {
    float va[4], vb[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      va[u] = row_a ? __ldg(row_a + (c + u) * 16 + j) : 0.0f;
      vb[u] = row_b ? __ldg(row_b + (c + u) * 16 + j) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float q = qf[(c + u) * 16 + j];
      float da = __fsub_rn(q, va[u]);
      float db = __fsub_rn(q, vb[u]);
      acc_a = __fmaf_rn(da, da, acc_a);
      acc_b = __fmaf_rn(db, db, acc_b);
    }
  }
  for (; c < chunks; ++c) {
    float va = row_a ? __ldg(row_a + c * 16 + j) : 0.0f;
    float vb = row_b ? __ldg(row_b + c * 16 + j) : 0.0f;
    float q = qf[c * 16 + j];
    float da = __fsub_rn(q, va), db = __fsub_rn(q, vb);
    acc_a = __fmaf_rn(da, da, acc_a);
    acc_b = __fmaf_rn(db, db, acc_b);
  }
  float ta = 0.0f, tb = 0.0f;
  if (rem) {
    float da = 0.0f, db = 0.0f;
    if ((uint32_t)j < rem) {
      float q = qf[chunks * 16 + j];
      if (row_a) da = __fsub_rn(q, __ldg(row_a + chunks * 16 + j));
      if (row_b) db = __fsub_rn(q, __ldg(row_b + chunks * 16 + j));
    }
    ta = tree16(__fmaf_rn(da, da, 0.0f));
    tb = tree16(__fmaf_rn(db, db, 0.0f));
  }
  *out_a = __fadd_rn(ta, tree16(acc_a));
  *out_b = __fadd_rn(tb, tree16(acc_b));
}

// f32 -> u32 key that orders like Rust's f32::total_cmp.
__device__ inline uint32_t total_order_key(float f) {
  int32_t b = __float_as_int(f);
  b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
  return (uint32_t)b ^ 0x80000000u;
}

// quantize: Rust f32::round (half away from zero), clamp(0, L), `as u8`.
__device__ inline uint32_t quantize(float v, float inv, float neg, float levels) {
  float q = roundf(__fmaf_rn(v, inv, neg));
  if (q != q) return 0u;
  q = fmaxf(q, 0.0f);
  q = fminf(q, levels);
  return (uint32_t)q;
}

// ---------------------------------------------------------------------------
// Navigation descent (src/graph/navigation.rs:609-653). Returns entry + f32
// distance; counts distance evaluations exactly as the reference does (an
// edge equal to the running node is skipped).
// ---------------------------------------------------------------------------
__device__ inline bool nav_descend(const SearchArgs& a, const WarpSmem& s, int lane, uint32_t* out_u,
                                   float* out_d, uint32_t* out_evals) {
  const int h = lane >> 4, j = lane & 15;
  uint32_t u = a.nav_entry;
  float du, dummy;
  hw_l2_pair(s.qf, a.vec + (size_t)u * a.dim, nullptr, a.dim, j, &du, &dummy);
  uint32_t evals = 1;
  uint32_t steps = 0;
  bool ok = true;
  if (a.nav_max_level > 0) {
    for (int level = (int)a.nav_max_level; level >= 1 && ok; --level) {
      while (true) {
        if (++steps > kNavStepLimit) {
          ok = false;
          break;
        }
        uint32_t slot = a.nav_slot[u];
        uint32_t off = 0, len = 0;
        if (slot != kSent) {
          off = a.nav_off[slot];
          len = a.nav_off[slot + 1] - off;
        }
        uint32_t start = (uint32_t)(level - 1) * a.nav_k;
        if (start >= len) break;
        uint32_t cnt = min(a.nav_k, len - start);
        uint32_t v = (uint32_t)lane < cnt ? a.nav_edges[off + start + lane] : kSent;
        for (uint32_t e0 = 0; e0 < cnt; e0 += 4) {
          uint32_t ea = e0 + h, eb = e0 + 2 + h;
          uint32_t va = __shfl_sync(kFull, v, ea & 31), vb = __shfl_sync(kFull, v, eb & 31);
          const float* ra = ea < cnt ? a.vec + (size_t)va * a.dim : nullptr;
          const float* rb = eb < cnt ? a.vec + (size_t)vb * a.dim : nullptr;
          float da, db;
          hw_l2_pair(s.qf, ra, rb, a.dim, j, &da, &db);
          if (j == 0) {
            if (ea < cnt) s.nd[ea] = da;
            if (eb < cnt) s.nd[eb] = db;
          }
        }
        __syncwarp();
        float d = (uint32_t)lane < cnt ? s.nd[lane] : __int_as_float(0x7f800000);
        // key: distance bits (non-negative floats order as integers; NaN sorts
        // after +inf and is never selected by `d < cur`) then edge index.
        unsigned long long key = ((unsigned long long)__float_as_uint(d) << 32) | (uint32_t)lane;
        if ((uint32_t)lane >= cnt) key = ~0ull;
        // Running node before edge e: the argmin over edges < e if it beats du.
        unsigned long long pre = key;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          unsigned long long t = __shfl_up_sync(kFull, pre, o);
          if (lane >= o && t < pre) pre = t;
        }
        unsigned long long excl = __shfl_up_sync(kFull, pre, 1);
        if (lane == 0) excl = ~0ull;
        const bool moved = excl != ~0ull && __uint_as_float((uint32_t)(excl >> 32)) < du;
        const uint32_t excl_v = __shfl_sync(kFull, v, moved ? (int)(excl & 31) : 0);
        const uint32_t run_u = moved ? excl_v : u;
        const bool counted = (uint32_t)lane < cnt && v != run_u;
        evals += __popc(__ballot_sync(kFull, counted));
        const unsigned long long best = __shfl_sync(kFull, pre, 31);
        const float bd = __uint_as_float((uint32_t)(best >> 32));
        const uint32_t best_v = __shfl_sync(kFull, v, (int)(best & 31));
        __syncwarp();
        if (best != ~0ull && bd < du) {
          du = bd;
          u = best_v;
        } else {
          break;
        }
      }
    }
  }
  *out_u = u;
  *out_d = du;
  *out_evals = evals;
  return ok;
}

// ---------------------------------------------------------------------------
// Visited set: open addressing in shared memory; after it passes 3/4 load the
// warp switches to its global spill table (lookups check both). Exact: every
// id lives in exactly one table.
// ---------------------------------------------------------------------------
__device__ inline uint32_t hash_slot(uint32_t id, uint32_t bits) { return (id * 0x9E3779B1u) >> (32 - bits); }

// Returns 1 if inserted (first visit), 0 if present. `insert` false: lookup only
// (returns 2 if absent).
template <bool kShared>
__device__ inline int probe_insert(uint32_t* t, uint32_t bits, uint32_t id, bool insert) {
  const uint32_t mask = (1u << bits) - 1u;
  uint32_t hsl = hash_slot(id, bits);
  for (uint32_t it = 0; it <= mask; ++it) {
    uint32_t cur = kShared ? t[hsl] : *(volatile uint32_t*)(t + hsl);
    if (cur == id) return 0;
    if (cur == kEmpty) {
      if (!insert) return 2;
      uint32_t old = atomicCAS(t + hsl, kEmpty, id);
      if (old == kEmpty) return 1;
      if (old == id) return 0;
    }
    hsl = (hsl + 1) & mask;
  }
  return insert ? 3 : 2;  // table full (not reached: load is capped at 3/4)
}

// Ascending bitonic sort of one u32 per lane.
__device__ inline uint32_t bitonic32(uint32_t key, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      uint32_t p = __shfl_xor_sync(kFull, key, j);
      bool up = (lane & k) == 0;
      bool lower = (lane & j) == 0;
      key = (lower == up) ? min(key, p) : max(key, p);
    }
  }
  return key;
}

__device__ inline int find_unchecked(const uint32_t* pool_id, int from, int sz, int lane) {
  for (int base = from & ~31; base < sz; base += 32) {
    int p = base + lane;
    bool ok = p >= from && p < sz && !(pool_id[p] & kChecked);
    uint32_t m = __ballot_sync(kFull, ok);
    if (m) return base + __ffs(m) - 1;
  }
  return sz;
}

// Integer SQ distance partial for one 16-byte chunk.
template <int QUANT>
struct QChunk;

template <>
struct QChunk<0> {  // SQ4: nibbles; per byte (q|0x80) - b never borrows, ^0x80 gives signed q-b
  uint32_t lo_or[4], hi_or[4];
  __device__ inline void load(const uint8_t* qcode, int chunk) {
    uint4 q = *(const uint4*)(qcode + chunk * 16);
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo_or[i] = (w[i] & 0x0F0F0F0Fu) | 0x80808080u;
      hi_or[i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | 0x80808080u;
    }
  }
  __device__ inline int dist(uint4 b) const {
    uint32_t w[4] = {b.x, b.y, b.z, b.w};
    int acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t blo = w[i] & 0x0F0F0F0Fu, bhi = (w[i] >> 4) & 0x0F0F0F0Fu;
      int dl = (int)((lo_or[i] - blo) ^ 0x80808080u);
      int dh = (int)((hi_or[i] - bhi) ^ 0x80808080u);
      acc = __dp4a(dl, dl, acc);
      acc = __dp4a(dh, dh, acc);
    }
    return acc;
  }
};

template <>
struct QChunk<1> {  // SQ8: |q-b| per byte, squared by dp4a
  uint32_t q[4];
  __device__ inline void load(const uint8_t* qcode, int chunk) {
    uint4 v = *(const uint4*)(qcode + chunk * 16);
    q[0] = v.x;
    q[1] = v.y;
    q[2] = v.z;
    q[3] = v.w;
  }
  __device__ inline int dist(uint4 b) const {
    uint32_t w[4] = {b.x, b.y, b.z, b.w};
    unsigned acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t d = __vabsdiffu4(q[i], w[i]);
      acc = __dp4a(d, d, acc);
    }
    return (int)acc;
  }
};

// ---------------------------------------------------------------------------
// The search kernel.
// ---------------------------------------------------------------------------
template <int QUANT, int CPL, int PT>
__global__ void __launch_bounds__(kWarpsPerBlock * 32) search_kernel(const SearchArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const WarpSmem s = carve(smem_raw + (size_t)wib * a.smem_per_warp, a, PT);
  const uint32_t slot = blockIdx.x * kWarpsPerBlock + wib;
  uint32_t* spill = a.spill ? a.spill + ((size_t)slot << a.spill_bits) : nullptr;
  const uint32_t H = 1u << a.hash_bits;
  const uint32_t h_limit = (H >> 2) * 3;
  const uint32_t S = 1u << a.spill_bits;
  const uint32_t s_limit = (S >> 2) * 3;
  constexpr int CPR = 32 / CPL;  // codes per gather round
  const int sub = lane & (CPL - 1);
  const int grp = lane / CPL;

  while (true) {
    unsigned long long qi_ = 0;
    if (lane == 0) qi_ = atomicAdd(a.counter, 1ull);
    const uint64_t qi = __shfl_sync(kFull, qi_, 0);
    if (qi >= a.nq) break;

    // 1. query to shared memory
    const float* qg = a.queries + qi * a.dim;
    for (uint32_t i = lane; i < a.dim_pad; i += 32) s.qf[i] = i < a.dim ? qg[i] : 0.0f;
    __syncwarp();
    int32_t status = 0;

    // 2. navigation descent (or the medoid)
    uint32_t entry = a.entry;
    float entry_f32 = 0.0f;
    uint32_t n_nav = 0;
    bool have_f32 = false;
    if (a.nav) {
      if (!nav_descend(a, s, lane, &entry, &entry_f32, &n_nav)) status = 2;
      have_f32 = true;
    }
    if (a.nav_only) {
      if (lane == 0) {
        a.ids[qi] = entry;
        a.dists[qi] = entry_f32;
        if (a.n_nav) a.n_nav[qi] = n_nav;
        if (a.status) a.status[qi] = status;
      }
      continue;
    }

    // 3. ef
    uint32_t ef = a.ef_fixed;
    if (a.adaptive) {
      if (!have_f32) {
        float d2, dummy;
        hw_l2_pair(s.qf, a.vec + (size_t)entry * a.dim, nullptr, a.dim, lane & 15, &d2, &dummy);
        entry_f32 = d2;
        n_nav += 1;
      }
      uint32_t e;
      if (a.n_samples <= 1) {
        e = a.ef_mid;
      } else {
        // rank = #samples < d (partition_point): the sorted samples are cut
        // into 32 segments; the segment heads locate the answer, one segment
        // is then counted.
        const uint32_t ns = a.n_samples;
        const uint32_t seg = (ns + 31) / 32;
        const uint32_t head = (uint32_t)lane * seg;
        const bool lt = head < ns && a.samples[head] < entry_f32;
        const int m = __popc(__ballot_sync(kFull, lt));
        uint32_t rank = 0;
        if (m > 0) {
          const uint32_t start = (uint32_t)(m - 1) * seg;
          const uint32_t end = min(ns, start + seg);
          uint32_t cnt = 0;
          for (uint32_t p0 = start; p0 < end; p0 += 32) {
            const uint32_t p = p0 + lane;
            cnt += __popc(__ballot_sync(kFull, p < end && a.samples[p] < entry_f32));
          }
          rank = start + cnt;
        }
        e = a.ef_table[rank];
      }
      ef = max(e, a.k);
    }
    if (ef == 0 || ef > 32u * PT) status = 3;  // RAVEN_Q_BAD_EF (host validation makes this unreachable)

    uint32_t vcount = 0, expansions = 0;
    int sz = 0;
    if (status != 3) {
      // encode the query
      if (QUANT == 0) {
        for (uint32_t b = lane; b < a.code_stride; b += 32) {
          uint32_t d0 = 2 * b, d1 = 2 * b + 1;
          uint32_t lo = d0 < a.dim ? quantize(s.qf[d0], a.q_inv[d0], a.q_neg[d0], a.levels) : 0u;
          uint32_t hi = d1 < a.dim ? quantize(s.qf[d1], a.q_inv[d1], a.q_neg[d1], a.levels) : 0u;
          s.qcode[b] = (uint8_t)(lo | (hi << 4));
        }
      } else {
        for (uint32_t b = lane; b < a.code_stride; b += 32)
          s.qcode[b] = b < a.dim ? (uint8_t)quantize(s.qf[b], a.q_inv[b], a.q_neg[b], a.levels) : (uint8_t)0;
      }
      // clear the visited table
      for (uint32_t i = lane * 4; i < H; i += 128) *(uint4*)(s.ht + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
      __syncwarp();
      QChunk<QUANT> qc;
      qc.load(s.qcode, sub);

      bool spilled = false;
      uint32_t tcount = 0, scount = 0;
      // 4. entry
      if (lane == 0) {
        probe_insert<true>(s.ht, a.hash_bits, entry, true);
        s.cand_id[0] = entry;
      }
      tcount = 1;
      if (a.history && lane == 0 && a.hist_cap > 0) a.history[qi * a.hist_cap] = entry;
      vcount = 1;
      __syncwarp();
      {
        int pd = 0;
        if (grp == 0) {
          uint4 v = __ldg((const uint4*)(a.codes + (size_t)entry * a.code_stride) + sub);
          pd = qc.dist(v);
        }
#pragma unroll
        for (int o = 1; o < CPL; o <<= 1) pd += __shfl_xor_sync(kFull, pd, o);
        if (lane == 0) {
          s.pool_d[0] = (uint32_t)pd;
          s.pool_id[0] = entry;
        }
      }
      sz = 1;
      __syncwarp();
      int cursor = 0;
      uint32_t pref_node = kSent;
      uint32_t pref_row[4];
      const uint32_t RL = a.r_pad >> 5;

      while (cursor < sz) {
        const uint32_t node = s.pool_id[cursor];
        __syncwarp();
        if (lane == 0) s.pool_id[cursor] = node | kChecked;
        __syncwarp();
        ++expansions;
        // neighbours (speculatively prefetched row of the next pool entry)
        uint32_t row[4];
        const uint32_t* rg = a.adj + (size_t)node * a.r_pad + lane;
        if (node == pref_node) {
#pragma unroll
          for (int r = 0; r < 4; ++r) row[r] = pref_row[r];
        } else {
#pragma unroll
          for (int r = 0; r < 4; ++r) row[r] = (uint32_t)r < RL ? __ldg(rg + 32 * r) : kSent;
        }
        {
          int nxt = find_unchecked(s.pool_id, cursor + 1, sz, lane);
          if (nxt < sz) {
            pref_node = s.pool_id[nxt] & ~kChecked;
            const uint32_t* pg = a.adj + (size_t)pref_node * a.r_pad + lane;
#pragma unroll
            for (int r = 0; r < 4; ++r) pref_row[r] = (uint32_t)r < RL ? __ldg(pg + 32 * r) : kSent;
          } else {
            pref_node = kSent;
          }
        }
        bool ended = false;  // first SENTINEL seen: degree reached
        bool overflow = false;
        for (uint32_t seg = 0; seg < RL && !ended; ++seg) {
          uint32_t id = seg == 0 ? row[0] : seg == 1 ? row[1] : seg == 2 ? row[2] : row[3];
          uint32_t sm = __ballot_sync(kFull, id == kSent);
          int deg = sm ? __ffs(sm) - 1 : 32;
          if (sm) ended = true;
          bool valid = lane < deg;
          // duplicates inside the row: the first (lowest lane) occurrence counts
          uint32_t peers = __match_any_sync(kFull, valid ? id : kSent);
          bool leader = valid && (__ffs(peers) - 1 == lane);
          if (!spilled && tcount + 32 > h_limit) {
            if (spill == nullptr) {
              overflow = true;
              break;
            }
            // switch to the global spill table: clear it first
            for (uint32_t i = lane * 4; i < S; i += 128) *(uint4*)(spill + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
            __syncwarp();
            spilled = true;
          }
          bool is_new = false;
          if (leader) {
            if (!spilled) {
              is_new = probe_insert<true>(s.ht, a.hash_bits, id, true) == 1;
            } else {
              int r = probe_insert<true>(s.ht, a.hash_bits, id, false);
              if (r == 2) is_new = probe_insert<false>(spill, a.spill_bits, id, true) == 1;
            }
          }
          uint32_t newm = __ballot_sync(kFull, is_new);
          int nn = __popc(newm);
          if (nn == 0) continue;
          if (!spilled) tcount += nn;
          else scount += nn;
          int rank = __popc(newm & lanemask_lt(lane));
          if (is_new) {
            s.cand_id[rank] = id;
            if (a.history && vcount + rank < a.hist_cap) a.history[qi * a.hist_cap + vcount + rank] = id;
          }
          vcount += nn;
          __syncwarp();
          // gather codes of the new neighbours, integer distances
          uint4 data[CPL];
#pragma unroll
          for (int r = 0; r < CPL; ++r) {
            int idx = r * CPR + grp;
            if (idx < nn) {
              uint32_t cid = s.cand_id[idx];
              data[r] = __ldg((const uint4*)(a.codes + (size_t)cid * a.code_stride) + sub);
            } else {
              data[r] = make_uint4(0, 0, 0, 0);
            }
          }
#pragma unroll
          for (int r = 0; r < CPL; ++r) {
            if (r * CPR < nn) {
              int pdist = qc.dist(data[r]);
#pragma unroll
              for (int o = 1; o < CPL; o <<= 1) pdist += __shfl_xor_sync(kFull, pdist, o);
              int idx = r * CPR + grp;
              if (sub == 0 && idx < nn) s.cand_d[idx] = (uint32_t)pdist;
            }
          }
          __syncwarp();
          const uint32_t my_d = lane < nn ? s.cand_d[lane] : 0xffffffffu;
          const uint32_t my_id = lane < nn ? s.cand_id[lane] : kSent;
          // merge into the pool (LinearPool::insert semantics, batched)
          const bool full = sz == (int)ef;
          const uint32_t worst = full ? s.pool_d[sz - 1] : 0xffffffffu;
          const bool acc = lane < nn && (!full || my_d < worst);
          const uint32_t am = __ballot_sync(kFull, acc);
          const int na = __popc(am);
          __syncwarp();
          if (na > 0) {
            uint32_t key = acc ? ((my_d << 5) | (uint32_t)lane) : 0xffffffffu;
            key = bitonic32(key, lane);
            const uint32_t cd = key >> 5;
            const uint32_t cid = __shfl_sync(kFull, my_id, (int)(key & 31));
            if (lane < na) s.cand_d[lane] = cd;
            __syncwarp();
            int cpos = 0, ub = 0;
            if (lane < na) {
              int lo = 0, hi = sz;  // # pool entries <= cd
              while (lo < hi) {
                int mid = (lo + hi) >> 1;
                if (s.pool_d[mid] <= cd) lo = mid + 1;
                else hi = mid;
              }
              ub = lo;
              cpos = lane + ub;
            }
            const int start = __shfl_sync(kFull, ub, 0);
            uint32_t rd[PT], ri[PT];
            int rnp[PT];
#pragma unroll
            for (int t = 0; t < PT; ++t) {
              int p = start + lane + 32 * t;
              rnp[t] = 1 << 30;
              if (p < sz) {
                rd[t] = s.pool_d[p];
                ri[t] = s.pool_id[p];
                int lo = 0, hi = na;  // # candidates < pool distance
                while (lo < hi) {
                  int mid = (lo + hi) >> 1;
                  if (s.cand_d[mid] < rd[t]) lo = mid + 1;
                  else hi = mid;
                }
                rnp[t] = p + lo;
              }
            }
            __syncwarp();
#pragma unroll
            for (int t = 0; t < PT; ++t) {
              if (rnp[t] < (int)ef) {
                s.pool_d[rnp[t]] = rd[t];
                s.pool_id[rnp[t]] = ri[t];
              }
            }
            if (lane < na && cpos < (int)ef) {
              s.pool_d[cpos] = cd;
              s.pool_id[cpos] = cid;
            }
            __syncwarp();
            sz = min(sz + na, (int)ef);
            if (start < cursor) cursor = start;
          }
          if (spilled && scount > s_limit) {
            overflow = true;
            break;
          }
        }
        if (overflow) {
          status = 1;
          break;
        }
        cursor = find_unchecked(s.pool_id, cursor, sz, lane);
      }
    }

    // 5. rerank: exact f32 L2 of the first min(k*rr, sz) pool entries
    const uint64_t krr = (uint64_t)a.k * (uint64_t)max(a.rr, 1u);
    const uint64_t krr_k = krr > (uint64_t)a.k ? krr : (uint64_t)a.k;
    const int rn = (int)(krr_k < (uint64_t)sz ? krr_k : (uint64_t)sz);
    float* rdist = (float*)s.ht;
    {
      const int h = lane >> 4, j = lane & 15;
      for (int e0 = 0; e0 < rn; e0 += 4) {
        int ea = e0 + h, eb = e0 + 2 + h;
        const float* ra = ea < rn ? a.vec + (size_t)(s.pool_id[ea] & ~kChecked) * a.dim : nullptr;
        const float* rb = eb < rn ? a.vec + (size_t)(s.pool_id[eb] & ~kChecked) * a.dim : nullptr;
        float da, db;
        hw_l2_pair(s.qf, ra, rb, a.dim, j, &da, &db);
        if (j == 0) {
          if (ea < rn) rdist[ea] = da;
          if (eb < rn) rdist[eb] = db;
        }
      }
    }
    __syncwarp();
    const int kout = min((int)a.k, rn);
    // stable ascending order by (total_cmp(dist), pool position)
    for (int i = lane; i < rn; i += 32) {
      const uint32_t ki = total_order_key(rdist[i]);
      int rank = 0;
      for (int jj = 0; jj < rn; ++jj) {
        const uint32_t kj = total_order_key(rdist[jj]);
        rank += (kj < ki) || (kj == ki && jj < i);
      }
      if (rank < kout) {
        a.ids[qi * a.k + rank] = s.pool_id[i] & ~kChecked;
        if (a.dists) a.dists[qi * a.k + rank] = rdist[i];
      }
    }
    for (int r = kout + lane; r < (int)a.k; r += 32) {
      a.ids[qi * a.k + r] = 0;
      if (a.dists) a.dists[qi * a.k + r] = 0.0f;
    }
    if (lane == 0) {
      if (a.counts) a.counts[qi] = (uint32_t)kout;
      if (a.visited) a.visited[qi] = vcount;
      if (a.ef_used) a.ef_used[qi] = ef;
      if (a.status) a.status[qi] = status;
      if (a.n_nav) a.n_nav[qi] = n_nav;
      if (a.expansions) a.expansions[qi] = expansions;
      if (a.hist_len) a.hist_len[qi] = vcount;
    }
    __syncwarp();
  }
}

}  // namespace raven_dev
