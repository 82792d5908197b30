// Small-batch search: one CTA of four warps per query.
//
// A batch smaller than the GPU leaves most SMs idle under the persistent
// one-warp-per-query kernel, and each query's latency is one warp's chain of
// dependent expansions. Here each query gets a whole CTA:
//   * VIS true (visited count or order requested): the visited set lives in a
//     shared-memory table of 2^14 slots (64 KB, over 14,000 visits; three CTAs
//     fit an SM), so a query does not reach the global spill levels in
//     practice (they remain, for exactness, behind the same capacity checks
//     as in the batch kernel). VIS false: no visited set; pool membership
//     decides new neighbours, with the same results (the argument is in
//     search_kernel.cuh), and a CTA needs only its pool and staging rows;
//   * the four warps share each expansion's work: with the visited set every
//     warp gathers the codes of eight of the row's neighbours and computes
//     their distances while warp 0 also runs the visited set; without it
//     warps 1-3 take eleven each while warp 0 finds the next unexpanded entry
//     and issues its prefetch; warp 0 then merges the pool. The navigation
//     descent and the rerank stage and score 16 rows per round across the
//     warps.
// The search itself is the batch kernel's (search_kernel.cuh): the same
// navigation descent, AdaptiveEf rank lookup, visited order, LinearPool merge
// and rerank tie rule, so results are identical (src/graph/vamana.rs:786-861,
// 1772-1829, src/graph/linear_pool.rs:100-171, src/graph/refiner.rs:45-61).
#pragma once
#include "search_kernel.cuh"

namespace raven_dev {

constexpr int kCtaWarps = 4;
constexpr int kCtaThreads = 32 * kCtaWarps;
constexpr int kCtaRowsPerWarp = 4;  // rows a warp stages per round (descent, rerank)
constexpr uint32_t kCtaHashBits = 14;

// Shared memory of one query (every piece 16-byte aligned).
struct CtaSmem {
  float* qf;          // dim_pad floats, lane-major
  uint8_t* qcode;     // code_stride bytes
  uint32_t* pool_d;   // pool_cap
  uint32_t* pool_id;  // pool_cap
  uint32_t* cand_id;  // 32: navigation edges / rerank ids
  uint32_t* cand_d;   // 2 x 32: beam distances of a segment's neighbours (by segment parity)
  float* nd;          // 32: navigation / rerank distances
  uint32_t* rowbuf;   // 2 x r_pad: adjacency rows prefetched by cp.async
  uint32_t* crow;     // 2 x r_pad: the row being expanded, for every warp (by expansion parity)
  uint32_t* ctl;      // 16 control words shared by the warps
  uint8_t* fbuf;      // 2 x 32 x code_stride: first 32 neighbour codes of a predicted expansion
  uint32_t* ht;       // cta_table_bytes: visited table (1 << hash_bits); row staging outside the beam
};

// The last region holds the visited table during the beam and the row staging
// of cta_rows_dist (kCtaWarps x kCtaRowsPerWarp rows) outside it: it is sized
// for the larger of the two (hash_bits 0: no visited table).
__host__ __device__ inline uint32_t cta_table_bytes(uint32_t dim_pad, uint32_t hash_bits) {
  const uint32_t table = hash_bits ? align16((1u << hash_bits) * 4) : 0u;
  const uint32_t stage = (uint32_t)(kCtaWarps * kCtaRowsPerWarp) * dim_pad * 4;
  return table > stage ? table : stage;
}

__host__ __device__ inline uint32_t cta_smem_bytes(uint32_t dim_pad, uint32_t code_stride, uint32_t pool_cap,
                                                   uint32_t hash_bits, uint32_t r_pad) {
  return align16(dim_pad * 4) + align16(code_stride) + 2 * align16(pool_cap * 4) + 128 + 256 + 128 +
         2 * r_pad * 4 + 2 * r_pad * 4 + 64 + 64 * code_stride + cta_table_bytes(dim_pad, hash_bits);
}

__device__ inline CtaSmem cta_carve(uint8_t* base, const SearchArgs& a) {
  CtaSmem s;
  uint32_t o = 0;
  s.qf = (float*)(base + o);
  o += align16(a.dim_pad * 4);
  s.qcode = base + o;
  o += align16(a.code_stride);
  s.pool_d = (uint32_t*)(base + o);
  o += align16(a.pool_cap * 4);
  s.pool_id = (uint32_t*)(base + o);
  o += align16(a.pool_cap * 4);
  s.cand_id = (uint32_t*)(base + o);
  o += 128;
  s.cand_d = (uint32_t*)(base + o);
  o += 256;
  s.nd = (float*)(base + o);
  o += 128;
  s.rowbuf = (uint32_t*)(base + o);
  o += 2 * a.r_pad * 4;
  s.crow = (uint32_t*)(base + o);
  o += 2 * a.r_pad * 4;
  s.ctl = (uint32_t*)(base + o);
  o += 64;
  s.fbuf = base + o;
  o += 64 * a.code_stride;
  s.ht = (uint32_t*)(base + o);
  return s;
}

// Distances of `n` rows (ids[r] resolved by row_ptr) into out[0..n): rounds of
// kCtaWarps x kCtaRowsPerWarp rows, warp w staging rows w*RW .. w*RW+RW-1 of
// the round in its own slice of `stage` and scoring them two at a time (one
// per half-warp, hw_dist's summation order). Every thread of the CTA calls;
// the caller synchronises the CTA before reading `out`.
template <class RowPtr>
__device__ inline void cta_rows_dist(const float* qf, float* stage, const uint32_t* ids, int n, uint32_t dim,
                                     uint32_t C, uint32_t rem, RowPtr row_ptr, float* out, int w, int lane) {
  constexpr int RW = kCtaRowsPerWarp;
  float* my = stage + (size_t)w * RW * dim;
  const int h = lane >> 4, j = lane & 15;
  for (int b0 = 0; b0 < n; b0 += kCtaWarps * RW) {
    const int r0 = b0 + w * RW;
    const int nb = max(0, min(RW, n - r0));
    if (nb > 0) {
      stage_rows(my, nb, dim, [&](uint32_t r) { return row_ptr(ids[r0 + r]); }, lane);
      for (int p = 0; p < nb; p += 2) {
        const int r = min(p + h, nb - 1);
        const float d = hw_dist(qf, my + (size_t)r * dim, C, rem, j);
        if (j == 0 && p + h < nb) out[r0 + p + h] = d;
      }
    }
    __syncwarp();
  }
}

// Navigation descent (src/graph/navigation.rs:609-653) with the CTA: warp 0
// reads each node's edges and makes the move decision exactly as nav_descend
// does; the candidates' distances are computed by all warps.
__device__ inline bool cta_nav_descend(const SearchArgs& a, const CtaSmem& s, int w, int lane, uint32_t* out_gid,
                                       float* out_d, uint32_t* out_evals) {
  auto row_of = [&](uint32_t hd) -> const float* {
    return (hd & kGidBit) ? a.vec + (size_t)(hd & ~kGidBit) * a.dim : a.nav_vec + (size_t)hd * a.dim;
  };
  float* stage = (float*)s.ht;
  uint32_t u = a.nav_entry_h;
  if (w == 0 && lane == 0) s.cand_id[0] = u;
  __syncthreads();
  cta_rows_dist(s.qf, stage, s.cand_id, 1, a.dim, a.vec_c, a.vec_rem, row_of, s.nd, w, lane);
  __syncthreads();
  float du = s.nd[0];
  uint32_t evals = 1, steps = 0;
  bool ok = true;
  const uint32_t K = a.nav_k;
  for (int level = (int)a.nav_max_level; level >= 1 && ok; --level) {
    while (true) {
      // warp 0: this node's edges at this level (ctl[0] = count, 0: level done)
      uint32_t v = kSent;
      if (w == 0) {
        uint32_t cnt = 0;
        if (++steps > kNavStepLimit) {
          ok = false;
        } else if (!(u & kGidBit) && (uint32_t)level <= a.nav_stride_levels) {
          v = (uint32_t)lane < K ? a.nav_e[((size_t)u * a.nav_stride_levels + (level - 1)) * K + lane] : kSent;
          const uint32_t sm = __ballot_sync(kFull, v == kSent);
          cnt = sm ? (uint32_t)(__ffs(sm) - 1) : 32u;
          if ((uint32_t)lane < cnt) s.cand_id[lane] = v;
        }
        if (lane == 0) {
          s.ctl[0] = cnt;
          s.ctl[1] = ok ? 1u : 0u;
        }
      }
      __syncthreads();
      const uint32_t cnt = s.ctl[0];
      ok = s.ctl[1] != 0;
      if (cnt == 0) break;
      cta_rows_dist(s.qf, stage, s.cand_id, (int)cnt, a.dim, a.vec_c, a.vec_rem, row_of, s.nd, w, lane);
      __syncthreads();
      // every warp takes the same decision from the same data
      {
        const float d = (uint32_t)lane < cnt ? s.nd[lane] : __int_as_float(0x7f800000);
        const uint32_t vv = (uint32_t)lane < cnt ? s.cand_id[lane] : kSent;
        unsigned long long key = ((unsigned long long)__float_as_uint(d) << 32) | (uint32_t)lane;
        if ((uint32_t)lane >= cnt) key = ~0ull;
        unsigned long long pre = key;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long t = __shfl_up_sync(kFull, pre, o);
          if (lane >= o && t < pre) pre = t;
        }
        unsigned long long excl = __shfl_up_sync(kFull, pre, 1);
        if (lane == 0) excl = ~0ull;
        const bool moved = excl != ~0ull && __uint_as_float((uint32_t)(excl >> 32)) < du;
        const uint32_t excl_v = __shfl_sync(kFull, vv, moved ? (int)(excl & 31) : 0);
        const uint32_t run_u = moved ? excl_v : u;
        evals += __popc(__ballot_sync(kFull, (uint32_t)lane < cnt && vv != run_u));
        const unsigned long long best = __shfl_sync(kFull, pre, 31);
        const float bd = __uint_as_float((uint32_t)(best >> 32));
        const uint32_t best_v = __shfl_sync(kFull, vv, (int)(best & 31));
        __syncthreads();  // cand_id / nd are rewritten by the next step
        if (best != ~0ull && bd < du) {
          du = bd;
          u = best_v;
        } else {
          break;
        }
      }
    }
  }
  *out_gid = (u & kGidBit) ? (u & ~kGidBit) : a.nav_gid[u];
  *out_d = du;
  *out_evals = evals;
  return ok;
}

// The small-batch kernel: grid = number of queries, kCtaThreads threads.
// QUANT 0 (SQ4) or 1 (SQ8); f16 reranks and the f32 traversal use the batch
// kernel. Level-A/B spill tables of query q start at a.spill + q * (9 <<
// spill_bits) (only touched by a query that fills the shared table).
template <int QUANT, int CPL, bool VIS>
__global__ void __launch_bounds__(kCtaThreads, 1) search_cta_kernel(const SearchArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const CtaSmem s = cta_carve(smem_raw, a);
  const uint64_t qi = blockIdx.x;
  if (qi >= a.nq) return;
  const uint32_t pool_cap = a.pool_cap;
  uint32_t* spill = a.spill ? a.spill + qi * (9ull << a.spill_bits) : nullptr;
  uint32_t* spill_b = a.spill ? spill + (1ull << a.spill_bits) : nullptr;
  const uint32_t H = 1u << a.hash_bits;
  const uint32_t h_limit = H - (H >> 3);
  const uint32_t S = 1u << a.spill_bits;
  const uint32_t s_limit = (S >> 2) * 3;
  const uint32_t SB = S << 3;
  const uint32_t sb_limit = (SB >> 2) * 3;
  constexpr int CPR = 32 / CPL;                              // codes per warp round
  // neighbours a gathering warp scores per segment: with the visited set all
  // four warps take eight (warp 0 also runs the visited set); without it
  // warps 1-3 take eleven, and warp 0 meanwhile finds the next entry and
  // issues its prefetch
  constexpr int kPer = VIS ? 8 : 11;
  constexpr int ROUNDS = (kPer + CPR - 1) / CPR;              // rounds for a warp's share
  const int gw = VIS ? w : w - 1;                             // gathering-warp index, -1: none
  const int sub = lane & (CPL - 1);
  const int grp = lane / CPL;
  auto vec_row = [&](uint32_t id) -> const float* { return a.vec + (size_t)id * a.dim; };

  // 1. query -> shared memory (lane-major)
  const float* qg = a.queries + qi * a.dim;
  for (uint32_t i = tid; i < a.dim_pad; i += kCtaThreads) {
    if (i < a.dim) s.qf[lane_major_pos(i, a.vec_c)] = qg[i];
    else s.qf[i] = 0.0f;
  }
  __syncthreads();
  int32_t status = 0;

  // 2. navigation descent (or the medoid)
  uint32_t entry = a.entry;
  float entry_f32 = 0.0f;
  uint32_t n_nav = 0;
  bool have_f32 = false;
  if (a.nav) {
    if (!cta_nav_descend(a, s, w, lane, &entry, &entry_f32, &n_nav)) status = 2;
    have_f32 = true;
  }

  // 3. ef (every warp computes the same value)
  uint32_t ef = a.ef_fixed;
  if (a.adaptive) {
    if (!have_f32) {
      if (w == 0 && lane == 0) s.cand_id[0] = entry;
      __syncthreads();
      cta_rows_dist(s.qf, (float*)s.ht, s.cand_id, 1, a.dim, a.vec_c, a.vec_rem, vec_row, s.nd, w, lane);
      __syncthreads();
      entry_f32 = s.nd[0];
      n_nav += 1;
    }
    uint32_t e;
    if (a.n_samples <= 1) {
      e = a.ef_mid;
    } else {
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
  if (ef == 0 || ef > pool_cap) status = 3;

  uint32_t vcount = 0, expansions = 0;
  int sz = 0;
  if (status != 3) {
    // encode the query
    if (QUANT == 0) {
      for (uint32_t b = tid; b < a.code_stride; b += kCtaThreads) {
        const uint32_t d0 = 2 * b, d1 = 2 * b + 1;
        const uint32_t lo =
            d0 < a.dim ? quantize(s.qf[lane_major_pos(d0, a.vec_c)], a.q_inv[d0], a.q_neg[d0], a.levels) : 0u;
        const uint32_t hi =
            d1 < a.dim ? quantize(s.qf[lane_major_pos(d1, a.vec_c)], a.q_inv[d1], a.q_neg[d1], a.levels) : 0u;
        s.qcode[b] = (uint8_t)(lo | (hi << 4));
      }
    } else {
      for (uint32_t b = tid; b < a.code_stride; b += kCtaThreads)
        s.qcode[b] =
            b < a.dim ? (uint8_t)quantize(s.qf[lane_major_pos(b, a.vec_c)], a.q_inv[b], a.q_neg[b], a.levels)
                      : (uint8_t)0;
    }
    if (VIS) {
      // clear the visited table (the descent's staging rows are done)
      for (uint32_t i = tid * 4; i < H; i += 4 * kCtaThreads)
        *(uint4*)(s.ht + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
    }
    __syncthreads();  // the query code (and the table) are written before any warp reads them
    QChunk<QUANT> qc;
    qc.load(s.qcode, sub);

    // warp 0's search state
    int level = 0;
    uint32_t tcount = 0, scount = 0;
    int cursor = 0;
    uint32_t pref_node = kSent;
    int pbuf = 0;
    int eb = 1;  // buffer of an early prediction during this expansion
    const uint32_t RL = a.r_pad >> 5;
    // Without the visited set, warp 0 prefetches the first 32 neighbour codes
    // of each predicted expansion (stored beside the rows) with its row, into
    // one of two buffers; the expansion that finds its codes there reads them
    // instead of gathering (ctl[8 + parity]: buffer + 1, 0 = gather), and new
    // prefetches go to the other buffer until every warp has read them.
    const bool use_fat = !VIS && a.fat != nullptr;
    const uint32_t fb_bytes = 32u * a.code_stride;
    if (w == 0) {
      // 4. entry
      if (VIS) {
        if (lane == 0) shared_insert2(s.ht, a.hash_bits - 2, entry);
        tcount = 1;
        if (a.history && lane == 0 && a.hist_cap > 0) a.history[qi * a.hist_cap] = entry;
      }
      vcount = 1;
      int pd = 0;
      if (grp == 0) {
        const uint4 v = __ldg((const uint4*)(a.codes + (size_t)entry * a.code_stride) + sub);
        pd = qc.dist(v);
      }
#pragma unroll
      for (int o = 1; o < CPL; o <<= 1) pd += __shfl_xor_sync(kFull, pd, o);
      if (lane == 0) {
        s.pool_d[0] = (uint32_t)pd;
        s.pool_id[0] = entry;
      }
      sz = 1;
      __syncwarp();
    }

    // Control words are double-buffered by the parity of a counter every warp
    // keeps in step, so that warp 0 never overwrites a word a slower warp has
    // yet to read: ctl[it & 1] "expand" flag, ctl[2 + par] overflow flag.
    uint32_t segs_done = 0;  // segments processed so far (cand_d / ctl parity)
    uint32_t it = 0;         // expansions started
    while (true) {
      // warp 0: pop the first unexpanded entry, publish its row
      int nxt = 0;
      int cur = -1;  // warp 0: prefetch buffer holding this expansion's row, or -1
      if (w == 0) {
        if (cursor < sz) {
          const uint32_t node = s.pool_id[cursor];
          __syncwarp();
          if (lane == 0) s.pool_id[cursor] = node | kChecked;
          ++expansions;
          cp_async_wait_all();
          __syncwarp();
          // a predicted row (and its codes) is read where it was prefetched;
          // otherwise warp 0 copies the row to crow's half for this
          // expansion's parity
          cur = node == pref_node ? pbuf : -1;
          if (cur < 0) {
            uint32_t* cw = s.crow + (it & 1) * a.r_pad;
            for (uint32_t i = lane; i < a.r_pad; i += 32) cw[i] = __ldg(a.adj + (size_t)node * a.r_pad + i);
          }
          if (lane == 0) s.ctl[8 + (it & 1)] = (uint32_t)(cur + 1);
        }
        if (lane == 0) s.ctl[it & 1] = cursor < sz ? 1u : 0u;
      }
      __syncthreads();
      if (s.ctl[it & 1] == 0) break;
      if (w == 0) {
        // while the other warps gather: the next unexpanded entry after this
        // one, and the prefetch of its row (and codes) into the buffer this
        // expansion does not read
        nxt = find_unchecked(s.pool_id, cursor + 1, sz, lane);
        const int nb = cur == 0 ? 1 : 0;  // the next in pool order; an early prediction takes the other
        eb = 1 - nb;
        if (nxt < sz) {
          pref_node = s.pool_id[nxt] & ~kChecked;
          if (use_fat) prefetch_fat(a.fat, a.r_pad, a.code_stride, s.fbuf + nb * fb_bytes, pref_node, lane, 32);
          prefetch_row(a.adj, a.r_pad, s.rowbuf + nb * a.r_pad, pref_node, lane);
          pbuf = nb;
        } else {
          pref_node = kSent;
        }
      }
      // the row: prefetch buffer + 1, or 0 for crow; the codes come from the
      // same buffer when they were prefetched with it
      const uint32_t rsel = s.ctl[8 + (it & 1)];
      const uint32_t* cr = rsel ? s.rowbuf + (rsel - 1) * a.r_pad : s.crow + (it & 1) * a.r_pad;
      const uint32_t fsel = use_fat ? rsel : 0u;
      ++it;

      uint32_t row[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) row[r] = (uint32_t)r < RL ? cr[32 * r + lane] : kSent;
      bool early = false;
      bool overflow = false;
      int first_insert = 0x7fffffff;
      for (uint32_t seg = 0; seg < RL; ++seg) {
        const uint32_t id = seg == 0 ? row[0] : seg == 1 ? row[1] : seg == 2 ? row[2] : row[3];
        const uint32_t sm = __ballot_sync(kFull, id == kSent);
        const int deg = sm ? __ffs(sm) - 1 : 32;
        if (deg == 0) break;  // the row ended at the previous segment
        const uint32_t par = segs_done & 1;
        uint32_t* cd = s.cand_d + 32 * par;
        ++segs_done;
        // gathering warps: codes of neighbours kPer gw .. kPer gw + kPer - 1 of this segment
        uint4 data[ROUNDS];
        int idxr[ROUNDS];
#pragma unroll
        for (int r = 0; r < ROUNDS; ++r) {
          const int loc = r * CPR + grp;  // neighbour within this warp's share
          const int idx = kPer * gw + loc;
          idxr[r] = (gw >= 0 && loc < kPer && idx < deg) ? idx : -1;
          if (gw < 0) {  // warp 0 without the visited set: no share
            data[r] = make_uint4(0, 0, 0, 0);
            continue;
          }
          const uint32_t cid = __shfl_sync(kFull, id, idx & 31);
          const uint32_t c = idxr[r] >= 0 ? cid : 0u;  // address always in range
          if (seg == 0 && fsel != 0)  // the prefetched copy (slot idx & 31 is always in the buffer)
            data[r] = *((const uint4*)(s.fbuf + (fsel - 1) * fb_bytes + (size_t)(idx & 31) * a.code_stride) + sub);
          else
            data[r] = __ldg((const uint4*)(a.codes + (size_t)c * a.code_stride) + sub);
        }
        // warp 0: the visited set, in adjacency order (the batch kernel's levels)
        bool is_new = false;
        const bool valid = lane < deg;
        if (VIS && w == 0) {
          if (level == 0 && tcount + 32 > h_limit) {
            if (spill == nullptr) {
              overflow = true;
            } else {
              for (uint32_t i = lane * 4; i < S; i += 128)
                *(uint4*)(spill + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
              __syncwarp();
              level = 1;
            }
          } else if (level == 1 && scount + 32 > s_limit) {
            for (uint32_t i = lane * 4; i < SB; i += 128)
              *(uint4*)(spill_b + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
            __syncwarp();
            level = 2;
            scount = 0;
          } else if (level == 2 && scount + 32 > sb_limit) {
            overflow = true;
          }
          if (!overflow) {
            if (level == 0) {
              const int r = valid ? shared_insert2(s.ht, a.hash_bits - 2, id) : 0;
              is_new = r == 1;
              const bool to_spill = r == 3;
              if (__any_sync(kFull, to_spill)) {
                if (spill == nullptr) {
                  overflow = true;
                } else {
                  for (uint32_t i = lane * 4; i < S; i += 128)
                    *(uint4*)(spill + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
                  __syncwarp();
                  level = 1;
                  const uint32_t sbk = hash_slot(id, a.spill_bits - 2);
                  const uint4 sv = to_spill ? __ldcv((const uint4*)(spill + 4 * sbk))
                                            : make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
                  is_new |= spill_insert_warp(spill, a.spill_bits, id, to_spill, sbk, sv, lane);
                }
              }
            } else if (level == 1) {
              const uint32_t sbk = hash_slot(id, a.spill_bits - 2);
              uint4 sv = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
              if (valid) sv = __ldcv((const uint4*)(spill + 4 * sbk));
              const bool need = valid && !shared_has2(s.ht, a.hash_bits - 2, id);
              is_new = spill_insert_warp(spill, a.spill_bits, id, need, sbk, sv, lane);
            } else if (valid && !shared_has2(s.ht, a.hash_bits - 2, id)) {
              is_new = probe_level_b(spill, spill_b, a.spill_bits, id);
            }
          }
          const uint32_t newm = __ballot_sync(kFull, is_new);
          const int nn = __popc(newm);
          if (level == 0) tcount += nn;
          else scount += nn;
          if (a.history && is_new) {
            const uint32_t pos = vcount + __popc(newm & lanemask_lt(lane));
            if (pos < a.hist_cap) a.history[qi * a.hist_cap + pos] = id;
          }
          vcount += nn;
          if (lane == 0) s.ctl[2 + par] = overflow ? 1u : 0u;
        }
        // gathering warps: distances of their share
#pragma unroll
        for (int r = 0; r < ROUNDS; ++r) {
          if (gw < 0) break;
          int pdist = qc.dist(data[r]);
#pragma unroll
          for (int o = 1; o < CPL; o <<= 1) pdist += __shfl_xor_sync(kFull, pdist, o);
          if (sub == 0 && idxr[r] >= 0) cd[idxr[r]] = (uint32_t)pdist;
        }
        __syncthreads();
        if (VIS && s.ctl[2 + par] != 0) {
          overflow = true;
          break;
        }
        if (w == 0) {
          // warp 0: LinearPool insert of the new neighbours, batched (as in the batch kernel)
          const bool cand = VIS ? is_new : valid;
          const uint32_t my_d = cand ? cd[lane] : 0xffffffffu;
          const bool full = sz == (int)ef;
          const uint32_t worst = full ? s.pool_d[sz - 1] : 0xffffffffu;
          bool acc = cand && (!full || my_d < worst);
          int lo = 0;  // # pool entries <= my_d (ties: pool first)
          if (acc) {
            lo = pool_upper_bound4(s.pool_d, sz, my_d);
            // without the visited set: a neighbour already in the pool sits
            // in the run of equal distances ending at lo - 1
            if (!VIS)
              for (int j = lo - 1; j >= 0 && s.pool_d[j] == my_d; --j)
                if ((s.pool_id[j] & ~kChecked) == id) {
                  acc = false;
                  break;
                }
          }
          const uint32_t am = __ballot_sync(kFull, acc);
          const int na = __popc(am);
          // (no sync needed here: the chunk moves sync before their first write)
          if (na > 0) {
            int cpos = acc ? lo : 0x7fffffff;
            const int start = (int)__reduce_min_sync(kFull, (unsigned)cpos);
            if (start <= min(nxt, first_insert)) {
              const uint32_t dmin = __reduce_min_sync(kFull, acc ? my_d : 0xffffffffu);
              pref_node = __shfl_sync(kFull, id, __ffs(__ballot_sync(kFull, acc && my_d == dmin)) - 1);
              if (early) {
                cp_async_wait_all();
                __syncwarp();
              }
              if (use_fat) prefetch_fat(a.fat, a.r_pad, a.code_stride, s.fbuf + eb * fb_bytes, pref_node, lane, 32);
              prefetch_row(a.adj, a.r_pad, s.rowbuf + eb * a.r_pad, pref_node, lane);
              pbuf = eb;
              early = true;
            }
            // rank among the accepted by (distance, lane), from the row's
            // distances in shared memory: 32 independent compares instead of
            // a chain of shuffles (an accepted lane's my_d is cd[lane])
            int crank = 0;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const uint4 q4 = *(const uint4*)(cd + 4 * j4);
              const uint32_t dq[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int jl = 4 * j4 + u;
                crank += (int)((am >> jl) & 1u) & ((dq[u] < my_d) | ((dq[u] == my_d) & (jl < lane)));
              }
            }
            if (acc) cpos += crank;
            const int nsz = min(sz + na, (int)ef);
            for (int t = (nsz - 1) >> 5; t >= (start >> 5); --t) {
              const int base = 32 * t;
              const uint32_t cw =
                  __reduce_or_sync(kFull, (acc && cpos >= base && cpos < base + 32) ? 1u << (cpos - base) : 0u);
              const int below = __popc(__ballot_sync(kFull, acc && cpos < base));
              const int j = base + lane;
              const bool mv = j >= start && j < nsz && !((cw >> lane) & 1u);
              uint32_t vd = 0, vi = 0;
              if (mv) {
                const int src = j - below - __popc(cw & lanemask_lt(lane));
                vd = s.pool_d[src];
                vi = s.pool_id[src];
              }
              __syncwarp();
              if (mv) {
                s.pool_d[j] = vd;
                s.pool_id[j] = vi;
              }
              // no sync here: a lower chunk reads only lower slots, and its
              // own sync orders this chunk's reads before its writes
            }
            if (acc && cpos < (int)ef) {
              s.pool_d[cpos] = my_d;
              s.pool_id[cpos] = id;
            }
            __syncwarp();
            sz = min(sz + na, (int)ef);
            if (start < first_insert) first_insert = start;
          }
        }
        if (sm) break;  // degree reached
      }
      if (overflow) {
        status = 1;
        break;
      }
      if (w == 0) {
        cursor = min(nxt, first_insert);
        if (cursor > sz) cursor = sz;
      }
    }
    if (w == 0) cp_async_wait_all();  // nothing left in flight
    // publish the pool size for the rerank
    if (w == 0 && lane == 0) s.ctl[6] = (uint32_t)sz;
    __syncthreads();
    sz = (int)s.ctl[6];
  }

  // 5. rerank: exact f32 L2 of the first min(k*rr, sz) pool entries
  const uint64_t krr = (uint64_t)a.k * (uint64_t)max(a.rr, 1u);
  const uint64_t krr_k = krr > (uint64_t)a.k ? krr : (uint64_t)a.k;
  const int rn = (int)(krr_k < (uint64_t)sz ? krr_k : (uint64_t)sz);
  float* rdist = (float*)s.pool_d;
  for (int c0 = 0; c0 < rn; c0 += 32) {
    const int cn = min(32, rn - c0);
    if (w == 0 && lane < cn) s.cand_id[lane] = s.pool_id[c0 + lane] & ~kChecked;
    __syncthreads();
    cta_rows_dist(s.qf, (float*)s.ht, s.cand_id, cn, a.dim, a.vec_c, a.vec_rem, vec_row, s.nd, w, lane);
    __syncthreads();
    if (w == 0 && lane < cn) rdist[c0 + lane] = s.nd[lane];
    __syncthreads();
  }
  if (w != 0) return;
  const int kout = min((int)a.k, rn);
  {
    uint32_t taken = 0;
    for (int r = 0; r < kout; ++r) {
      uint32_t best = 0xffffffffu;
      int bt = -1;
      for (int t = 0; lane + 32 * t < rn; ++t) {
        if (taken & (1u << t)) continue;
        const uint32_t kk = total_order_key(rdist[lane + 32 * t]);
        if (bt < 0 || kk < best) {
          best = kk;
          bt = t;
        }
      }
      const uint32_t m = __reduce_min_sync(kFull, best);
      const int myt = (best == m && bt >= 0) ? bt : 0x7fff;
      const int mt = (int)__reduce_min_sync(kFull, (unsigned)myt);
      const uint32_t who = __ballot_sync(kFull, best == m && bt == mt);
      const int wl = __ffs(who) - 1;
      if (lane == wl) {
        const int i = lane + 32 * bt;
        taken |= 1u << bt;
        a.ids[qi * a.k + r] = s.pool_id[i] & ~kChecked;
        if (a.dists) a.dists[qi * a.k + r] = rdist[i];
      }
    }
  }
  for (int r = kout + lane; r < (int)a.k; r += 32) {
    a.ids[qi * a.k + r] = 0;
    if (a.dists) a.dists[qi * a.k + r] = 0.0f;
  }
  if (lane == 0) {
    if (a.counts) a.counts[qi] = (uint32_t)kout;
    if (VIS && a.visited) a.visited[qi] = vcount;
    if (a.ef_used) a.ef_used[qi] = ef;
    if (a.status) a.status[qi] = status;
    if (a.n_nav) a.n_nav[qi] = n_nav;
    if (a.expansions) a.expansions[qi] = expansions;
    if (VIS && a.hist_len) a.hist_len[qi] = vcount;
  }
}

}  // namespace raven_dev
