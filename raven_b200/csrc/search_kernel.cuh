// Device side of the query engine: one warp per query, persistent grid.
//
// Per query (all inside one warp, warp-synchronous, no block barriers):
//   1. query -> shared memory, SQ4/SQ8 encode          (src/quant/sq4.rs:93-105, sq8.rs:89-97)
//   2. layered-navigation greedy descent, f32 L2 in    (src/graph/navigation.rs:609-653,
//      the reference's AVX-512 lane/tree order          src/distance/avx512.rs:31-62)
//   3. AdaptiveEf rank -> ef table lookup, .max(k)      (src/graph/adaptive_ef.rs:340-359,
//                                                        src/graph/vamana.rs:1803)
//   4. beam search over the fixed-degree adjacency      (src/graph/vamana.rs:786-861 / 683-773,
//      with the LinearPool ordering; new neighbours     src/graph/linear_pool.rs:100-171,
//      by pool membership or an exact visited set        src/memory/visited.rs:88-103)
//      (VIS below); SQ4 distances of a row on the
//      tensor cores when the pool is run-time sized
//   5. f32 rerank of min(k*rr, |pool|) survivors        (src/graph/refiner.rs:45-61)
//
// QUANT selects the beam's distance: 0 SQ4 codes, 1 SQ8 codes, 2 the f32
// vectors themselves (GraphSearcher::search, src/graph/vamana.rs:1627-1672, and
// the build's greedy_search_vec_build, :530-567). With f32 distances there is
// no query code and no rerank: the result is the first k entries of the pool.
//
// VIS selects how step 4 decides that a neighbour is new. true: an exact
// visited set (VisitedTracker), which the visited count, the visited order
// and the f32 beam need. false (SQ4/SQ8 only): membership in the pool. Every
// visited node that is not in the pool has a distance >= the pool's current
// worst entry once the pool is full (it was rejected at or above an earlier
// worst, or evicted from the last slot, and the worst never rises), and while
// the pool is not full every visited node is in it. So "not visited" and "not
// in the pool" accept exactly the same candidates, and ids, distances,
// expansion order and every other result are unchanged; a visited neighbour
// that the pool has dropped is merely scored again (its code was gathered
// anyway) and rejected. The duplicate test costs one shared read after the
// search that places the candidate: an equal id can only sit in the
// run of equal distances just before its slot.
//
// LinearPool equivalence used by the batch merge: the pool always holds the
// first `ef` of all inserted candidates ordered by (distance, insertion order)
// and the cursor is the first unexpanded entry. A new candidate therefore loses
// every distance tie against an entry already in the pool, and candidates of
// one expansion tie-break by adjacency order, so merging one expansion's
// candidates at once gives the same pool as inserting them one by one.
//
// f32 rows (vectors, queries) use a lane-major layout: with C = dim/16, row
// position j*C + c holds element 16c + j (j < 16, c < C) and the dim%16 tail
// follows unpermuted. Lane j of a half-warp then reads its whole fma chain
// (elements j, 16+j, 32+j, ...) contiguously, in the reference's order.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace raven_dev {

constexpr uint32_t kFull = 0xffffffffu;
constexpr uint32_t kSent = 0xffffffffu;
constexpr uint32_t kChecked = 0x80000000u;
constexpr uint32_t kGidBit = 0x80000000u;  // nav handle: global id (node without upper list)
constexpr uint32_t kEmpty = 0xffffffffu;
constexpr int kWarpsPerBlock = 4;
constexpr int kMinBlocksPerSm = 6;  // 80 registers/thread: the measured best residency trade-off
constexpr int kMinBlocksPerSmPool = 7;  // without a visited set: 72 registers, 7 blocks (measured best of 6/7/8)
constexpr uint32_t kNavStepLimit = 1u << 16;

struct SearchArgs {
  // index
  const float* __restrict__ vec;  // n x dim, lane-major rows
  uint32_t dim;
  uint32_t dim_pad;  // dim rounded up to 16 (query buffer)
  uint32_t vec_c;    // dim / 16
  uint32_t vec_rem;  // dim % 16
  const uint32_t* __restrict__ adj;
  uint32_t r_pad;  // row stride in ids (multiple of 32)
  uint32_t pool_cap;  // beam pool capacity per warp (multiple of 32, >= every query's ef)
  const uint16_t* vec16;  // n x dim f16, lane-major (with_f16), or null
  int rerank_f16;         // 1: rerank with the f16 vectors
  const uint8_t* __restrict__ codes;
  uint32_t code_stride;  // bytes per code row (power of two, >= 16)
  const float* __restrict__ q_inv;
  const float* __restrict__ q_neg;
  float levels;  // 15 (SQ4) or 255 (SQ8)
  uint32_t entry;
  // layered navigation, slot based (see raven_gpu.cu)
  int nav;
  uint32_t nav_entry_h;  // handle of the top entry
  uint32_t nav_max_level, nav_k, nav_stride_levels;
  const float* __restrict__ nav_vec;     // slots x dim, lane-major
  const uint32_t* __restrict__ nav_e;    // slots x stride_levels x k handles, kSent padded
  const uint32_t* __restrict__ nav_gid;  // slot -> global id
  // AdaptiveEf
  int adaptive;
  const float* __restrict__ samples;
  uint32_t n_samples;
  const uint32_t* __restrict__ ef_table;  // n_samples + 1 entries
  uint32_t ef_mid;
  uint32_t ef_fixed, k, rr;
  uint32_t dist_bits;   // bits of the largest possible quantised distance
  uint32_t hash_bits;   // shared-memory visited table: 1 << hash_bits slots
  uint32_t spill_bits;  // global spill tables per warp slot: level A 1 << spill_bits slots
  uint32_t* spill;      // (all slots' A tables contiguous), then level B tables 8x larger
  uint64_t n_slots;     // warp slots of the launch (A region = n_slots << spill_bits)
  uint32_t smem_per_warp;
  // queries (natural layout)
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
  uint32_t f32_stage_rows;  // QUANT 2: rows staged per round for the beam's f32 distances
  // neighbour codes beside each row (n x r_pad x code_stride), or null; read
  // by the small-batch kernel without a visited set
  const uint8_t* __restrict__ fat;
  // SQ4: sum of squared nibbles per node (n entries): the batch kernel's
  // tensor-core distance path needs it (always set for SQ4)
  const uint32_t* __restrict__ xnorm;
};

// Per-warp shared-memory carve-up (every piece 16-byte aligned).
struct WarpSmem {
  float* qf;          // dim_pad floats, lane-major
  uint8_t* qcode;     // code_stride bytes
  uint32_t* pool_d;   // pool_cap
  uint32_t* pool_id;  // pool_cap
  uint32_t* cand_id;  // 32
  uint32_t* cand_d;   // 32
  float* nd;          // 32
  uint32_t* rowbuf;   // 2 x r_pad: adjacency rows prefetched by cp.async
  uint32_t* ht;       // 1 << hash_bits; also the row staging area outside the beam search
  float* fstage;      // QUANT 2: f32_stage_rows rows of the beam's new neighbours
};

__host__ __device__ inline uint32_t align16(uint32_t x) { return (x + 15u) & ~15u; }

__host__ __device__ inline uint32_t warp_smem_bytes(uint32_t dim_pad, uint32_t code_stride, uint32_t pool_cap,
                                                    uint32_t hash_bits, uint32_t r_pad, uint32_t f32_stage_rows = 0) {
  return align16(dim_pad * 4) + align16(code_stride) + 2 * align16(pool_cap * 4) + 3 * 128 + 2 * r_pad * 4 +
         align16((1u << hash_bits) * 4) + f32_stage_rows * dim_pad * 4;
}

__device__ inline WarpSmem carve(uint8_t* base, const SearchArgs& a, uint32_t pool_cap) {
  WarpSmem s;
  uint32_t o = 0;
  s.qf = (float*)(base + o);
  o += align16(a.dim_pad * 4);
  s.qcode = base + o;
  o += align16(a.code_stride);
  s.pool_d = (uint32_t*)(base + o);
  o += align16(pool_cap * 4);
  s.pool_id = (uint32_t*)(base + o);
  o += align16(pool_cap * 4);
  s.cand_id = (uint32_t*)(base + o);
  o += 128;
  s.cand_d = (uint32_t*)(base + o);
  o += 128;
  s.nd = (float*)(base + o);
  o += 128;
  s.rowbuf = (uint32_t*)(base + o);
  o += 2 * a.r_pad * 4;
  s.ht = (uint32_t*)(base + o);
  o += align16((1u << a.hash_bits) * 4);
  s.fstage = (float*)(base + o);
  return s;
}

__device__ inline uint32_t lanemask_lt(int lane) { return (1u << lane) - 1u; }

// Position of natural element d in a lane-major row.
__host__ __device__ inline uint32_t lane_major_pos(uint32_t d, uint32_t c_count) {
  const uint32_t main = 16u * c_count;
  return d < main ? (d & 15u) * c_count + (d >> 4) : d;
}

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (cp.async; completion by wait_group,
// a hardware wait, no spinning).
// ---------------------------------------------------------------------------
__device__ inline void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ inline void cp_async4(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem) : "memory");
}
// Asynchronous copy of node's adjacency row (r_pad ids, 16 B per lane) into
// `buf`, as its own commit group.
__device__ inline void prefetch_row(const uint32_t* adj, uint32_t r_pad, uint32_t* buf, uint32_t node, int lane) {
  if ((uint32_t)lane < (r_pad >> 2)) cp_async16(buf + 4 * lane, adj + (size_t)node * r_pad + 4 * lane);
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
// The first 32 neighbour codes of `node` (32 x stride bytes) into shared
// memory, copied by the `nthreads` threads t = 0.. of the caller.
__device__ inline void prefetch_fat(const uint8_t* fat, uint32_t r_pad, uint32_t stride, uint8_t* buf, uint32_t node,
                                    int t, int nthreads) {
  const uint8_t* src = fat + (size_t)node * r_pad * stride;
  for (uint32_t i = (uint32_t)t; i < 2u * stride; i += (uint32_t)nthreads) cp_async16(buf + 16 * i, src + 16 * i);
}
__device__ inline void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Stage `nrows` f32 rows (row r from row_ptr(r)) into shared memory
// (row r at stage + r*dim). All lanes issue copies, then wait.
template <class RowPtr>
__device__ inline void stage_rows(float* stage, int nrows, uint32_t dim, RowPtr row_ptr, int lane) {
  if ((dim & 3u) == 0) {
    const uint32_t per = dim >> 2;  // 16-byte pieces per row
    if (per <= 32 && (per & (per - 1)) == 0) {
      // several rows per pass: lane -> (row offset, piece) by shift/mask
      const uint32_t sh = __ffs(per) - 1;
      const uint32_t rows_per_pass = 32u >> sh;
      const uint32_t ro = (uint32_t)lane >> sh, o = (uint32_t)lane & (per - 1);
      for (uint32_t r0 = 0; r0 < (uint32_t)nrows; r0 += rows_per_pass) {
        const uint32_t r = r0 + ro;
        if (r < (uint32_t)nrows) cp_async16(stage + r * dim + o * 4, row_ptr(r) + o * 4);
      }
    } else {
      for (uint32_t r = 0; r < (uint32_t)nrows; ++r) {
        const float* src = row_ptr(r);
        for (uint32_t o = lane; o < per; o += 32) cp_async16(stage + r * dim + o * 4, src + o * 4);
      }
    }
  } else {
    for (uint32_t r = 0; r < (uint32_t)nrows; ++r) {
      const float* src = row_ptr(r);
      for (uint32_t o = lane; o < dim; o += 32) cp_async4(stage + r * dim + o, src + o);
    }
  }
  cp_async_wait_all();
  __syncwarp();
}

// Halving tree over the 16 lanes of each half-warp (xor 8, 4, 2, 1): the
// _mm512_reduce_add_ps order.
__device__ inline float tree16(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 8));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 4));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(kFull, v, 1));
  return v;
}

// Squared L2 of the (lane-major) query against a lane-major row in shared
// memory, by a half-warp (lane j = lane & 15): lane j's fma chain over
// c = 0..C-1 then the tree; the tail is its own masked vector reduced the
// same way; result = tail + main (src/distance/avx512.rs:31-62). All 32 lanes
// must call (both half-warps, each with its own row).
__device__ inline float hw_dist(const float* __restrict__ qf, const float* __restrict__ row, uint32_t C,
                                uint32_t rem, int j) {
  float acc = 0.0f;
  const float* q = qf + j * C;
  const float* r = row + j * C;
  uint32_t c = 0;
  // 16-byte loads only when both rows are 16-byte aligned (a staged row of a
  // dim that is not a multiple of 4 is not); same summation order either way
  if ((C & 3u) == 0 && (((uintptr_t)q | (uintptr_t)r) & 15u) == 0) {
    for (; c < C; c += 4) {
      const float4 qa = *(const float4*)(q + c);
      const float4 ra = *(const float4*)(r + c);
      float d;
      d = __fsub_rn(qa.x, ra.x);
      acc = __fmaf_rn(d, d, acc);
      d = __fsub_rn(qa.y, ra.y);
      acc = __fmaf_rn(d, d, acc);
      d = __fsub_rn(qa.z, ra.z);
      acc = __fmaf_rn(d, d, acc);
      d = __fsub_rn(qa.w, ra.w);
      acc = __fmaf_rn(d, d, acc);
    }
  } else {
    for (; c < C; ++c) {
      const float d = __fsub_rn(q[c], r[c]);
      acc = __fmaf_rn(d, d, acc);
    }
  }
  float tail = 0.0f;
  if (rem) {
    float d = 0.0f;
    if ((uint32_t)j < rem) d = __fsub_rn(qf[16 * C + j], row[16 * C + j]);
    tail = tree16(__fmaf_rn(d, d, 0.0f));
  }
  return __fadd_rn(tail, tree16(acc));
}

// ---------------------------------------------------------------------------
// f16 rerank (GraphSearcher::with_f16, src/graph/vamana.rs:1559, 1824-1828).
// ---------------------------------------------------------------------------
// F16::to_f32 (src/distance/f16.rs:86-115) as the reference computes it in
// software: exact for normal numbers; a denormal comes out at half its value.
__device__ inline float f16_to_f32_soft(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const int32_t exp = (h >> 10) & 0x1F;
  const uint32_t mant = h & 0x3FFu;
  if (exp == 0) {
    if (mant == 0) return __uint_as_float(sign);
    int32_t e = -1;
    uint32_t m = mant;
    while ((m & 0x400u) == 0) {
      m <<= 1;
      e -= 1;
    }
    return __uint_as_float(sign | ((uint32_t)(127 + e - 14) << 23) | ((m & 0x3FFu) << 13));
  }
  if (exp == 0x1F) return __uint_as_float(sign | 0x7F800000u | (mant << 13));
  return __uint_as_float(sign | ((uint32_t)(exp - 15 + 127) << 23) | (mant << 13));
}

// l2_f16_mixed_avx512 (src/distance/f16.rs:213-262) by a half-warp, against a
// lane-major f16 row: lane j's fma chain over c (hardware f16 -> f32, exact),
// the tree; the dim%16 tail element by element with the software conversion
// and a separate multiply and add (every lane computes it; same value);
// result = tail + tree.
__device__ inline float hw_dist_f16(const float* __restrict__ qf, const uint16_t* __restrict__ row, uint32_t C,
                                   uint32_t rem, int j) {
  float acc = 0.0f;
  const float* q = qf + j * C;
  const uint16_t* r = row + j * C;
  for (uint32_t c = 0; c < C; ++c) {
    const float d = __fsub_rn(q[c], __half2float(__ushort_as_half(r[c])));
    acc = __fmaf_rn(d, d, acc);
  }
  float tail = 0.0f;
  for (uint32_t i = 0; i < rem; ++i) {
    const float d = __fsub_rn(qf[16 * C + i], f16_to_f32_soft(row[16 * C + i]));
    tail = __fadd_rn(tail, __fmul_rn(d, d));
  }
  return __fadd_rn(tail, tree16(acc));
}

// Stage `nrows` f16 rows (dim halves each, row r from row_ptr(r)) at stage +
// r*dim; 16-byte copies when rows are multiples of 8 halves, 4-byte copies for
// even dims, plain loads otherwise. All lanes issue, then wait.
template <class RowPtr>
__device__ inline void stage_rows_f16(uint16_t* stage, int nrows, uint32_t dim, RowPtr row_ptr, int lane) {
  if ((dim & 7u) == 0) {
    const uint32_t per = dim >> 3;
    for (uint32_t t = lane; t < (uint32_t)nrows * per; t += 32) {
      const uint32_t r = t / per, o = t - r * per;
      cp_async16(stage + r * dim + o * 8, row_ptr(r) + o * 8);
    }
  } else if ((dim & 1u) == 0) {
    const uint32_t per = dim >> 1;
    for (uint32_t t = lane; t < (uint32_t)nrows * per; t += 32) {
      const uint32_t r = t / per, o = t - r * per;
      cp_async4(stage + r * dim + o * 2, row_ptr(r) + o * 2);
    }
  } else {
    for (uint32_t t = lane; t < (uint32_t)nrows * dim; t += 32) {
      const uint32_t r = t / dim, o = t - r * dim;
      stage[r * dim + o] = row_ptr(r)[o];
    }
  }
  cp_async_wait_all();
  __syncwarp();
}

template <class RowPtr>
__device__ inline void rows_dist_f16(const float* qf, uint16_t* stage, uint32_t stage_rows_max, const uint32_t* ids,
                                     int n, uint32_t dim, uint32_t C, uint32_t rem, RowPtr row_ptr, float* out,
                                     int lane) {
  const int h = lane >> 4, j = lane & 15;
  for (int b0 = 0; b0 < n; b0 += (int)stage_rows_max) {
    const int nb = min((int)stage_rows_max, n - b0);
    stage_rows_f16(stage, nb, dim, [&](uint32_t r) { return row_ptr(ids[b0 + r]); }, lane);
    for (int r0 = 0; r0 < nb; r0 += 2) {
      const int r = min(r0 + h, nb - 1);
      const float d = hw_dist_f16(qf, stage + (size_t)r * dim, C, rem, j);
      if (j == 0 && r0 + h < nb) out[b0 + r0 + h] = d;
    }
    __syncwarp();
  }
}

// Distances of `n` rows (handles/ids in `ids` smem, resolved by row_ptr) into
// out[0..n), staging up to `stage_rows_max` rows per round in `stage`.
template <class RowPtr>
__device__ inline void rows_dist(const float* qf, float* stage, uint32_t stage_rows_max, const uint32_t* ids, int n,
                                 uint32_t dim, uint32_t C, uint32_t rem, RowPtr row_ptr, float* out, int lane) {
  const int h = lane >> 4, j = lane & 15;
  for (int b0 = 0; b0 < n; b0 += (int)stage_rows_max) {
    const int nb = min((int)stage_rows_max, n - b0);
    stage_rows(stage, nb, dim, [&](uint32_t r) { return row_ptr(ids[b0 + r]); }, lane);
    for (int r0 = 0; r0 < nb; r0 += 2) {
      const int r = min(r0 + h, nb - 1);
      const float d = hw_dist(qf, stage + (size_t)r * dim, C, rem, j);
      if (j == 0 && r0 + h < nb) out[b0 + r0 + h] = d;
    }
    __syncwarp();
  }
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
// Navigation descent (src/graph/navigation.rs:609-653). Works on handles
// (slot index, or kGidBit|id for a node without upper list). Returns the
// entry's global id + f32 distance and counts distance evaluations exactly as
// the reference does (an edge equal to the running node is skipped).
// ---------------------------------------------------------------------------
__device__ inline bool nav_descend(const SearchArgs& a, const WarpSmem& s, float* stage, uint32_t stage_rows_max,
                                   int lane, uint32_t* out_gid, float* out_d, uint32_t* out_evals) {
  auto row_of = [&](uint32_t hd) -> const float* {
    return (hd & kGidBit) ? a.vec + (size_t)(hd & ~kGidBit) * a.dim : a.nav_vec + (size_t)hd * a.dim;
  };
  uint32_t u = a.nav_entry_h;
  if (lane == 0) s.cand_id[0] = u;
  __syncwarp();
  rows_dist(s.qf, stage, stage_rows_max, s.cand_id, 1, a.dim, a.vec_c, a.vec_rem, row_of, s.nd, lane);
  float du = s.nd[0];
  __syncwarp();
  uint32_t evals = 1;
  uint32_t steps = 0;
  bool ok = true;
  const uint32_t K = a.nav_k;
  for (int level = (int)a.nav_max_level; level >= 1 && ok; --level) {
    while (true) {
      if (++steps > kNavStepLimit) {
        ok = false;
        break;
      }
      if ((u & kGidBit) || (uint32_t)level > a.nav_stride_levels) break;
      const uint32_t v =
          (uint32_t)lane < K ? a.nav_e[((size_t)u * a.nav_stride_levels + (level - 1)) * K + lane] : kSent;
      const uint32_t sm = __ballot_sync(kFull, v == kSent);
      const uint32_t cnt = sm ? (uint32_t)(__ffs(sm) - 1) : 32u;
      if (cnt == 0) break;
      if ((uint32_t)lane < cnt) s.cand_id[lane] = v;
      __syncwarp();
      rows_dist(s.qf, stage, stage_rows_max, s.cand_id, (int)cnt, a.dim, a.vec_c, a.vec_rem, row_of, s.nd, lane);
      const float d = (uint32_t)lane < cnt ? s.nd[lane] : __int_as_float(0x7f800000);
      // key: distance bits (non-negative floats order as integers; NaN sorts
      // after +inf and is never selected by `d < cur`) then edge index.
      unsigned long long key = ((unsigned long long)__float_as_uint(d) << 32) | (uint32_t)lane;
      if ((uint32_t)lane >= cnt) key = ~0ull;
      unsigned long long pre = key;  // inclusive prefix minimum
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long t = __shfl_up_sync(kFull, pre, o);
        if (lane >= o && t < pre) pre = t;
      }
      unsigned long long excl = __shfl_up_sync(kFull, pre, 1);
      if (lane == 0) excl = ~0ull;
      // running node before edge e: the argmin over earlier edges if it beat du
      const bool moved = excl != ~0ull && __uint_as_float((uint32_t)(excl >> 32)) < du;
      const uint32_t excl_v = __shfl_sync(kFull, v, moved ? (int)(excl & 31) : 0);
      const uint32_t run_u = moved ? excl_v : u;
      evals += __popc(__ballot_sync(kFull, (uint32_t)lane < cnt && v != run_u));
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
  *out_gid = (u & kGidBit) ? (u & ~kGidBit) : a.nav_gid[u];
  *out_d = du;
  *out_evals = evals;
  return ok;
}

// ---------------------------------------------------------------------------
// Visited set: open addressing in shared memory; past 3/4 load the warp
// switches to its global spill table (lookups check both). Exact: every id
// lives in exactly one table.
// ---------------------------------------------------------------------------
__device__ inline uint32_t hash_slot(uint32_t id, uint32_t bits) { return (id * 0x9E3779B1u) >> (32 - bits); }

// Bucketed open addressing: 4-slot buckets (one 16-byte read), linear over
// buckets. Returns 1 if inserted (first visit), 0 if present. `insert`
// false: lookup only (returns 2 if absent). `bits` = log2(slots) >= 2.
template <bool kShared>
__device__ inline int probe_insert(uint32_t* t, uint32_t bits, uint32_t id, bool insert) {
  const uint32_t nb = 1u << (bits - 2);
  uint32_t b = hash_slot(id, bits - 2);
  for (uint32_t it = 0; it < nb; ++it) {
    uint4 v;
    if (kShared) {
      v = *(const uint4*)(t + 4 * b);
    } else {
      v = __ldcv((const uint4*)(t + 4 * b));  // the spill table lives in L2: bypass L1
    }
    if (v.x == id || v.y == id || v.z == id || v.w == id) return 0;
    const int e = v.x == kEmpty ? 0 : v.y == kEmpty ? 1 : v.z == kEmpty ? 2 : v.w == kEmpty ? 3 : -1;
    if (e >= 0) {
      if (!insert) return 2;
      const uint32_t old = atomicCAS(t + 4 * b + e, kEmpty, id);
      if (old == kEmpty) return 1;
      if (old == id) return 0;
      --it;  // lost the slot to another lane: re-read this bucket
      continue;
    }
    b = (b + 1) & (nb - 1);
  }
  return insert ? 3 : 2;  // table full (not reached: load is capped at 3/4)
}

// Level 0 of the visited set: a two-choice bucketed table in shared memory.
// An id lives in bucket h1(id) or h2(id) (4 slots each), so a lookup is two
// independent 16-byte reads and never a probe chain, and inserts fill the
// emptier bucket, which keeps the buckets even up to high load.
__device__ inline uint32_t hash2_slot(uint32_t id, uint32_t bits) {
  return ((id ^ (id >> 15)) * 0x2C1B3C6Du) >> (32 - bits);
}
__device__ inline bool bucket_has(uint4 v, uint32_t id) { return v.x == id || v.y == id || v.z == id || v.w == id; }
__device__ inline int bucket_free(uint4 v) {
  return (int)(v.x == kEmpty) + (int)(v.y == kEmpty) + (int)(v.z == kEmpty) + (int)(v.w == kEmpty);
}
// 1 inserted (first visit), 0 present, 3 both buckets full (the id belongs
// in the spill table). `bbits` = log2(buckets). Lanes insert distinct ids;
// a lost atomicCAS means another lane filled one of this id's (at most 8)
// slots, so nine rounds always reach a verdict.
__device__ inline int shared_insert2(uint32_t* t, uint32_t bbits, uint32_t id) {
  const uint32_t b1 = hash_slot(id, bbits), b2 = hash2_slot(id, bbits);
  for (int it = 0; it < 9; ++it) {
    const uint4 v1 = *(const uint4*)(t + 4 * b1);
    const uint4 v2 = *(const uint4*)(t + 4 * b2);
    if (bucket_has(v1, id) || bucket_has(v2, id)) return 0;
    const int n1 = bucket_free(v1), n2 = bucket_free(v2);
    if (n1 + n2 == 0) return 3;
    const uint4 v = n1 >= n2 ? v1 : v2;
    const uint32_t b = n1 >= n2 ? b1 : b2;
    const int e = v.x == kEmpty ? 0 : v.y == kEmpty ? 1 : v.z == kEmpty ? 2 : 3;
    if (atomicCAS(t + 4 * b + e, kEmpty, id) == kEmpty) return 1;
  }
  return 3;
}
__device__ inline bool shared_has2(const uint32_t* t, uint32_t bbits, uint32_t id) {
  const uint4 v1 = *(const uint4*)(t + 4 * hash_slot(id, bbits));
  const uint4 v2 = *(const uint4*)(t + 4 * hash2_slot(id, bbits));
  return bucket_has(v1, id) || bucket_has(v2, id);
}

// Level B of the visited set (outlier queries only): look up level A, then
// insert into B. Out of line to keep the common path compact.
__device__ __noinline__ bool probe_level_b(uint32_t* spill_a, uint32_t* spill_b, uint32_t bits_a, uint32_t id) {
  if (probe_insert<false>(spill_a, bits_a, id, false) != 2) return false;
  return probe_insert<false>(spill_b, bits_a + 3, id, true) == 1;
}

// Level A of the visited set, warp-cooperative. The table belongs to this
// warp alone and the lanes' ids are distinct, so insertion needs no atomics:
// each lane looks for its id in the bucket `v` it has already read (bucket `b`,
// read early so that the read overlaps the code gather), then claims the first
// empty slot it sees; lanes claiming the same slot are settled by
// __match_any_sync (lowest lane wins, the others see the slot taken and try
// again), and a lane whose bucket is full reads the next one. Stores are plain
// and need no reply. Returns true for a first visit. Linear probing over
// 4-slot buckets with no deletions, so "absent" = an empty slot was reached.
// The loop ends: every round either places one lane per contended slot or
// moves every unplaced lane to its next bucket, and the load is capped at 3/4.
__device__ inline bool spill_insert_warp(uint32_t* t, uint32_t bits, uint32_t id, bool need, uint32_t b, uint4 v,
                                         int lane) {
  constexpr uint32_t kTaken = 0xFFFFFFFEu;  // slot claimed this round by another lane (never an id)
  const uint32_t bmask = (1u << (bits - 2)) - 1u;
  bool pending = need, is_new = false;
  for (uint32_t round = 0; round <= bmask + 33u; ++round) {
    int e = -1;
    if (pending) {
      if (v.x == id || v.y == id || v.z == id || v.w == id) pending = false;
      else e = v.x == kEmpty ? 0 : v.y == kEmpty ? 1 : v.z == kEmpty ? 2 : v.w == kEmpty ? 3 : -1;
    }
    const bool want = pending && e >= 0;
    const uint32_t wm = __ballot_sync(kFull, want);
    if (want) {
      const uint32_t key = 4u * b + (uint32_t)e;
      const uint32_t same = __match_any_sync(wm, key);
      if (__ffs(same) - 1 == lane) {
        t[key] = id;
        pending = false;
        is_new = true;
      } else if (e == 0) v.x = kTaken;
      else if (e == 1) v.y = kTaken;
      else if (e == 2) v.z = kTaken;
      else v.w = kTaken;
    }
    __syncwarp();  // this round's stores are visible to the lanes that read next
    if (pending && e < 0) {
      b = (b + 1) & bmask;
      v = __ldcv((const uint4*)(t + 4 * b));
    }
    if (!__any_sync(kFull, pending)) break;
  }
  return is_new;
}

// Number of entries <= d in the sorted pool prefix [0, sz), for a candidate
// that the pool accepts (so the answer is < 256 at the engine's pool limit of
// 256): four steps of three independent shared reads each, a quarter of the
// dependent chain of a binary search and no divergent loop (measured +1.6 %
// at ef=140 in the batch kernel, -5 % latency in the small-batch kernel).
__device__ inline int pool_upper_bound4(const uint32_t* pool_d, int sz, uint32_t d) {
  int pos = 0;
#pragma unroll
  for (int step = 64; step > 0; step >>= 2) {
    const int p1 = pos + step, p2 = pos + 2 * step, p3 = pos + 3 * step;
    const bool c1 = p1 <= sz && pool_d[p1 - 1] <= d;
    const bool c2 = p2 <= sz && pool_d[p2 - 1] <= d;
    const bool c3 = p3 <= sz && pool_d[p3 - 1] <= d;
    pos += step * ((int)c1 + (int)c2 + (int)c3);
  }
  return pos;
}

__device__ inline int find_unchecked(const uint32_t* pool_id, int from, int sz, int lane) {
  for (int base = from & ~31; base < sz; base += 32) {
    const int p = base + lane;
    const bool ok = p >= from && p < sz && !(pool_id[p] & kChecked);
    const uint32_t m = __ballot_sync(kFull, ok);
    if (m) return base + __ffs(m) - 1;
  }
  return sz;
}

// D += A (16 x 32 u8, row) x B (32 x 8 s8, col): the warp-level integer MMA,
// exact. Fragments (thread t = 4 g + u): a0 = A[g][4u..4u+3], a1 = A[g+8][4u..],
// a2 = A[g][16+4u..], a3 = A[g+8][16+4u..]; b0 = B[4u..4u+3][g], b1 =
// B[16+4u..][g]; d0, d1 = D[g][2u, 2u+1], d2, d3 = D[g+8][2u, 2u+1].
__device__ inline void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ inline uint32_t u4_word(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// dot product of 4 unsigned bytes (a) with 4 signed bytes (b), plus c.
__device__ inline int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Integer SQ distance partial for one 16-byte chunk.
template <int QUANT>
struct QChunk;

template <>
struct QChunk<0> {  // SQ4: sum (q-x)^2 = sum q^2 + sum x (x - 2q), nibbles unpacked to bytes
  int m2q_lo[4], m2q_hi[4];  // -2q per byte (signed)
  int qq;                    // sum of q^2 over this lane's 32 nibbles
  __device__ inline void load(const uint8_t* qcode, int chunk) {
    const uint4 q = *(const uint4*)(qcode + chunk * 16);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    qq = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
      qq = __dp4a(lo, lo, (unsigned)qq);
      qq = __dp4a(hi, hi, (unsigned)qq);
      // -2q per byte as a signed byte: 0 - 2q never borrows across bytes
      // when done as (0x80 - 2q) ^ 0x80 with 2q <= 30
      m2q_lo[i] = (int)((0x80808080u - 2u * lo) ^ 0x80808080u);
      m2q_hi[i] = (int)((0x80808080u - 2u * hi) ^ 0x80808080u);
    }
  }
  __device__ inline int dist(uint4 b) const {
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
    int acc = qq;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t blo = w[i] & 0x0F0F0F0Fu, bhi = (w[i] >> 4) & 0x0F0F0F0Fu;
      acc = dp4a_us(blo, (int)blo, acc);
      acc = dp4a_us(blo, m2q_lo[i], acc);
      acc = dp4a_us(bhi, (int)bhi, acc);
      acc = dp4a_us(bhi, m2q_hi[i], acc);
    }
    return acc;
  }
};

template <>
struct QChunk<2> {  // f32 beam: no code (distances come from the vectors)
  __device__ inline void load(const uint8_t*, int) {}
  __device__ inline int dist(uint4) const { return 0; }
};

template <>
struct QChunk<1> {  // SQ8: |q-b| per byte, squared by dp4a
  uint32_t q[4];
  __device__ inline void load(const uint8_t* qcode, int chunk) {
    const uint4 v = *(const uint4*)(qcode + chunk * 16);
    q[0] = v.x;
    q[1] = v.y;
    q[2] = v.z;
    q[3] = v.w;
  }
  __device__ inline int dist(uint4 b) const {
    const uint32_t w[4] = {b.x, b.y, b.z, b.w};
    unsigned acc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t d = __vabsdiffu4(q[i], w[i]);
      acc = __dp4a(d, d, acc);
    }
    return (int)acc;
  }
};

// ---------------------------------------------------------------------------
// The search kernel.
// ---------------------------------------------------------------------------
// POOLMAX: 64 for pools of at most 64 entries (layout and merge bounds fixed
// at compile time), 0 for a run-time capacity (a.pool_cap).
template <int QUANT, int CPL, int POOLMAX, bool VIS, bool MMA = false>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, VIS ? kMinBlocksPerSm : kMinBlocksPerSmPool)
    search_kernel(const SearchArgs a) {
  static_assert(!MMA || (QUANT == 0 && CPL == 4 && POOLMAX == 0), "tensor-core distances: SQ4, 4 lanes, run-time pool");
  static_assert(VIS || QUANT != 2, "the f32 beam scores new neighbours only: it needs the visited set");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const uint32_t pool_cap = POOLMAX ? (uint32_t)POOLMAX : a.pool_cap;
  const WarpSmem s = carve(smem_raw + (size_t)wib * a.smem_per_warp, a, pool_cap);
  const uint32_t slot = blockIdx.x * kWarpsPerBlock + wib;
  // level A tables are contiguous (TLB friendly); level B only for outliers
  uint32_t* spill = a.spill ? a.spill + ((size_t)slot << a.spill_bits) : nullptr;
  uint32_t* spill_b = a.spill ? a.spill + (a.n_slots << a.spill_bits) + ((size_t)slot << (a.spill_bits + 3)) : nullptr;
  const uint32_t H = 1u << a.hash_bits;
  const uint32_t h_limit = H - (H >> 3);  // two-choice buckets stay short-probed to 7/8 load
  const uint32_t S = 1u << a.spill_bits;
  const uint32_t s_limit = (S >> 2) * 3;
  const uint32_t SB = S << 3;
  const uint32_t sb_limit = (SB >> 2) * 3;
  float* stage = (float*)s.ht;
  const uint32_t stage_rows_max = min(32u, (H * 4u) / (a.dim * 4u));
  constexpr int CPR = 32 / CPL;  // codes per gather round
  const int sub = lane & (CPL - 1);
  const int grp = lane / CPL;
  auto vec_row = [&](uint32_t id) -> const float* { return a.vec + (size_t)id * a.dim; };

  while (true) {
    unsigned long long qi_ = 0;
    if (lane == 0) qi_ = atomicAdd(a.counter, 1ull);
    const uint64_t qi = __shfl_sync(kFull, qi_, 0);
    if (qi >= a.nq) break;

    // 1. query -> shared memory (lane-major)
    const float* qg = a.queries + qi * a.dim;
    for (uint32_t i = lane; i < a.dim_pad; i += 32) {
      if (i < a.dim) s.qf[lane_major_pos(i, a.vec_c)] = qg[i];
      else s.qf[i] = 0.0f;
    }
    __syncwarp();
    int32_t status = 0;

    // 2. navigation descent (or the medoid)
    uint32_t entry = a.entry;
    float entry_f32 = 0.0f;
    uint32_t n_nav = 0;
    bool have_f32 = false;
    if (a.nav) {
      if (!nav_descend(a, s, stage, stage_rows_max, lane, &entry, &entry_f32, &n_nav)) status = 2;
      have_f32 = true;
    }
    if (a.nav_only) {
      if (lane == 0) {
        a.ids[qi] = entry;
        a.dists[qi] = entry_f32;
        if (a.n_nav) a.n_nav[qi] = n_nav;
        if (a.status) a.status[qi] = status;
      }
      __syncwarp();
      continue;
    }

    // 3. ef
    uint32_t ef = a.ef_fixed;
    if (a.adaptive) {
      if (!have_f32) {
        if (lane == 0) s.cand_id[0] = entry;
        __syncwarp();
        rows_dist(s.qf, stage, stage_rows_max, s.cand_id, 1, a.dim, a.vec_c, a.vec_rem, vec_row, s.nd, lane);
        entry_f32 = s.nd[0];
        n_nav += 1;
      }
      uint32_t e;
      if (a.n_samples <= 1) {
        e = a.ef_mid;
      } else {
        // rank = #samples < d (partition_point): 32 segment heads locate the
        // segment, which is then counted.
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
    if (ef == 0 || ef > pool_cap) status = 3;  // RAVEN_Q_BAD_EF (host validation makes this unreachable)

    uint32_t vcount = 0, expansions = 0;
    int sz = 0;
    if (status != 3) {
      // encode the query (natural dims read through the lane-major map)
      if (QUANT == 2) {
        // f32 beam: no query code
      } else if (QUANT == 0) {
        for (uint32_t b = lane; b < a.code_stride; b += 32) {
          const uint32_t d0 = 2 * b, d1 = 2 * b + 1;
          const uint32_t lo =
              d0 < a.dim ? quantize(s.qf[lane_major_pos(d0, a.vec_c)], a.q_inv[d0], a.q_neg[d0], a.levels) : 0u;
          const uint32_t hi =
              d1 < a.dim ? quantize(s.qf[lane_major_pos(d1, a.vec_c)], a.q_inv[d1], a.q_neg[d1], a.levels) : 0u;
          s.qcode[b] = (uint8_t)(lo | (hi << 4));
        }
      } else {
        for (uint32_t b = lane; b < a.code_stride; b += 32)
          s.qcode[b] = b < a.dim ? (uint8_t)quantize(s.qf[lane_major_pos(b, a.vec_c)], a.q_inv[b], a.q_neg[b],
                                                     a.levels)
                                 : (uint8_t)0;
      }
      if (VIS) {
        // clear the visited table (the staging rows of the descent are done)
        for (uint32_t i = lane * 4; i < H; i += 128) *(uint4*)(s.ht + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
      }
      __syncwarp();  // the query code (and the table) are written before any lane reads them
      QChunk<QUANT> qc;
      qc.load(s.qcode, sub);
      // MMA (SQ4, four lanes per code, run-time pool): a row's distances on
      // the tensor cores as sum q^2 + sum x^2 - 2 sum qx (exact integers):
      // sum q^2 over all four chunks here, sum x^2 per node from the upload.
      // A separate instantiation: the host picks it per launch, and a kernel
      // holding both paths measured slower on either.
      constexpr bool kMma = MMA;
      int qqf = 0;
      if constexpr (kMma) {
        qqf = qc.qq + __shfl_xor_sync(kFull, qc.qq, 1);
        qqf += __shfl_xor_sync(kFull, qqf, 2);
      }

      int level = 0;
      uint32_t tcount = 0, scount = 0;
      // 4. entry
      if (VIS) {
        if (lane == 0) shared_insert2(s.ht, a.hash_bits - 2, entry);
        tcount = 1;
        if (a.history && lane == 0 && a.hist_cap > 0) a.history[qi * a.hist_cap] = entry;
      }
      vcount = 1;
      if (QUANT == 2) {
        // l2_simd(query, vectors[entry]) (src/graph/vamana.rs:603-606); non-negative
        // f32 distances order like their bit patterns, which the pool compares
        if (lane == 0) s.cand_id[0] = entry;
        __syncwarp();
        rows_dist(s.qf, s.fstage, a.f32_stage_rows, s.cand_id, 1, a.dim, a.vec_c, a.vec_rem, vec_row, s.nd, lane);
        if (lane == 0) {
          s.pool_d[0] = __float_as_uint(s.nd[0]);
          s.pool_id[0] = entry;
        }
      } else {
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
      }
      sz = 1;
      __syncwarp();
      int cursor = 0;
      uint32_t pref_node = kSent;  // node whose row was prefetched into rowbuf[pbuf]
      int pbuf = 0;
      const uint32_t RL = a.r_pad >> 5;

      while (cursor < sz) {
        const uint32_t node = s.pool_id[cursor];
        __syncwarp();
        if (lane == 0) s.pool_id[cursor] = node | kChecked;
        ++expansions;
        // neighbours: the row of the predicted expansion was prefetched into
        // rowbuf (cp.async); every prefetch has landed after this wait
        cp_async_wait_all();
        __syncwarp();
        uint32_t row[4];
        if (node == pref_node) {
          const uint32_t* rb = s.rowbuf + pbuf * a.r_pad + lane;
#pragma unroll
          for (int r = 0; r < 4; ++r) row[r] = (uint32_t)r < RL ? rb[32 * r] : kSent;
        } else {
          const uint32_t* rg = a.adj + (size_t)node * a.r_pad + lane;
#pragma unroll
          for (int r = 0; r < 4; ++r) row[r] = (uint32_t)r < RL ? __ldg(rg + 32 * r) : kSent;
        }
        __syncwarp();  // both buffers read before new copies are issued
        const int nxt = find_unchecked(s.pool_id, cursor + 1, sz, lane);
        // next expansion if nothing lands before it: prefetch into buffer 0
        if (nxt < sz) {
          pref_node = s.pool_id[nxt] & ~kChecked;
          prefetch_row(a.adj, a.r_pad, s.rowbuf, pref_node, lane);
          pbuf = 0;
        } else {
          pref_node = kSent;
        }
        bool early = false;  // buffer 1 holds (or is receiving) a prediction of this expansion
        bool ended = false;  // first SENTINEL seen: degree reached
        bool overflow = false;
        int first_insert = 0x7fffffff;
        for (uint32_t seg = 0; seg < RL && !ended; ++seg) {
          const uint32_t id = seg == 0 ? row[0] : seg == 1 ? row[1] : seg == 2 ? row[2] : row[3];
          const uint32_t sm = __ballot_sync(kFull, id == kSent);
          const int deg = sm ? __ffs(sm) - 1 : 32;
          if (sm) ended = true;
          if (deg == 0) continue;
          // speculative gather: codes of every neighbour in the row are
          // requested before the visited check, so the two latencies overlap
          // (a neighbour that turns out visited costs one wasted 16 B load per lane)
          uint4 data[CPL];
#pragma unroll
          for (int r = 0; r < (QUANT == 2 ? 0 : CPL); ++r) {
            const int idx = r * CPR + grp;
            const uint32_t cid_raw = __shfl_sync(kFull, id, idx & 31);
            const uint32_t cid = idx < deg ? cid_raw : 0u;  // address always in range
            // lanes past the degree load node 0's codes; their distances are never stored
            data[r] = __ldg((const uint4*)(a.codes + (size_t)cid * a.code_stride) + sub);
          }
          // rows hold no repeated id (the upload drops later repeats, which the
          // reference treats as already visited), so every valid lane probes.
          const bool valid = lane < deg;
          const uint32_t xn = (kMma && valid) ? __ldg(a.xnorm + id) : 0u;
          bool is_new = false;
          uint32_t newm = 0;  // lanes holding a first visit
          if (VIS) {
            // visited-set level: 0 shared table, 1 spill A, 2 spill B
            if (level == 0 && tcount + 32 > h_limit) {
              if (spill == nullptr) {
                overflow = true;
                break;
              }
              for (uint32_t i = lane * 4; i < S; i += 128)
                *(uint4*)(spill + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
              __syncwarp();
              level = 1;
            } else if (level == 1 && scount + 32 > s_limit) {
              for (uint32_t i = lane * 4; i < SB; i += 128)
                *(uint4*)(spill_b + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
              __syncwarp();
              level = 2;
              scount = 0;
            } else if (level == 2 && scount + 32 > sb_limit) {
              overflow = true;
              break;
            }
            // every id lives in exactly one level; insert into the current one
            if (level == 0) {
              const int r = valid ? shared_insert2(s.ht, a.hash_bits - 2, id) : 0;
              is_new = r == 1;
              const bool to_spill = r == 3;  // both buckets full: this id starts level A
              if (__any_sync(kFull, to_spill)) {
                if (spill == nullptr) {
                  overflow = true;
                  break;
                }
                for (uint32_t i = lane * 4; i < S; i += 128)
                  *(uint4*)(spill + i) = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
                __syncwarp();
                level = 1;
                const uint32_t sbk = hash_slot(id, a.spill_bits - 2);
                const uint4 sv = to_spill ? __ldcv((const uint4*)(spill + 4 * sbk)) : make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
                is_new |= spill_insert_warp(spill, a.spill_bits, id, to_spill, sbk, sv, lane);
              }
            } else if (level == 1) {
              // home bucket of level A read before the shared lookup: the two overlap
              const uint32_t sbk = hash_slot(id, a.spill_bits - 2);
              uint4 sv = make_uint4(kEmpty, kEmpty, kEmpty, kEmpty);
              if (valid) sv = __ldcv((const uint4*)(spill + 4 * sbk));
              const bool need = valid && !shared_has2(s.ht, a.hash_bits - 2, id);
              is_new = spill_insert_warp(spill, a.spill_bits, id, need, sbk, sv, lane);
            } else if (valid && !shared_has2(s.ht, a.hash_bits - 2, id)) {
              is_new = probe_level_b(spill, spill_b, a.spill_bits, id);
            }
            newm = __ballot_sync(kFull, is_new);
            if (newm == 0) continue;
            const int nn = __popc(newm);
            if (level == 0) tcount += nn;
            else scount += nn;
            if (a.history && is_new) {
              const uint32_t pos = vcount + __popc(newm & lanemask_lt(lane));
              if (pos < a.hist_cap) a.history[qi * a.hist_cap + pos] = id;
            }
            vcount += nn;
          }
          uint32_t my_d;
          if constexpr (QUANT == 2) {
            // f32 distances of the new neighbours only, in adjacency order
            // (compacted), their rows staged in shared memory
            const int cpos = __popc(newm & lanemask_lt(lane));
            if (is_new) s.cand_id[cpos] = id;
            __syncwarp();
            rows_dist(s.qf, s.fstage, a.f32_stage_rows, s.cand_id, __popc(newm), a.dim, a.vec_c, a.vec_rem, vec_row,
                      s.nd, lane);
            my_d = is_new ? __float_as_uint(s.nd[cpos]) : 0xffffffffu;
          } else if constexpr (kMma) {
            // the row's 32 codes as two 16 x 128 tiles (rounds 0-1, 2-3: row
            // m of tile t is neighbour 16 t + m) against -2q: K block kb takes
            // word kb of every lane's 16-byte chunk, low nibbles as columns
            // 4u.., high nibbles as 16 + 4u.. (the same order for the query)
            // (two accumulators per tile, even and odd K blocks, halve the
            // dependent MMA chain)
            int t0[4] = {0, 0, 0, 0}, t1[4] = {0, 0, 0, 0}, u0[4] = {0, 0, 0, 0}, u1[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              const uint32_t w0 = u4_word(data[0], kb), w1 = u4_word(data[1 % CPL], kb);
              const uint32_t w2 = u4_word(data[2 % CPL], kb), w3 = u4_word(data[3 % CPL], kb);
              const uint32_t m = 0x0F0F0F0Fu;
              const uint32_t b0 = (uint32_t)qc.m2q_lo[kb], b1 = (uint32_t)qc.m2q_hi[kb];
              if (kb & 1) {
                mma_u8s8(u0, w0 & m, w1 & m, (w0 >> 4) & m, (w1 >> 4) & m, b0, b1);
                mma_u8s8(u1, w2 & m, w3 & m, (w2 >> 4) & m, (w3 >> 4) & m, b0, b1);
              } else {
                mma_u8s8(t0, w0 & m, w1 & m, (w0 >> 4) & m, (w1 >> 4) & m, b0, b1);
                mma_u8s8(t1, w2 & m, w3 & m, (w2 >> 4) & m, (w3 >> 4) & m, b0, b1);
              }
            }
            t0[0] += u0[0];
            t0[2] += u0[2];
            t1[0] += u1[0];
            t1[2] += u1[2];
            // neighbour `lane`: tile lane >> 4, row lane & 15, held by thread 4 (lane & 7)
            const int src = (lane & 7) << 2;
            const int e0 = __shfl_sync(kFull, t0[0], src), e1 = __shfl_sync(kFull, t0[2], src);
            const int e2 = __shfl_sync(kFull, t1[0], src), e3 = __shfl_sync(kFull, t1[2], src);
            const int dot = lane < 16 ? ((lane & 8) ? e1 : e0) : ((lane & 8) ? e3 : e2);
            my_d = (VIS ? is_new : valid) ? (uint32_t)(qqf + (int)xn + dot) : 0xffffffffu;
          } else {
            // integer distances of the row (candidate idx -> cand_d[idx])
#pragma unroll
            for (int r = 0; r < CPL; ++r) {
              if (r * CPR < deg) {
                int pdist = qc.dist(data[r]);
#pragma unroll
                for (int o = 1; o < CPL; o <<= 1) pdist += __shfl_xor_sync(kFull, pdist, o);
                const int idx = r * CPR + grp;
                if (sub == 0 && idx < deg) s.cand_d[idx] = (uint32_t)pdist;
              }
            }
            __syncwarp();
            my_d = (VIS ? is_new : valid) ? s.cand_d[lane] : 0xffffffffu;
          }
          // merge the new neighbours (adjacency order) into the pool:
          // LinearPool::insert semantics, batched
          const bool full = sz == (int)ef;
          const uint32_t worst = full ? s.pool_d[sz - 1] : 0xffffffffu;
          bool acc = (VIS ? is_new : valid) && (!full || my_d < worst);
          int slot_lo = 0;  // without the visited set: # pool entries <= my_d
          if (!VIS && acc) {
            const int lo = pool_upper_bound4(s.pool_d, sz, my_d);
            slot_lo = lo;
            // already in the pool: an equal id sits in the run of equal
            // distances ending at lo - 1
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
            // pool entries from the first insertion point onward move right
            int cpos = 0x7fffffff;
            if (acc && !VIS) cpos = slot_lo;
            if (acc && VIS) {
              cpos = pool_upper_bound4(s.pool_d, sz, my_d);  // ties: pool first
            }
            const int start = (int)__reduce_min_sync(kFull, (unsigned)cpos);
            if (start <= min(nxt, first_insert)) {
              // the closest accepted candidate lands before every unexpanded
              // entry, so it is the next expansion: fetch its row now, while
              // the merge runs
              const uint32_t dmin = __reduce_min_sync(kFull, acc ? my_d : 0xffffffffu);
              pref_node = __shfl_sync(kFull, id, __ffs(__ballot_sync(kFull, acc && my_d == dmin)) - 1);
              if (early) {  // rows longer than 32: a later segment overrides; let the earlier copy land
                cp_async_wait_all();
                __syncwarp();
              }
              prefetch_row(a.adj, a.r_pad, s.rowbuf + a.r_pad, pref_node, lane);
              pbuf = 1;
              early = true;
            }
            // rank among the accepted candidates by (distance, lane): the
            // reference inserts them one by one in adjacency order and an
            // equal distance goes after, so equal candidates keep lane order
            int crank = 0;
            for (uint32_t m = am; m; m &= m - 1) {
              const int jl = __ffs(m) - 1;
              const uint32_t dj = __shfl_sync(kFull, my_d, jl);
              crank += (dj < my_d) | ((dj == my_d) & (jl < lane));
            }
            if (acc) cpos += crank;  // final slot; >= ef: falls off the end
            const int nsz = min(sz + na, (int)ef);
            // Pool entries move right past the candidate slots. Output slot j
            // (not a candidate slot) takes old entry j - #(candidate slots < j);
            // chunks of 32 slots from the top down, so a chunk's sources (all
            // <= its slots) are read before a lower chunk is written.
            // the chunks holding [start, nsz), top down (fixed bounds for small pools)
            const int t_lo = POOLMAX ? 0 : start >> 5;
            const int t_hi = POOLMAX ? POOLMAX / 32 - 1 : (nsz - 1) >> 5;
#pragma unroll
            for (int t = t_hi; t >= t_lo; --t) {
              const int base = 32 * t;
              if (POOLMAX && (base >= nsz || base + 32 <= start)) continue;
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
        if (overflow) {
          status = 1;
          break;
        }
        // Entries before the popped one are expanded and `nxt` was the first
        // unexpanded after it; an insert before `nxt` leaves it in place, so
        // the next pop is the earlier of the two.
        cursor = min(nxt, first_insert);
        if (cursor > sz) cursor = sz;
      }
    }

    // 5. rerank: exact f32 L2 of the first min(k*rr, sz) pool entries. With
    // the f32 beam the pool already holds those distances (the same values):
    // the result is its first min(k, sz) entries (search(), vamana.rs:1667-1671)
    const uint64_t krr = QUANT == 2 ? (uint64_t)a.k : (uint64_t)a.k * (uint64_t)max(a.rr, 1u);
    const uint64_t krr_k = krr > (uint64_t)a.k ? krr : (uint64_t)a.k;
    const int rn = (int)(krr_k < (uint64_t)sz ? krr_k : (uint64_t)sz);
    float* rdist = (float*)s.pool_d;  // pool distances are no longer needed
    for (int c0 = 0; c0 < (QUANT == 2 ? 0 : rn); c0 += 32) {
      const int cn = min(32, rn - c0);
      if (lane < cn) s.cand_id[lane] = s.pool_id[c0 + lane] & ~kChecked;
      __syncwarp();
      if (a.rerank_f16)
        rows_dist_f16(s.qf, (uint16_t*)s.ht, min(32u, (H * 4u) / (a.dim * 2u)), s.cand_id, cn, a.dim, a.vec_c,
                      a.vec_rem, [&](uint32_t id) { return a.vec16 + (size_t)id * a.dim; }, s.nd, lane);
      else
        rows_dist(s.qf, stage, stage_rows_max, s.cand_id, cn, a.dim, a.vec_c, a.vec_rem, vec_row, s.nd, lane);
      if (lane < cn) rdist[c0 + lane] = s.nd[lane];
      __syncwarp();
    }
    const int kout = min((int)a.k, rn);
    // k smallest by (total_cmp(dist), pool position): repeated warp minimum;
    // each lane owns positions lane, lane+32, ...
    {
      uint32_t taken = 0;  // bit t: position lane+32t already output
      for (int r = 0; r < kout; ++r) {
        uint32_t best = 0xffffffffu;
        int bt = -1;
        for (int t = 0; lane + 32 * t < rn; ++t) {
          if (taken & (1u << t)) continue;
          const uint32_t kk = total_order_key(rdist[lane + 32 * t]);
          if (bt < 0 || kk < best) {  // strict: the lowest position wins a tie within a lane
            best = kk;
            bt = t;
          }
        }
        const uint32_t m = __reduce_min_sync(kFull, best);
        // ties across lanes: the smallest position, i.e. lowest t, then lowest lane
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
    __syncwarp();
  }
}

}  // namespace raven_dev
