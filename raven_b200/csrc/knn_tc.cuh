// Exact k-nearest neighbours (recall ground truth) on the 5th-generation
// tensor cores: squared L2 as |q|^2 + |x|^2 - 2 q.x, the q.x tile computed by
// tcgen05.mma kind::tf32 into tensor memory, operands staged by TMA.
//
// Precision. TF32 keeps 11 significant bits. Integer-valued data with
// |v| <= 2048 is exact in TF32, every product is exact in the f32
// accumulator, and as long as |q|^2 + |x|^2 < 2^24 every partial sum and the
// final distance are exact integers: one pass gives the same distances (and,
// with ties broken by id, the same neighbours) as a direct f32 sum of squared
// differences. Other data runs three passes on a hi/lo split,
// q.x ~ qh.xh + qh.xl + ql.xh with xh = tf32(x), xl = x - xh (the dropped
// ql.xl term is ~2^-22 relative), i.e. f32-level accuracy.
//
// Work split. One CTA per (128-query tile, base split); the base rows of a
// split stream through a ring of shared-memory stages (128 rows x 32 floats,
// one 128-byte swizzled row per base vector and K block), the query tile stays
// resident. Warp roles: warp 0 lane 0 issues TMA loads, warp 1 lane 0 issues
// the MMAs, warp 2 owns the tensor memory (two 128 x 128 f32 accumulators so
// the epilogue of one base tile overlaps the MMAs of the next), warps 4-7 are
// the epilogue: thread r owns query r of the tile (tensor-memory lane r),
// reads its 128 dot products per base tile and keeps a sorted top-k in
// registers (ties by id). Every mbarrier wait is bounded; a wait that runs out
// sets an error flag. Before the tensor memory is freed and the CTA exits, the
// producer waits for every TMA load it issued to land and the MMA issuer for
// every MMA it issued to complete (both bounded), so no copy or MMA of this CTA
// can write into shared or tensor memory that a later CTA is given.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace raven_tc {

constexpr int kBM = 128;      // queries per tile = tensor-memory lanes
constexpr int kBN = 128;      // base rows per tile = accumulator columns
constexpr int kBK = 32;       // floats per K block: one 128-byte swizzled row
constexpr int kMaxKB = 4;     // K blocks: dim <= 128
constexpr int kEpiWarps = 8;  // two per lane quadrant: columns 0-63 and 64-127 of a tile
constexpr int kThreads = 32 * (4 + kEpiWarps);
constexpr uint32_t kBlockBytes = kBN * kBK * 4;  // one operand block: 16 KB
constexpr uint32_t kTmemCols = 2 * kBN;
constexpr long long kWaitCycles = 1ll << 32;     // ~2 s: a longer wait is a fault

template <int PASSES>
struct Layout {
  static constexpr int kStages = PASSES == 1 ? 6 : 2;
  static constexpr int kParts = PASSES == 1 ? 1 : 2;  // hi (and lo) per operand block
  static constexpr uint32_t kA = 0;                   // query blocks: [part][kb]
  static constexpr uint32_t kB = kParts * kMaxKB * kBlockBytes;
  static constexpr uint32_t kBars = kB + kStages * kParts * kBlockBytes;
  // barriers: a_full, full[S], empty[S], acc_full[2], acc_empty[2], drain; then the tmem slot
  static constexpr uint32_t kNumBars = 1 + 2 * kStages + 5;
  static constexpr uint32_t kTmemSlot = kBars + kNumBars * 8;
  static constexpr uint32_t kBytes = kTmemSlot + 16 + 1024;  // + alignment slack
};

struct Params {
  uint64_t n;           // base rows
  uint64_t nq;          // queries
  uint32_t kb;          // K blocks (dim / 32 rounded up)
  uint32_t k;           // neighbours per query (<= KT)
  uint64_t split_rows;  // base rows per split (multiple of kBN)
  uint32_t qtiles;      // query tiles
  const float* xn;      // base squared norms, +inf from row n up to a multiple of kBN
  const float* qn;      // query squared norms
  uint32_t* out_i;      // [split][column half][nq][k]
  float* out_d;
  int* err;             // set to 1 when a wait ran out
};

__device__ inline uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ inline void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ inline void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ inline void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// Waits until the phase with parity `parity` has completed; false after
// kWaitCycles.
__device__ inline bool mbar_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kWaitCycles) return false;
  }
}
__device__ inline void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ inline void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ inline void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Shared-memory operand descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), leading offset unused for this layout (1), version 1.
__device__ inline uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}
// Instruction descriptor: D f32, A and B tf32, both K-major, N = kBN, M = kBM.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);

__device__ inline void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ inline void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
// 32 consecutive accumulator columns of this thread's lane.
__device__ inline void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// 32 dot products of one query against base rows id0..id0+31: distances
// |q|^2 + |x|^2 - 2 q.x, and any that beat the current k-th distance go into
// the sorted list. The common case (nothing qualifies) costs an FMA and a
// min per element; insertions use one compact site, the candidate's value
// picked by a select chain (no dynamic register indexing). Ids rise along the
// scan, so an equal distance never displaces an entry already held and the
// strict test keeps ties ordered by id.
template <int KT>
__device__ inline void scan_chunk(const uint32_t (&v)[32], const float* xn, float qnorm, uint32_t id0, uint32_t k,
                                  float (&kd)[KT], uint32_t (&ki)[KT], float& thr) {
  const float4* xp = (const float4*)xn;
  float dv[32];
  float dmin = __int_as_float(0x7f800000);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 f = __ldg(xp + j);
    dv[4 * j] = fmaf(-2.0f, __uint_as_float(v[4 * j]), qnorm + f.x);
    dv[4 * j + 1] = fmaf(-2.0f, __uint_as_float(v[4 * j + 1]), qnorm + f.y);
    dv[4 * j + 2] = fmaf(-2.0f, __uint_as_float(v[4 * j + 2]), qnorm + f.z);
    dv[4 * j + 3] = fmaf(-2.0f, __uint_as_float(v[4 * j + 3]), qnorm + f.w);
    dmin = fminf(dmin, fminf(fminf(dv[4 * j], dv[4 * j + 1]), fminf(dv[4 * j + 2], dv[4 * j + 3])));
  }
  if (!(dmin < thr)) return;
  uint32_t cand = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) cand |= (uint32_t)(dv[j] < thr) << j;
  while (cand) {
    const int j = __ffs(cand) - 1;
    cand &= cand - 1;
    float cd = 0.0f;
#pragma unroll
    for (int m = 0; m < 32; ++m) cd = m == j ? dv[m] : cd;
    if (!(cd < thr)) continue;  // an earlier insertion of this chunk raised the bar
    uint32_t ci = id0 + (uint32_t)j;
#pragma unroll
    for (int m = 0; m < KT; ++m) {
      const bool sw = cd < kd[m] || (cd == kd[m] && ci < ki[m]);
      const float td = kd[m];
      const uint32_t ti = ki[m];
      kd[m] = sw ? cd : td;
      ki[m] = sw ? ci : ti;
      cd = sw ? td : cd;
      ci = sw ? ti : ci;
    }
#pragma unroll
    for (int m = 0; m < KT; ++m) thr = (uint32_t)m == k - 1 ? kd[m] : thr;
  }
}

template <int PASSES, int KT>
__global__ void __launch_bounds__(kThreads, 1)
    knn_tc_kernel(const __grid_constant__ CUtensorMap tm_qh, const __grid_constant__ CUtensorMap tm_ql,
                  const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                  const Params p) {
  using L = Layout<PASSES>;
  constexpr int S = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBars;
  const uint32_t a_full = bar0;
  auto full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto empty = [&](int s) { return bar0 + 8u * (1 + S + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (1 + 2 * S + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (3 + 2 * S + b); };
  const uint32_t drain = bar0 + 8u * (5 + 2 * S);  // completion of every MMA this CTA issued
  auto a_blk = [&](int part, int kb) { return sbase + L::kA + (uint32_t)(part * kMaxKB + kb) * kBlockBytes; };
  auto b_blk = [&](int s, int part) { return sbase + L::kB + (uint32_t)(s * L::kParts + part) * kBlockBytes; };
  uint32_t* tmem_slot = (uint32_t*)(smem + L::kTmemSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t qt = blockIdx.x % p.qtiles, sp = blockIdx.x / p.qtiles;
  const uint64_t q0 = (uint64_t)qt * kBM;
  const uint64_t r_begin = (uint64_t)sp * p.split_rows;
  const uint64_t r_end = r_begin + p.split_rows < p.n ? r_begin + p.split_rows : p.n;
  const uint32_t ntiles = r_begin < r_end ? (uint32_t)((r_end - r_begin + kBN - 1) / kBN) : 0u;
  const uint32_t KB = p.kb;

  if (threadIdx.x == 0) {
    mbar_init(a_full, 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), kEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      mbar_expect_tx(a_full, KB * kBlockBytes * L::kParts);
      for (uint32_t kb = 0; kb < KB; ++kb) {
        tma_load_2d(a_blk(0, kb), &tm_qh, (int)(kb * kBK), (int)q0, a_full);
        if (PASSES == 3) tma_load_2d(a_blk(1, kb), &tm_ql, (int)(kb * kBK), (int)q0, a_full);
      }
      int s = 0;
      uint32_t ph = 0;
      uint32_t used = 0, last_ph = 0;  // bit s: stage s was loaded; its last load's phase parity
      for (uint32_t t = 0; t < ntiles && ok; ++t) {
        const int row = (int)(r_begin + (uint64_t)t * kBN);
        for (uint32_t kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(empty(s), ph ^ 1u)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full(s), kBlockBytes * L::kParts);
          tma_load_2d(b_blk(s, 0), &tm_xh, (int)(kb * kBK), row, full(s));
          if (PASSES == 3) tma_load_2d(b_blk(s, 1), &tm_xl, (int)(kb * kBK), row, full(s));
          used |= 1u << s;
          last_ph = (last_ph & ~(1u << s)) | (ph << s);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // drain: every load issued has landed (immediate unless a wait ran out)
      bool landed = mbar_wait(a_full, 0);
#pragma unroll
      for (int st = 0; st < S; ++st)
        if ((used >> st) & 1u) landed &= mbar_wait(full(st), (last_ph >> st) & 1u);
      ok &= landed;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      ok = mbar_wait(a_full, 0);
      tc_fence_after();
      int s = 0;
      uint32_t ph = 0;
      for (uint32_t t = 0; t < ntiles && ok; ++t) {
        const int b = (int)(t & 1u);
        if (!mbar_wait(acc_empty(b), ((t >> 1) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * kBN);
        for (uint32_t kb = 0; kb < KB && ok; ++kb) {
          if (!mbar_wait(full(s), ph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ah = sw128_desc(a_blk(0, (int)kb)), bh = sw128_desc(b_blk(s, 0));
#pragma unroll
          for (int k = 0; k < kBK / 8; ++k) {  // K = 8 per tf32 MMA: +32 bytes along the swizzled row
            const uint64_t step = (uint64_t)(2 * k);
            mma_tf32(d_tmem, ah + step, bh + step, (kb | (uint32_t)k) != 0u ? 1u : 0u);
            if (PASSES == 3) {
              const uint64_t al = sw128_desc(a_blk(1, (int)kb)), bl = sw128_desc(b_blk(s, 1));
              mma_tf32(d_tmem, ah + step, bl + step, 1u);
              mma_tf32(d_tmem, al + step, bh + step, 1u);
            }
          }
          mma_commit(empty(s));  // the stage is free once these MMAs have read it
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) mma_commit(acc_full(b));
      }
      // drain: every MMA issued has completed (immediate unless a wait ran out)
      mma_commit(drain);
      ok &= mbar_wait(drain, 0);
    }
  } else if (warp >= 4) {
    // epilogue: warp w reads tensor-memory lanes 32*(w%4).. (query rows) and
    // one half of each tile's columns; thread <-> (query r, column half)
    const int quad = warp & 3, half = (warp - 4) >> 2;
    const int r = quad * 32 + lane;
    const uint64_t qi = q0 + (uint64_t)r;
    const float qnorm = qi < p.nq ? p.qn[qi] : 0.0f;
    float kd[KT];
    uint32_t ki[KT];
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      kd[j] = __int_as_float(0x7f800000);
      ki[j] = 0xffffffffu;
    }
    float thr = __int_as_float(0x7f800000);  // distance of the k-th entry held
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    constexpr int kHalf = kBN / 2;
    for (uint32_t t = 0; t < ntiles; ++t) {
      const int b = (int)(t & 1u);
      const bool got = mbar_wait(acc_full(b), (t >> 1) & 1u);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint64_t row0 = r_begin + (uint64_t)t * kBN;
      // the next tile's norms into L1 while this one is scanned (two 128-byte lines per half)
      if (lane < 2 && t + 1 < ntiles)
        asm volatile("prefetch.global.L1 [%0];\n" ::"l"(p.xn + row0 + kBN + half * kHalf + 32 * lane));
      uint32_t va[32], vb[32];
      tmem_ld32(tmem + lane_base + (uint32_t)(b * kBN + half * kHalf), va);
      // second chunk requested now, waited for after the first chunk's work
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
          "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
          : "=r"(vb[0]), "=r"(vb[1]), "=r"(vb[2]), "=r"(vb[3]), "=r"(vb[4]), "=r"(vb[5]), "=r"(vb[6]), "=r"(vb[7]),
            "=r"(vb[8]), "=r"(vb[9]), "=r"(vb[10]), "=r"(vb[11]), "=r"(vb[12]), "=r"(vb[13]), "=r"(vb[14]),
            "=r"(vb[15]), "=r"(vb[16]), "=r"(vb[17]), "=r"(vb[18]), "=r"(vb[19]), "=r"(vb[20]), "=r"(vb[21]),
            "=r"(vb[22]), "=r"(vb[23]), "=r"(vb[24]), "=r"(vb[25]), "=r"(vb[26]), "=r"(vb[27]), "=r"(vb[28]),
            "=r"(vb[29]), "=r"(vb[30]), "=r"(vb[31])
          : "r"(tmem + lane_base + (uint32_t)(b * kBN + half * kHalf + 32)));
      scan_chunk<KT>(va, p.xn + row0 + half * kHalf, qnorm, (uint32_t)(row0 + half * kHalf), p.k, kd, ki, thr);
      asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
      scan_chunk<KT>(vb, p.xn + row0 + half * kHalf + 32, qnorm, (uint32_t)(row0 + half * kHalf + 32), p.k, kd, ki, thr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(b));
    }
    if (qi < p.nq) {
      const size_t o = (((size_t)sp * 2 + (size_t)half) * p.nq + qi) * p.k;
#pragma unroll
      for (int m = 0; m < KT; ++m)
        if ((uint32_t)m < p.k) {
          p.out_i[o + m] = ki[m];
          p.out_d[o + m] = kd[m];
        }
    }
  }
  if (!ok && lane == 0) atomicOr(p.err, 1);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace raven_tc
