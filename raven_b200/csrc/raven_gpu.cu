// C-ABI implementation of the B200 query engine (include/raven_gpu.h).
//
// Device data layout (HBM):
//   vectors   n x dim f32 (row-major, as given)
//   adj       n x r_pad u32, r_pad = roundup(r_max, 32): the HybridBlockedCsr
//             main block, SENTINEL padded; one 128 B line per 32 neighbours
//   sq4/sq8   n x stride u8 codes, stride = pow2 >= 16 bytes (64 B for dim 128
//             SQ4, 128 B for dim 128 SQ8), zero padded past the real code
//   nav       slot[n] -> nav_off[slot..slot+1] into nav_edges (global ids)
//   adaptive  sorted sample distances (<= 2000) + per-call rank->ef table
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/raven_gpu.h"
#include "host_index.h"
#include "knn_tc.cuh"
#include "search_cta.cuh"
#include "search_kernel.cuh"

using namespace raven_dev;

struct raven_graph {
  raven::HostGraph g;
};

struct raven_index {
  int device = 0;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  uint64_t n = 0;
  uint32_t dim = 0, dim_pad = 0, r_max = 0, r_pad = 0, entry = 0;
  float* d_vec = nullptr;
  uint16_t* d_vec16 = nullptr;  // f16 copy for with_f16 reranks (F16Dataset), lane-major like d_vec
  uint32_t* d_adj = nullptr;
  bool has_q[2] = {false, false};
  uint32_t q_stride[2] = {0, 0};
  uint8_t* d_codes[2] = {nullptr, nullptr};
  // neighbour codes beside each row: node i's slot j holds the code of
  // adj[i][j] (zeros past the degree), n x r_pad x q_stride bytes, or null
  uint8_t* d_fat[2] = {nullptr, nullptr};
  // SQ4: sum of the squared nibbles of each node's code (the search's
  // distance is sum q^2 + sum x^2 - 2 sum qx, the last on tensor cores)
  uint32_t* d_xnorm = nullptr;
  float* d_qparams[2] = {nullptr, nullptr};  // 5*dim
  std::vector<float> h_qparams[2];
  bool has_nav = false;
  uint32_t nav_entry_h = 0, nav_max_level = 0, nav_k = 0, nav_stride_levels = 0;
  float* d_nav_vec = nullptr;      // slots x dim, lane-major
  uint32_t* d_nav_e = nullptr;     // slots x stride_levels x k handles
  uint32_t* d_nav_gid = nullptr;   // slot -> global id
  std::vector<float> h_samples;
  float* d_samples = nullptr;
  // launch tuning
  int hash_bits_override = 0;
  int spill_bits_override = 0;
  uint64_t small_batch_max = ~0ull;  // batches of at most this many queries run one CTA per query (~0: one wave)
};

namespace {

// NVTX range around a host-side phase (upload, search, exact kNN, merge,
// build batches): shows on a profiler's timeline, no cost without one.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define CU(call)                                                                        \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess) return fail(RAVEN_ECUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
  } while (0)

// The CUDA context current on the calling thread (driver entry point looked up
// once through the runtime; null if it is unavailable).
void* current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuCtxGetCurrent_v4000)p;
    else
      (void)cudaGetLastError();
  });
  CUcontext c = nullptr;
  if (fn && fn(&c) != CUDA_SUCCESS) c = nullptr;
  return (void*)c;
}

// Per-context cache of kernel launch attributes: the dynamic shared memory a
// kernel has been allowed and its resident blocks per SM at a given shared
// memory size. Both are queried once instead of on every search (a context
// created after a device reset starts with an empty cache).
struct LaunchCache {
  std::mutex mu;
  std::vector<std::pair<std::pair<void*, const void*>, uint32_t>> allowed;          // (ctx, kernel) -> bytes
  std::vector<std::pair<std::pair<void*, const void*>, std::pair<uint32_t, int>>> occ;  // (ctx, kernel) -> (bytes, blocks)
};
LaunchCache& launch_cache() {
  static LaunchCache c;
  return c;
}
cudaError_t allow_smem(const void* k, uint32_t smem) {
  const auto key = std::make_pair(current_context(), k);
  LaunchCache& c = launch_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  for (auto& e : c.allowed)
    if (e.first == key && e.second >= smem) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) {
    bool found = false;
    for (auto& x : c.allowed)
      if (x.first == key) {
        x.second = smem;
        found = true;
      }
    if (!found) c.allowed.push_back({key, smem});
  }
  return e;
}
// Drops the cached attributes of `k` in the current context: a context
// created after a reset can reuse an old context's handle, and a launch that
// fails on the shared-memory size is retried once with the attribute set anew.
void forget_kernel(const void* k) {
  const auto key = std::make_pair(current_context(), k);
  LaunchCache& c = launch_cache();
  std::lock_guard<std::mutex> lk(c.mu);
  c.allowed.erase(std::remove_if(c.allowed.begin(), c.allowed.end(), [&](auto& e) { return e.first == key; }),
                  c.allowed.end());
  c.occ.erase(std::remove_if(c.occ.begin(), c.occ.end(), [&](auto& e) { return e.first == key; }), c.occ.end());
}

cudaError_t blocks_per_sm(const void* k, int threads, uint32_t smem, int* blocks) {
  const auto key = std::make_pair(current_context(), k);
  {
    LaunchCache& c = launch_cache();
    std::lock_guard<std::mutex> lk(c.mu);
    for (auto& e : c.occ)
      if (e.first == key && e.second.first == smem) {
        *blocks = e.second.second;
        return cudaSuccess;
      }
  }
  cudaError_t e = allow_smem(k, smem);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, k, threads, smem);
  if (e == cudaSuccess) {
    LaunchCache& c = launch_cache();
    std::lock_guard<std::mutex> lk(c.mu);
    c.occ.push_back({key, {smem, *blocks}});
  }
  return e;
}

uint32_t next_pow2(uint32_t x) {
  uint32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

// ---------------------------------------------------------------------------
// Quantisation on the device: SQ4Params::encode_all (src/quant/sq4.rs:108-125)
// and SQ8Params::encode_all (src/quant/sq8.rs:100-111). One thread per output
// 4-byte word; padding bytes are zero.
// ---------------------------------------------------------------------------

// Neighbour codes beside each row: fat[i][j] = codes[adj[i][j]], zeros for
// SENTINEL slots. One warp per row, 16-byte pieces (stride is a multiple of
// 16). Grid-stride over rows.
__global__ void fat_rows_kernel(const uint32_t* __restrict__ adj, const uint8_t* __restrict__ codes, uint64_t n,
                                uint32_t r_pad, uint32_t stride, uint8_t* __restrict__ fat) {
  const int lane = threadIdx.x & 31;
  const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
  const uint32_t pieces = stride >> 4;  // per code
  const uint32_t total = r_pad * pieces;
  for (uint64_t row = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < n; row += warps) {
    uint4* dst = (uint4*)(fat + row * r_pad * stride);
    for (uint32_t t = lane; t < total; t += 32) {
      const uint32_t j = t / pieces, pc = t - j * pieces;
      const uint32_t id = adj[row * r_pad + j];
      dst[t] = id == 0xFFFFFFFFu ? make_uint4(0, 0, 0, 0) : ((const uint4*)(codes + (size_t)id * stride))[pc];
    }
  }
}

// Sum of squared nibbles of each SQ4 code row (padding nibbles are zero).
__global__ void code_norms_kernel(const uint8_t* __restrict__ codes, uint64_t n, uint32_t stride,
                                  uint32_t* __restrict__ out) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t* w = (const uint32_t*)(codes + i * stride);
    uint32_t acc = 0;
    for (uint32_t j = 0; j < stride / 4; ++j) {
      const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
      acc = __dp4a(lo, lo, acc);
      acc = __dp4a(hi, hi, acc);
    }
    out[i] = acc;
  }
}

__global__ void encode_kernel(const float* __restrict__ v, uint64_t n, uint32_t dim, const float* __restrict__ inv,
                              const float* __restrict__ neg, float levels, int sq4, uint32_t stride,
                              uint32_t* __restrict__ out) {
  const uint32_t words = stride / 4;
  const uint64_t total = n * words;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = t / words;
    const uint32_t w = (uint32_t)(t % words);
    const float* r = v + row * dim;
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = w * 4 + b;
      uint32_t val = 0;
      if (sq4) {
        const uint32_t d0 = 2 * byte, d1 = 2 * byte + 1;
        uint32_t lo = d0 < dim ? quantize(r[d0], inv[d0], neg[d0], levels) : 0u;
        uint32_t hi = d1 < dim ? quantize(r[d1], inv[d1], neg[d1], levels) : 0u;
        val = lo | (hi << 4);
      } else {
        val = byte < dim ? quantize(r[byte], inv[byte], neg[byte], levels) : 0u;
      }
      word |= (val & 0xFFu) << (8 * b);
    }
    out[t] = word;
  }
}

// Natural -> lane-major rows (see search_kernel.cuh).
__global__ void permute_rows_kernel(const float* __restrict__ in, float* __restrict__ out, uint64_t n, uint32_t dim) {
  const uint32_t C = dim / 16;
  const uint64_t total = n * dim;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = t / dim;
    const uint32_t d = (uint32_t)(t - r * dim);
    out[r * dim + lane_major_pos(d, C)] = in[t];
  }
}

// out[s] = rows[gid[s]] (row copies, any layout).
__global__ void gather_rows_kernel(const float* __restrict__ rows, const uint32_t* __restrict__ gid, uint64_t m,
                                   uint32_t dim, float* __restrict__ out) {
  const uint64_t total = m * dim;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t s_ = t / dim;
    const uint32_t d = (uint32_t)(t - s_ * dim);
    out[t] = rows[(uint64_t)gid[s_] * dim + d];
  }
}

// ---------------------------------------------------------------------------
// Exact kNN (recall ground truth). Block: 64 queries x 64-row tiles of the
// base, 256 threads, 4x4 register micro-tile of squared distances
// (sum of fma(d,d) over dims: exact for integer-valued data), then a per-query
// sorted top-k (k <= 32) kept in shared memory, ties by id. The base range is
// split over gridDim.y; a second kernel merges the splits.
// ---------------------------------------------------------------------------
constexpr int KQ = 64, KB = 64, KD = 16, KMAXK = 32;

__global__ void __launch_bounds__(256) knn_tile_kernel(const float* __restrict__ base, uint64_t n,
                                                        const float* __restrict__ q, uint64_t nq, uint32_t dim,
                                                        uint32_t k, uint64_t split_rows, uint32_t* __restrict__ out_i,
                                                        float* __restrict__ out_d) {
  __shared__ float qs[KD][KQ + 1];
  __shared__ float bs[KD][KB + 1];
  __shared__ float dt[KQ][KB + 1];
  __shared__ float tk_d[KQ][KMAXK];
  __shared__ uint32_t tk_i[KQ][KMAXK];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const uint64_t q0 = (uint64_t)blockIdx.x * KQ;
  const uint64_t r_begin = (uint64_t)blockIdx.y * split_rows;
  const uint64_t r_end = min(n, r_begin + split_rows);
  for (int i = tid; i < KQ * KMAXK; i += 256) {
    tk_d[i / KMAXK][i % KMAXK] = __int_as_float(0x7f800000);
    tk_i[i / KMAXK][i % KMAXK] = 0xffffffffu;
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  for (uint64_t b0 = r_begin; b0 < r_end; b0 += KB) {
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (uint32_t d0 = 0; d0 < dim; d0 += KD) {
      for (int i = tid; i < KD * KQ; i += 256) {
        int qq = i / KD, dd = i % KD;
        uint64_t qi = q0 + qq;
        // base rows are lane-major: fetch the query element that sits at the
        // same position (position p < 16C holds element 16*(p%C) + p/C)
        const uint32_t p = d0 + dd, C = dim / 16;
        const uint32_t e = p < 16 * C ? 16 * (p % C) + p / C : p;
        qs[dd][qq] = (qi < nq && p < dim) ? q[qi * dim + e] : 0.0f;
      }
      for (int i = tid; i < KD * KB; i += 256) {
        int bb = i / KD, dd = i % KD;
        uint64_t bi = b0 + bb;
        bs[dd][bb] = (bi < r_end && d0 + dd < dim) ? base[bi * dim + d0 + dd] : 0.0f;
      }
      __syncthreads();
#pragma unroll 8
      for (int dd = 0; dd < KD; ++dd) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = qs[dd][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = bs[dd][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float t = a[i] - b[j];
            acc[i][j] = fmaf(t, t, acc[i][j]);
          }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) dt[ty * 4 + i][tx * 4 + j] = acc[i][j];
    __syncthreads();
    // top-k update: warp w owns queries w, w+8, ...
    for (int qq = warp; qq < KQ; qq += 8) {
      const float thr = tk_d[qq][k - 1];
      const uint32_t thr_i = tk_i[qq][k - 1];
      for (int c = lane; c < KB; c += 32) {
        uint64_t bi = b0 + c;
        float d = dt[qq][c];
        bool cand = bi < r_end && (d < thr || (d == thr && (uint32_t)bi < thr_i));
        uint32_t m = __ballot_sync(0xffffffffu, cand);
        while (m) {
          int src = __ffs(m) - 1;
          m &= m - 1;
          float cd = __shfl_sync(0xffffffffu, d, src);
          uint32_t ci = (uint32_t)(b0 + c - lane + src);
          // insert (cd, ci) into the sorted list (lane 0 does it)
          if (lane == 0) {
            int pos = (int)k;
            while (pos > 0 && (tk_d[qq][pos - 1] > cd || (tk_d[qq][pos - 1] == cd && tk_i[qq][pos - 1] > ci))) --pos;
            if (pos < (int)k) {
              for (int t = (int)k - 1; t > pos; --t) {
                tk_d[qq][t] = tk_d[qq][t - 1];
                tk_i[qq][t] = tk_i[qq][t - 1];
              }
              tk_d[qq][pos] = cd;
              tk_i[qq][pos] = ci;
            }
          }
          __syncwarp();
        }
      }
    }
    __syncthreads();
  }
  for (int i = tid; i < KQ * (int)k; i += 256) {
    int qq = i / k, j = i % k;
    uint64_t qi = q0 + qq;
    if (qi < nq) {
      size_t o = ((size_t)blockIdx.y * nq + qi) * k + j;
      out_i[o] = tk_i[qq][j];
      out_d[o] = tk_d[qq][j];
    }
  }
}

// Merge sorted top-k lists: per query, `lists` lists of k (dist, id) entries,
// ascending (dist, id) -> k. One warp per query, rank counting.
__global__ void knn_merge_kernel(const uint32_t* __restrict__ in_i, const float* __restrict__ in_d, uint32_t lists,
                                 uint64_t nq, uint32_t k, uint32_t* __restrict__ out_i, float* __restrict__ out_d) {
  const uint64_t qi = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (qi >= nq) return;
  const uint32_t total = lists * k;
  for (uint32_t e = lane; e < total; e += 32) {
    const uint32_t l = e / k, j = e % k;
    const size_t o = ((size_t)l * nq + qi) * k + j;
    const float d = in_d[o];
    const uint32_t id = in_i[o];
    uint32_t rank = 0;
    for (uint32_t f = 0; f < total; ++f) {
      const size_t p = ((size_t)(f / k) * nq + qi) * k + f % k;
      const float df = in_d[p];
      const uint32_t idf = in_i[p];
      rank += (df < d) || (df == d && (idf < id || (idf == id && f < e)));
    }
    if (rank < k) {
      out_i[qi * k + rank] = id;
      out_d[qi * k + rank] = d;
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core exact kNN: operand preparation (knn_tc.cuh holds the kernel).
// ---------------------------------------------------------------------------
// TF32 value of x, rounded to nearest (ties away), low 13 bits zero.
__device__ inline float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// flags[0] bit 0: a value not exact in TF32 (non-integer or |v| > 2048);
// flags[1], flags[2]: largest base / query squared norm (f32 bits).
__device__ inline bool tf32_exact_int(float v) { return v == rintf(v) && fabsf(v) <= 2048.0f; }

// One warp per base row: squared norm and exactness flags; rows n..n_pad-1
// get +inf (rows past the base never qualify as neighbours).
__global__ void tc_base_norms_kernel(const float* __restrict__ vec, uint64_t n, uint64_t n_pad, uint32_t dim,
                                     float* __restrict__ xn, unsigned* __restrict__ flags) {
  const uint64_t row = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= n_pad) return;
  if (row >= n) {
    if (lane == 0) xn[row] = __int_as_float(0x7f800000);
    return;
  }
  const float* v = vec + row * dim;
  float acc = 0.0f;
  bool inexact = false;
  for (uint32_t j = lane; j < dim; j += 32) {
    const float x = v[j];
    acc = fmaf(x, x, acc);
    inexact |= !tf32_exact_int(x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (__any_sync(0xffffffffu, inexact) && lane == 0) atomicOr(&flags[0], 1u);
  if (lane == 0) {
    xn[row] = acc;
    atomicMax(&flags[1], __float_as_uint(acc));
  }
}

// One warp per query: the row in the base rows' lane-major order (position
// p < 16C holds element 16*(p%C) + p/C), zero-padded to kpad, split into
// TF32 hi and lo parts, its squared norm and the exactness flags. Rows
// nq..nq_pad-1 are zero.
__global__ void tc_query_prep_kernel(const float* __restrict__ q, uint64_t nq, uint64_t nq_pad, uint32_t dim,
                                     uint32_t C, uint32_t kpad, float* __restrict__ qh, float* __restrict__ ql,
                                     float* __restrict__ qn, unsigned* __restrict__ flags) {
  const uint64_t row = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= nq_pad) return;
  float acc = 0.0f;
  bool inexact = false;
  for (uint32_t p = lane; p < kpad; p += 32) {
    float x = 0.0f;
    if (row < nq && p < dim) {
      const uint32_t e = p < 16 * C ? 16 * (p % C) + p / C : p;
      x = q[row * dim + e];
    }
    acc = fmaf(x, x, acc);
    inexact |= !tf32_exact_int(x);
    const float h = tf32_round(x);
    qh[row * kpad + p] = h;
    ql[row * kpad + p] = x - h;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (__any_sync(0xffffffffu, inexact) && lane == 0) atomicOr(&flags[0], 1u);
  if (lane == 0 && row < nq) {
    qn[row] = acc;
    atomicMax(&flags[2], __float_as_uint(acc));
  }
}

// Base hi/lo split for the three-pass form.
__global__ void tc_base_split_kernel(const float* __restrict__ vec, uint64_t total, float* __restrict__ xh,
                                     float* __restrict__ xl) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const float x = vec[i];
    const float h = tf32_round(x);
    xh[i] = h;
    xl[i] = x - h;
  }
}

// F16::from_f32 (src/distance/f16.rs:26-76) with the reference's exact
// behaviour: normal results OR the round bit into the truncated mantissa (an
// odd mantissa is never rounded up), denormal results are truncated, overflow
// gives Inf, NaN gives 0x7E00.
__device__ inline uint16_t f16_from_f32_ref(float f) {
  const uint32_t bits = __float_as_uint(f);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
  const int32_t exp = (int32_t)((bits >> 23) & 0xFFu);
  const uint32_t mant = bits & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | (mant ? 0x7E00u : 0x7C00u));
  const int32_t new_exp = exp - 127 + 15;
  if (new_exp >= 0x1F) return (uint16_t)(sign | 0x7C00u);
  if (new_exp <= 0) {
    if (new_exp < -10) return sign;
    const uint32_t m = mant | 0x800000u;
    return (uint16_t)(sign | (uint16_t)(m >> (14 - new_exp)));
  }
  const uint16_t mant_f16 = (uint16_t)(mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  const uint16_t round = (rem > 0x1000u || (rem == 0x1000u && (mant_f16 & 1u))) ? 1 : 0;
  uint16_t result = (uint16_t)(sign | ((uint16_t)new_exp << 10) | mant_f16 | round);
  if ((result & 0x7C00u) == 0x7C00u) result = (uint16_t)(sign | 0x7C00u);
  return result;
}
// The element-wise conversion commutes with the lane-major permutation, so
// the f16 rows are converted straight from the device's f32 rows.
__global__ void f16_convert_kernel(const float* __restrict__ in, uint64_t total, uint16_t* __restrict__ out) {
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x)
    out[t] = f16_from_f32_ref(in[t]);
}

// Shard merge: ids are shard-local; global id = shard * shard_size + local.
// Shard s's lists start at block b(s) = (s % W) * P + s / W of each array:
// ids at ids + b(s) * stride_i, distances at ds + b(s) * stride_d, counts at
// counts + b(s) * stride_c, each [nq][k] (counts [nq]). W = 1, P = n_shards
// is the shard-major layout; W ranks x P blocks is the layout an all-gather
// of per-rank blocks (shard s on rank s % W, slot s / W) leaves behind.
// One warp per query: each valid entry's output rank is the number of valid
// entries before it in (distance, shard, rank) order.
struct MergeLayout {
  uint32_t W, P;
  uint64_t stride_i, stride_d, stride_c;
  __device__ uint64_t block(uint32_t s) const { return (uint64_t)(s % W) * P + s / W; }
};

constexpr uint32_t kMergeStage = 256;  // candidates per query staged in shared memory (n_shards * k)
constexpr int kMergeThreads = 256;

__global__ void shard_merge_kernel(const uint32_t* __restrict__ ids, const float* __restrict__ ds,
                                   const uint32_t* __restrict__ counts, MergeLayout L, uint32_t n_shards, uint64_t nq,
                                   uint32_t k, uint64_t shard_size, uint32_t* __restrict__ out_i,
                                   float* __restrict__ out_d, uint32_t* __restrict__ out_c) {
  __shared__ float merge_stage[kMergeThreads / 32][kMergeStage];
  const uint64_t qi = (blockIdx.x * (uint64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (qi >= nq) return;  // whole warps
  const uint32_t total = n_shards * k;
  auto cnt_of = [&](uint32_t sh) { return counts ? min(counts[L.block(sh) * L.stride_c + qi], k) : k; };
  auto dist_at = [&](uint32_t sh, uint32_t r) { return ds[L.block(sh) * L.stride_d + qi * k + r]; };
  uint32_t valid_total = 0;
  for (uint32_t sh = 0; sh < n_shards; ++sh) valid_total += cnt_of(sh);
  if (total <= kMergeStage) {
    // the query's candidates staged once, in shard-major order (entry e =
    // shard e / k, rank e % k); entries past a shard's count are NaN, which
    // no comparison counts. Ties by (distance, shard, rank) = (distance, e).
    float* sd = merge_stage[threadIdx.x >> 5];
    for (uint32_t e = lane; e < total; e += 32) {
      const uint32_t sh = e / k, r = e - sh * k;
      sd[e] = r < cnt_of(sh) ? dist_at(sh, r) : __int_as_float(0x7fc00000);
    }
    __syncwarp();
    for (uint32_t e = lane; e < total; e += 32) {
      const float d = sd[e];
      if (d != d) continue;  // past its shard's count
      uint32_t rank = 0;
      for (uint32_t f = 0; f < total; ++f) {
        const float df = sd[f];
        rank += (df < d) || (df == d && f < e);
      }
      if (rank < k) {
        const uint32_t sh = e / k, r = e - sh * k;
        out_i[qi * k + rank] = (uint32_t)(sh * shard_size + ids[L.block(sh) * L.stride_i + qi * k + r]);
        out_d[qi * k + rank] = d;
      }
    }
  } else {
  for (uint32_t e = lane; e < total; e += 32) {
    const uint32_t sh = e / k, r = e % k;
    if (r >= cnt_of(sh)) continue;
    const float d = dist_at(sh, r);
    uint32_t rank = 0;
    for (uint32_t f = 0; f < total; ++f) {
      const uint32_t fs = f / k, fr = f % k;
      if (fr >= cnt_of(fs)) continue;
      const float df = dist_at(fs, fr);
      rank += (df < d) || (df == d && (fs < sh || (fs == sh && fr < r)));
    }
    if (rank < k) {
      out_i[qi * k + rank] = (uint32_t)(sh * shard_size + ids[L.block(sh) * L.stride_i + qi * k + r]);
      out_d[qi * k + rank] = d;
    }
  }
  }
  const uint32_t outc = min(valid_total, k);
  for (uint32_t r = outc + lane; r < k; r += 32) {
    out_i[qi * k + r] = 0;
    out_d[qi * k + r] = 0.0f;
  }
  if (lane == 0 && out_c) out_c[qi] = outc;
}

// ---------------------------------------------------------------------------
// Search launch.
// ---------------------------------------------------------------------------
// The instantiation for a launch: fixed 64-entry pool, run-time pool, or (SQ4
// with four lanes per code, when the host enabled it through a.xnorm) the
// run-time pool with tensor-core distances.
template <int QUANT, int CPL, bool VIS>
auto search_variant(uint32_t pool_cap, bool mma) {
  if constexpr (QUANT == 0 && CPL == 4)
    if (pool_cap > 64 && mma) return search_kernel<QUANT, CPL, 0, VIS, true>;
  return pool_cap <= 64 ? search_kernel<QUANT, CPL, 64, VIS> : search_kernel<QUANT, CPL, 0, VIS>;
}
template <int QUANT, int CPL, bool VIS>
cudaError_t launch_t(const SearchArgs& a, uint32_t smem_per_block, int grid, cudaStream_t st) {
  auto k = search_variant<QUANT, CPL, VIS>(a.pool_cap, a.xnorm != nullptr);
  cudaError_t e = allow_smem((const void*)k, smem_per_block);
  if (e != cudaSuccess) return e;
  k<<<grid, kWarpsPerBlock * 32, smem_per_block, st>>>(a);
  e = cudaGetLastError();
  if (e == cudaErrorInvalidValue) {
    forget_kernel((const void*)k);
    if ((e = allow_smem((const void*)k, smem_per_block)) != cudaSuccess) return e;
    k<<<grid, kWarpsPerBlock * 32, smem_per_block, st>>>(a);
    e = cudaGetLastError();
  }
  return e;
}
template <int QUANT, int CPL, bool VIS>
cudaError_t occupancy_t(uint32_t pool_cap, bool mma, uint32_t smem_per_block, int* blocks) {
  auto k = search_variant<QUANT, CPL, VIS>(pool_cap, mma);
  return blocks_per_sm((const void*)k, kWarpsPerBlock * 32, smem_per_block, blocks);
}

template <int QUANT, bool VIS>
cudaError_t dispatch_cpl(int cpl, bool occ, const SearchArgs& a, uint32_t smem, int grid, cudaStream_t st,
                         int* blocks) {
  switch (cpl) {
    case 1:
      return occ ? occupancy_t<QUANT, 1, VIS>(a.pool_cap, a.xnorm != nullptr, smem, blocks)
                 : launch_t<QUANT, 1, VIS>(a, smem, grid, st);
    case 2:
      return occ ? occupancy_t<QUANT, 2, VIS>(a.pool_cap, a.xnorm != nullptr, smem, blocks)
                 : launch_t<QUANT, 2, VIS>(a, smem, grid, st);
    case 4:
      return occ ? occupancy_t<QUANT, 4, VIS>(a.pool_cap, a.xnorm != nullptr, smem, blocks)
                 : launch_t<QUANT, 4, VIS>(a, smem, grid, st);
    case 8:
      return occ ? occupancy_t<QUANT, 8, VIS>(a.pool_cap, a.xnorm != nullptr, smem, blocks)
                 : launch_t<QUANT, 8, VIS>(a, smem, grid, st);
  }
  return cudaErrorInvalidValue;
}
// vis: the exact visited set (visited counts or the visited order requested,
// or the f32 beam); otherwise pool membership decides new neighbours, with
// the same results and no visited tables (search_kernel.cuh).
cudaError_t dispatch(int quant, int cpl, bool vis, bool occ, const SearchArgs& a, uint32_t smem, int grid,
                     cudaStream_t st, int* blocks) {
  if (quant == RAVEN_QUANT_F32)
    return occ ? occupancy_t<2, 1, true>(a.pool_cap, false, smem, blocks) : launch_t<2, 1, true>(a, smem, grid, st);
  if (vis)
    return quant == 0 ? dispatch_cpl<0, true>(cpl, occ, a, smem, grid, st, blocks)
                      : dispatch_cpl<1, true>(cpl, occ, a, smem, grid, st, blocks);
  return quant == 0 ? dispatch_cpl<0, false>(cpl, occ, a, smem, grid, st, blocks)
                    : dispatch_cpl<1, false>(cpl, occ, a, smem, grid, st, blocks);
}

// Whether a batch-kernel launch needs the exact visited set.
bool needs_visited(int quant, const raven_search_outputs* o) {
  return quant == RAVEN_QUANT_F32 || o->visited || o->history || o->history_len;
}

template <int QUANT, int CPL>
cudaError_t launch_cta_t(const SearchArgs& a, bool vis, uint32_t smem, uint64_t nq, cudaStream_t st) {
  auto k = vis ? search_cta_kernel<QUANT, CPL, true> : search_cta_kernel<QUANT, CPL, false>;
  cudaError_t e = allow_smem((const void*)k, smem);
  if (e != cudaSuccess) return e;
  k<<<(unsigned)nq, kCtaThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e == cudaErrorInvalidValue) {
    forget_kernel((const void*)k);
    if ((e = allow_smem((const void*)k, smem)) != cudaSuccess) return e;
    k<<<(unsigned)nq, kCtaThreads, smem, st>>>(a);
    e = cudaGetLastError();
  }
  return e;
}
template <int QUANT, int CPL>
cudaError_t occupancy_cta_t(bool vis, uint32_t smem, int* per_sm) {
  auto k = vis ? search_cta_kernel<QUANT, CPL, true> : search_cta_kernel<QUANT, CPL, false>;
  return blocks_per_sm((const void*)k, kCtaThreads, smem, per_sm);
}
template <int QUANT>
cudaError_t occupancy_cta_cpl(int cpl, bool vis, uint32_t smem, int* per_sm) {
  switch (cpl) {
    case 1: return occupancy_cta_t<QUANT, 1>(vis, smem, per_sm);
    case 2: return occupancy_cta_t<QUANT, 2>(vis, smem, per_sm);
    case 4: return occupancy_cta_t<QUANT, 4>(vis, smem, per_sm);
    case 8: return occupancy_cta_t<QUANT, 8>(vis, smem, per_sm);
  }
  return cudaErrorInvalidValue;
}
template <int QUANT>
cudaError_t dispatch_cta_cpl(int cpl, const SearchArgs& a, bool vis, uint32_t smem, uint64_t nq, cudaStream_t st) {
  switch (cpl) {
    case 1: return launch_cta_t<QUANT, 1>(a, vis, smem, nq, st);
    case 2: return launch_cta_t<QUANT, 2>(a, vis, smem, nq, st);
    case 4: return launch_cta_t<QUANT, 4>(a, vis, smem, nq, st);
    case 8: return launch_cta_t<QUANT, 8>(a, vis, smem, nq, st);
  }
  return cudaErrorInvalidValue;
}

constexpr int kCtaAutoPerSm = 4;  // small-batch kernel: default limit, resident CTAs per SM
constexpr uint32_t kMmaMaxPool = 160;        // tensor-core distances: largest pool
constexpr uint64_t kMmaMaxNodes = 4u << 20;  // ... and largest index (16 MB of norms)

constexpr uint32_t kMaxEf = 256;
constexpr uint32_t kMaxDimSq4 = 256;
constexpr uint32_t kMaxDimSq8 = 128;
constexpr uint32_t kMaxR = 128;
constexpr uint32_t kMaxNavK = 32;

// AdaptiveEf::estimate_ef for every rank 0..S (src/graph/adaptive_ef.rs:340-359),
// evaluated on the host with the platform powf like the reference.
std::vector<uint32_t> ef_table(uint32_t S, uint32_t min_ef, uint32_t max_ef, float gamma) {
  std::vector<uint32_t> t(S + 1);
  for (uint32_t r = 0; r <= S; ++r) {
    float pct = (float)r / (float)S;
    float shaped = powf(pct, gamma);
    float ef = std::fma(shaped, (float)(max_ef - min_ef), (float)min_ef);
    float rd = std::round(ef);
    uint32_t v = 0;
    if (rd > 0.0f) v = rd >= 4294967295.0f ? 0xFFFFFFFFu : (uint32_t)rd;
    t[r] = v;
  }
  return t;
}

struct Plan {
  int quant, cpl, hash_bits, spill_bits;
  uint32_t f32_stage_rows;  // f32 traversal: neighbour rows staged per round
  uint32_t pool_cap;  // beam pool entries per warp: ef_cap rounded up to 32
  uint32_t ef_cap;
  uint32_t smem_warp, smem_block;
  std::vector<uint32_t> table;
  uint32_t ef_mid;
};

int make_plan(const raven_index* ix, const raven_search_params* p, Plan* pl) {
  if (!p) return fail(RAVEN_EINVAL, "null search params");
  if (p->quant != RAVEN_QUANT_SQ4 && p->quant != RAVEN_QUANT_SQ8 && p->quant != RAVEN_QUANT_F32)
    return fail(RAVEN_EINVAL, "unknown quant");
  if (p->quant != RAVEN_QUANT_F32 && !ix->has_q[p->quant])
    return fail(RAVEN_ESTATE, p->quant == 0 ? "search_sq4 requires with_sq4() first (index uploaded without SQ4)"
                                            : "search_sq8 requires with_sq8() first (index uploaded without SQ8)");
  if (p->k == 0) return fail(RAVEN_EINVAL, "k must be >= 1");
  if (p->rerank_f16 && !ix->d_vec16)
    return fail(RAVEN_ESTATE, "with_f16 requires an index uploaded with build_f16");
  pl->quant = p->quant;
  const bool f32 = p->quant == RAVEN_QUANT_F32;
  pl->cpl = f32 ? 1 : (int)(ix->q_stride[p->quant] / 16);
  pl->f32_stage_rows = f32 ? (ix->dim_pad <= 128 ? 16u : 8u) : 0u;
  uint32_t ef_cap;
  if (p->adaptive) {
    if (p->max_ef < p->min_ef) return fail(RAVEN_EINVAL, "max_ef must be >= min_ef");
    uint32_t S = (uint32_t)ix->h_samples.size();
    if (S == 0 && !ix->has_nav) return fail(RAVEN_ESTATE, "AdaptiveEf requires layered nav samples");
    pl->table = ef_table(S, p->min_ef, p->max_ef, p->gamma);
    pl->ef_mid = p->min_ef + (p->max_ef - p->min_ef) / 2;  // usize::midpoint
    ef_cap = pl->ef_mid;
    if (S > 1)
      for (uint32_t v : pl->table) ef_cap = std::max(ef_cap, v);
    ef_cap = std::max(ef_cap, p->k);
    if (S <= 1 && std::max(pl->ef_mid, p->k) == 0) return fail(RAVEN_EINVAL, "ef must be >= 1");
  } else {
    if (p->ef == 0) return fail(RAVEN_EINVAL, "ef must be >= 1");
    ef_cap = p->ef;
  }
  if (ef_cap > kMaxEf) return fail(RAVEN_ELIMIT, "ef above the engine limit of 256");
  pl->ef_cap = ef_cap;
  pl->pool_cap = ef_cap <= 64 ? 64u : (ef_cap + 31) & ~31u;  // <= 64: the fixed-layout kernel
  uint32_t hb = ix->hash_bits_override;
  if (hb == 0) {
    // Shared-memory visited slots per warp. Past 3/4 load a query continues
    // in its global spill table, whose probes overlap the code
    // gather; a smaller shared table buys residency. Measured on a 1M-node
    // graph: 2048 slots best at ef <= 64, 1024 beyond.
    hb = ef_cap <= 64 ? 11 : 10;
  }
  // Level A slots per warp; level B (8x) catches outliers. A query visits
  // ~25 nodes per unit of ef, and a sparser table means fewer lanes of a row
  // contending for one bucket in the warp-cooperative insert. Measured on a
  // 1M-node graph (B200, 10k-query batches): ef=140 with 2^12 / 2^13 / 2^14 /
  // 2^15 slots 2.83 / 3.49 / 3.70 / 3.45 M QPS; ef=50 with 2^12 / 2^13 / 2^14
  // slots 7.56 / 7.65 / 7.50 M QPS. Sized by the ef a typical query runs at:
  // the fixed ef, or the median of the AdaptiveEf rank -> ef table.
  uint32_t ef_typ = ef_cap;
  if (p->adaptive)  // with <= 1 sample every query runs at ef_mid
    ef_typ = std::max(pl->table.size() > 2 ? pl->table[pl->table.size() / 2] : pl->ef_mid, p->k);
  uint32_t sb = ix->spill_bits_override;
  if (sb == 0) sb = ef_typ <= 80 ? 13 : 14;
  pl->spill_bits = (int)sb;
  // the visited table doubles as the row staging area: it must hold a row
  while ((1u << hb) < ix->dim_pad) ++hb;
  pl->hash_bits = (int)hb;
  pl->smem_warp = warp_smem_bytes(ix->dim_pad, f32 ? 0u : ix->q_stride[p->quant], pl->pool_cap, hb, ix->r_pad,
                                  pl->f32_stage_rows);
  pl->smem_block = pl->smem_warp * kWarpsPerBlock;
  return RAVEN_OK;
}

// The per-node code norms when a batch launch should use the tensor-core SQ4
// distances (the instantiation is chosen from them), else null (dp4a).
// Measured faster for pools of up to 160 entries while the norms stay in L2
// (1M nodes: ef 100-160 +4-5 %); slower at ef 200 (-14 %) and on 10M nodes,
// whose 40 MB of norms cost a DRAM sector per neighbour (-4 % at ef 100).
const uint32_t* mma_norms(const raven_index* ix, const Plan& pl) {
  const bool on = pl.quant == RAVEN_QUANT_SQ4 && pl.cpl == 4 && pl.pool_cap > 64 && pl.pool_cap <= kMmaMaxPool &&
                  ix->n <= kMmaMaxNodes;
  return on ? ix->d_xnorm : nullptr;
}

// Kernel arguments shared by every search launch (the caller sets the
// queries, the scratch areas and the work counter).
void fill_args(const raven_index* ix, const Plan& pl, const raven_search_params* p, const raven_search_outputs* o,
               SearchArgs* out) {
  SearchArgs& a = *out;
  const bool f32 = pl.quant == RAVEN_QUANT_F32;
  a.vec = ix->d_vec;
  a.dim = ix->dim;
  a.dim_pad = ix->dim_pad;
  a.vec_c = ix->dim / 16;
  a.vec_rem = ix->dim % 16;
  a.adj = ix->d_adj;
  a.r_pad = ix->r_pad;
  a.vec16 = ix->d_vec16;
  a.rerank_f16 = p->rerank_f16 ? 1 : 0;
  a.pool_cap = pl.pool_cap;
  a.codes = f32 ? nullptr : ix->d_codes[pl.quant];
  a.code_stride = f32 ? 0u : ix->q_stride[pl.quant];
  a.q_inv = f32 ? nullptr : ix->d_qparams[pl.quant] + 3 * ix->dim;
  a.q_neg = f32 ? nullptr : ix->d_qparams[pl.quant] + 4 * ix->dim;
  a.levels = pl.quant == 0 ? 15.0f : 255.0f;
  a.dist_bits = 32;
  if (!f32) {
    // largest SQ distance: (levels^2) per dimension over the padded code
    const uint64_t per_dim = pl.quant == 0 ? 225ull : 65025ull;
    const uint64_t dims = pl.quant == 0 ? (uint64_t)ix->q_stride[0] * 2 : (uint64_t)ix->q_stride[1];
    const uint64_t mx = per_dim * dims;
    uint32_t b = 0;
    while (b < 32 && (mx >> b) != 0) ++b;
    a.dist_bits = b;
  }
  a.entry = ix->entry;
  a.nav = ix->has_nav ? 1 : 0;
  a.nav_entry_h = ix->nav_entry_h;
  a.nav_max_level = ix->nav_max_level;
  a.nav_k = ix->nav_k;
  a.nav_stride_levels = ix->nav_stride_levels;
  a.nav_vec = ix->d_nav_vec;
  a.nav_e = ix->d_nav_e;
  a.nav_gid = ix->d_nav_gid;
  a.adaptive = p->adaptive ? 1 : 0;
  a.samples = ix->d_samples;
  a.n_samples = (uint32_t)ix->h_samples.size();
  a.ef_mid = pl.ef_mid;
  a.ef_fixed = p->ef;
  a.k = p->k;
  a.rr = std::max<uint32_t>(p->rerank_factor, 1);
  a.hash_bits = pl.hash_bits;
  // neighbour codes beside the rows (read by the small-batch search without a visited set)
  a.fat = f32 ? nullptr : ix->d_fat[pl.quant];
  a.xnorm = mma_norms(ix, pl);
  a.spill_bits = pl.spill_bits;
  a.smem_per_warp = pl.smem_warp;
  a.f32_stage_rows = pl.f32_stage_rows;
  a.ids = o->ids;
  a.dists = o->dists;
  a.counts = o->counts;
  a.visited = o->visited;
  a.ef_used = o->ef_used;
  a.status = o->status;
  a.n_nav = o->n_nav;
  a.expansions = o->expansions;
  a.history = o->history;
  a.hist_cap = o->history ? o->history_cap : 0;
  a.hist_len = o->history_len;
}

// Shared-memory visited-table bits of the small-batch kernel (0: none).
uint32_t cta_hash_bits(const raven_index* ix, bool vis) {
  if (!vis) return 0;
  // the tuning hook can shrink the table (tests reach the spill levels this way)
  uint32_t hb = ix->hash_bits_override ? std::min<uint32_t>((uint32_t)ix->hash_bits_override, kCtaHashBits)
                                       : kCtaHashBits;
  while ((1u << hb) < ix->dim_pad) ++hb;
  return hb;
}

// Small batches: one CTA of four warps per query (search_cta.cuh). With the
// visited count or order requested, the visited set lives in a 2^14-slot
// shared table, and per-query global spill tables (2^13-slot level A, level B
// 8x) stay allocated for exactness, touched only by a query that fills the
// shared table; otherwise pool membership decides and nothing is allocated
// but the ef table. Same results as the batch kernel.
int run_search_cta(raven_index* ix, const float* d_q, uint64_t nq, const raven_search_params* p, const Plan& pl,
                   const raven_search_outputs* o, cudaStream_t st) {
  const bool vis = needs_visited(pl.quant, o);
  const uint32_t hb = cta_hash_bits(ix, vis);
  const uint32_t kSpill = ix->spill_bits_override ? std::min<uint32_t>((uint32_t)ix->spill_bits_override, 13u) : 13u;
  const uint32_t smem = cta_smem_bytes(ix->dim_pad, ix->q_stride[pl.quant], pl.pool_cap, hb, ix->r_pad);
  const size_t spill_bytes = vis ? (size_t)nq * (9ull << kSpill) * 4 : 0;
  const size_t table_bytes = pl.table.size() * 4;
  uint8_t* scratch = nullptr;
  CU(cudaMallocAsync((void**)&scratch, spill_bytes + ((table_bytes + 255) & ~(size_t)255) + 256, st));
  uint32_t* spill = (uint32_t*)scratch;
  uint32_t* table = (uint32_t*)(scratch + spill_bytes);
  cudaError_t e = cudaSuccess;
  if (table_bytes) e = cudaMemcpyAsync(table, pl.table.data(), table_bytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) {
    SearchArgs a{};
    fill_args(ix, pl, p, o, &a);
    a.hash_bits = hb;
    a.spill_bits = kSpill;
    a.ef_table = table;
    a.spill = vis ? spill : nullptr;
    a.n_slots = nq;
    a.queries = d_q;
    a.nq = nq;
    a.counter = nullptr;
    a.nav_only = 0;
    e = pl.quant == 0 ? dispatch_cta_cpl<0>(pl.cpl, a, vis, smem, nq, st)
                      : dispatch_cta_cpl<1>(pl.cpl, a, vis, smem, nq, st);
  }
  cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("small-batch search launch: ") + cudaGetErrorString(e));
  return RAVEN_OK;
}

// Runs the search (or the nav-only descent) for device buffers.
int run_search(raven_index* ix, const float* d_q, uint64_t nq, const raven_search_params* p,
               const raven_search_outputs* o, cudaStream_t st, int nav_only) {
  Plan pl;
  raven_search_params nav_p{};
  if (nav_only) {
    nav_p.quant = ix->has_q[0] ? RAVEN_QUANT_SQ4 : ix->has_q[1] ? RAVEN_QUANT_SQ8 : RAVEN_QUANT_F32;
    nav_p.ef = 1;
    nav_p.k = 1;
    p = &nav_p;
  }
  int rc = make_plan(ix, p, &pl);
  if (rc) return rc;
  if (nq == 0) return RAVEN_OK;
  if (!o || !o->ids) return fail(RAVEN_EINVAL, "outputs.ids is required");
  CU(cudaSetDevice(ix->device));
  if (!nav_only && pl.quant != RAVEN_QUANT_F32 && !p->rerank_f16 && nq <= ix->small_batch_max) {
    uint64_t lim = ix->small_batch_max;
    if (lim == ~0ull) {  // as many queries as one wave of CTAs holds
      int per_sm = 0;
      const bool vis = needs_visited(pl.quant, o);
      const uint32_t smem =
          cta_smem_bytes(ix->dim_pad, ix->q_stride[pl.quant], pl.pool_cap, vis ? kCtaHashBits : 0u, ix->r_pad);
      CU(pl.quant == 0 ? occupancy_cta_cpl<0>(pl.cpl, vis, smem, &per_sm)
                       : occupancy_cta_cpl<1>(pl.cpl, vis, smem, &per_sm));
      // measured on a 1M-node graph (ef 50 and 140): the persistent kernel
      // takes over between 3 and 6 resident CTAs per SM
      lim = (uint64_t)std::min(std::max(per_sm, 0), kCtaAutoPerSm) * (uint64_t)ix->num_sms;
    }
    if (nq <= lim) return run_search_cta(ix, d_q, nq, p, pl, o, st);
  }
  int blocks_per_sm = 0;
  SearchArgs occ_args{};
  occ_args.pool_cap = pl.pool_cap;  // selects the kernel variant whose occupancy is asked
  occ_args.xnorm = mma_norms(ix, pl);
  const bool vis = nav_only || needs_visited(pl.quant, o);
  CU(dispatch(pl.quant, pl.cpl, vis, true, occ_args, pl.smem_block, 0, st, &blocks_per_sm));
  if (blocks_per_sm <= 0) return fail(RAVEN_ELIMIT, "search kernel does not fit on an SM with this configuration");
  uint64_t grid64 = (uint64_t)blocks_per_sm * ix->num_sms;
  uint64_t need = (nq + kWarpsPerBlock - 1) / kWarpsPerBlock;
  int grid = (int)std::max<uint64_t>(1, std::min(grid64, need));
  const uint64_t slots = (uint64_t)grid * kWarpsPerBlock;
  // per-call scratch: work counter, spill tables (exact visited set only), ef table (stream ordered)
  const size_t spill_bytes = vis && !nav_only ? (size_t)slots * (9ull << pl.spill_bits) * 4 : 0;  // levels A + B
  const size_t table_bytes = pl.table.size() * 4;
  size_t total = 256 + spill_bytes + ((table_bytes + 255) & ~(size_t)255);
  uint8_t* scratch = nullptr;
  CU(cudaMallocAsync((void**)&scratch, total, st));
  unsigned long long* counter = (unsigned long long*)scratch;
  uint32_t* spill = (uint32_t*)(scratch + 256);
  uint32_t* table = (uint32_t*)(scratch + 256 + spill_bytes);
  cudaError_t e = cudaMemsetAsync(counter, 0, 8, st);
  if (e == cudaSuccess && table_bytes)
    e = cudaMemcpyAsync(table, pl.table.data(), table_bytes, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) {
    cudaFreeAsync(scratch, st);
    return fail(RAVEN_ECUDA, std::string("scratch setup: ") + cudaGetErrorString(e));
  }
  SearchArgs a{};
  fill_args(ix, pl, p, o, &a);
  a.ef_table = table;
  a.spill = spill_bytes ? spill : nullptr;
  a.n_slots = slots;
  a.queries = d_q;
  a.nq = nq;
  a.rerank_f16 = (!nav_only && p->rerank_f16) ? 1 : 0;
  a.counter = counter;
  a.nav_only = nav_only;
  e = dispatch(pl.quant, pl.cpl, vis, false, a, pl.smem_block, grid, st, nullptr);
  cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("search launch: ") + cudaGetErrorString(e));
  return RAVEN_OK;
}

template <class T>
int dev_alloc_copy(T** dst, const T* src, size_t count) {
  CU(cudaMalloc((void**)dst, std::max<size_t>(count, 1) * sizeof(T)));
  if (count) CU(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice));
  return RAVEN_OK;
}

// Builds (or frees) the neighbour codes beside each row for quantiser q.
// Skipped, not failed, when they would take more than half of the free device
// memory: the search then gathers the codes from the code array instead.
int set_fat_rows(raven_index* ix, int q, bool enable) {
  cudaFree(ix->d_fat[q]);
  ix->d_fat[q] = nullptr;
  if (!enable || !ix->has_q[q]) return RAVEN_OK;
  const size_t bytes = (size_t)ix->n * ix->r_pad * ix->q_stride[q];
  size_t free_b = 0, total_b = 0;
  CU(cudaMemGetInfo(&free_b, &total_b));
  if (bytes > free_b / 2) return RAVEN_OK;
  if (cudaMalloc((void**)&ix->d_fat[q], bytes) != cudaSuccess) {
    cudaGetLastError();
    ix->d_fat[q] = nullptr;
    return RAVEN_OK;
  }
  fat_rows_kernel<<<ix->num_sms * 8, 256, 0, ix->stream>>>(ix->d_adj, ix->d_codes[q], ix->n, ix->r_pad,
                                                          ix->q_stride[q], ix->d_fat[q]);
  CU(cudaGetLastError());
  CU(cudaStreamSynchronize(ix->stream));
  return RAVEN_OK;
}

void free_index(raven_index* ix) {
  if (!ix) return;
  cudaSetDevice(ix->device);
  cudaFree(ix->d_vec);
  cudaFree(ix->d_vec16);
  cudaFree(ix->d_adj);
  for (int q = 0; q < 2; ++q) {
    cudaFree(ix->d_codes[q]);
    cudaFree(ix->d_fat[q]);
    cudaFree(ix->d_qparams[q]);
  }
  cudaFree(ix->d_xnorm);
  cudaFree(ix->d_nav_vec);
  cudaFree(ix->d_nav_e);
  cudaFree(ix->d_nav_gid);
  cudaFree(ix->d_samples);
  if (ix->stream) cudaStreamDestroy(ix->stream);
  delete ix;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* raven_last_error(void) { return g_err.c_str(); }
const char* raven_version(void) { return "raven-b200 0.1 (sm_100a)"; }

void raven_limits(raven_limits_t* out) {
  if (!out) return;
  out->max_ef = kMaxEf;
  out->max_dim = kMaxDimSq4;
  out->max_r = kMaxR;
  out->max_nav_k = kMaxNavK;
}

int raven_graph_build(const float* vectors, uint64_t n, uint32_t dim, const raven_build_config* cfg,
                      raven_graph** out) {
  NvtxRange nvtx_range("raven.graph_build");
  if (!out || (!vectors && n) || !cfg) return fail(RAVEN_EINVAL, "null argument");
  raven::BuildConfig c;
  c.alpha = cfg->alpha;
  c.l_build = cfg->l_build;
  c.r_max = cfg->r_max;
  c.r_soft = cfg->r_soft;
  c.max_iterations = cfg->max_iterations;
  c.saturate = cfg->saturate != 0;
  c.enable_layered_nav = cfg->layered_nav != 0;
  c.nav_m = cfg->nav_m;
  c.directional = cfg->directional != 0;
  c.seed = cfg->seed;
  c.threads = cfg->threads;
  c.verbose = cfg->verbose;
  if (c.nav_m < 2) return fail(RAVEN_EINVAL, "nav_m must be >= 2");
  raven_graph* g = new raven_graph();
  std::string err;
  int rc = raven::build_vamana(vectors, n, dim, c, &g->g, &err);
  if (rc) {
    delete g;
    return fail(rc, err);
  }
  *out = g;
  return RAVEN_OK;
}

int raven_graph_load_bytes(const void* bytes, size_t len, raven_graph** out) {
  if (!out || (!bytes && len)) return fail(RAVEN_EINVAL, "null argument");
  raven_graph* g = new raven_graph();
  std::string err;
  int rc = raven::parse_annx((const uint8_t*)bytes, len, &g->g, &err);
  if (rc) {
    delete g;
    return fail(rc, err);
  }
  *out = g;
  return RAVEN_OK;
}

int raven_graph_load(const char* path, raven_graph** out) {
  if (!path || !out) return fail(RAVEN_EINVAL, "null argument");
  std::ifstream f(path, std::ios::binary);
  if (!f) return fail(RAVEN_EIO, std::string("cannot open ") + path);
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return raven_graph_load_bytes(bytes.data(), bytes.size(), out);
}

int raven_graph_save(const raven_graph* g, const char* path) {
  if (!g || !path) return fail(RAVEN_EINVAL, "null argument");
  std::vector<uint8_t> bytes = raven::serialize_annx(g->g);
  std::ofstream f(path, std::ios::binary);
  if (!f) return fail(RAVEN_EIO, std::string("cannot open ") + path + " for writing");
  f.write((const char*)bytes.data(), (std::streamsize)bytes.size());
  if (!f) return fail(RAVEN_EIO, std::string("write failed: ") + path);
  return RAVEN_OK;
}

void raven_graph_free(raven_graph* g) { delete g; }

int raven_graph_info(const raven_graph* g, raven_graph_info_t* out) {
  if (!g || !out) return fail(RAVEN_EINVAL, "null argument");
  out->n = g->g.n;
  out->dim = g->g.dim;
  out->r_max = g->g.r_max;
  out->entry_point = g->g.entry;
  out->has_nav = g->g.nav.present ? 1 : 0;
  out->nav_entry = g->g.nav.entry;
  out->nav_max_level = g->g.nav.max_level;
  out->nav_k = g->g.nav.k;
  uint64_t c = 0;
  for (auto& l : g->g.nav.upper) c += !l.empty();
  out->nav_upper_nodes = c;
  return RAVEN_OK;
}

int raven_graph_neighbors(const raven_graph* g, uint32_t node, uint32_t* out, uint32_t cap, uint32_t* deg) {
  if (!g || node >= g->g.n) return fail(RAVEN_EINVAL, "node out of range");
  uint32_t d = g->g.degrees[node];
  const uint32_t* row = g->g.main_block.data() + (size_t)node * g->g.r_max;
  for (uint32_t i = 0; i < d && i < cap; ++i) out[i] = row[i];
  if (deg) *deg = d;
  return RAVEN_OK;
}

int raven_index_upload(const raven_graph* gr, const float* vectors, uint64_t n, uint32_t dim,
                       const raven_upload_options* opt, raven_index** out) {
  NvtxRange nvtx_range("raven.index_upload");
  if (!gr || !out || (!vectors && n)) return fail(RAVEN_EINVAL, "null argument");
  const raven::HostGraph& g = gr->g;
  if (n != g.n) return fail(RAVEN_EINVAL, "vector count does not match the graph");
  if (dim != g.dim) return fail(RAVEN_EINVAL, "dim mismatch: expected " + std::to_string(g.dim) + ", got " + std::to_string(dim));
  if (n == 0) return fail(RAVEN_EINVAL, "empty index");
  if (n >= 0x7FFFFFFFull) return fail(RAVEN_ELIMIT, "node ids must fit in 31 bits");
  raven_upload_options o{0, 1, 0, 0, 0};
  if (opt) o = *opt;
  if (g.r_max > kMaxR) return fail(RAVEN_ELIMIT, "graph degree above the engine limit of 128");
  if (o.build_sq4 && dim > kMaxDimSq4) return fail(RAVEN_ELIMIT, "dim above the SQ4 engine limit of 256");
  if (o.build_sq8 && dim > kMaxDimSq8) return fail(RAVEN_ELIMIT, "dim above the SQ8 engine limit of 128");
  // validate ids before any device work (ids index device arrays)
  if (g.entry >= n) return fail(RAVEN_EFORMAT, "entry point out of range");
  for (size_t i = 0; i < g.main_block.size(); ++i)
    if (g.main_block[i] != raven::kSentinel && g.main_block[i] >= n)
      return fail(RAVEN_EFORMAT, "adjacency id out of range at slot " + std::to_string(i));
  const bool nav = g.nav.present;
  if (nav) {
    if (g.nav.entry >= n) return fail(RAVEN_EFORMAT, "navigation entry out of range");
    if (g.nav.max_level > 0 && (g.nav.k == 0 || g.nav.k > kMaxNavK))
      return fail(RAVEN_ELIMIT, "navigation degree K must be in 1..32");
    if (g.nav.upper.size() > n) return fail(RAVEN_EFORMAT, "navigation covers more nodes than the graph");
    for (auto& l : g.nav.upper)
      for (uint32_t v : l)
        if (v >= n) return fail(RAVEN_EFORMAT, "navigation edge out of range");
  }
  int dev_count = 0;
  CU(cudaGetDeviceCount(&dev_count));
  if (o.device < 0 || o.device >= dev_count) return fail(RAVEN_EINVAL, "no such CUDA device");
  CU(cudaSetDevice(o.device));
  raven_index* ix = new raven_index();
  ix->device = o.device;
  auto bail = [&](int rc) {
    free_index(ix);
    return rc;
  };
  if (cudaDeviceGetAttribute(&ix->num_sms, cudaDevAttrMultiProcessorCount, o.device) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ix->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(fail(RAVEN_ECUDA, "device query / stream creation failed"));
  ix->small_batch_max = ~0ull;  // one wave of CTAs (resolved per call)

  {
    // per-call scratch comes from the device's stream-ordered pool; keep freed
    // blocks cached instead of returning them to the driver at every sync
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, o.device) == cudaSuccess) {
      uint64_t thr = ~0ull;
      cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
    }
  }
  ix->n = n;
  ix->dim = dim;
  ix->dim_pad = (dim + 15) & ~15u;
  ix->r_max = (uint32_t)g.r_max;
  ix->r_pad = (ix->r_max + 31) & ~31u;
  ix->entry = g.entry;
  int rc;
  float* d_nat = nullptr;  // natural layout, needed until codes and samples exist
  if ((rc = dev_alloc_copy(&d_nat, vectors, n * (size_t)dim))) return bail(rc);
  auto bail2 = [&](int code) {
    cudaFree(d_nat);
    return bail(code);
  };
  if (cudaMalloc((void**)&ix->d_vec, n * (size_t)dim * 4) != cudaSuccess)
    return bail2(fail(RAVEN_ENOMEM, "vector allocation failed"));
  permute_rows_kernel<<<ix->num_sms * 8, 256, 0, ix->stream>>>(d_nat, ix->d_vec, n, dim);
  if (cudaGetLastError() != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "permute launch failed"));
  // adjacency, padded to r_pad. Each row is cut at its first SENTINEL (the
  // degree rule of HybridBlockedCsr::from_parts, src/memory/graph.rs:234-240)
  // and later repeats of an id are dropped: the reference marks a repeat as
  // already visited and does nothing else with it (src/graph/vamana.rs:824-832),
  // so the search sees the same sequence of new neighbours.
  {
    std::vector<uint32_t> pad((size_t)n * ix->r_pad, raven::kSentinel);
    const uint32_t rm = (uint32_t)g.r_max, rp = ix->r_pad;
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; ++i) {
      const uint32_t* src = g.main_block.data() + (size_t)i * rm;
      uint32_t* dst = pad.data() + (size_t)i * rp;
      uint32_t m = 0;
      for (uint32_t t = 0; t < rm && src[t] != raven::kSentinel; ++t) {
        bool dup = false;
        for (uint32_t u = 0; u < m; ++u) dup |= dst[u] == src[t];
        if (!dup) dst[m++] = src[t];
      }
    }
    if ((rc = dev_alloc_copy(&ix->d_adj, pad.data(), pad.size()))) return bail2(rc);
  }
  // quantisers: fit on the host (exact sequential min/max semantics), encode on the device
  for (int q = 0; q < 2; ++q) {
    if (!(q == 0 ? o.build_sq4 : o.build_sq8)) continue;
    uint32_t bytes = q == 0 ? (dim + 1) / 2 : dim;
    uint32_t stride = std::max<uint32_t>(16, next_pow2(bytes));
    ix->q_stride[q] = stride;
    ix->h_qparams[q].resize(5 * (size_t)dim);
    raven::sq_fit_host(vectors, n, dim, q == 0 ? 15.0f : 255.0f, ix->h_qparams[q].data(), 0);
    if ((rc = dev_alloc_copy(&ix->d_qparams[q], ix->h_qparams[q].data(), ix->h_qparams[q].size()))) return bail2(rc);
    if (cudaMalloc((void**)&ix->d_codes[q], (size_t)n * stride) != cudaSuccess)
      return bail2(fail(RAVEN_ENOMEM, "code allocation failed"));
    encode_kernel<<<ix->num_sms * 8, 256, 0, ix->stream>>>(d_nat, n, dim, ix->d_qparams[q] + 3 * dim,
                                                          ix->d_qparams[q] + 4 * dim, q == 0 ? 15.0f : 255.0f,
                                                          q == 0, stride, (uint32_t*)ix->d_codes[q]);
    if (cudaGetLastError() != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "encode launch failed"));
    ix->has_q[q] = true;
    if (q == 0) {
      if (cudaMalloc((void**)&ix->d_xnorm, (size_t)n * 4) != cudaSuccess)
        return bail2(fail(RAVEN_ENOMEM, "code norm allocation failed"));
      code_norms_kernel<<<ix->num_sms * 8, 256, 0, ix->stream>>>(ix->d_codes[0], n, stride, ix->d_xnorm);
      if (cudaGetLastError() != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "code norm launch failed"));
    }
    if ((rc = set_fat_rows(ix, q, true))) return bail2(rc);
  }
  // navigation layers: every node with an upper list gets a slot; its edges
  // are stored per level at a fixed stride (stride_levels x k, kSent padded)
  // as handles (slot, or kGidBit|id for a target without upper list), and
  // its vector is copied into a compact lane-major array.
  if (nav) {
    ix->has_nav = true;
    ix->nav_max_level = g.nav.max_level;
    ix->nav_k = std::max<uint32_t>(g.nav.k, 1);
    const uint32_t K = ix->nav_k;
    std::vector<uint32_t> slot(n, raven::kSentinel), gid;
    uint32_t levels = 0;
    for (size_t i = 0; i < g.nav.upper.size(); ++i) {
      if (g.nav.upper[i].empty()) continue;
      slot[i] = (uint32_t)gid.size();
      gid.push_back((uint32_t)i);
      levels = std::max<uint32_t>(levels, (uint32_t)((g.nav.upper[i].size() + K - 1) / K));
    }
    ix->nav_stride_levels = levels;
    auto handle = [&](uint32_t v) { return slot[v] != raven::kSentinel ? slot[v] : (kGidBit | v); };
    std::vector<uint32_t> e((size_t)gid.size() * levels * K, raven::kSentinel);
    for (size_t sl = 0; sl < gid.size(); ++sl) {
      const auto& l = g.nav.upper[gid[sl]];
      for (size_t t = 0; t < l.size(); ++t) e[sl * levels * K + t] = handle(l[t]);
    }
    ix->nav_entry_h = handle(g.nav.entry);
    if ((rc = dev_alloc_copy(&ix->d_nav_e, e.data(), e.size()))) return bail2(rc);
    if ((rc = dev_alloc_copy(&ix->d_nav_gid, gid.data(), gid.size()))) return bail2(rc);
    if (cudaMalloc((void**)&ix->d_nav_vec, std::max<size_t>(gid.size(), 1) * dim * 4) != cudaSuccess)
      return bail2(fail(RAVEN_ENOMEM, "nav vector allocation failed"));
    if (!gid.empty()) {
      gather_rows_kernel<<<ix->num_sms * 4, 256, 0, ix->stream>>>(ix->d_vec, ix->d_nav_gid, gid.size(), dim,
                                                                  ix->d_nav_vec);
      if (cudaGetLastError() != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "nav gather failed"));
    }
  }
  if (o.build_f16) {
    if (cudaMalloc((void**)&ix->d_vec16, n * dim * 2) != cudaSuccess) return bail2(fail(RAVEN_ENOMEM, "f16 vectors"));
    f16_convert_kernel<<<ix->num_sms * 4, 256, 0, ix->stream>>>(ix->d_vec, n * dim, ix->d_vec16);
    if (cudaGetLastError() != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "f16 conversion failed"));
  }
  if (cudaStreamSynchronize(ix->stream) != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "upload failed"));
  // AdaptiveEf samples: nav.initialize distances of base vectors 0..min(n,2000)
  if (o.build_adaptive) {
    if (!nav) return bail2(fail(RAVEN_ESTATE, "AdaptiveEf requires layered nav (enable_layered_nav=true)"));
    uint32_t S = (uint32_t)std::min<uint64_t>(n, 2000);
    uint32_t* d_e = nullptr;
    float* d_d = nullptr;
    if (cudaMalloc((void**)&d_e, S * 4) != cudaSuccess || cudaMalloc((void**)&d_d, S * 4) != cudaSuccess) {
      cudaFree(d_e);
      return bail2(fail(RAVEN_ENOMEM, "sample buffers"));
    }
    raven_search_outputs so{};
    so.ids = d_e;
    so.dists = d_d;
    rc = run_search(ix, d_nat, S, nullptr, &so, ix->stream, 1);
    ix->h_samples.resize(S);
    cudaError_t e = rc ? cudaSuccess : cudaMemcpyAsync(ix->h_samples.data(), d_d, S * 4, cudaMemcpyDeviceToHost, ix->stream);
    cudaError_t e2 = cudaStreamSynchronize(ix->stream);
    cudaFree(d_e);
    cudaFree(d_d);
    if (rc) return bail2(rc);
    if (e != cudaSuccess || e2 != cudaSuccess) return bail2(fail(RAVEN_ECUDA, "sample distances"));
    std::sort(ix->h_samples.begin(), ix->h_samples.end());
    if ((rc = dev_alloc_copy(&ix->d_samples, ix->h_samples.data(), ix->h_samples.size()))) return bail2(rc);
  }
  cudaFree(d_nat);
  *out = ix;
  return RAVEN_OK;
}

int raven_index_free(raven_index* ix) {
  free_index(ix);
  return RAVEN_OK;
}

int raven_index_adaptive_samples(const raven_index* ix, float* out, uint32_t cap, uint32_t* n_out) {
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  uint32_t S = (uint32_t)ix->h_samples.size();
  if (out)
    for (uint32_t i = 0; i < S && i < cap; ++i) out[i] = ix->h_samples[i];
  if (n_out) *n_out = S;
  return RAVEN_OK;
}

int raven_index_sq_params(const raven_index* ix, int32_t quant, float* out5dim) {
  if (!ix || !out5dim || (quant != 0 && quant != 1)) return fail(RAVEN_EINVAL, "bad argument");
  if (!ix->has_q[quant]) return fail(RAVEN_ESTATE, "quantiser not built");
  std::memcpy(out5dim, ix->h_qparams[quant].data(), ix->h_qparams[quant].size() * 4);
  return RAVEN_OK;
}

int raven_index_codes(const raven_index* ix, int32_t quant, uint8_t* out, uint64_t cap_bytes) {
  if (!ix || !out || (quant != 0 && quant != 1)) return fail(RAVEN_EINVAL, "bad argument");
  if (!ix->has_q[quant]) return fail(RAVEN_ESTATE, "quantiser not built");
  const uint32_t bytes = quant == 0 ? (ix->dim + 1) / 2 : ix->dim;
  if (cap_bytes < ix->n * bytes) return fail(RAVEN_EINVAL, "output buffer too small");
  CU(cudaSetDevice(ix->device));
  CU(cudaMemcpy2D(out, bytes, ix->d_codes[quant], ix->q_stride[quant], bytes, ix->n, cudaMemcpyDeviceToHost));
  return RAVEN_OK;
}

int raven_search_batch_device(raven_index* ix, const float* d_q, uint64_t nq, const raven_search_params* p,
                              const raven_search_outputs* d_out, void* stream) {
  NvtxRange nvtx_range("raven.search_batch_device");
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  if (nq && !d_q) return fail(RAVEN_EINVAL, "null queries");
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the CUDA default stream
  return run_search(ix, d_q, nq, p, d_out, st, 0);
}

int raven_search_batch(raven_index* ix, const float* q, uint64_t nq, const raven_search_params* p,
                       const raven_search_outputs* out, void* stream) {
  NvtxRange nvtx_range("raven.search_batch");
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  if (!out || !out->ids) return fail(RAVEN_EINVAL, "outputs.ids is required");
  if (!p) return fail(RAVEN_EINVAL, "null search params");
  if (nq == 0) return RAVEN_OK;
  if (!q) return fail(RAVEN_EINVAL, "null queries");
  CU(cudaSetDevice(ix->device));
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the CUDA default stream
  const uint64_t k = p->k;
  const uint64_t hc = out->history ? out->history_cap : 0;
  // one device block for queries + every requested output
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~(size_t)255;
    return o;
  };
  const size_t o_q = take(nq * ix->dim * 4), o_ids = take(nq * k * 4);
  const size_t o_d = out->dists ? take(nq * k * 4) : 0;
  const size_t o_c = out->counts ? take(nq * 4) : 0, o_v = out->visited ? take(nq * 4) : 0;
  const size_t o_e = out->ef_used ? take(nq * 4) : 0, o_s = out->status ? take(nq * 4) : 0;
  const size_t o_n = out->n_nav ? take(nq * 4) : 0, o_x = out->expansions ? take(nq * 4) : 0;
  const size_t o_h = hc ? take(nq * hc * 4) : 0, o_hl = hc ? take(nq * 4) : 0;
  uint8_t* buf = nullptr;
  CU(cudaMallocAsync((void**)&buf, off, st));
  raven_search_outputs d{};
  d.ids = (uint32_t*)(buf + o_ids);
  d.dists = out->dists ? (float*)(buf + o_d) : nullptr;
  d.counts = out->counts ? (uint32_t*)(buf + o_c) : nullptr;
  d.visited = out->visited ? (uint32_t*)(buf + o_v) : nullptr;
  d.ef_used = out->ef_used ? (uint32_t*)(buf + o_e) : nullptr;
  d.status = out->status ? (int32_t*)(buf + o_s) : nullptr;
  d.n_nav = out->n_nav ? (uint32_t*)(buf + o_n) : nullptr;
  d.expansions = out->expansions ? (uint32_t*)(buf + o_x) : nullptr;
  d.history = hc ? (uint32_t*)(buf + o_h) : nullptr;
  d.history_cap = (uint32_t)hc;
  d.history_len = hc ? (uint32_t*)(buf + o_hl) : nullptr;
  int rc = RAVEN_OK;
  cudaError_t e = cudaMemcpyAsync(buf + o_q, q, nq * ix->dim * 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess && hc) e = cudaMemsetAsync(d.history, 0, nq * hc * 4, st);  // entries past history_len read 0
  if (e == cudaSuccess) rc = run_search(ix, (const float*)(buf + o_q), nq, p, &d, st, 0);
  auto back = [&](void* dst, const void* src, size_t bytes) {
    if (dst && e == cudaSuccess) e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, st);
  };
  if (rc == RAVEN_OK && e == cudaSuccess) {
    back(out->ids, d.ids, nq * k * 4);
    back(out->dists, d.dists, nq * k * 4);
    back(out->counts, d.counts, nq * 4);
    back(out->visited, d.visited, nq * 4);
    back(out->ef_used, d.ef_used, nq * 4);
    back(out->status, d.status, nq * 4);
    back(out->n_nav, d.n_nav, nq * 4);
    back(out->expansions, d.expansions, nq * 4);
    if (hc) {
      back(out->history, d.history, nq * hc * 4);
      back(out->history_len, d.history_len, nq * 4);
    }
  }
  cudaFreeAsync(buf, st);
  cudaError_t es = cudaStreamSynchronize(st);
  if (rc) return rc;
  if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("search copies: ") + cudaGetErrorString(e));
  if (es != cudaSuccess) return fail(RAVEN_ECUDA, std::string("search: ") + cudaGetErrorString(es));
  return RAVEN_OK;
}

}  // extern "C"

namespace {

// cuTensorMapEncodeTiled, looked up once through the runtime (no link-time
// dependency on the driver library).
PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    else
      (void)cudaGetLastError();
  });
  return fn;
}

// f32 matrix of `rows` rows, `cols` used columns, row stride `ld` floats
// (ld * 4 a multiple of 16 bytes); box 32 columns x 128 rows, 128-byte
// swizzle (the K-major SW128 operand layout), out-of-range elements read 0.
bool make_tile_map(CUtensorMap* m, const float* base, uint64_t cols, uint64_t rows, uint64_t ld) {
  PFN_cuTensorMapEncodeTiled_v12000 f = encode_tiled();
  if (!f) return false;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld * 4};
  cuuint32_t box[2] = {(cuuint32_t)raven_tc::kBK, (cuuint32_t)raven_tc::kBM};
  cuuint32_t estr[2] = {1, 1};
  return f(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <int PASSES, int KT>
cudaError_t launch_knn_tc(const CUtensorMap& qh, const CUtensorMap& ql, const CUtensorMap& xh, const CUtensorMap& xl,
                          const raven_tc::Params& p, unsigned grid, cudaStream_t st) {
  auto kern = raven_tc::knn_tc_kernel<PASSES, KT>;
  const int smem = (int)raven_tc::Layout<PASSES>::kBytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, raven_tc::kThreads, smem, st>>>(qh, ql, xh, xl, p);
  return cudaGetLastError();
}

// Splits of the base range: as many CTAs as keep the last wave full, at
// least 8 base tiles per CTA.
uint64_t tc_splits(uint64_t n, uint64_t qtiles, int sms) {
  const uint64_t tiles = (n + raven_tc::kBN - 1) / raven_tc::kBN;
  uint64_t best = 1;
  double best_eff = -1.0;
  for (uint64_t s = 1; s <= 64 && s * 8 <= std::max<uint64_t>(tiles, 8); ++s) {
    const uint64_t items = qtiles * s;
    const uint64_t waves = (items + sms - 1) / sms;
    const double eff = (double)items / (double)(waves * sms) - 0.002 * (double)s;  // prefer fewer merges
    if (eff > best_eff) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

}  // namespace

extern "C" {

int raven_knn_exact_device(raven_index* ix, const float* d_q, uint64_t nq, uint32_t k, uint32_t* d_ids,
                           float* d_dists, void* stream) {
  NvtxRange nvtx_range("raven.knn_exact");
  if (!ix || (!d_q && nq) || !d_ids || !d_dists) return fail(RAVEN_EINVAL, "null argument");
  if (k == 0 || k > KMAXK) return fail(RAVEN_ELIMIT, "k must be in 1..32");
  if (nq == 0) return RAVEN_OK;
  CU(cudaSetDevice(ix->device));
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the CUDA default stream
  const uint32_t dim = ix->dim;
  const bool tc = dim % 4 == 0 && dim <= (uint32_t)(raven_tc::kBK * raven_tc::kMaxKB) && encode_tiled() != nullptr;
  if (tc) {
    // tensor-core path (knn_tc.cuh): prepare operands, pick one or three passes
    const uint32_t kb = (dim + raven_tc::kBK - 1) / raven_tc::kBK, kpad = kb * raven_tc::kBK;
    const uint64_t qtiles = (nq + raven_tc::kBM - 1) / raven_tc::kBM, nq_pad = qtiles * raven_tc::kBM;
    const uint64_t splits = tc_splits(ix->n, qtiles, ix->num_sms);
    uint64_t split_rows = (ix->n + splits - 1) / splits;
    split_rows = (split_rows + raven_tc::kBN - 1) / raven_tc::kBN * raven_tc::kBN;
    const uint64_t nsplit = (ix->n + split_rows - 1) / split_rows;
    const size_t qbytes = nq_pad * kpad * 4, per = 2 * nsplit * nq * k;  // two column halves per split
    const uint64_t n_pad = (ix->n + raven_tc::kBN - 1) / raven_tc::kBN * raven_tc::kBN;
    const size_t bytes = 2 * qbytes + nq_pad * 4 + n_pad * 4 + 16 + per * 8;
    uint8_t* tmp = nullptr;
    CU(cudaMallocAsync((void**)&tmp, bytes, st));
    float* qh = (float*)tmp;
    float* ql = (float*)(tmp + qbytes);
    float* qn = (float*)(tmp + 2 * qbytes);
    float* xn = qn + nq_pad;
    unsigned* flags = (unsigned*)(xn + n_pad);
    uint32_t* ti = (uint32_t*)(flags + 4);
    float* td = (float*)(ti + per);
    float* xsplit = nullptr;
    int* d_err = (int*)(flags + 3);
    unsigned h_flags[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemsetAsync(flags, 0, 16, st);
    if (e == cudaSuccess) {
      tc_base_norms_kernel<<<(unsigned)((n_pad * 32 + 255) / 256), 256, 0, st>>>(ix->d_vec, ix->n, n_pad, dim, xn,
                                                                                 flags);
      tc_query_prep_kernel<<<(unsigned)((nq_pad * 32 + 255) / 256), 256, 0, st>>>(d_q, nq, nq_pad, dim, dim / 16, kpad,
                                                                                    qh, ql, qn, flags);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_flags, flags, 16, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    int passes = 3;
    if (e == cudaSuccess) {
      float mx, mq;
      std::memcpy(&mx, &h_flags[1], 4);
      std::memcpy(&mq, &h_flags[2], 4);
      // exact in one pass: TF32-exact integers, norms and their sum below 2^24
      if (!(h_flags[0] & 1u) && (double)mx + (double)mq < 16777216.0) passes = 1;
    }
    if (e == cudaSuccess && passes == 3) {
      e = cudaMallocAsync((void**)&xsplit, ix->n * dim * 8, st);
      if (e == cudaSuccess) {
        tc_base_split_kernel<<<(unsigned)std::min<uint64_t>((ix->n * dim + 255) / 256, 65535u * 4), 256, 0, st>>>(
            ix->d_vec, ix->n * dim, xsplit, xsplit + ix->n * dim);
        e = cudaGetLastError();
      }
    }
    if (e == cudaSuccess) {
      CUtensorMap m_qh, m_ql, m_xh, m_xl;
      const float* xh = passes == 1 ? ix->d_vec : xsplit;
      const float* xl = passes == 1 ? ix->d_vec : xsplit + ix->n * dim;
      bool ok = make_tile_map(&m_qh, qh, kpad, nq_pad, kpad) && make_tile_map(&m_ql, ql, kpad, nq_pad, kpad) &&
                make_tile_map(&m_xh, xh, dim, ix->n, dim) && make_tile_map(&m_xl, xl, dim, ix->n, dim);
      if (!ok) {
        e = cudaErrorInvalidValue;
      } else {
        raven_tc::Params prm{};
        prm.n = ix->n;
        prm.nq = nq;
        prm.kb = kb;
        prm.k = k;
        prm.split_rows = split_rows;
        prm.qtiles = (uint32_t)qtiles;
        prm.xn = xn;
        prm.qn = qn;
        prm.out_i = ti;
        prm.out_d = td;
        prm.err = d_err;
        const unsigned grid = (unsigned)(qtiles * nsplit);
        if (passes == 1)
          e = k <= 16 ? launch_knn_tc<1, 16>(m_qh, m_ql, m_xh, m_xl, prm, grid, st)
                      : launch_knn_tc<1, 32>(m_qh, m_ql, m_xh, m_xl, prm, grid, st);
        else
          e = k <= 16 ? launch_knn_tc<3, 16>(m_qh, m_ql, m_xh, m_xl, prm, grid, st)
                      : launch_knn_tc<3, 32>(m_qh, m_ql, m_xh, m_xl, prm, grid, st);
      }
    }
    if (e == cudaSuccess) {
      knn_merge_kernel<<<(unsigned)((nq * 32 + 255) / 256), 256, 0, st>>>(ti, td, (uint32_t)(2 * nsplit), nq, k, d_ids,
                                                                          d_dists);
      e = cudaGetLastError();
    }
    int h_err = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&h_err, d_err, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (xsplit) cudaFreeAsync(xsplit, st);
    cudaFreeAsync(tmp, st);
    if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("knn (tensor cores): ") + cudaGetErrorString(e));
    if (h_err) return fail(RAVEN_ECUDA, "knn (tensor cores): a pipeline wait ran out");
    return RAVEN_OK;
  }
  // CUDA-core path (dims the tensor-core path does not take)
  const uint64_t qblocks = (nq + KQ - 1) / KQ;
  uint64_t splits = std::max<uint64_t>(1, (uint64_t)ix->num_sms * 4 / std::max<uint64_t>(qblocks, 1));
  splits = std::min<uint64_t>(splits, (ix->n + KB - 1) / KB);
  splits = std::min<uint64_t>(splits, 64);
  uint64_t split_rows = (ix->n + splits - 1) / splits;
  split_rows = (split_rows + KB - 1) / KB * KB;
  splits = (ix->n + split_rows - 1) / split_rows;
  uint8_t* tmp = nullptr;
  const size_t per = splits * nq * k;
  CU(cudaMallocAsync((void**)&tmp, per * 8, st));
  uint32_t* ti = (uint32_t*)tmp;
  float* td = (float*)(tmp + per * 4);
  dim3 grid((unsigned)qblocks, (unsigned)splits);
  knn_tile_kernel<<<grid, 256, 0, st>>>(ix->d_vec, ix->n, d_q, nq, ix->dim, k, split_rows, ti, td);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    knn_merge_kernel<<<(unsigned)((nq * 32 + 255) / 256), 256, 0, st>>>(ti, td, (uint32_t)splits, nq, k, d_ids, d_dists);
    e = cudaGetLastError();
  }
  cudaFreeAsync(tmp, st);
  if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("knn: ") + cudaGetErrorString(e));
  return RAVEN_OK;
}

int raven_merge_topk_device(const uint32_t* d_ids, const float* d_dists, const uint32_t* d_counts, uint32_t n_shards,
                            uint64_t nq, uint32_t k, uint64_t shard_size, uint32_t* d_out_ids, float* d_out_dists,
                            uint32_t* d_out_counts, void* stream) {
  NvtxRange nvtx_range("raven.merge_topk");
  if (!d_ids || !d_dists || !d_out_ids || !d_out_dists) return fail(RAVEN_EINVAL, "null argument");
  if (n_shards == 0 || k == 0) return fail(RAVEN_EINVAL, "n_shards and k must be >= 1");
  if (nq == 0) return RAVEN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const MergeLayout lay{1u, n_shards, nq * k, nq * k, nq};
  const unsigned blocks = (unsigned)((nq * 32 + kMergeThreads - 1) / kMergeThreads);
  shard_merge_kernel<<<blocks, kMergeThreads, 0, st>>>(d_ids, d_dists, d_counts, lay, n_shards, nq, k, shard_size,
                                                       d_out_ids, d_out_dists, d_out_counts);
  CU(cudaGetLastError());
  return RAVEN_OK;
}

int raven_merge_topk_gathered_device(const void* d_gathered, uint32_t n_shards, uint32_t world, uint32_t per_rank,
                                     uint64_t nq, uint32_t k, uint64_t shard_size, uint32_t* d_out_ids,
                                     float* d_out_dists, uint32_t* d_out_counts, void* stream) {
  NvtxRange nvtx_range("raven.merge_topk_gathered");
  if (!d_gathered || !d_out_ids || !d_out_dists) return fail(RAVEN_EINVAL, "null argument");
  if (n_shards == 0 || k == 0 || world == 0) return fail(RAVEN_EINVAL, "n_shards, world and k must be >= 1");
  if ((uint64_t)per_rank * world < n_shards || (uint64_t)(per_rank - 1) * world >= n_shards)
    return fail(RAVEN_EINVAL, "per_rank must be ceil(n_shards / world)");
  if (nq == 0) return RAVEN_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const uint64_t block = nq * (2ull * k + 1);  // words per shard block: ids, distances, counts
  const uint32_t* base = (const uint32_t*)d_gathered;
  const MergeLayout lay{world, per_rank, block, block, block};
  const unsigned blocks = (unsigned)((nq * 32 + kMergeThreads - 1) / kMergeThreads);
  shard_merge_kernel<<<blocks, kMergeThreads, 0, st>>>(
      base, (const float*)(base + nq * k), base + 2 * nq * k, lay, n_shards, nq, k, shard_size, d_out_ids, d_out_dists,
      d_out_counts);
  CU(cudaGetLastError());
  return RAVEN_OK;
}

int raven_index_set_small_batch(raven_index* ix, uint64_t max_nq) {
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  ix->small_batch_max = max_nq;
  return RAVEN_OK;
}

// Tuning hooks (benchmark sweeps): 0 keeps the default.
int raven_index_set_tuning(raven_index* ix, int32_t hash_bits, int32_t spill_bits) {
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  if (hash_bits && (hash_bits < 8 || hash_bits > 14)) return fail(RAVEN_EINVAL, "hash_bits must be in 8..14");
  if (spill_bits && (spill_bits < 10 || spill_bits > 20)) return fail(RAVEN_EINVAL, "spill_bits must be in 10..20");
  ix->hash_bits_override = hash_bits;
  ix->spill_bits_override = spill_bits;
  return RAVEN_OK;
}

// Neighbour codes beside each row (no reference counterpart): built by
// default at upload; disabling frees them (the search gathers codes instead).
int raven_index_set_fat_rows(raven_index* ix, int32_t enable) {
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  CU(cudaSetDevice(ix->device));
  for (int q = 0; q < 2; ++q) {
    const int rc = set_fat_rows(ix, q, enable != 0);
    if (rc) return rc;
  }
  return RAVEN_OK;
}

}  // extern "C"

// ===========================================================================
// Search without allocation: scratch from a fixed device array.
//
// Some callers cannot allocate device memory at search time: a serving loop
// whose GPU memory is entirely reserved up front by another allocator (a
// framework's caching pool), a process that has to keep a hard memory budget
// and fail at start-up rather than mid-request, or code that must not make the
// allocator calls that can synchronise the device. For them this entry point
// takes the per-call scratch (work counter, AdaptiveEf table, visited-set spill
// tables) from g_noalloc_scratch, a file-scope device array of
// kNoAllocScratchBytes that every GPU which loads this library holds until the
// process exits. The caller still provides queries and outputs.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;  // 64 MiB per GPU
constexpr size_t kNoAllocHeader = 16384;               // counter (256 B) + ef table (<= 4032 u32)
constexpr uint32_t kNoAllocMaxSpillBits = 11;          // spill level A 8 KB, level B 64 KB per warp

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];


std::mutex g_noalloc_mu;
struct NoAllocSlot {
  void* ctx = nullptr;    // context the address was taken in
  uint8_t* ptr = nullptr;  // device address of g_noalloc_scratch in that context
};
NoAllocSlot g_noalloc_slot[256];  // per device ordinal

// In host code g_noalloc_scratch names a host-side stand-in, not device memory:
// the device address comes from cudaGetSymbolAddress, taken once per device
// with that device current, and taken again if the device's context has been
// replaced since (cudaDeviceReset destroys the array with its context).
int noalloc_scratch(int device, uint8_t** out) {
  if (device < 0 || device >= 256) return fail(RAVEN_EINVAL, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocSlot& sl = g_noalloc_slot[device];
  void* ctx = current_context();
  if (!sl.ptr || ctx != sl.ctx) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return fail(RAVEN_ECUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    sl.ptr = (uint8_t*)ptr;
    sl.ctx = current_context();  // the lookup may have created the primary context
  }
  *out = sl.ptr;
  return RAVEN_OK;
}

}  // namespace

extern "C" {

int raven_search_batch_device_noalloc(raven_index* ix, const float* d_q, uint64_t nq, const raven_search_params* p,
                                      const raven_search_outputs* o, void* stream) {
  NvtxRange nvtx_range("raven.search_batch_device_noalloc");
  if (!ix) return fail(RAVEN_EINVAL, "null index");
  if (nq && !d_q) return fail(RAVEN_EINVAL, "null queries");
  Plan pl;
  int rc = make_plan(ix, p, &pl);
  if (rc) return rc;
  if (nq == 0) return RAVEN_OK;
  if (!o || !o->ids) return fail(RAVEN_EINVAL, "outputs.ids is required");
  if (pl.table.size() * 4 + 256 > kNoAllocHeader)
    return fail(RAVEN_ELIMIT, "AdaptiveEf table larger than the fixed scratch header (max 4032 samples)");
  CU(cudaSetDevice(ix->device));
  uint8_t* scratch = nullptr;
  if ((rc = noalloc_scratch(ix->device, &scratch))) return rc;
  cudaStream_t st = (cudaStream_t)stream;  // NULL: the CUDA default stream
  // spill tables sized to fit the fixed array: smaller level A, and as many
  // resident warps as the remaining bytes allow
  const uint32_t sb = std::min<uint32_t>((uint32_t)pl.spill_bits, kNoAllocMaxSpillBits);
  const size_t per_slot = (9ull << sb) * 4;
  const uint64_t max_slots = (kNoAllocScratchBytes - kNoAllocHeader) / per_slot;
  int blocks_per_sm = 0;
  SearchArgs occ_args{};
  occ_args.pool_cap = pl.pool_cap;  // selects the kernel variant whose occupancy is asked
  occ_args.xnorm = mma_norms(ix, pl);
  // without visited counts or the visited order the search keeps no visited
  // tables, and the array holds only the counter and the ef table
  const bool vis = needs_visited(pl.quant, o);
  CU(dispatch(pl.quant, pl.cpl, vis, true, occ_args, pl.smem_block, 0, st, &blocks_per_sm));
  if (blocks_per_sm <= 0) return fail(RAVEN_ELIMIT, "search kernel does not fit on an SM with this configuration");
  const uint64_t need = (nq + kWarpsPerBlock - 1) / kWarpsPerBlock;
  const uint64_t grid64 = std::min<uint64_t>(
      {(uint64_t)blocks_per_sm * ix->num_sms, need, vis ? max_slots / kWarpsPerBlock : ~0ull});
  if (grid64 == 0) return fail(RAVEN_ELIMIT, "fixed scratch array too small for one block of spill tables");
  const int grid = (int)grid64;
  const uint64_t slots = (uint64_t)grid * kWarpsPerBlock;
  unsigned long long* counter = (unsigned long long*)scratch;
  uint32_t* table = (uint32_t*)(scratch + 256);
  uint32_t* spill = (uint32_t*)(scratch + kNoAllocHeader);
  // the array keeps the previous call's contents: the work counter must start
  // at zero; spill tables are cleared by each query on first use
  CU(cudaMemsetAsync(counter, 0, 8, st));
  if (!pl.table.empty())
    CU(cudaMemcpyAsync(table, pl.table.data(), pl.table.size() * 4, cudaMemcpyHostToDevice, st));
  SearchArgs a{};
  fill_args(ix, pl, p, o, &a);
  a.ef_table = table;
  a.spill_bits = sb;
  a.spill = vis ? spill : nullptr;
  a.n_slots = slots;
  a.queries = d_q;
  a.nq = nq;
  a.counter = counter;
  a.nav_only = 0;
  const cudaError_t e = dispatch(pl.quant, pl.cpl, vis, false, a, pl.smem_block, grid, st, nullptr);
  if (e != cudaSuccess) return fail(RAVEN_ECUDA, std::string("search launch: ") + cudaGetErrorString(e));
  return RAVEN_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Vamana build on the GPU (no reference counterpart on a GPU: it replaces the
// per-batch candidate step of VamanaGraph::build, src/graph/vamana.rs:106-201).
// Per batch: the search kernel in its f32 mode (greedy_search_vec_build,
// vamana.rs:530-567: entry = medoid, L = l_build, visited history recorded)
// gives each node's candidate set, build_prune_kernel applies DirectionalPrune
// to it; the host build keeps the batch order, the connect step and the final
// prune, and sends back every changed row.
// ---------------------------------------------------------------------------
namespace {

constexpr int kPruneThreads = 256;
constexpr uint32_t kBuildHistCap = 16384;  // visited ids kept per node (the rest are dropped, and counted)

// DirectionalPrune (src/graph/robust_prune.rs:280-385) of one node's visited
// set, one CTA per node. d(q, c) and l2(a, c) are f32 squared L2 in the
// AVX-512 summation order (hw_dist). Candidates (node itself excluded) are
// sorted by (distance, id) with a bitonic sort in shared memory; then in that
// order a candidate is kept when no kept neighbour a has l2(a, c) < d(q, c),
// until r_max are kept; if fewer than r_min are kept, a second pass adds, in
// order, candidates not yet kept with l2(a, c) != 0 and d(q, c) / l2(a, c) <=
// backfill_alpha for every kept a.
__global__ void __launch_bounds__(kPruneThreads) build_prune_kernel(
    const float* __restrict__ vec, uint32_t dim, uint32_t C, uint32_t rem, const uint32_t* __restrict__ nodes,
    const uint32_t* __restrict__ hist, const uint32_t* __restrict__ hist_len, uint32_t hcap, uint32_t sortn,
    uint32_t r_max, uint32_t r_min, float backfill_alpha, uint32_t* __restrict__ out, uint32_t* __restrict__ out_len) {
  extern __shared__ __align__(16) uint8_t sm[];
  const uint32_t stride = (dim + 3u) & ~3u;                    // 16-byte aligned rows
  unsigned long long* keys = (unsigned long long*)sm;          // sortn
  const uint32_t bit_words = ((sortn / 32) + 3u) & ~3u;       // 16-byte multiple: later rows stay aligned
  uint32_t* kept_bits = (uint32_t*)(keys + sortn);             // bit i: sorted candidate i kept
  uint32_t* kept_id = kept_bits + bit_words;                   // r_max (+ pad)
  float* rows = (float*)(kept_id + ((r_max + 3u) & ~3u));      // r_max kept rows, then 16 candidate rows
  float* crow = rows + (size_t)r_max * stride;
  __shared__ uint32_t nk, ncand;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, h = lane >> 4, j = lane & 15;
  const uint32_t b = blockIdx.x;
  const uint32_t node = nodes[b];
  const float* qrow = vec + (size_t)node * dim;
  const uint32_t len = min(hist_len[b], hcap);
  const uint32_t* hb = hist + (size_t)b * hcap;
  if (tid == 0) {
    nk = 0;
    ncand = 0;
  }
  for (uint32_t i = tid; i < bit_words; i += kPruneThreads) kept_bits[i] = 0;
  __syncthreads();
  // 1. keys = (distance bits, id); the node itself and padding sort last
  //    (distances are >= 0, so their bit patterns order like the values)
  for (uint32_t i0 = 2u * warp; i0 < sortn; i0 += 2u * (kPruneThreads / 32)) {
    const uint32_t i = i0 + h;
    const bool in = i < len;
    const uint32_t id = in ? hb[i] : node;
    float d = 0.0f;
    if (i0 < len) d = hw_dist(qrow, vec + (size_t)id * dim, C, rem, j);  // both half-warps take this branch
    if (j == 0) {
      const bool ok = in && id != node;
      keys[i] = ok ? ((unsigned long long)__float_as_uint(d) << 32) | id : ~0ull;
      if (ok) atomicAdd(&ncand, 1u);
    }
  }
  __syncthreads();
  // 2. bitonic sort, ascending
  for (uint32_t k2 = 2; k2 <= sortn; k2 <<= 1)
    for (uint32_t jj = k2 >> 1; jj > 0; jj >>= 1) {
      for (uint32_t i = tid; i < sortn; i += kPruneThreads) {
        const uint32_t ixj = i ^ jj;
        if (ixj > i) {
          const unsigned long long x = keys[i], y = keys[ixj];
          if ((x > y) == ((i & k2) == 0)) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  // 3. greedy selection, then the backfill pass, 16 candidates at a time:
  //    each half-warp tests one candidate against every row kept before the
  //    chunk, then warp 0 walks the chunk in order and tests the survivors
  //    against the candidates it accepted earlier in the same chunk, which
  //    gives the decisions of the one-at-a-time loop.
  const uint32_t nc = ncand;
  constexpr int kChunk = 2 * (kPruneThreads / 32);
  __shared__ uint32_t cidx[kChunk];
  __shared__ int cviol[kChunk];
  __shared__ uint32_t cn, next_i;
  if (tid == 0) next_i = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const uint32_t target = pass == 0 ? r_max : r_min;
    if (tid == 0) next_i = 0;
    __syncthreads();
    while (true) {
      if (tid == 0) {
        uint32_t c = 0, i = next_i;
        for (; i < nc && c < (uint32_t)kChunk; ++i)
          if (pass == 0 || !((kept_bits[i >> 5] >> (i & 31)) & 1u)) cidx[c++] = i;
        cn = c;
        next_i = i;
      }
      __syncthreads();
      const uint32_t m = nk, n_chunk = cn;
      if (n_chunk == 0 || m >= target) break;
      // stage the chunk's rows after the kept rows
      for (uint32_t e = tid; e < n_chunk * dim; e += kPruneThreads) {
        const uint32_t t = e / dim, d = e - t * dim;
        crow[t * stride + d] = vec[(size_t)(uint32_t)keys[cidx[t]] * dim + d];
      }
      __syncthreads();
      {
        const uint32_t t = 2u * warp + h;  // this half-warp's candidate
        const uint32_t tt = min(t, n_chunk - 1);
        const float dq = __uint_as_float((uint32_t)(keys[cidx[tt]] >> 32));
        bool bad = false;
        for (uint32_t a = 0; a < m; ++a) {
          if (__all_sync(kFull, bad)) break;  // both half-warps decided (the distance needs the whole warp)
          const float d = hw_dist(rows + (size_t)a * stride, crow + (size_t)tt * stride, C, rem, j);
          bad |= pass == 0 ? d < dq : (d == 0.0f || __fdiv_rn(dq, d) > backfill_alpha);
        }
        if (j == 0 && t < n_chunk) cviol[t] = bad ? 1 : 0;
      }
      __syncthreads();
      if (warp == 0) {
        uint32_t first_new = m, cnt = m;
        for (uint32_t t = 0; t < n_chunk && cnt < target; ++t) {
          if (cviol[t]) continue;
          const float dq = __uint_as_float((uint32_t)(keys[cidx[t]] >> 32));
          bool bad = false;
          for (uint32_t s2 = first_new; s2 < cnt && !bad; ++s2) {
            const float d = hw_dist(rows + (size_t)s2 * stride, crow + (size_t)t * stride, C, rem, j);
            bad = pass == 0 ? d < dq : (d == 0.0f || __fdiv_rn(dq, d) > backfill_alpha);
          }
          if (bad) continue;
          for (uint32_t e = lane; e < dim; e += 32) rows[(size_t)cnt * stride + e] = crow[(size_t)t * stride + e];
          if (lane == 0) {
            kept_id[cnt] = (uint32_t)keys[cidx[t]];
            kept_bits[cidx[t] >> 5] |= 1u << (cidx[t] & 31);
          }
          __syncwarp();
          ++cnt;
        }
        if (lane == 0) nk = cnt;
      }
      __syncthreads();
    }
  }
  for (uint32_t t = tid; t < nk; t += kPruneThreads) out[(size_t)b * r_max + t] = kept_id[t];
  if (tid == 0) out_len[b] = nk;
}

__global__ void build_scatter_rows_kernel(const uint32_t* __restrict__ ids, const uint32_t* __restrict__ rows,
                                          uint64_t count, uint32_t r, uint32_t r_pad, uint32_t* __restrict__ adj) {
  const uint64_t total = count * r_pad;
  for (uint64_t t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; t < total; t += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t i = t / r_pad;
    const uint32_t c = (uint32_t)(t - i * r_pad);
    adj[(uint64_t)ids[i] * r_pad + c] = c < r ? rows[i * r + c] : raven::kSentinel;
  }
}

struct GpuBuild : raven::BuildAccelerator {
  const float* h_vec;
  uint64_t n;
  uint32_t dim;
  raven::BuildConfig cfg;
  int device;
  raven_index* ix = nullptr;
  float* d_nat = nullptr;
  uint8_t* d_buf = nullptr;
  uint32_t *d_nodes = nullptr, *d_hist = nullptr, *d_hlen = nullptr, *d_ids = nullptr, *d_pruned = nullptr,
           *d_plen = nullptr, *d_rows = nullptr;
  float *d_q = nullptr, *d_dists = nullptr;
  int32_t* d_status = nullptr;
  size_t cap_nodes = 0, cap_rows = 0;
  uint64_t truncated = 0;  // nodes whose visited set exceeded kBuildHistCap
  double t_search = 0, t_prune = 0, t_rows = 0;  // seconds, reported in verbose builds
  static double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
  }

  GpuBuild(const float* v, uint64_t n_, uint32_t d, const raven::BuildConfig& c, int dev)
      : h_vec(v), n(n_), dim(d), cfg(c), device(dev) {}
  ~GpuBuild() override {
    if (d_nat) cudaFree(d_nat);
    if (d_buf) cudaFree(d_buf);
    if (d_rows) cudaFree(d_rows);
    if (ix) raven_index_free(ix);
  }
  static int cuda_err(cudaError_t e, std::string* err, const char* what) {
    if (e == cudaSuccess) return 0;
    if (err) *err = std::string(what) + ": " + cudaGetErrorString(e);
    return RAVEN_ECUDA;
  }
  int begin(const uint32_t* main_block, uint64_t n_, uint64_t r, uint32_t entry, std::string* err) override {
    raven_graph gr;
    gr.g.n = n_;
    gr.g.dim = dim;
    gr.g.r_max = r;
    gr.g.entry = entry;
    gr.g.main_block.assign(main_block, main_block + n_ * r);
    gr.g.degrees.resize(n_);
    gr.g.overflow.resize(n_);
    for (uint64_t v = 0; v < n_; ++v) {
      uint16_t d = 0;
      while (d < r && main_block[v * r + d] != raven::kSentinel) ++d;
      gr.g.degrees[v] = d;
    }
    raven_upload_options o{device, 0, 0, 0, 0};  // the f32 traversal needs no codes
    int rc = raven_index_upload(&gr, h_vec, n_, dim, &o, &ix);
    if (rc) {
      if (err) *err = raven_last_error();
      return rc;
    }
    if (int e = cuda_err(cudaMalloc((void**)&d_nat, n_ * dim * 4), err, "build: vectors")) return e;
    return cuda_err(cudaMemcpy(d_nat, h_vec, n_ * dim * 4, cudaMemcpyHostToDevice), err, "build: vectors");
  }
  int ensure(size_t count, std::string* err) {
    if (count <= cap_nodes) return 0;
    if (d_buf) cudaFree(d_buf);
    d_buf = nullptr;
    const size_t per = 4 * (1 + kBuildHistCap + 1 + 1 + cfg.r_max + 1 + 1) + 4 * (size_t)dim + 4;
    if (int e = cuda_err(cudaMalloc((void**)&d_buf, count * per + 256), err, "build: batch buffers")) return e;
    uint8_t* p = d_buf;
    auto take = [&](size_t bytes) { uint8_t* q = p; p += (bytes + 15) & ~(size_t)15; return q; };
    d_nodes = (uint32_t*)take(count * 4);
    d_hist = (uint32_t*)take(count * kBuildHistCap * 4);
    d_hlen = (uint32_t*)take(count * 4);
    d_ids = (uint32_t*)take(count * 4);
    d_pruned = (uint32_t*)take(count * cfg.r_max * 4);
    d_plen = (uint32_t*)take(count * 4);
    d_status = (int32_t*)take(count * 4);
    d_q = (float*)take(count * dim * 4);
    d_dists = (float*)take(count * 4);
    cap_nodes = count;
    return 0;
  }
  int search_prune(const uint32_t* nodes, size_t count, float alpha, std::vector<std::vector<uint32_t>>* pruned,
                   std::string* err) override {
    NvtxRange nvtx_range("raven.build.search_prune");
    if (int e = ensure(count, err)) return e;
    const double t0 = now();
    cudaStream_t st = ix->stream;
    if (int e = cuda_err(cudaMemcpyAsync(d_nodes, nodes, count * 4, cudaMemcpyHostToDevice, st), err, "build: ids"))
      return e;
    gather_rows_kernel<<<ix->num_sms * 4, 256, 0, st>>>(d_nat, d_nodes, count, dim, d_q);
    raven_search_params p{};
    p.ef = cfg.l_build;
    p.k = 1;
    p.rerank_factor = 1;
    p.quant = RAVEN_QUANT_F32;  // greedy_search_vec_build: the f32 beam
    raven_search_outputs o{};
    o.ids = d_ids;
    o.dists = d_dists;
    o.status = d_status;
    o.history = d_hist;
    o.history_cap = kBuildHistCap;
    o.history_len = d_hlen;
    int rc = raven_search_batch_device(ix, d_q, count, &p, &o, st);
    if (rc) {
      if (err) *err = raven_last_error();
      return rc;
    }
    std::vector<uint32_t> hlen(count);
    if (int e = cuda_err(cudaMemcpyAsync(hlen.data(), d_hlen, count * 4, cudaMemcpyDeviceToHost, st), err,
                         "build: history lengths"))
      return e;
    if (int e = cuda_err(cudaStreamSynchronize(st), err, "build: search")) return e;
    const double t1 = now();
    t_search += t1 - t0;
    uint32_t mx = 32;
    for (uint32_t v : hlen) {
      mx = std::max(mx, std::min(v, kBuildHistCap));
      if (v > kBuildHistCap) ++truncated;
    }
    uint32_t sortn = 32;
    while (sortn < mx) sortn <<= 1;
    const uint32_t stride = (dim + 3u) & ~3u;
    const size_t bit_words = ((sortn / 32) + 3u) & ~3u;
    const size_t smem = (size_t)sortn * 8 + bit_words * 4 + ((cfg.r_max + 3u) & ~3u) * 4 +
                        (size_t)(cfg.r_max + 2 * (kPruneThreads / 32)) * stride * 4;
    if (smem > 227 * 1024) {
      if (err) *err = "build: prune workspace above the shared-memory limit";
      return RAVEN_ELIMIT;
    }
    const uint32_t div = cfg.rmin_divisor ? cfg.rmin_divisor : 4;
    const uint32_t r_min = std::max<uint32_t>(cfg.r_max / div, 1);
    const float bf_alpha = std::max(alpha, 1.0f);
    cudaFuncSetAttribute(build_prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    build_prune_kernel<<<(unsigned)count, kPruneThreads, smem, st>>>(ix->d_vec, dim, dim / 16, dim % 16, d_nodes,
                                                                      d_hist, d_hlen, kBuildHistCap, sortn, cfg.r_max,
                                                                      r_min, bf_alpha, d_pruned, d_plen);
    if (int e = cuda_err(cudaGetLastError(), err, "build: prune")) return e;
    std::vector<uint32_t> pr(count * cfg.r_max), pl(count);
    cudaMemcpyAsync(pr.data(), d_pruned, pr.size() * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(pl.data(), d_plen, count * 4, cudaMemcpyDeviceToHost, st);
    if (int e = cuda_err(cudaStreamSynchronize(st), err, "build: prune")) return e;
    for (size_t i = 0; i < count; ++i)
      (*pruned)[i].assign(pr.begin() + i * cfg.r_max, pr.begin() + i * cfg.r_max + pl[i]);
    t_prune += now() - t1;
    return 0;
  }
  int update_rows(const uint32_t* ids, size_t count, const uint32_t* main_block, std::string* err) override {
    NvtxRange nvtx_range("raven.build.update_rows");
    if (count == 0) return 0;
    const double t0 = now();
    const uint32_t r = cfg.r_max;
    if (count > cap_rows) {
      if (d_rows) cudaFree(d_rows);
      d_rows = nullptr;
      if (int e = cuda_err(cudaMalloc((void**)&d_rows, count * (r + 1) * 4), err, "build: row staging")) return e;
      cap_rows = count;
    }
    std::vector<uint32_t> stage(count * (size_t)(r + 1));
    uint32_t* sid = stage.data();
    uint32_t* srow = stage.data() + count;
    for (size_t i = 0; i < count; ++i) {
      sid[i] = ids[i];
      std::memcpy(srow + i * r, main_block + (size_t)ids[i] * r, r * 4);
    }
    cudaStream_t st = ix->stream;
    if (int e = cuda_err(cudaMemcpyAsync(d_rows, stage.data(), stage.size() * 4, cudaMemcpyHostToDevice, st), err,
                         "build: rows"))
      return e;
    build_scatter_rows_kernel<<<ix->num_sms * 4, 256, 0, st>>>(d_rows, d_rows + count, count, r, ix->r_pad, ix->d_adj);
    const int e = cuda_err(cudaStreamSynchronize(st), err, "build: rows");
    t_rows += now() - t0;
    return e;
  }
};

}  // namespace

extern "C" {

int raven_graph_build_gpu(const float* vectors, uint64_t n, uint32_t dim, const raven_build_config* cfg, int device,
                          raven_graph** out) {
  NvtxRange nvtx_range("raven.graph_build_gpu");
  if (!out || (!vectors && n) || !cfg) return fail(RAVEN_EINVAL, "null argument");
  raven::BuildConfig c;
  c.alpha = cfg->alpha;
  c.l_build = cfg->l_build;
  c.r_max = cfg->r_max;
  c.r_soft = cfg->r_soft;
  c.max_iterations = cfg->max_iterations;
  c.saturate = cfg->saturate != 0;
  c.enable_layered_nav = cfg->layered_nav != 0;
  c.nav_m = cfg->nav_m;
  c.directional = cfg->directional != 0;
  c.seed = cfg->seed;
  c.threads = cfg->threads;
  c.verbose = cfg->verbose;
  if (c.nav_m < 2) return fail(RAVEN_EINVAL, "nav_m must be >= 2");
  if (!c.directional) return fail(RAVEN_EINVAL, "the GPU build implements DirectionalPrune (directional=1)");
  if (c.l_build == 0 || c.l_build > kMaxEf) return fail(RAVEN_ELIMIT, "l_build must be in 1..256 for the GPU build");
  if (c.r_max == 0 || c.r_max > 64) return fail(RAVEN_ELIMIT, "r_max must be in 1..64 for the GPU build");
  if (dim == 0 || dim > kMaxDimSq4) return fail(RAVEN_ELIMIT, "dim must be in 1..256 for the GPU build");
  if (n < 2) return fail(RAVEN_EINVAL, "the GPU build needs at least 2 vectors");
  raven_graph* g = new raven_graph();
  std::string err;
  int rc;
  {
    GpuBuild acc(vectors, n, dim, c, device);
    const double t0 = GpuBuild::now();
    rc = raven::build_vamana(vectors, n, dim, c, &g->g, &err, &acc);
    if (!rc && c.verbose)
      fprintf(stderr, "[build] total %.1f s: GPU search %.1f s, GPU prune %.1f s, row updates %.1f s, host rest %.1f s\n",
              GpuBuild::now() - t0, acc.t_search, acc.t_prune, acc.t_rows,
              GpuBuild::now() - t0 - acc.t_search - acc.t_prune - acc.t_rows);
    if (!rc && acc.truncated && c.verbose)
      fprintf(stderr, "[build] %llu nodes had more than %u visited ids (first ones kept)\n",
              (unsigned long long)acc.truncated, kBuildHistCap);
  }
  if (rc) {
    delete g;
    return fail(rc < 0 ? RAVEN_ECUDA : rc, err);
  }
  *out = g;
  return RAVEN_OK;
}

}  // extern "C"
