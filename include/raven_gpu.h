/*
 * raven_gpu.h — C ABI of the B200 query engine for RAVEN's Vamana graph search.
 *
 * This is the boundary a host binding (a Rust FFI crate, the pybind/ctypes
 * layer, a C program) calls. Plain pointers and sizes only; every call returns
 * a status code (RAVEN_OK or a negative RAVEN_E*) and never aborts the
 * process; raven_last_error() gives a thread-local message for the last
 * failure on the calling thread.
 *
 * Each entry point names the reference interface it replaces (paths relative
 * to the Juwan-Hwang/RAVEN source tree).
 *
 * Ownership: the caller owns every buffer it passes; the library copies what
 * it keeps. A raven_graph owns host memory, a raven_index owns device memory
 * on one GPU. Threading: a raven_graph is immutable after load/build; a
 * raven_index is immutable after upload, and concurrent searches on distinct
 * CUDA streams are allowed (each call uses its own work counter; the
 * visited-set spill area is per call, see raven_search_batch_device). Two
 * exceptions: raven_index_set_tuning changes the index and must not overlap a
 * search call on it, and raven_search_batch_device_noalloc calls share one
 * scratch array per GPU (see there).
 */
#ifndef RAVEN_GPU_H
#define RAVEN_GPU_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RAVEN_API __attribute__((visibility("default")))
#else
#define RAVEN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes -------------------------------------------------------- */
#define RAVEN_OK 0
#define RAVEN_EINVAL (-1)   /* bad argument (PyO3 ValueError, e.g. dim mismatch src/python.rs:100-105) */
#define RAVEN_EIO (-2)      /* file could not be read/written (PyO3 IOError src/python.rs:191,199) */
#define RAVEN_EMAGIC (-3)   /* SerializeError::MagicMismatch src/memory/serialize.rs:38 */
#define RAVEN_EVERSION (-4) /* SerializeError::VersionMismatch src/memory/serialize.rs:40 */
#define RAVEN_ECRC (-5)     /* SerializeError::CrcMismatch src/memory/serialize.rs:45 */
#define RAVEN_EFORMAT (-6)  /* truncated / inconsistent file (SerializeError::Io UnexpectedEof/InvalidData) */
#define RAVEN_ESTATE (-7)   /* wrong state, e.g. search_sq4 without with_sq4 (src/graph/vamana.rs:1773 panic) */
#define RAVEN_ECUDA (-8)    /* CUDA runtime error */
#define RAVEN_ENOMEM (-9)   /* allocation failed */
#define RAVEN_ELIMIT (-10)  /* a size is above a compiled limit of this engine (see raven_limits) */

/* per-query status written to outputs.status */
#define RAVEN_Q_OK 0
#define RAVEN_Q_VISITED_OVERFLOW 1 /* visited set exceeded shared+spill capacity; result truncated */
#define RAVEN_Q_NAV_LIMIT 2        /* navigation descent exceeded its step bound */
#define RAVEN_Q_BAD_EF 3           /* ef resolved to 0 or above the engine limit (host validation prevents it) */

#define RAVEN_QUANT_SQ4 0 /* GraphSearcher::with_sq4 / search_sq4  src/graph/vamana.rs:1578,1772 */
#define RAVEN_QUANT_SQ8 1 /* GraphSearcher::with_sq8 / search_sq8  src/graph/vamana.rs:1568,1752 */
#define RAVEN_QUANT_F32 2 /* GraphSearcher::search: the f32 traversal (greedy_search_vec_reuse),
                             results = the first k of the pool, no rerank  src/graph/vamana.rs:1627-1672 */

typedef struct raven_graph raven_graph; /* VamanaGraph (host)            src/graph/vamana.rs:85 */
typedef struct raven_index raven_index; /* searcher state on one GPU     src/graph/vamana.rs:1428 */

/* VamanaBuildConfig as PyO3 fills it (src/graph/vamana.rs:33-60, src/python.rs:109-123). */
typedef struct {
  float alpha;             /* 1.2 */
  uint32_t l_build;        /* 200 */
  uint32_t r_max;          /* 32  */
  uint32_t r_soft;         /* 48 (= r_max * 1.5 in PyO3) */
  uint32_t max_iterations; /* 2 */
  int32_t saturate;        /* !directional */
  int32_t layered_nav;     /* 1 */
  uint32_t nav_m;          /* 32 */
  int32_t directional;     /* 1 = DirectionalPrune, 0 = RobustPrune */
  uint64_t seed;           /* 42 */
  int32_t threads;         /* 0 = all host threads */
  int32_t verbose;
} raven_build_config;

typedef struct {
  uint64_t n, dim, r_max;
  uint32_t entry_point;  /* medoid */
  int32_t has_nav;
  uint32_t nav_entry, nav_max_level, nav_k;
  uint64_t nav_upper_nodes; /* nodes with a non-empty upper list */
} raven_graph_info_t;

/* ---- host graph (build / load / save) ------------------------------------ */
/* VamanaGraph::build (src/graph/vamana.rs:106-201) via PyIndex::build (src/python.rs:97-129). */
RAVEN_API int raven_graph_build(const float* vectors, uint64_t n, uint32_t dim, const raven_build_config* cfg,
                      raven_graph** out);

/* Vamana build with the per-batch candidate step on a GPU (no reference
 * counterpart on a GPU; replaces the search + prune loop of VamanaGraph::build,
 * src/graph/vamana.rs:106-201). Same batches, random stream, connect step and
 * final prune as raven_graph_build; each batch's nodes are searched by the
 * engine's search kernel in its f32 mode (greedy_search_vec_build,
 * src/graph/vamana.rs:530-567: entry = medoid, ef = l_build, f32 distances in
 * the AVX-512 summation order) and their visited sets pruned by
 * DirectionalPrune on the GPU with the same distances, so the graph is the one
 * raven_graph_build makes, byte for byte. DirectionalPrune only
 * (cfg->directional = 1); l_build <= 256, r_max <= 64, dim <= 256. The layered
 * navigation is built on the host as in raven_graph_build. */
RAVEN_API int raven_graph_build_gpu(const float* vectors, uint64_t n, uint32_t dim, const raven_build_config* cfg,
                                    int device, raven_graph** out);
/* Serializable::load + VamanaGraph::deserialize (src/memory/serialize.rs:146, src/graph/vamana.rs:1326). */
RAVEN_API int raven_graph_load(const char* path, raven_graph** out);
RAVEN_API int raven_graph_load_bytes(const void* bytes, size_t len, raven_graph** out);
/* Serializable::save (src/memory/serialize.rs:140). */
RAVEN_API int raven_graph_save(const raven_graph* g, const char* path);
RAVEN_API void raven_graph_free(raven_graph* g);
RAVEN_API int raven_graph_info(const raven_graph* g, raven_graph_info_t* out);
/* HybridBlockedCsr::neighbors (src/memory/graph.rs:78-82): copies <= cap ids, returns degree in *deg. */
RAVEN_API int raven_graph_neighbors(const raven_graph* g, uint32_t node, uint32_t* out, uint32_t cap, uint32_t* deg);

/* ---- device index (searcher creation) ------------------------------------ */
typedef struct {
  int32_t device;         /* CUDA ordinal */
  int32_t build_sq4;      /* SQ4Dataset::build (src/quant/sq4.rs:303) on the device */
  int32_t build_sq8;      /* SQ8Dataset::build (src/quant/sq8.rs:395) on the device */
  int32_t build_adaptive; /* AdaptiveEfConfig::build_with_layered_nav samples (src/graph/adaptive_ef.rs:307-327) */
  int32_t build_f16;      /* F16Dataset::build (src/distance/f16.rs:344-349) for rerank_f16 */
} raven_upload_options;

/* PyIndex::searcher (src/python.rs:134-181) / GraphSearcher::new + with_sq4/with_sq8
 * (src/graph/vamana.rs:1478,1568,1578): copies the graph (as a fixed-degree
 * R_pad=roundup(r_max,32) SENTINEL-padded u32 array), the f32 vectors and the
 * navigation layers to HBM, and quantises the vectors there. The caller keeps
 * `g` and `vectors`. */
RAVEN_API int raven_index_upload(const raven_graph* g, const float* vectors, uint64_t n, uint32_t dim,
                       const raven_upload_options* opt, raven_index** out);
RAVEN_API int raven_index_free(raven_index* ix);
/* Sorted AdaptiveEf sample distances (<= 2000), copied to `out`. */
RAVEN_API int raven_index_adaptive_samples(const raven_index* ix, float* out, uint32_t cap, uint32_t* n_out);
/* SQ params: 5*dim floats (min, max, scale, inv_scale, neg_min_div) — SQ4Params/SQ8Params fields. */
RAVEN_API int raven_index_sq_params(const raven_index* ix, int32_t quant, float* out5dim);
/* Device codes copied to host, unpadded: n * ceil(dim/2) (SQ4) or n * dim (SQ8) bytes. */
RAVEN_API int raven_index_codes(const raven_index* ix, int32_t quant, uint8_t* out, uint64_t cap_bytes);

/* ---- search -------------------------------------------------------------- */
/* GraphSearcher knobs (src/graph/vamana.rs:1478-1616; PyO3 defaults src/python.rs:171-179). */
typedef struct {
  uint32_t ef;              /* ef_search (fixed mode); 50 */
  uint32_t k;               /* results per query; 10 */
  uint32_t rerank_factor;   /* with_rerank_factor, clamped >= 1 (vamana.rs:1547-1550) */
  uint32_t prefetch_offset; /* with_prefetch_offset: accepted, no effect on results or the device */
  int32_t quant;            /* RAVEN_QUANT_SQ4 / RAVEN_QUANT_SQ8 */
  int32_t adaptive;         /* with_adaptive_ef(base.with_params(min_ef, max_ef, gamma)) */
  float gamma;
  uint32_t min_ef, max_ef;
  int32_t rerank_f16;       /* with_f16 (vamana.rs:1559): rerank with the f16 vectors (rerank_f16,
                               src/graph/refiner.rs:87-104); needs an index uploaded with build_f16 */
} raven_search_params;

/* Per-query outputs. ids/dists: nq*k, results in ascending f32 distance,
 * unfilled slots id 0 / dist 0 (PyO3 batch_search padding, src/python.rs:344-349).
 * Any pointer but ids may be NULL. history (optional): nq*history_cap, the
 * visited nodes of each query in VisitedTracker order, with the full count in
 * history_len (entries beyond history_cap are not stored).
 *
 * visited / history / history_len cost time: with any of them set, an SQ4/SQ8
 * search keeps the exact visited set (a shared-memory table per query with
 * global spill tables behind it). With all three NULL it decides new
 * neighbours by pool membership instead, which accepts exactly the same
 * candidates (a visited node outside the pool never beats the pool's worst
 * entry), so every other output is identical; it needs no spill tables and
 * runs faster. The f32 traversal always keeps the visited set. */
typedef struct {
  uint32_t* ids;
  float* dists;
  uint32_t* counts;      /* results returned (<= k) */
  uint32_t* visited;     /* last_visited_count (vamana.rs:1942) */
  uint32_t* ef_used;     /* last_ef_used (vamana.rs:1950) */
  int32_t* status;       /* RAVEN_Q_* */
  uint32_t* n_nav;       /* f32 distance evaluations in the navigation descent */
  uint32_t* expansions;  /* beam pops */
  uint32_t* history;
  uint32_t history_cap;
  uint32_t* history_len;
} raven_search_outputs;

/* GraphSearcher::batch_search (src/graph/vamana.rs:1983-2095) with host
 * buffers: copies queries in, runs on `stream` (a cudaStream_t; NULL = the
 * CUDA default stream), copies outputs back and synchronises that stream. */
RAVEN_API int raven_search_batch(raven_index* ix, const float* queries, uint64_t nq, const raven_search_params* p,
                       const raven_search_outputs* out, void* stream);
/* Same with device buffers; asynchronous on `stream` (NULL = the CUDA default stream). */
RAVEN_API int raven_search_batch_device(raven_index* ix, const float* d_queries, uint64_t nq, const raven_search_params* p,
                              const raven_search_outputs* d_out, void* stream);

/* Device-buffer search that allocates nothing (no counterpart in the
 * reference). For callers that cannot allocate device memory while serving —
 * e.g. when another allocator has reserved the GPU's memory up front, or a hard
 * memory budget must be fixed at start-up — the per-call scratch (work counter,
 * AdaptiveEf table, visited-set spill tables) comes from one fixed 64 MiB
 * device array that every GPU loading this library holds until the process
 * exits, instead of the stream-ordered pool used by raven_search_batch_device.
 * Same inputs, outputs and results. The first call on a device looks up that
 * array's device address (cudaGetSymbolAddress), as does the first call after
 * the device's context was replaced (cudaDeviceReset); make those calls before
 * any stream capture. All calls share the array: calls that overlap on the GPU
 * (e.g. on two streams) race and must be serialised by the caller. To fit the
 * array, spill tables are smaller (each query can still hold over 14,000 visited
 * nodes before reporting RAVEN_Q_VISITED_OVERFLOW) and fewer warps may be
 * resident. Returns RAVEN_ELIMIT if a call cannot fit (an AdaptiveEf table of
 * more than 4032 samples). */
RAVEN_API int raven_search_batch_device_noalloc(raven_index* ix, const float* d_queries, uint64_t nq,
                                                const raven_search_params* p, const raven_search_outputs* d_out,
                                                void* stream);

/* Exact k-nearest neighbours over the uploaded f32 vectors (recall ground
 * truth; no reference counterpart — the reference reads SIFT groundtruth
 * files, src/bin/sq4_ef_sweep.rs:61). Device buffers; ties broken by id.
 * Every wait inside the tensor-core kernel is bounded: if one runs out, the
 * call returns RAVEN_ECUDA and its outputs are not valid, and the kernel lets
 * its own copies and MMAs finish before it frees tensor memory and exits. */
RAVEN_API int raven_knn_exact_device(raven_index* ix, const float* d_queries, uint64_t nq, uint32_t k, uint32_t* d_ids,
                           float* d_dists, void* stream);

/* Merge per-shard top-k lists (shard-major [n_shards][nq][k], ids local to
 * each shard, shard s covering global ids [s*shard_size, ...)) into global
 * top-k per query, ties by (dist, shard, rank). No reference counterpart
 * (the reference has no sharding). Device buffers. */
RAVEN_API int raven_merge_topk_device(const uint32_t* d_ids, const float* d_dists, const uint32_t* d_counts,
                            uint32_t n_shards, uint64_t nq, uint32_t k, uint64_t shard_size, uint32_t* d_out_ids,
                            float* d_out_dists, uint32_t* d_out_counts, void* stream);

/* The same merge read straight from the buffer an all-gather of per-rank
 * blocks leaves behind (no reference counterpart). The buffer holds world x
 * per_rank shard blocks, per_rank = ceil(n_shards / world); shard s (on rank
 * s % world, its slot s / world there) is block (s % world) * per_rank +
 * s / world. A block is nq*(2k+1) 32-bit words: ids u32 [nq][k], distances
 * f32 [nq][k], counts u32 [nq] (a search's ids / dists / counts outputs laid
 * end to end). Blocks past the last shard are ignored. Device buffers. */
RAVEN_API int raven_merge_topk_gathered_device(const void* d_gathered, uint32_t n_shards, uint32_t world,
                                               uint32_t per_rank, uint64_t nq, uint32_t k, uint64_t shard_size,
                                               uint32_t* d_out_ids, float* d_out_dists, uint32_t* d_out_counts,
                                               void* stream);

typedef struct {
  uint32_t max_ef;      /* largest pool capacity (fixed ef or adaptive max) */
  uint32_t max_dim;     /* largest vector dimension */
  uint32_t max_r;       /* largest graph degree */
  uint32_t max_nav_k;   /* largest navigation-layer degree */
} raven_limits_t;
RAVEN_API void raven_limits(raven_limits_t* out);

/* Launch tuning for benchmark sweeps (no reference counterpart): log2 of the
 * shared-memory visited-table slots per query (8..14, 0 = automatic) and of the
 * global spill-table slots per resident warp (10..20, 0 = keep). */
RAVEN_API int raven_index_set_tuning(raven_index* ix, int32_t hash_bits, int32_t spill_bits);

/* Small-batch path (no reference counterpart): a search of at most `max_nq`
 * queries runs one CTA of four warps per query (with the visited set, when
 * requested, in a 2^14-slot shared-memory table) instead of the persistent
 * one-warp-per-query kernel; results are identical. RAVEN_SMALL_BATCH_AUTO
 * (the default after upload): as many queries as one wave of such CTAs holds,
 * at most four per SM (592 queries on 148 SMs); 0 disables it (every batch
 * uses the persistent kernel). Applies to SQ4/SQ8 searches without
 * rerank_f16 through raven_search_batch and raven_search_batch_device. */
#define RAVEN_SMALL_BATCH_AUTO (~(uint64_t)0)
RAVEN_API int raven_index_set_small_batch(raven_index* ix, uint64_t max_nq);

/* Neighbour codes beside each row (no reference counterpart): for every
 * uploaded quantiser, n x R_pad x code-stride bytes in which node i's slot j
 * holds the code of its j-th neighbour (2 GB for 1M nodes, R_pad 32, SQ4 at
 * dim 128). A search without visited counts then reads an expansion's codes
 * as one contiguous piece, prefetched with the row, instead of gathering them
 * from R scattered nodes. Built at upload when they fit in half of the free
 * device memory; enable = 0 frees them, 1 (re)builds them. Results are
 * identical either way. */
RAVEN_API int raven_index_set_fat_rows(raven_index* ix, int32_t enable);

RAVEN_API const char* raven_last_error(void);
RAVEN_API const char* raven_version(void);

#ifdef __cplusplus
}
#endif
#endif /* RAVEN_GPU_H */
