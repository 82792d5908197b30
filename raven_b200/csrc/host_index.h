// Host-side index: the in-memory form of a RAVEN ANNX v1 index file
// (VamanaGraph + HybridBlockedCsr + LayeredNavigation), its reader/writer,
// and the CPU Vamana build that produces it.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace raven {

constexpr uint32_t kSentinel = 0xFFFFFFFFu;        // src/lib.rs:37
constexpr uint32_t kIndexMagic = 0x414E4E58u;      // src/memory/serialize.rs:19
constexpr uint32_t kIndexVersion = 1;              // src/memory/serialize.rs:23
constexpr uint32_t kFlagHasMetadata = 0x1;         // src/memory/serialize.rs:26
constexpr uint32_t kFlagHasLayeredNav = 0x2;       // src/memory/serialize.rs:29

// LayeredNavigation (src/graph/navigation.rs:218-234).
struct LayeredNav {
  bool present = false;
  uint32_t entry = 0;
  uint8_t max_level = 0;
  uint32_t k = 0;
  std::vector<uint8_t> node_levels;
  std::vector<std::vector<uint32_t>> upper;       // per node: level l edges at [(l-1)k, lk)
  std::vector<uint32_t> entry_candidates;
};

// VamanaGraph + HybridBlockedCsr (src/graph/vamana.rs:85-100, src/memory/graph.rs:22-40).
struct HostGraph {
  uint64_t n = 0;
  uint64_t dim = 0;
  uint64_t r_max = 0;
  uint32_t entry = 0;
  std::vector<uint32_t> main_block;                // n * r_max, SENTINEL padded
  std::vector<uint16_t> degrees;                   // first SENTINEL position
  std::vector<std::vector<uint32_t>> overflow;     // build-time spill (never read by search)
  std::string metadata_toml;                       // FLAG_HAS_METADATA trailer (may be empty)
  LayeredNav nav;
};

// Build configuration (src/graph/vamana.rs:33-60 and the PyO3 mapping
// src/python.rs:109-123).
struct BuildConfig {
  float alpha = 1.2f;
  uint32_t l_build = 200;
  uint32_t r_max = 32;
  uint32_t r_soft = 48;
  uint32_t max_iterations = 2;
  bool saturate = false;
  bool enable_layered_nav = true;
  uint32_t nav_m = 32;
  bool directional = true;     // DirectionalPrune (true) or RobustPrune
  uint32_t rmin_divisor = 4;   // RAVEN_RMIN_DIVISOR default (src/graph/robust_prune.rs:223-234)
  uint64_t seed = 42;
  int threads = 0;             // 0 = all hardware threads
  int verbose = 0;
};

uint32_t crc32_ieee(const uint8_t* p, size_t n, uint32_t crc = 0);

// Returns 0 or a negative RAVEN_E* code; *err gets a message.
int parse_annx(const uint8_t* bytes, size_t len, HostGraph* g, std::string* err);
std::vector<uint8_t> serialize_annx(const HostGraph& g);

// The per-batch candidate step of the Vamana build (greedy search of the
// current graph from the entry, then DirectionalPrune of the visited set),
// done elsewhere (the GPU). build_vamana keeps the batch order, the
// connect step and the final prune; the accelerator sees every change to
// the searched rows through update_rows.
struct BuildAccelerator {
  virtual ~BuildAccelerator() = default;
  // Once, before the first batch: the graph's main blocks (n * r, SENTINEL
  // padded) and the entry point.
  virtual int begin(const uint32_t* main_block, uint64_t n, uint64_t r, uint32_t entry, std::string* err) = 0;
  // For each node of the batch: the pruned neighbour list.
  virtual int search_prune(const uint32_t* nodes, size_t count, float alpha,
                           std::vector<std::vector<uint32_t>>* pruned, std::string* err) = 0;
  // Rows whose main block changed in the connect step.
  virtual int update_rows(const uint32_t* ids, size_t count, const uint32_t* main_block, std::string* err) = 0;
};

int build_vamana(const float* vectors, uint64_t n, uint32_t dim, const BuildConfig& cfg, HostGraph* out,
                 std::string* err, BuildAccelerator* acc = nullptr);

// SQ4Params::fit / SQ8Params::fit (src/quant/sq4.rs:46-77, src/quant/sq8.rs:41-75):
// out = 5*dim floats (min, max, scale, inv_scale, neg_min_div). The min/max
// scan is split over row blocks and merged in block order with the same
// strict comparisons, so the result equals the reference's sequential scan.
void sq_fit_host(const float* data, uint64_t n, uint32_t dim, float levels, float* out, int threads);

}  // namespace raven
