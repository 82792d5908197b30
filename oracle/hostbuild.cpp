// C entry point of the host Vamana build for the reference arm of the
// benchmark. TEST AND BENCHMARK INFRASTRUCTURE ONLY.
//
// The reference builds its index offline with its Rayon pipeline
// (VamanaGraph::build, src/graph/vamana.rs:106-201, with the PyO3 build
// parameters of src/python.rs:109-123) and searches the saved file. Its C++
// restatement lives in raven_b200/csrc/host_index.cpp; this file links that
// restatement into its own library (oracle/_build/libhostbuild.so) so that the
// reference arm can build and save an index without loading the engine's
// CUDA library.
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>

#include "../raven_b200/csrc/host_index.h"

extern "C" {

// Builds the Vamana graph of `n` x `dim` vectors and writes it as an ANNX v1
// file at `path`. Returns 0, or a negative code with a message in `err`.
int hostbuild_build_save(const float* vectors, unsigned long long n, unsigned dim, float alpha, unsigned l_build,
                         unsigned r_max, unsigned r_soft, unsigned max_iterations, int directional, unsigned nav_m,
                         unsigned long long seed, int threads, const char* path, char* err, size_t err_len) {
  raven::BuildConfig c;
  c.alpha = alpha;
  c.l_build = l_build;
  c.r_max = r_max;
  c.r_soft = r_soft;
  c.max_iterations = max_iterations;
  c.saturate = directional == 0;
  c.enable_layered_nav = true;
  c.nav_m = nav_m;
  c.directional = directional != 0;
  c.seed = seed;
  c.threads = threads;
  raven::HostGraph g;
  std::string msg;
  auto report = [&](int rc, const std::string& m) {
    if (err && err_len) snprintf(err, err_len, "%s", m.c_str());
    return rc;
  };
  int rc = raven::build_vamana(vectors, n, dim, c, &g, &msg);
  if (rc) return report(rc < 0 ? rc : -rc, msg);
  const std::vector<uint8_t> bytes = raven::serialize_annx(g);
  std::ofstream f(path, std::ios::binary);
  if (!f) return report(-2, std::string("cannot open ") + path);
  f.write((const char*)bytes.data(), (std::streamsize)bytes.size());
  if (!f) return report(-2, std::string("write failed: ") + path);
  return 0;
}

}  // extern "C"
