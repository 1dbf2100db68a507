// State of the CPU stand-in for the C ABI (mock_uv.cpp): what the C++ host
// API passed to the library, and failures to inject.  Test infrastructure.
#ifndef ULTRAVEC_MOCK_UV_H
#define ULTRAVEC_MOCK_UV_H

#include "ultravec_b200.h"

#include <string>
#include <vector>

struct MockState {
  std::vector<std::string> calls;  // entry points in call order
  std::string error;               // uv_last_error()
  std::string fail_call;           // this entry point fails with fail_code
  int fail_code = UV_ECUDA;
  uv_config cfg{};                 // last uv_codec_create
  std::vector<float> rows;         // last rows / queries / centroids passed
  std::vector<int64_t> ids;        // last ids passed to uv_index_add
  int64_t nq = 0, reserved = 0, n_db = 0;
  int32_t k = 0, mode = -1, nprobe = 0, rdepth = 0, iters = 0, centered = -1, nlist = 0;
  int32_t n_centroids = 0, sl_c = -1, sl_asym = -1, sl_rnorm = -1;
  uint64_t seed = 0;
  std::string path;
  int live_codecs = 0, live_indexes = 0, live_prepared = 0;
  int order_errors = 0;  // codecs destroyed while an index on them was alive

  void reset() { *this = MockState(); }
  bool called(const std::string &name) const {
    for (const auto &c : calls)
      if (c == name) return true;
    return false;
  }
};

extern MockState mock;

#endif
