// The C++ host API (include/ultravec_b200.hpp) linked against the real
// library on a machine without a GPU: a codec cannot be made, and the
// failure arrives as ultravec::Error with the library's status, after the
// configuration checks that need no device.  Prints "ok" and exits 0.
#include "ultravec_b200.hpp"

#include <cstdio>

using namespace ultravec;

static int expect(int want_a, int want_b, const TrellisConfig &cfg) {
  try {
    TrellisQuantizer::from_config(cfg);
  } catch (const Error &e) {
    if (e.code() == want_a || e.code() == want_b) return 0;
    std::printf("FAILED: status %d (%s)\n", e.code(), e.what());
    return 1;
  }
  std::printf("FAILED: no ultravec::Error\n");
  return 1;
}

int main() {
  if (uv_abi_version() != UV_ABI_VERSION) return 1;
  // no device: a status, not a crash
  if (expect(UV_EINVAL, UV_ECUDA, TrellisConfig::make(128, 2, 8))) return 1;
  // 5 bits per coordinate: refused before any device work
  if (expect(UV_EINVAL, UV_EINVAL, TrellisConfig::make(128, 5, 8))) return 1;
  std::printf("ok\n");
  return 0;
}
