// The host-side arithmetic of the C++ API (include/ultravec_b200.hpp) against
// the oracle: reconstruct_unit's normalization (detail::unit_direction over
// a decoded record, l2_norm in the reference's order) gives the bits of the
// oracle's reconstruct_unit, for uncentered and centered records.  Built
// with FMA contraction on (-mfma -ffp-contract=fast) to show the header's
// sums keep their roundings under any flags.  Links the oracle only (test
// infrastructure); prints "ok <records>".
#include "ultravec_b200.hpp"
#include "uv_oracle.h"

#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

int main() {
  std::mt19937 rng(11);
  std::normal_distribution<float> nd(0.0f, 1.0f);
  int records = 0;
  for (int centered = 0; centered < 2; centered++) {
    for (int dim : {32, 64, 96}) {
      uvo_codec *c = uvo_codec_new(dim, 2, 6, 42, 3, 6, 0, 0.0f);
      std::vector<float> cen;
      const int ncen = centered ? 3 : 0;
      if (centered) {
        cen.resize((size_t)ncen * dim);
        for (auto &v : cen) v = 0.3f * nd(rng);
        uvo_codec_set_centroids(c, cen.data(), ncen);
      }
      const int cb = uvo_codec_code_bytes(c);
      for (int r = 0; r < 40; r++) {
        std::vector<float> row(dim);
        for (auto &v : row) v = nd(rng);
        std::vector<uint8_t> codes(cb);
        uint32_t start = 0, cidx = 0;
        float rescale = 0.0f, rnorm = 1.0f;
        uvo_encode(c, row.data(), codes.data(), &start, &rescale, &rnorm, &cidx);
        std::vector<float> want(dim), dec(dim);
        uvo_reconstruct_unit(c, codes.data(), start, rnorm, cidx, want.data());
        uvo_decode_codes(c, codes.data(), start, dec.data());
        const std::vector<float> got = ultravec::detail::unit_direction(
            dec, centered ? cen.data() + (size_t)cidx * dim : nullptr, rnorm);
        if (std::memcmp(got.data(), want.data(), sizeof(float) * dim) != 0) {
          std::printf("FAILED: dim %d centered %d record %d\n", dim, centered, r);
          return 1;
        }
        records++;
      }
      uvo_codec_free(c);
    }
  }
  std::printf("ok %d\n", records);
  return 0;
}
