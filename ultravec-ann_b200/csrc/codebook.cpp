// codebook.cpp -- host-side construction of the data-oblivious codec state:
// the normalized Gaussian code table and the seeded rotation signs.  Both are
// pure functions of the configuration, computed once per codec on the host in
// the reference's own arithmetic (f64 inverse CDF, sequential f32 sums) and
// uploaded verbatim, so the device decodes with the exact table bits.
#include "codebook.h"

#include <cmath>

namespace uvb {

// dist.rs:158-201 inv_norm_cdf (Beasley-Springer-Moro), in f64.
static double inv_norm_cdf(double p) {
  static const double a[6] = {-3.969683028665376e1, 2.209460984245205e2, -2.759285104469687e2,
                              1.383577518672690e2,  -3.066479806614716e1, 2.506628277459239e0};
  static const double b[5] = {-5.447609879822406e1, 1.615858368580409e2, -1.556989798598866e2,
                              6.680131188771972e1,  -1.328068155288572e1};
  static const double c[6] = {-7.784894002430293e-3, -3.223964580411365e-1, -2.400758277161838e0,
                              -2.549732539343734e0,  4.374664141464968e0,   2.938163982698783e0};
  static const double d[4] = {7.784695709041462e-3, 3.224671290700398e-1, 2.445134137142996e0,
                              3.754408661907416e0};
  const double p_low = 0.02425;
  if (p < p_low) {
    const double q = std::sqrt(-2.0 * std::log(p));
    return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
           ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
  }
  if (p <= 1.0 - p_low) {
    const double q = p - 0.5;
    const double r = q * q;
    return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
           (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0);
  }
  const double q = std::sqrt(-2.0 * std::log(1.0 - p));
  return -((((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
           ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0));
}

// trellis.rs:136-145: lowbias32 finalizer -> (h + 0.5) / 2^32 -> inverse CDF.
static float gaussian_code(uint32_t w) {
  uint32_t h = w;
  h ^= h >> 16;
  h *= 0x7feb352dU;
  h ^= h >> 15;
  h *= 0x846ca68bU;
  h ^= h >> 16;
  return (float)inv_norm_cdf(((double)h + 0.5) / 4294967296.0);
}

// trellis.rs:593-610: the table over all 2^(mem+bits) windows, then shifted
// and scaled by its own mean and std (sequential f32 folds, from -0.0 like
// Rust's f32 Sum).
std::vector<float> build_code_table(int mem, int bits) {
  const size_t n = (size_t)1 << (mem + bits);
  std::vector<float> code(n);
  for (size_t k = 0; k < n; k++) code[k] = gaussian_code((uint32_t)k);
  // built with -ffp-contract=off and no fast-math: each fold stays sequential
  float s = -0.0f;
  for (size_t k = 0; k < n; k++) s = s + code[k];
  const float mean = s / (float)n;
  float v = -0.0f;
  for (size_t k = 0; k < n; k++) {
    const float dlt = code[k] - mean;
    const float sq = dlt * dlt;
    v = v + sq;
  }
  const float var = v / (float)n;
  const float inv_std = 1.0f / std::fmax(std::sqrt(var), 1e-9f);
  for (size_t k = 0; k < n; k++) code[k] = (code[k] - mean) * inv_std;
  return code;
}

// lib.rs:259-265
uint64_t splitmix64(uint64_t *state) {
  *state += 0x9E3779B97F4A7C15ULL;
  uint64_t z = *state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

// lib.rs:428-463: greedy power-of-two blocks; rounds x dim signs, -1 when the
// splitmix64 draw is even.
RotationHost build_rotation(int dim, uint64_t seed, int rounds) {
  RotationHost r;
  r.dim = dim;
  r.rounds = rounds < 1 ? 1 : rounds;
  int remaining = dim, offset = 0;
  while (remaining > 0) {
    int bs = 1;
    while (bs * 2 <= remaining) bs *= 2;
    r.blk_off.push_back(offset);
    r.blk_len.push_back(bs);
    // fwht's normalization: 1.0 / (n as f32).sqrt() (lib.rs:293)
    r.blk_inv.push_back(1.0f / std::sqrt((float)bs));
    offset += bs;
    remaining -= bs;
  }
  r.signs.resize((size_t)r.rounds * dim);
  uint64_t st = seed;
  for (int k = 0; k < r.rounds; k++)
    for (int i = 0; i < dim; i++)
      r.signs[(size_t)k * dim + i] = (splitmix64(&st) & 1) == 0 ? -1.0f : 1.0f;
  return r;
}

}  // namespace uvb
