// codebook.h -- host construction of the code table and rotation signs.
#pragma once

#include <cstdint>
#include <vector>

namespace uvb {

struct RotationHost {
  int dim = 0, rounds = 0;
  std::vector<int> blk_off, blk_len;
  std::vector<float> blk_inv;
  std::vector<float> signs;  // rounds x dim
};

std::vector<float> build_code_table(int mem, int bits);
RotationHost build_rotation(int dim, uint64_t seed, int rounds);
// lib.rs:259-265: one splitmix64 step (advances *state, returns the mix)
uint64_t splitmix64(uint64_t *state);

}  // namespace uvb
