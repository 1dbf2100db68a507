// uv_common.cuh -- device helpers shared by the trellis encode and scan kernels.
//
// Rounding contract: every f32 operation that the reference performs as a
// separate IEEE op is written with an explicit round-to-nearest intrinsic
// (__fadd_rn, __fmul_rn, ...), which the compiler never fuses, so device
// results are bit-identical to the reference's rustc-compiled arithmetic.
// fmaf() appears only where the reference itself issues _mm256_fmadd_ps.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace uvb {

constexpr float kF32Eps = 1.1920928955078125e-7f;  // f32::EPSILON

__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float fsqrt(float a) { return __fsqrt_rn(a); }
// Rust f32::max: the non-NaN operand wins, like fmaxf.
__device__ __forceinline__ float fmax_rs(float a, float b) { return fmaxf(a, b); }

// core::f32::total_cmp as a signed key: key(a) < key(b) <=> a orders first.
__device__ __forceinline__ int32_t total_key(float f) {
  int32_t x = __float_as_int(f);
  return x ^ (int32_t)(((uint32_t)(x >> 31)) >> 1);
}

// Ranking key for top-k: larger is better.  NaN ranks as -inf and -0.0 as
// +0.0, so equal scores tie exactly as `partial_cmp` sees them.  The low 32
// bits carry ~index so that, at equal score, the smaller index is larger.
__device__ __forceinline__ uint32_t score_key32(float s) {
  if (s != s) s = -INFINITY;
  if (s == 0.0f) s = 0.0f;
  uint32_t u = __float_as_uint(s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key32_score(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
__device__ __forceinline__ uint64_t rank_key(float s, uint32_t idx) {
  return ((uint64_t)score_key32(s) << 32) | (uint64_t)(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t rank_key_index(uint64_t key) {
  return 0xffffffffu - (uint32_t)(key & 0xffffffffu);
}
// Key of an empty slot: below every real candidate.
constexpr uint64_t kEmptyKey = 0ull;

// Rotation parameters: greedy power-of-two blocks (src/lib.rs:430-440), the
// +-1 signs of each round, and each block's 1/sqrt(len) computed as the
// reference does (f32 sqrt, f32 divide, src/lib.rs:293).
constexpr int kMaxBlocks = 16;
struct RotParams {
  int dim;
  int rounds;
  int n_blocks;
  int blk_off[kMaxBlocks];
  int blk_len[kMaxBlocks];
  float blk_inv[kMaxBlocks];
  const float *signs;  // rounds x dim (device)
};

}  // namespace uvb
