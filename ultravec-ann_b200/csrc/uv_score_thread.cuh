// uv_score_thread.cuh -- one thread computes the codes-only dot of one record
// with a rotated query, in the association of src/simd.rs:202-262.
//
// The thread keeps the 16 accumulators of the two 8-lane FMA chains itself
// (acc[c & 15] over the 16-blocks, acc[0..7] for a trailing 8-block), folds
// them with the hsum256 tree and adds the scalar tail with a separate
// multiply and add -- bit-identical to lut_dot_u32 over the record's
// windows.  Window c is the (mem + BITS)-bit field of the big-endian
// [start || codes] stream that ends at bit 32 + (c + 1) * BITS.
//
// At BITS 1, 2, 4 the record's code words arrive 16 bytes at a time and
// every window of a chunk is cut from two adjacent words with shifts known
// at compile time (code rows are padded to 16 bytes).  BITS 3 reads the two
// words of each window through the cache.  The table is read at
// table[w * rstride + rsel], so callers may keep bank-private copies.
#pragma once

#include "uv_common.cuh"

namespace uvb {

// window_at(c) for any width, reading the code words through the cache
__device__ __forceinline__ uint32_t window_any(const uint32_t *cw, int rw, uint32_t st, int c,
                                               int bits, int mem) {
  const int pos = 32 + c * bits - mem;
  const int w0 = pos >> 5, sh = pos & 31;
  const uint32_t hi = w0 == 0 ? st : (w0 <= rw ? __byte_perm(__ldg(cw + w0 - 1), 0, 0x0123) : 0u);
  const uint32_t lo = w0 + 1 <= rw ? __byte_perm(__ldg(cw + w0), 0, 0x0123) : 0u;
  return __funnelshift_l(lo, hi, sh) >> (32 - mem - bits);
}

template <int BITS>
__device__ __forceinline__ float record_dot_thread(const float *qv, const uint8_t *codes,
                                                   uint32_t st, int dim, int mem, int code_stride,
                                                   const float *table, int rstride, int rsel) {
  const uint32_t wmask = (1u << (mem + BITS)) - 1u;
  const int nb16 = dim >> 4;
  const int rw = code_stride >> 2;
  const uint32_t *cw = (const uint32_t *)codes;
  float acc[16];
#pragma unroll
  for (int t = 0; t < 16; t++) acc[t] = 0.0f;
  if constexpr (BITS == 1 || BITS == 2 || BITS == 4) {
    constexpr int CPC = 128 / BITS;  // coordinates per 16-byte chunk
    const int nchunks = (nb16 * 16 + CPC - 1) / CPC;
    const uint4 *cw4 = (const uint4 *)codes;
    uint32_t prev = st;
    for (int k = 0; k < nchunks; k++) {
      const uint4 raw = __ldg(cw4 + k);
      const uint32_t w[4] = {__byte_perm(raw.x, 0, 0x0123), __byte_perm(raw.y, 0, 0x0123),
                             __byte_perm(raw.z, 0, 0x0123), __byte_perm(raw.w, 0, 0x0123)};
#pragma unroll
      for (int blk = 0; blk < CPC / 16; blk++) {
        const int c0 = k * CPC + blk * 16;
        if (c0 < nb16 * 16) {
          float qq[16];
#pragma unroll
          for (int v = 0; v < 4; v++) {
            const float4 f = *((const float4 *)(qv + c0) + v);
            qq[4 * v] = f.x;
            qq[4 * v + 1] = f.y;
            qq[4 * v + 2] = f.z;
            qq[4 * v + 3] = f.w;
          }
#pragma unroll
          for (int t = 0; t < 16; t++) {
            const int e = (blk * 16 + t + 1) * BITS;  // chunk bits consumed
            const int wi = (e - 1) >> 5;
            const int sh = 31 - ((e - 1) & 31);
            const uint32_t hiw = wi == 0 ? prev : w[wi > 0 ? wi - 1 : 0];
            const uint64_t v = ((uint64_t)hiw << 32) | w[wi];
            const uint32_t win = (uint32_t)(v >> sh) & wmask;
            acc[t] = fmaf(qq[t], table[win * rstride + rsel], acc[t]);
          }
        }
      }
      prev = w[3];
    }
  } else {
    for (int b = 0; b < nb16; b++) {
#pragma unroll
      for (int t = 0; t < 16; t++) {
        const int c = b * 16 + t;
        acc[t] = fmaf(qv[c], table[window_any(cw, rw, st, c, BITS, mem) * rstride + rsel],
                      acc[t]);
      }
    }
  }
  int c = nb16 * 16;
  if ((dim & 15) >= 8) {
#pragma unroll
    for (int t = 0; t < 8; t++)
      acc[t] = fmaf(qv[c + t], table[window_any(cw, rw, st, c + t, BITS, mem) * rstride + rsel],
                    acc[t]);
    c += 8;
  }
  float v8[8];
#pragma unroll
  for (int t = 0; t < 8; t++) v8[t] = fadd(acc[t], acc[t + 8]);
  const float s0 = fadd(v8[0], v8[4]), s1 = fadd(v8[1], v8[5]);
  const float s2 = fadd(v8[2], v8[6]), s3 = fadd(v8[3], v8[7]);
  float dot = fadd(fadd(s0, s1), fadd(s2, s3));
  for (; c < dim; c++)
    dot = fadd(dot, fmul(qv[c], table[window_any(cw, rw, st, c, BITS, mem) * rstride + rsel]));
  return dot;
}

}  // namespace uvb
