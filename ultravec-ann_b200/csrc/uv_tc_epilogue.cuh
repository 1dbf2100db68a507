// uv_tc_epilogue.cuh -- the per-tile epilogue of the tensor-core prefilter
// kernels (tcscan.cu, tcwide.cu): one thread holds one query's bounds for a
// run of records (nl chunks of 32 accumulator columns, already in
// registers).  Pass 1 writes the run's largest lower bound; pass 2 appends
// every record whose upper bound reaches the query's threshold to its
// candidate list; mode 3 (the IVF probe) stores every value.
// bounds_run takes bounds that the MMA formed (the extra K slice);
// bounds_run_cmax forms them from s * g * dot and the chunk constants.
#pragma once

#include "uv_kernels.h"

namespace uvb {
namespace tcep {

// 3-input maximum (NaN-ignoring like fmaxf)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float chunk_max(const uint32_t (&v)[32]) {
  float m = max3(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
#pragma unroll
  for (int j = 3; j < 31; j += 2) m = max3(m, __uint_as_float(v[j]), __uint_as_float(v[j + 1]));
  return fmaxf(m, __uint_as_float(v[31]));
}

// r: the bounds of records rec0 .. rec0 + 32 * NL - 1 for query q; group:
// the tile-maxima slot of this run (pass 1).  Pass 2 appends to this
// thread's own segment of the query's candidate list (dst, region_cap
// slots), counting in `count`: one thread per (query, record split, column
// half) owns a segment, so no append waits on an atomic.
template <int MODE, int NL>
__device__ __forceinline__ void bounds_run(const TcScanParams &p, const uint32_t (&r)[NL][32],
                                           int64_t q, bool qok, float theta, int64_t group,
                                           int64_t rec0, uint32_t *dst = nullptr,
                                           int *count = nullptr) {
  if (MODE == 3) {
    // every value: row q of p.tmax (leading dimension n_groups), the dot
    // itself (the IVF probe bounds it on the host side of the contract)
    if (q < p.nq) {
      float *dst = p.tmax + q * p.n_groups;
#pragma unroll
      for (int l = 0; l < NL; l++)
#pragma unroll
        for (int j = 0; j < 32; j++)
          if (rec0 + 32 * l + j < p.n) dst[rec0 + 32 * l + j] = __uint_as_float(r[l][j]);
    }
    return;
  }
  float mc[NL];
#pragma unroll
  for (int l = 0; l < NL; l++) mc[l] = chunk_max(r[l]);
  float m = mc[0];
#pragma unroll
  for (int l = 1; l < NL; l++) m = fmaxf(m, mc[l]);
  if (MODE == 1) {
    if (q < p.nq) p.tmax[q * p.n_groups + group] = qok ? m : -INFINITY;
  } else if (qok && !(m < theta)) {
    // rare: every record of the chunks whose maximum reaches theta
    uint32_t mask[NL];
#pragma unroll
    for (int l = 0; l < NL; l++) {
      uint32_t mk = 0;
      if (!(mc[l] < theta)) {
#pragma unroll
        for (int j = 0; j < 32; j++) mk |= (!(__uint_as_float(r[l][j]) < theta) ? 1u : 0u) << j;
      }
      mask[l] = mk;
    }
    if (rec0 + 32 * NL > p.n) {
      const int64_t lim = p.n - rec0;  // records past n are padding
#pragma unroll
      for (int l = 0; l < NL; l++) {
        const int64_t room = lim - 32 * l;
        mask[l] &= room >= 32 ? 0xffffffffu : (room <= 0 ? 0u : ((1u << room) - 1u));
      }
    }
    int pos = *count;
#pragma unroll
    for (int l = 0; l < NL; l++) {
      uint32_t mk = mask[l];
      while (mk != 0u) {
        const int j = __ffs(mk) - 1;
        mk &= mk - 1u;
        if (pos < p.region_cap) dst[pos] = (uint32_t)(rec0 + 32 * l + j);
        pos++;
      }
    }
    *count = pos;
  }
}

// maximum of 16 accumulator values (NaN-ignoring like fmaxf)
__device__ __forceinline__ float chunk_max16(const uint32_t (&v)[16]) {
  float m = max3(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
#pragma unroll
  for (int j = 3; j < 15; j += 2) m = max3(m, __uint_as_float(v[j]), __uint_as_float(v[j + 1]));
  return fmaxf(m, __uint_as_float(v[15]));
}

// The same for accumulators of s * g * dot alone (no extra K slice), one
// thread's run of NC chunks of 16 records: the bound constant is applied per
// chunk with its largest C' (cm[c], from p.cmax), rounded outwards.
//   pass 1: max_chunk(dot) - cm rounded down lower-bounds the score of the
//           chunk's largest-dot record (padding rows of the last tile are
//           left out of the maximum);
//   pass 2: a record is kept when dot >= t = theta - cm rounded down, which
//           every record whose own upper bound dot + C' reaches theta
//           satisfies (C' <= cm).
template <int MODE, int NC>
__device__ __forceinline__ void bounds_run_cmax(const TcScanParams &p,
                                                const uint32_t (&r)[NC][16],
                                                const float (&cm)[NC], int64_t q, bool qok,
                                                float theta, int64_t group, int64_t rec0,
                                                uint32_t *dst, int *count) {
  float mc[NC];
#pragma unroll
  for (int c = 0; c < NC; c++) {
    const uint32_t *v = r[c];
    float m = max3(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
#pragma unroll
    for (int j = 3; j < 15; j += 2) m = max3(m, __uint_as_float(v[j]), __uint_as_float(v[j + 1]));
    mc[c] = fmaxf(m, __uint_as_float(v[15]));
  }
  if (MODE == 1) {
    if (rec0 + 16 * NC > p.n) {
#pragma unroll
      for (int c = 0; c < NC; c++) {
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < 16; j++)
          if (rec0 + 16 * c + j < p.n) mx = fmaxf(mx, __uint_as_float(r[c][j]));
        mc[c] = mx;
      }
    }
    float m = __fsub_rd(mc[0], cm[0]);
#pragma unroll
    for (int c = 1; c < NC; c++) m = fmaxf(m, __fsub_rd(mc[c], cm[c]));
    if (q < p.nq) p.tmax[q * p.n_groups + group] = qok ? m : -INFINITY;
    return;
  }
  float t[NC];
  bool any = false;
#pragma unroll
  for (int c = 0; c < NC; c++) {
    t[c] = __fsub_rd(theta, cm[c]);
    any |= !(mc[c] < t[c]);
  }
  if (!qok || !any) return;
  // rare: every record of the chunks whose maximum reaches their threshold
  static_assert(NC * 16 <= 64, "one 64-bit mask per run");
  uint64_t mask = 0;
#pragma unroll
  for (int c = 0; c < NC; c++) {
    if (!(mc[c] < t[c])) {
      uint32_t mk = 0;
#pragma unroll
      for (int j = 0; j < 16; j++) mk |= (!(__uint_as_float(r[c][j]) < t[c]) ? 1u : 0u) << j;
      mask |= (uint64_t)mk << (16 * c);
    }
  }
  if (rec0 + 16 * NC > p.n) {
    const int64_t room = p.n - rec0;  // records past n are padding
    mask &= room <= 0 ? 0ull : ((1ull << room) - 1ull);  // room < 16 * NC <= 64 here
  }
  int pos = *count;
  while (mask != 0ull) {
    const int j = __ffsll((long long)mask) - 1;
    mask &= mask - 1ull;
    if (pos < p.region_cap) dst[pos] = (uint32_t)(rec0 + j);
    pos++;
  }
  *count = pos;
}

}  // namespace tcep
}  // namespace uvb
