// candidates.cu -- batched per-candidate scoring: the codes-only graph walk's
// CandidateScorer (src/lib.rs:83-102) as one launch over many
// (query, record) pairs.
//
// PreparedQuery::score_at (src/trellis.rs:2016-2036) scores one stored record
// against a prepared query with the search estimator qm + rnorm*(dot/rescale)
// (src/trellis.rs:1483-1536); a graph walk calls it for scattered records.
// Here a batch of queries is prepared once (prep_queries_kernel) and their
// candidate lists arrive as CSR (offsets, positions).  Half a warp scores one
// candidate: lane j accumulates coordinates 16b + j (the two 8-lane FMA chains
// of src/simd.rs:202-240: lanes 0-7 are acc0, lanes 8-15 acc1), a remaining
// 8-block goes to lanes 0-7 (acc0), the xor 8, 4, 1, 2 shuffles are the
// hsum256 tree (src/simd.rs:251-262) and lane 0 adds the scalar tail with a
// separate multiply and add -- the reference's association, so every score
// is bit-identical to score_at's.
//
// Records are read where they lie (SoA arrays of the index): a candidate costs
// its code bytes plus one 32-byte sector of each sidecar.  The code table sits
// in shared memory when it fits.
#include "uv_common.cuh"
#include "uv_kernels.h"
#include "uv_score_thread.cuh"

namespace uvb {

__global__ void __launch_bounds__(256) score_candidates_kernel(const CandParams p) {
  extern __shared__ __align__(16) float table_s[];
  if (p.table_in_smem) {
    for (int i = threadIdx.x; i < p.table_len; i += blockDim.x) table_s[i] = __ldg(p.code + i);
    __syncthreads();
  }
  const float *code = p.table_in_smem ? table_s : p.code;
  const int lane = threadIdx.x & 31, j = lane & 15;
  const int hw = threadIdx.x >> 4;  // half-warp of the block
  const unsigned hmask = lane < 16 ? 0x0000ffffu : 0xffff0000u;
  const int W = p.mem + p.bits;
  const int rw = p.code_stride >> 2;
  const int nb16 = p.dim >> 4;
  const bool has8 = (p.dim & 15) >= 8;
  const int tail0 = (nb16 << 4) + (has8 ? 8 : 0);
  const int64_t step = (int64_t)gridDim.x * (blockDim.x >> 4);

  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 4) + hw; i < p.n; i += step) {
    // the query of candidate i: the last q with offsets[q] <= i
    int64_t q = 0;
    bool ok = true;
    if (p.offsets) {
      if (__ldg(p.offsets) > i || __ldg(p.offsets + p.nq) <= i) ok = false;
      int64_t lo = 0, hi = p.nq;
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (__ldg(p.offsets + mid) <= i)
          lo = mid;
        else
          hi = mid;
      }
      q = lo;
    }
    const int64_t rec = __ldg(p.positions + i);
    if (rec < 0 || rec >= p.n_records) ok = false;
    if (!ok) {
      if (j == 0) {
        p.out[i] = __int_as_float(0x7fc00000);
        atomicAdd(p.n_bad, 1);
      }
      continue;
    }
    if (p.degenerate[q]) {  // src/trellis.rs:2031-2033
      if (j == 0) p.out[i] = 0.0f;
      continue;
    }
    const float *qv = p.q_r + q * (int64_t)p.q_stride;
    const uint32_t *cw = (const uint32_t *)(p.codes + rec * (int64_t)p.code_stride);
    const uint32_t st = __ldg(p.start + rec);
    // window_at(c): W bits of the big-endian [start || codes] stream at bit
    // 32 + c*bits - mem
    auto window = [&](int c) -> uint32_t {
      const int pos = 32 + c * p.bits - p.mem;
      const int w0 = pos >> 5, sh = pos & 31;
      const uint32_t hi =
          w0 == 0 ? st : (w0 <= rw ? __byte_perm(__ldg(cw + w0 - 1), 0, 0x0123) : 0u);
      const uint32_t lo = w0 + 1 <= rw ? __byte_perm(__ldg(cw + w0), 0, 0x0123) : 0u;
      return __funnelshift_l(lo, hi, sh) >> (32 - W);
    };
    float acc = 0.0f;
    for (int b = 0; b < nb16; b++) {
      const int c = (b << 4) + j;
      acc = fmaf(__ldg(qv + c), code[window(c)], acc);
    }
    if (has8 && j < 8) {
      const int c = (nb16 << 4) + j;
      acc = fmaf(__ldg(qv + c), code[window(c)], acc);
    }
    acc = fadd(acc, __shfl_xor_sync(hmask, acc, 8));
    acc = fadd(acc, __shfl_xor_sync(hmask, acc, 4));
    acc = fadd(acc, __shfl_xor_sync(hmask, acc, 1));
    acc = fadd(acc, __shfl_xor_sync(hmask, acc, 2));
    if (j == 0) {
      for (int c = tail0; c < p.dim; c++) acc = fadd(acc, fmul(__ldg(qv + c), code[window(c)]));
      float qm = 0.0f;  // qc.get(cidx).unwrap_or(0.0), src/trellis.rs:2035
      if (p.n_centroids > 0) {
        const uint32_t ci = p.cidx ? __ldg(p.cidx + rec) : 0u;
        if (ci < (uint32_t)p.n_centroids) qm = __ldg(p.qc + q * p.n_centroids + ci);
      }
      const float rn = p.rnorm ? __ldg(p.rnorm + rec) : 1.0f;
      p.out[i] = fadd(qm, fmul(rn, fdiv(acc, __ldg(p.rescale + rec))));
    }
  }
}

// ---------------------------------------------------------------------------
// The lane kernel: one thread per candidate, a warp per 32
// consecutive candidates, each thread running record_dot_thread
// (uv_score_thread.cuh: its own 16 accumulators, windows cut from 16-byte
// code chunks with compile-time shifts).  The code table is replicated in
// shared memory so that lane l reads copy l % R at word e * R + l % R: with
// R = 32 every lane owns a bank and the table gathers never conflict.
template <int BITS>
__global__ void __launch_bounds__(1024, 1) score_candidates_lane_kernel(const CandParams p) {
  extern __shared__ __align__(16) float tab[];
  const int R = p.table_rep;
  if (R > 0) {
    for (int e = threadIdx.x; e < p.table_len; e += blockDim.x) {
      const float v = __ldg(p.code + e);
      for (int r = 0; r < R; r++) tab[e * R + r] = v;
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31;
  const int rsel = R > 0 ? (lane & (R - 1)) : 0;
  const int rstride = R > 0 ? R : 1;
  const float *table = R > 0 ? tab : p.code;
  const int64_t ngroups = (p.n + 31) >> 5;
  const int warps = blockDim.x >> 5;

  for (int64_t g = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); g < ngroups;
       g += (int64_t)gridDim.x * warps) {
    const int64_t i = (g << 5) + lane;
    const bool live = i < p.n;
    // the query of candidate i: first and last of the group by binary search,
    // then a search between them (usually empty)
    int64_t q = 0;
    bool ok = live;
    if (p.offsets) {
      const int64_t last = min((g << 5) + 31, p.n - 1);
      const int64_t target = lane == 0 ? (g << 5) : last;
      int64_t lo = 0, hi = p.nq;
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (__ldg(p.offsets + mid) <= target)
          lo = mid;
        else
          hi = mid;
      }
      int64_t qa = __shfl_sync(0xffffffffu, lo, 0);
      int64_t qb = __shfl_sync(0xffffffffu, lo, 31) + 1;
      if (live) {
        while (qb - qa > 1) {
          const int64_t mid = (qa + qb) >> 1;
          if (__ldg(p.offsets + mid) <= i)
            qa = mid;
          else
            qb = mid;
        }
        if (__ldg(p.offsets) > i || __ldg(p.offsets + p.nq) <= i) ok = false;
      }
      q = qa;
    }
    const int64_t rec = live ? __ldg(p.positions + i) : 0;
    if (rec < 0 || rec >= p.n_records) ok = false;
    if (!ok) {
      if (live) {
        p.out[i] = __int_as_float(0x7fc00000);
        atomicAdd(p.n_bad, 1);
      }
      continue;
    }
    if (p.degenerate[q]) {  // src/trellis.rs:2031-2033
      p.out[i] = 0.0f;
      continue;
    }
    const float *qv = p.q_r + q * (int64_t)p.q_stride;
    const float dot = record_dot_thread<BITS>(qv, p.codes + rec * (int64_t)p.code_stride,
                                              __ldg(p.start + rec), p.dim, p.mem, p.code_stride,
                                              table, rstride, rsel);
    float qm = 0.0f;  // qc.get(cidx).unwrap_or(0.0), src/trellis.rs:2035
    if (p.n_centroids > 0) {
      const uint32_t ci = p.cidx ? __ldg(p.cidx + rec) : 0u;
      if (ci < (uint32_t)p.n_centroids) qm = __ldg(p.qc + q * p.n_centroids + ci);
    }
    const float rn = p.rnorm ? __ldg(p.rnorm + rec) : 1.0f;
    p.out[i] = fadd(qm, fmul(rn, fdiv(dot, __ldg(p.rescale + rec))));
  }
}

const void *score_candidates_lane_kernel_ptr(int bits) {
  switch (bits) {
    case 1:
      return (const void *)score_candidates_lane_kernel<1>;
    case 2:
      return (const void *)score_candidates_lane_kernel<2>;
    case 3:
      return (const void *)score_candidates_lane_kernel<3>;
    case 4:
      return (const void *)score_candidates_lane_kernel<4>;
  }
  return nullptr;
}

}  // namespace uvb
