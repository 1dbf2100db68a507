// uv_team.cuh -- a "team" is the group of threads that owns one vector
// (encode) or one query (query preparation).  Teams of <= 32 threads are
// aligned lane groups inside a warp and synchronize with __syncwarp(); a team
// larger than a warp is the whole CTA and uses __syncthreads().  Every lane of
// a warp runs the same sequence of team syncs, so packed teams never diverge
// on a barrier.
#pragma once

#include "uv_common.cuh"

namespace uvb {

struct Team {
  int t;     // rank inside the team
  int T;     // team size (power of two)
  bool cta;  // team spans the CTA
  __device__ __forceinline__ void sync() const {
    if (cta)
      __syncthreads();
    else
      __syncwarp();
  }
  __device__ __forceinline__ bool leader() const { return t == 0; }
};

// Rust `.sum::<f32>()` of x*x: a left fold from -0.0, one rounding per op.
// Eight operands are read ahead of the fold (the adds stay in order), so
// the one dependent chain is the adds, not the loads.
__device__ __forceinline__ float seq_sum_sq(const float *x, int n) {
  float s = -0.0f;
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    float v[8];
#pragma unroll
    for (int t = 0; t < 8; t++) v[t] = x[i + t];
#pragma unroll
    for (int t = 0; t < 8; t++) s = fadd(s, fmul(v[t], v[t]));
  }
  for (; i < n; i++) s = fadd(s, fmul(x[i], x[i]));
  return s;
}

__device__ __forceinline__ float seq_dot(const float *a, const float *b, int n) {
  float s = -0.0f;
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    float va[8], vb[8];
#pragma unroll
    for (int t = 0; t < 8; t++) {
      va[t] = a[i + t];
      vb[t] = b[i + t];
    }
#pragma unroll
    for (int t = 0; t < 8; t++) s = fadd(s, fmul(va[t], vb[t]));
  }
  for (; i < n; i++) s = fadd(s, fmul(a[i], b[i]));
  return s;
}

// std_about_mean (src/lib.rs:251-256)
__device__ __forceinline__ float seq_std_about_mean(const float *x, int n) {
  float nf = (float)n;
  float s = -0.0f;
  for (int i = 0; i < n; i++) s = fadd(s, x[i]);
  float mean = fdiv(s, nf);
  float v = -0.0f;
  for (int i = 0; i < n; i++) {
    float d = fsub(x[i], mean);
    v = fadd(v, fmul(d, d));
  }
  return fsqrt(fdiv(v, nf));
}

// In-place normalized FWHT of one block (src/lib.rs:281-295): stages h = 1,
// 2, 4, ... in order, each output a single add or subtract, then x * inv.
// The stage order is what fixes the rounding; within a stage the butterflies
// are independent, so the team splits them freely.
__device__ __forceinline__ void team_fwht(float *blk, int len, float inv, const Team &tm) {
  const int half = len >> 1;
  for (int h = 1; h < len; h <<= 1) {
    for (int bi = tm.t; bi < half; bi += tm.T) {
      int i = ((bi & ~(h - 1)) << 1) | (bi & (h - 1));
      float u = blk[i], v = blk[i + h];
      blk[i] = fadd(u, v);
      blk[i + h] = fsub(u, v);
    }
    tm.sync();
  }
  for (int i = tm.t; i < len; i += tm.T) blk[i] = fmul(blk[i], inv);
  tm.sync();
}

// Rotation::apply (src/lib.rs:472-484) or apply_inverse (487-499) on a
// shared-memory row.
__device__ __forceinline__ void team_rotate(float *x, const RotParams &rp, const Team &tm,
                                            bool inverse) {
  for (int r = 0; r < rp.rounds; r++) {
    const int rr = inverse ? rp.rounds - 1 - r : r;
    const float *sg = rp.signs + (size_t)rr * rp.dim;
    for (int b = 0; b < rp.n_blocks; b++) {
      const int off = rp.blk_off[b], len = rp.blk_len[b];
      float *blk = x + off;
      if (!inverse) {
        for (int i = tm.t; i < len; i += tm.T) blk[i] = fmul(blk[i], sg[off + i]);
        tm.sync();
      }
      team_fwht(blk, len, rp.blk_inv[b], tm);
      if (inverse) {
        for (int i = tm.t; i < len; i += tm.T) blk[i] = fmul(blk[i], sg[off + i]);
        tm.sync();
      }
    }
  }
}

}  // namespace uvb
