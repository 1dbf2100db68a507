// uv_encode_row.cuh -- the per-row stages shared by the trellis encoders
// (encode.cu: one team per row inside a CTA; encode_cluster.cu: one thread-
// block cluster per row): prep before the Viterbi forward pass and the
// finalize after the traceback.
#pragma once

#include "uv_kernels.h"
#include "uv_team.cuh"

namespace uvb {

// Team-wide maximum of a 64-bit key.  `scratch` holds 32 u64 in shared memory
// (only used when the team spans the CTA).
__device__ __forceinline__ uint64_t team_max_u64(uint64_t v, const Team &tm,
                                                 uint64_t *scratch) {
  if (!tm.cta) {
    for (int o = tm.T >> 1; o > 0; o >>= 1) {
      uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w > v ? w : v;
    }
    return v;
  }
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  uint64_t r = scratch[0];
  for (int w = 1; w < (tm.T >> 5); w++) r = scratch[w] > r ? scratch[w] : r;
  __syncthreads();
  return r;
}


// Prep (src/trellis.rs:1144-1160, 1172-1176, src/lib.rs:472-484): load row
// vv, normalize, center (flat centroids by first maximum, or the IVF list
// centroid), rotate, standardize.  Leaves u_r in xbuf and u_rs in ubuf;
// misc[0] = |row|, misc[2] = rnorm, misc[3] = scale, misc_u[4] = cidx.
__device__ __forceinline__ void encode_row_prep(const EncodeParams &p, int64_t vv, float *xbuf,
                                                float *ubuf, float *misc, uint64_t *red,
                                                const Team &tm) {
  const int d = p.dim;
  const int T = tm.T;
  uint32_t *misc_u = (uint32_t *)misc;
  const float *row = p.rows + (p.row_index ? p.row_index[vv] : vv) * (int64_t)d;
  for (int i = tm.t; i < d; i += T) xbuf[i] = row[i];
  tm.sync();
  if (!p.rotated_input) {
    if (tm.leader()) {
      float l2 = fsqrt(seq_sum_sq(xbuf, d));
      misc[0] = l2;
      misc[1] = fmax_rs(l2, kF32Eps);
      misc[2] = 1.0f;
      misc_u[4] = 0u;
    }
    tm.sync();
    const float nrm = misc[1];
    for (int i = tm.t; i < d; i += T) xbuf[i] = fdiv(xbuf[i], nrm);
    tm.sync();
    const float *cen = nullptr;
    if (p.list_centroids != nullptr) {
      cen = p.list_centroids + (size_t)p.row_list[vv] * d;
    } else if (p.n_centroids > 0) {
      // assign (src/trellis.rs:993-1004): first strict maximum of <u, c_j>
      uint64_t best = 0;
      for (int j = tm.t; j < p.n_centroids; j += T) {
        float dj = seq_dot(xbuf, p.centroids + (size_t)j * d, d);
        uint64_t key = ((uint64_t)score_key32(dj) << 32) | (uint32_t)(~(uint32_t)j);
        best = key > best ? key : best;
      }
      best = team_max_u64(best, tm, red);
      uint32_t j = ~(uint32_t)(best & 0xffffffffu);
      // every dot NaN or -inf: the reference keeps index 0
      if ((uint32_t)(best >> 32) <= score_key32(-INFINITY)) j = 0;
      if (tm.leader()) misc_u[4] = j;
      cen = p.centroids + (size_t)j * d;
    }
    if (cen != nullptr) {
      for (int i = tm.t; i < d; i += T) xbuf[i] = fsub(xbuf[i], cen[i]);
      tm.sync();
      if (tm.leader()) misc[2] = fmax_rs(fsqrt(seq_sum_sq(xbuf, d)), kF32Eps);
      tm.sync();
      const float rn = misc[2];
      for (int i = tm.t; i < d; i += T) xbuf[i] = fdiv(xbuf[i], rn);
      tm.sync();
    }
    team_rotate(xbuf, p.rot, tm, false);
  }
  if (tm.leader()) misc[3] = fmax_rs(seq_std_about_mean(xbuf, d), kF32Eps);
  tm.sync();
  const float scale = misc[3];
  for (int i = tm.t; i < d; i += T) ubuf[i] = fdiv(xbuf[i], scale);
}

// Finalize (src/trellis.rs:1009-1133, src/lib.rs:610-627): rescale =
// sequential sum of code[w_i] * u_r[i] (leader), MSB-first packing of the
// windows' emissions (team), and the record's outputs.  wv holds the
// windows, misc_u[5] the start state.
template <int B>
__device__ __forceinline__ void encode_row_finalize(const EncodeParams &p, int64_t vv, bool valid,
                                                    const uint32_t *wv, const float *xbuf,
                                                    float *misc, const Team &tm) {
  const int d = p.dim;
  const int T = tm.T;
  uint32_t *misc_u = (uint32_t *)misc;
  if (tm.leader()) {
    float rs = 0.0f;
    for (int i = 0; i < d; i++) rs = fadd(rs, fmul(__ldg(p.code + wv[i]), xbuf[i]));
    if (p.rescale_bits > 0 && rs > 1e-6f) {
      const float levels = (float)((1u << p.rescale_bits) - 1u);
      const float sq = fsqrt((float)d);
      const float lo = fmul(0.0f, sq), hi = fmul(1.25f, sq);
      float t = fdiv(fsub(rs, lo), fsub(hi, lo));
      t = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
      rs = fadd(lo, fmul(fdiv(roundf(fmul(t, levels)), levels), fsub(hi, lo)));
    }
    misc[6] = rs > 1e-6f ? rs : INFINITY;
  }
  if (valid && p.codes != nullptr) {
    uint8_t *out = p.codes + vv * (int64_t)p.code_stride;
    const int nbits = d * B;
    for (int bi = tm.t; bi < p.code_stride; bi += T) {
      uint32_t val = 0;
      if (bi < p.code_bytes) {
#pragma unroll
        for (int bit = 0; bit < 8; bit++) {
          const int pos = bi * 8 + bit;
          if (pos < nbits) {
            const int i = pos / B;
            const int off = B - 1 - (pos - i * B);
            val |= ((wv[i] >> off) & 1u) << (7 - bit);
          }
        }
      }
      out[bi] = (uint8_t)val;
    }
  }
  if (valid && p.signs != nullptr) {
    // the shortlist's 1-bit code: pack_indices(u_r > 0, 1), MSB-first
    // (src/trellis.rs:1084-1094), zero-padded to sign_stride
    uint8_t *out = p.signs + vv * (int64_t)p.sign_stride;
    for (int bi = tm.t; bi < p.sign_stride; bi += T) {
      uint32_t val = 0;
#pragma unroll
      for (int bit = 0; bit < 8; bit++) {
        const int i = bi * 8 + bit;
        if (i < d && xbuf[i] > 0.0f) val |= 0x80u >> bit;
      }
      out[bi] = (uint8_t)val;
    }
  }
  tm.sync();
  if (valid && tm.leader()) {
    if (p.start) p.start[vv] = misc_u[5];
    if (p.rescale) p.rescale[vv] = misc[6];
    if (p.rnorm) p.rnorm[vv] = p.rotated_input ? 1.0f : misc[2];
    if (p.cidx) p.cidx[vv] = p.rotated_input ? 0u : misc_u[4];
    if (p.norms) p.norms[vv] = p.rotated_input ? 0.0f : misc[0];
  }
  tm.sync();
}

}  // namespace uvb
