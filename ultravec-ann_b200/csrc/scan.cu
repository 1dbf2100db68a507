// scan.cu -- codes-only scan of a trellis index with a fused per-query top-k,
// plus query preparation and the top-k merge.
//
// Score of query q against record r (src/trellis.rs:1483-1536, 1576-1618):
//   dot   = sum_i q_r[i] * code[w_i(r)], in the association of
//           simd::lut_dot_u32 (src/simd.rs:202-262): lane j in 0..16 keeps a
//           sequential FMA chain over the 16-wide blocks; then
//           v_j = a_j + a_{j+8}, s_j = v_j + v_{j+4}, ((s0+s1) + (s2+s3)).
//   score = qm + rnorm * (dot / rescale)          (1517)
//   mips  = score * |x_r|                          (src/bench.rs:1029-1037)
// Top-k: score descending, index ascending (the reference sorts by score with
// an unstable sort, so only exact ties can differ).
//
// Tile: a CTA of 256 threads holds TQ = 32 prepared queries (transposed in
// shared memory) and walks a contiguous range of records TN = 32 at a time.
// Each record tile is decoded once into shared memory (x-bar = code[window],
// the windows read straight from the packed bit stream) and reused by all 32
// queries, so the inner loop is an f32 decode-GEMM: thread (j, p) accumulates
// lane j of an 8x8 (query, record) sub-tile.  The 16 lanes are then combined
// by an order-preserving transpose-reduction over shuffles (xor 8, 4, 1, 2
// reproduces the reference tree exactly), the estimator and the MIPS norm are
// applied, and candidates above the query's running k-th key are appended to
// a shared-memory buffer that is merged (bitonic) into the query's top-k when
// it nears capacity.
#include "uv_kernels.h"
#include "uv_team.cuh"

namespace uvb {

// ---------------------------------------------------------------------------
// Query preparation (src/trellis.rs:2120-2136): u = q/|q| (degenerate when
// |q| < EPS), qc[j] = <u, c_j>, q_r = rotate(u).  One warp per query.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prep_queries_kernel(const PrepParams p) {
  extern __shared__ __align__(16) float smem[];
  const int team = threadIdx.x >> 5;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  float *x = smem + (size_t)team * (p.dim_pad + 4);
  float *misc = x + p.dim_pad;
  const int d = p.dim;
  const int64_t iters = (p.nq + (int64_t)gridDim.x * 8 - 1) / ((int64_t)gridDim.x * 8);
  for (int64_t it = 0; it < iters; it++) {
    const int64_t q = ((int64_t)it * gridDim.x + blockIdx.x) * 8 + team;
    const bool valid = q < p.nq;
    const int64_t qq = valid ? q : p.nq - 1;
    const float *src = p.queries + qq * (int64_t)d;
    for (int i = tm.t; i < d; i += 32) x[i] = src[i];
    tm.sync();
    if (tm.leader()) misc[0] = fsqrt(seq_sum_sq(x, d));
    tm.sync();
    const float qn = misc[0];
    const bool degenerate = !(qn >= kF32Eps);
    if (!degenerate) {
      for (int i = tm.t; i < d; i += 32) x[i] = fdiv(x[i], qn);
      tm.sync();
      for (int j = tm.t; j < p.n_centroids; j += 32) {
        float dj = seq_dot(x, p.centroids + (size_t)j * d, d);
        if (valid) p.qc[qq * p.n_centroids + j] = dj;
      }
      team_rotate(x, p.rot, tm, false);
    } else {
      for (int i = tm.t; i < d; i += 32) x[i] = 0.0f;
      for (int j = tm.t; j < p.n_centroids; j += 32)
        if (valid) p.qc[qq * p.n_centroids + j] = 0.0f;
      tm.sync();
    }
    if (valid) {
      for (int i = tm.t; i < d; i += 32) p.q_r[qq * (int64_t)p.dim_pad + i] = x[i];
      if (tm.leader()) p.degenerate[qq] = degenerate ? 1u : 0u;
    }
    tm.sync();
  }
}

// ---------------------------------------------------------------------------
// Flat scan + top-k.
// ---------------------------------------------------------------------------
constexpr int TQ = 32;       // queries per CTA
constexpr int TN = 32;       // records per tile
constexpr int QSTR = TQ + 4;  // padded row of the transposed query tile
constexpr int XSTR = TN + 4;  // padded row of the transposed record tile
constexpr int KCAP = 128;     // top-k capacity per query
constexpr int BCAP = 128;     // candidate buffer per query
constexpr int SLOTS = KCAP + BCAP;

// Bitonic sort (descending) of n = 256 keys in shared memory by one warp.
__device__ __forceinline__ void warp_sort_desc_256(uint64_t *a) {
  const int lane = threadIdx.x & 31;
  for (int size = 2; size <= SLOTS; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < SLOTS / 2; pi += 32) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int jx = i + stride;
        const bool desc = (i & size) == 0;
        const uint64_t x = a[i], y = a[jx];
        const bool swap = desc ? (x < y) : (x > y);
        if (swap) {
          a[i] = y;
          a[jx] = x;
        }
      }
      __syncwarp();
    }
  }
}

// Merge the candidate buffer of one query into its top-k (one warp).
__device__ __forceinline__ void flush_query(uint64_t *slots, int *cnt, uint64_t *theta, int k) {
  warp_sort_desc_256(slots);
  const int lane = threadIdx.x & 31;
  for (int i = KCAP + lane; i < SLOTS; i += 32) slots[i] = kEmptyKey;
  __syncwarp();
  if (lane == 0) {
    *cnt = 0;
    *theta = slots[k - 1];
  }
  __syncwarp();
}

// Read the 64 bits that start at bit `pos` of a big-endian byte image held as
// little-endian u32 words in shared memory.
__device__ __forceinline__ uint64_t read_bits64(const uint32_t *w, int pos) {
  const int wi = pos >> 5, off = pos & 31;
  const uint32_t a = __byte_perm(w[wi], 0, 0x0123);
  const uint32_t b = __byte_perm(w[wi + 1], 0, 0x0123);
  const uint32_t c = __byte_perm(w[wi + 2], 0, 0x0123);
  const uint64_t hi = ((uint64_t)a << 32) | b;
  return off ? (hi << off) | (c >> (32 - off)) : hi;
}

__global__ void __launch_bounds__(256) flat_scan_kernel(const ScanParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x;
  const int d = p.dim;
  const int W = p.mem + p.bits;
  const uint32_t wmask = (1u << W) - 1u;

  // shared-memory carve-up (all offsets 16-byte aligned)
  float *qT = (float *)sm;                                   // d x QSTR
  float *xT = qT + (size_t)d * QSTR;                         // d x XSTR
  uint64_t *slots = (uint64_t *)(xT + (size_t)d * XSTR);     // TQ x SLOTS
  uint64_t *theta = slots + (size_t)TQ * SLOTS;              // TQ
  int *cnt = (int *)(theta + TQ);                            // TQ
  float *qm_s = (float *)(cnt + TQ);                         // TQ
  uint32_t *degen = (uint32_t *)(qm_s + TQ);                 // TQ
  float *rs_s = (float *)(degen + TQ);                       // TN rescale
  float *rn_s = rs_s + TN;                                   // TN rnorm
  float *nm_s = rn_s + TN;                                   // TN norm
  uint32_t *ci_s = (uint32_t *)(nm_s + TN);                  // TN cidx
  int *flag = (int *)(ci_s + TN);                            // 4
  uint32_t *img = (uint32_t *)(flag + 4);                    // TN x img_words
  const int img_words = p.img_words;                         // per record
  float *table = (float *)(img + (size_t)TN * img_words + 4);  // code table (optional)
  const float *code = p.table_in_smem ? table : p.code;

  const int64_t q_base = (int64_t)blockIdx.x * TQ;
  const int split = blockIdx.y;
  const int64_t r_begin = p.n * split / gridDim.y;
  const int64_t r_end = p.n * (split + 1) / gridDim.y;

  // ---- load queries (transposed), per-query state, table ----
  for (int e = tid; e < TQ * d; e += 256) {
    const int qi = e / d, i = e - qi * d;
    const int64_t q = q_base + qi;
    qT[(size_t)i * QSTR + qi] = q < p.nq ? p.q_r[q * (int64_t)p.q_stride + i] : 0.0f;
  }
  for (int e = tid; e < TQ * SLOTS; e += 256) slots[e] = kEmptyKey;
  if (tid < TQ) {
    const int64_t q = q_base + tid;
    theta[tid] = kEmptyKey;
    cnt[tid] = 0;
    degen[tid] = q < p.nq ? p.degenerate[q] : 1u;
    qm_s[tid] = 0.0f;
  }
  if (p.table_in_smem)
    for (int e = tid; e < p.table_len; e += 256) table[e] = __ldg(p.code + e);
  __syncthreads();

  const int j = tid & 15;         // accumulator lane
  const int pp = tid >> 4;        // position 0..15
  const int pq = pp >> 2;         // query octet
  const int pn = pp & 3;          // record octet
  // after the reduction this thread owns queries qsel and records rsel..rsel+3
  const int qsel = pq * 8 + (((j >> 3) & 1) << 2) + (((j >> 2) & 1) << 1) + (j & 1);
  const int rsel = pn * 8 + (((j >> 1) & 1) << 2);

  const int kblocks = d >> 4;
  const int per_thread_win = d / 8;  // windows decoded per thread per tile

  for (int64_t r0 = r_begin; r0 < r_end; r0 += TN) {
    const int nr = (int)((r_end - r0) < (int64_t)TN ? (r_end - r0) : (int64_t)TN);
    // ---- stage the tile: record images (start word + codes) and scalars ----
    {
      const int rw = p.code_stride >> 2;  // code words per record
      for (int e = tid; e < TN * rw; e += 256) {
        const int r = e / rw, wi = e - r * rw;
        uint32_t val = 0;
        if (r < nr) val = __ldg((const uint32_t *)(p.codes + (r0 + r) * (int64_t)p.code_stride) + wi);
        img[r * img_words + 4 + wi] = val;
      }
      if (tid < TN) {
        const int r = tid;
        const bool ok = r < nr;
        const uint32_t st = ok ? __ldg(p.start + r0 + r) : 0u;
        img[r * img_words + 3] = __byte_perm(st, 0, 0x0123);  // big-endian start word
        img[r * img_words + 0] = 0u;
        img[r * img_words + 1] = 0u;
        img[r * img_words + 2] = 0u;
        for (int w = 4 + rw; w < img_words; w++) img[r * img_words + w] = 0u;
        rs_s[r] = ok ? __ldg(p.rescale + r0 + r) : INFINITY;
        rn_s[r] = (ok && p.rnorm) ? __ldg(p.rnorm + r0 + r) : 1.0f;
        nm_s[r] = (ok && p.norms) ? __ldg(p.norms + r0 + r) : 1.0f;
        ci_s[r] = (ok && p.cidx) ? __ldg(p.cidx + r0 + r) : 0u;
      }
    }
    __syncthreads();
    // ---- decode: x-bar[i][r] = code[window_i(r)] ----
    {
      const int r = tid & 31;
      const int c = tid >> 5;  // 8 coordinate chunks
      const uint32_t *rec = img + r * img_words;
      const int i0 = c * per_thread_win;
      // window i = image bits [128 + i*B - M, 128 + i*B + B)
      int done = 0;
      while (done < per_thread_win) {
        const int i = i0 + done;
        const int pos = 128 + i * p.bits - p.mem;
        const uint64_t bits64 = read_bits64(rec, pos);
        const int group = min(per_thread_win - done, (64 - W) / p.bits + 1);
        for (int g = 0; g < group; g++) {
          const uint32_t w = (uint32_t)(bits64 >> (64 - W - g * p.bits)) & wmask;
          xT[(size_t)(i + g) * XSTR + r] = code[w];
        }
        done += group;
      }
    }
    __syncthreads();

    // ---- decode-GEMM: acc[a][c] = lane j of dot(query a, record c) ----
    float acc[8][8];
#pragma unroll
    for (int a = 0; a < 8; a++)
#pragma unroll
      for (int c = 0; c < 8; c++) acc[a][c] = 0.0f;
    for (int b = 0; b < kblocks; b++) {
      const int coord = (b << 4) + j;
      const float4 qa = *(const float4 *)(qT + (size_t)coord * QSTR + pq * 8);
      const float4 qb = *(const float4 *)(qT + (size_t)coord * QSTR + pq * 8 + 4);
      const float4 xa = *(const float4 *)(xT + (size_t)coord * XSTR + pn * 8);
      const float4 xb = *(const float4 *)(xT + (size_t)coord * XSTR + pn * 8 + 4);
      const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
      const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
      for (int a = 0; a < 8; a++)
#pragma unroll
        for (int c = 0; c < 8; c++) acc[a][c] = fmaf(qv[a], xv[c], acc[a][c]);
    }

    // ---- order-preserving transpose-reduction over the 16 lanes ----
    // level 1 (xor 8): keep query half by bit 3 of j    -> 32 values
    float l1[4][8];
    {
      const bool hi = (j & 8) != 0;
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float keep = hi ? acc[a + 4][c] : acc[a][c];
          const float send = hi ? acc[a][c] : acc[a + 4][c];
          l1[a][c] = fadd(keep, __shfl_xor_sync(0xffffffffu, send, 8));
        }
    }
    // level 2 (xor 4): keep query pair by bit 2          -> 16 values
    float l2[2][8];
    {
      const bool hi = (j & 4) != 0;
#pragma unroll
      for (int a = 0; a < 2; a++)
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const float keep = hi ? l1[a + 2][c] : l1[a][c];
          const float send = hi ? l1[a][c] : l1[a + 2][c];
          l2[a][c] = fadd(keep, __shfl_xor_sync(0xffffffffu, send, 4));
        }
    }
    // level 3 (xor 1): keep query by bit 0               -> 8 values
    float l3[8];
    {
      const bool hi = (j & 1) != 0;
#pragma unroll
      for (int c = 0; c < 8; c++) {
        const float keep = hi ? l2[1][c] : l2[0][c];
        const float send = hi ? l2[0][c] : l2[1][c];
        l3[c] = fadd(keep, __shfl_xor_sync(0xffffffffu, send, 1));
      }
    }
    // level 4 (xor 2): keep record half by bit 1         -> 4 values
    float dot4[4];
    {
      const bool hi = (j & 2) != 0;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const float keep = hi ? l3[c + 4] : l3[c];
        const float send = hi ? l3[c] : l3[c + 4];
        dot4[c] = fadd(keep, __shfl_xor_sync(0xffffffffu, send, 2));
      }
    }

    // ---- estimator, MIPS norm, threshold test ----
    if (!degen[qsel]) {
      const uint64_t th = theta[qsel];
      const int64_t q = q_base + qsel;
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int r = rsel + c;
        if (r < nr) {
          const float qm = p.n_centroids > 0 ? p.qc[q * p.n_centroids + ci_s[r]] : 0.0f;
          float s = fadd(qm, fmul(rn_s[r], fdiv(dot4[c], rs_s[r])));
          if (p.mips) s = fmul(s, nm_s[r]);
          const uint64_t key = rank_key(s, (uint32_t)(r0 - r_begin + r));
          if (key > th) {
            const int pos = atomicAdd(&cnt[qsel], 1);
            slots[(size_t)qsel * SLOTS + KCAP + pos] = key;
          }
        }
      }
    }
    __syncthreads();
    // ---- merge buffers that are close to full ----
    {
      const int warp = tid >> 5;
      for (int qi = warp; qi < TQ; qi += 8)
        if (cnt[qi] > BCAP - TN) flush_query(slots + (size_t)qi * SLOTS, &cnt[qi], &theta[qi], p.k);
    }
    __syncthreads();
  }

  // ---- final merge and write-out of this split's top-k ----
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int qi = warp; qi < TQ; qi += 8) {
      const int64_t q = q_base + qi;
      if (cnt[qi] > 0) flush_query(slots + (size_t)qi * SLOTS, &cnt[qi], &theta[qi], p.k);
      if (q < p.nq) {
        uint32_t *ok = p.part_key + (q * gridDim.y + split) * (int64_t)p.k;
        int64_t *oid = p.part_id + (q * gridDim.y + split) * (int64_t)p.k;
        for (int i = lane; i < p.k; i += 32) {
          const uint64_t key = slots[(size_t)qi * SLOTS + i];
          if (key == kEmptyKey) {
            ok[i] = 0u;
            oid[i] = -1;
          } else {
            const uint32_t local = rank_key_index(key);
            const int64_t rec = r_begin + local;
            ok[i] = (uint32_t)(key >> 32);
            oid[i] = p.ids ? p.ids[rec] : p.id_base + rec;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Top-k merge of n_lists sorted lists per query (one warp per query).
// Elements compare by (score key desc, id asc); empty slots (id -1, key 0)
// sort last.
// ---------------------------------------------------------------------------
struct KeyId {
  uint32_t key;
  int64_t id;
};

__device__ __forceinline__ bool kid_better(const KeyId &a, const KeyId &b) {
  if (a.id < 0) return false;
  if (b.id < 0) return true;
  return a.key > b.key || (a.key == b.key && a.id < b.id);
}

__global__ void __launch_bounds__(256) merge_topk_kernel(const MergeParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * p.warps + warp;
  const int n = p.pow2;
  KeyId *a = (KeyId *)sm + (size_t)warp * n;
  if (q >= p.nq) return;  // whole warp exits together
  const int total = p.n_lists * p.k_in;
  for (int i = lane; i < n; i += 32) {
    KeyId e;
    e.key = 0u;
    e.id = -1;
    if (i < total) {
      const int64_t src = q * total + i;
      e.id = p.in_id[src];
      e.key = p.in_key ? p.in_key[src] : 0u;
      if (p.in_score) e.key = score_key32(p.in_score[src]);
      if (e.id < 0) e.key = 0u;
    }
    a[i] = e;
  }
  __syncwarp();
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < n / 2; pi += 32) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int jx = i + stride;
        const bool desc = (i & size) == 0;
        const KeyId x = a[i], y = a[jx];
        const bool swap = desc ? kid_better(y, x) : kid_better(x, y);
        if (swap) {
          a[i] = y;
          a[jx] = x;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    const KeyId e = a[i];
    p.out_id[q * p.k + i] = e.id;
    p.out_score[q * p.k + i] = e.id < 0 ? -INFINITY : key32_score(e.key);
  }
}

}  // namespace uvb

namespace uvb {

// Must match the carve-up at the top of flat_scan_kernel.
size_t scan_smem_bytes(int dim, int img_words, int table_len, bool table_in_smem) {
  size_t b = 0;
  b += (size_t)dim * QSTR * 4;
  b += (size_t)dim * XSTR * 4;
  b += (size_t)TQ * SLOTS * 8;
  b += (size_t)TQ * 8;          // theta
  b += (size_t)TQ * 4 * 3;      // cnt, qm, degenerate
  b += (size_t)TN * 4 * 4;      // rescale, rnorm, norm, cidx
  b += 16;                      // flags
  b += (size_t)TN * img_words * 4 + 16;
  if (table_in_smem) b += (size_t)table_len * 4;
  return b;
}

}  // namespace uvb
