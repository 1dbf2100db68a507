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
// |q| < EPS), qc[j] = <u, c_j>, q_r = rotate(u).  One warp per query.  With
// clamp_norm (src/coset_trellis.rs:473-476) |q| is clamped at EPS instead.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prep_queries_kernel(const PrepParams p) {
  extern __shared__ __align__(16) float smem[];
  // teams of 256 / teams threads, one query each: warps for narrow rows, the
  // whole CTA for wide ones (the FWHT stages then spread over 256 threads)
  const int teams = p.teams > 0 ? p.teams : 8;
  Team tm;
  tm.T = 256 / teams;
  tm.cta = teams == 1;
  tm.t = threadIdx.x % tm.T;
  const int team = threadIdx.x / tm.T;
  const int T = tm.T;
  float *x = smem + (size_t)team * (p.dim_pad + 4);
  float *misc = x + p.dim_pad;
  const int d = p.dim;
  const int64_t per = (int64_t)gridDim.x * teams;
  const int64_t iters = (p.nq + per - 1) / per;
  for (int64_t it = 0; it < iters; it++) {
    const int64_t qq = ((int64_t)it * gridDim.x + blockIdx.x) * teams + team;
    if (qq >= p.nq) continue;  // uniform over the team; teams never wait on each other
    const float *src = p.queries + qq * (int64_t)d;
    for (int i = tm.t; i < d; i += T) x[i] = src[i];
    tm.sync();
    if (tm.leader()) {
      const float l2 = fsqrt(seq_sum_sq(x, d));
      misc[0] = p.clamp_norm ? fmax_rs(l2, kF32Eps) : l2;
    }
    tm.sync();
    const float qn = misc[0];
    const bool degenerate = !p.clamp_norm && !(qn >= kF32Eps);
    if (!degenerate) {
      for (int i = tm.t; i < d; i += T) x[i] = fdiv(x[i], qn);
      tm.sync();
      if (p.u != nullptr)
        for (int i = tm.t; i < d; i += T) p.u[qq * (int64_t)p.dim_pad + i] = x[i];
      for (int j = tm.t; j < p.n_centroids; j += T)
        p.qc[qq * p.n_centroids + j] = seq_dot(x, p.centroids + (size_t)j * d, d);
      team_rotate(x, p.rot, tm, false);
    } else {
      for (int i = tm.t; i < d; i += T) x[i] = 0.0f;
      if (p.u != nullptr)
        for (int i = tm.t; i < d; i += T) p.u[qq * (int64_t)p.dim_pad + i] = 0.0f;
      for (int j = tm.t; j < p.n_centroids; j += T) p.qc[qq * p.n_centroids + j] = 0.0f;
      tm.sync();
    }
    for (int i = tm.t; i < d; i += T) p.q_r[qq * (int64_t)p.dim_pad + i] = x[i];
    if (tm.leader()) p.degenerate[qq] = degenerate ? 1u : 0u;
    tm.sync();
  }
}

int prep_teams(int dim) { return dim >= 512 ? 1 : 8; }

// ---------------------------------------------------------------------------
// Flat scan + top-k.
// ---------------------------------------------------------------------------
constexpr int TQ = 32;        // queries per CTA
constexpr int TN = 32;        // records per tile
constexpr int QSTR = TQ + 4;  // padded row of the transposed query tile (LDS.128)
constexpr int XSTR = TN + 4;  // padded row of the transposed record tile (LDS.128)
constexpr int KCAP = 128;     // top-k capacity per query
constexpr int BCAP = 64;      // candidate buffer per query (power of two)

// Sort N keys descending (bitonic, one warp).
template <int N>
__device__ __forceinline__ void warp_sort_desc(uint64_t *a) {
  const int lane = threadIdx.x & 31;
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < N / 2; pi += 32) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int jx = i + stride;
        const bool desc = (i & size) == 0;
        const uint64_t x = a[i], y = a[jx];
        if (desc ? (x < y) : (x > y)) {
          a[i] = y;
          a[jx] = x;
        }
      }
      __syncwarp();
    }
  }
}

// Number of keys in the descending array a[0..n) that are larger than x.
__device__ __forceinline__ int count_larger(const uint64_t *a, int n, uint64_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] > x)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Merge one query's candidate buffer into its sorted top-k list (one warp).
// Keys are unique, so every element's merged position is its own rank plus
// the number of larger keys in the other list; positions >= KC_ drop out.
template <int KC_, int BC_>
__device__ __forceinline__ void flush_query(uint64_t *top, uint64_t *buf, int *cnt, uint64_t *theta,
                                            float *theta_s, int k) {
  const int lane = threadIdx.x & 31;
  const int m = *cnt;
  for (int i = m + lane; i < BC_; i += 32) buf[i] = kEmptyKey;
  __syncwarp();
  warp_sort_desc<BC_>(buf);
  uint64_t tv[KC_ / 32], bv[BC_ / 32];
  int tp[KC_ / 32], bp[BC_ / 32];
#pragma unroll
  for (int u = 0; u < KC_ / 32; u++) {
    const int i = lane + 32 * u;
    tv[u] = top[i];
    tp[u] = i + count_larger(buf, BC_, tv[u]);
  }
#pragma unroll
  for (int u = 0; u < BC_ / 32; u++) {
    const int i = lane + 32 * u;
    bv[u] = buf[i];
    bp[u] = i + count_larger(top, KC_, bv[u]);
  }
  __syncwarp();
#pragma unroll
  for (int u = 0; u < KC_ / 32; u++)
    if (tv[u] != kEmptyKey && tp[u] < KC_) top[tp[u]] = tv[u];
#pragma unroll
  for (int u = 0; u < BC_ / 32; u++)
    if (bv[u] != kEmptyKey && bp[u] < KC_) top[bp[u]] = bv[u];
  __syncwarp();
  if (lane == 0) {
    *cnt = 0;
    const uint64_t th = top[k - 1];
    *theta = th;
    *theta_s = th == kEmptyKey ? -INFINITY : key32_score((uint32_t)(th >> 32));
  }
  __syncwarp();
}

// Per-tile record scalars in shared memory: rescale, rnorm, norm, cidx and
// the ratio g = rnorm / rescale used by the cheap pre-filter below.
constexpr int NSC = 5;

// Decode coordinates [k0, k0 + kc) of one record tile into x-bar (transposed,
// rows relative to k0) and, when `scalars` is set, stage its scalars.
// Thread (r, c) decodes windows [k0 + c*kc/8, k0 + (c+1)*kc/8) of record r in
// chunks of 16, reading the packed stream straight from global memory:
// window i is the field [i*B, i*B + M + B) of [start (M bits) || codes]
// (src/trellis.rs:1576-1600), i.e. bits [32 + i*B - M, ...) of the image whose
// first 32-bit word is the start state.  k0 is a multiple of 16.
// Coset records (src/coset_trellis.rs:414-434): [start state, ceil(mem/8)
// bytes little-endian | (2 + m)-bit symbols (branch << m | book index),
// MSB first].  Thread (r, c) decodes a contiguous range of 8-wide blocks of
// record r.  The state entering block b is fixed by the start state and the
// branches before b, of which only the last ceil(mem/2) still show, so each
// thread replays at most that many symbols before its range.  x-bar values
// come from the 32-entry table of (R/2 - mean)/std over raw coordinates R;
// coordinates from the row's width up to the padded width are zeros.
__device__ __forceinline__ uint32_t coset_sym(const uint32_t *cw, int rw, int bitpos, int W) {
  const int wi = bitpos >> 5;
  const uint32_t w0 = wi < rw ? __byte_perm(__ldg(cw + wi), 0, 0x0123) : 0u;
  const uint32_t w1 = wi + 1 < rw ? __byte_perm(__ldg(cw + wi + 1), 0, 0x0123) : 0u;
  const uint32_t top = __funnelshift_l(w1, w0, bitpos & 31);
  return top >> (32 - W);
}

__device__ __forceinline__ void decode_tile_coset(const ScanParams &p, int64_t r0, int nr,
                                                  float *xT, float *sc, int k0, int kc,
                                                  bool scalars) {
  const CosetModel &m = p.coset;
  const int tid = threadIdx.x;
  const int r = tid & 31;
  const int c = tid >> 5;
  const bool ok = r < nr;
  const int64_t rec = ok ? r0 + r : r0;
  const uint8_t *bytes = p.codes + rec * (int64_t)p.code_stride;
  const uint32_t *cw = (const uint32_t *)bytes;
  const int rw = p.code_stride >> 2;
  const int nb = m.dim >> 3;
  const int W = 2 + m.m_bits;
  const uint32_t mask = (1u << m.mem) - 1, imask = (1u << m.m_bits) - 1;
  const int L = (m.mem + 1) >> 1;
  const int sbits = 8 * m.start_bytes;
  // blocks of coordinates [k0, k0 + kc) that hold data (k0 is a multiple of 16)
  const int kb0 = k0 >> 3;
  const int kbn = max(0, min(nb, (k0 + kc) >> 3) - kb0);
  const int b0 = kb0 + c * kbn / 8, b1 = kb0 + (c + 1) * kbn / 8;
  uint32_t st = 0;
  if (b0 <= L)
    for (int i = 0; i < m.start_bytes; i++) st |= (uint32_t)__ldg(bytes + i) << (8 * i);
  for (int i = b0 > L ? b0 - L : 0; i < b0; i++)
    st = ((st << 2) | (coset_sym(cw, rw, sbits + i * W, W) >> m.m_bits)) & mask;
  for (int b = b0; b < b1; b++) {
    const uint32_t sym = coset_sym(cw, rw, sbits + b * W, W);
    const uint32_t br = sym >> m.m_bits;
    const int cs = (int)(((__popc(st) & 1) << 2) | br);
    const uint64_t key = __ldg(m.books + (size_t)cs * m.per_coset + (sym & imask));
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int i = b * 8 + j;
      const int R = (int)((key >> (5 * (7 - j))) & 31);  // R + 16
      const float v = ok ? __ldg(m.xval + R) : 0.0f;
      xT[(size_t)(i - k0) * XSTR + (r ^ (((i >> 1) & 1) << 2))] = v;
    }
    st = ((st << 2) | br) & mask;
  }
  if (c == 7)
    for (int i = max(m.dim, k0); i < k0 + kc; i++)
      xT[(size_t)(i - k0) * XSTR + (r ^ (((i >> 1) & 1) << 2))] = 0.0f;
  if (scalars && tid < TN) {
    const bool okr = tid < nr;
    const float rs = okr ? __ldg(p.rescale + r0 + tid) : INFINITY;
    const float rn = okr ? __ldg(p.rnorm + r0 + tid) : 1.0f;
    sc[tid] = rs;
    sc[TN + tid] = rn;
    sc[2 * TN + tid] = 1.0f;
    ((uint32_t *)sc)[3 * TN + tid] = (okr && p.cidx) ? __ldg(p.cidx + r0 + tid) : 0u;
    sc[4 * TN + tid] = fdiv(rn, rs);
  }
}

template <int B, bool TSMEM>
__device__ __forceinline__ void decode_tile(const ScanParams &p, const float *code, int64_t r0,
                                            int nr, float *xT, float *sc, int k0, int kc,
                                            bool scalars) {
  if constexpr (B == 0) {
    decode_tile_coset(p, r0, nr, xT, sc, k0, kc, scalars);
    return;
  }
  const int tid = threadIdx.x;
  const int W = p.mem + B;
  const int rshift = 32 - W;
  const int r = tid & 31;
  const int c = tid >> 5;
  const int per_thread = kc >> 3;
  const bool ok = r < nr;
  const int64_t rec = ok ? r0 + r : r0;
  const uint32_t *cw = (const uint32_t *)(p.codes + rec * (int64_t)p.code_stride);
  const int rw = p.code_stride >> 2;
  const uint32_t st = __ldg(p.start + rec);
  // column of record r in rows read by lanes with bit 1 clear / set
  float *col0 = xT + r;
  float *col1 = xT + (r ^ 4);
  const int end = (c + 1) * per_thread;
  for (int base = c * per_thread; base < end; base += 16) {
    const int lim = end - base;  // windows in this chunk: 16 unless kc < 128
    const int pos0 = 32 + (k0 + base) * B - p.mem;
    const int w0 = pos0 >> 5;
    uint32_t w[5];
#pragma unroll
    for (int u = 0; u < 5; u++) {
      const int wi = w0 + u;
      w[u] = wi == 0 ? st : (wi <= rw ? __byte_perm(__ldg(cw + wi - 1), 0, 0x0123) : 0u);
    }
    const int sh = pos0 & 31;
    uint32_t a[4];
#pragma unroll
    for (int u = 0; u < 4; u++) a[u] = __funnelshift_l(w[u + 1], w[u], sh);
    // row base+g is read by accumulator lane (base+g) & 15, whose record half
    // is bit 1 of that lane; base is even, so that bit is (base>>1 ^ g>>1) & 1
    const bool fb = (base >> 1) & 1;
    float *row0 = (fb ? col1 : col0) + (size_t)base * XSTR;
    float *row1 = (fb ? col0 : col1) + (size_t)base * XSTR;
#pragma unroll
    for (int g = 0; g < 16; g++) {
      const int bit = g * B;  // compile-time: word and offset of window g
      const uint32_t top = __funnelshift_l(a[(bit >> 5) + 1], a[bit >> 5], bit & 31);
      const uint32_t win = top >> rshift;
      float v = 0.0f;
      if (ok) v = TSMEM ? code[win] : __ldg(code + win);
      if (g < lim) ((g >> 1) & 1 ? row1 : row0)[g * XSTR] = v;
    }
  }
  if (scalars && tid < TN) {
    const bool okr = tid < nr;
    const float rs = okr ? __ldg(p.rescale + r0 + tid) : INFINITY;
    const float rn = (okr && p.rnorm) ? __ldg(p.rnorm + r0 + tid) : 1.0f;
    sc[tid] = rs;
    sc[TN + tid] = rn;
    sc[2 * TN + tid] = (okr && p.norms) ? __ldg(p.norms + r0 + tid) : 1.0f;
    ((uint32_t *)sc)[3 * TN + tid] = (okr && p.cidx) ? __ldg(p.cidx + r0 + tid) : 0u;
    sc[4 * TN + tid] = fdiv(rn, rs);
  }
}

template <int B, bool TSMEM>
__global__ void __launch_bounds__(256, 2) flat_scan_kernel(const ScanParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x;
  const int d = p.dim;

  // shared-memory carve-up (must match scan_smem_bytes)
  float *xT0 = (float *)sm;                                  // d x XSTR
  float *xT1 = xT0 + (size_t)d * XSTR;                       // d x XSTR
  float *qT = xT1 + (size_t)d * XSTR;                        // d x QSTR
  uint64_t *top = (uint64_t *)(qT + (((size_t)d * QSTR + 3) & ~(size_t)3));  // TQ x KCAP
  uint64_t *buf = top + (size_t)TQ * KCAP;                   // TQ x BCAP
  uint64_t *theta = buf + (size_t)TQ * BCAP;                 // TQ
  int *cnt = (int *)(theta + TQ);                            // TQ
  uint32_t *degen = (uint32_t *)(cnt + TQ);                  // TQ
  float *theta_s = (float *)(degen + TQ);                    // TQ: score of theta
  float *sc = theta_s + TQ;                                  // 2 x NSC x TN scalars
  int *flag = (int *)(sc + 2 * NSC * TN);                    // 4
  float *qtail = (float *)(flag + 4);                        // TQ x 8 tail coordinates
  float *table = qtail + TQ * 8;                             // optional code table
  const float *code = TSMEM ? table : p.code;
  // coordinates [d8, d8 + ntail) are the scalar tail (dim_data % 8 of them)
  const int d8 = p.dim_data > 0 ? (p.dim_data & ~7) : d;
  const int ntail = p.dim_data > 0 ? p.dim_data - d8 : 0;

  const int64_t q_base = (int64_t)blockIdx.x * TQ;
  const int split = blockIdx.y;
  const int64_t r_begin = p.n * split / gridDim.y;
  const int64_t r_end = p.n * (split + 1) / gridDim.y;
  const int ntiles = (int)((r_end - r_begin + TN - 1) / TN);

  for (int e = tid; e < TQ * d; e += 256) {
    const int qi = e / d, i = e - qi * d;
    const int64_t q = q_base + qi;
    // row i is read only by accumulator lane j = i & 15: store its queries
    // pre-permuted by that lane's mask (bits 3, 2, 0 of j)
    const int jm = i & 15;
    const int qm = (((jm >> 3) & 1) << 2) | (((jm >> 2) & 1) << 1) | (jm & 1);
    const bool live = q < p.nq && (B != 0 ? i < d8 : i < p.coset.dim);
    qT[(size_t)i * QSTR + (qi ^ qm)] = live ? p.q_r[q * (int64_t)p.q_stride + i] : 0.0f;
  }
  for (int e = tid; e < TQ * 8; e += 256) {
    const int qi = e >> 3, t = e & 7;
    const int64_t q = q_base + qi;
    qtail[e] = (t < ntail && q < p.nq) ? p.q_r[q * (int64_t)p.q_stride + d8 + t] : 0.0f;
  }
  for (int e = tid; e < TQ * KCAP; e += 256) top[e] = kEmptyKey;
  if (tid < TQ) {
    const int64_t q = q_base + tid;
    theta[tid] = kEmptyKey;
    theta_s[tid] = -INFINITY;
    cnt[tid] = 0;
    degen[tid] = q < p.nq ? p.degenerate[q] : 1u;
  }
  if (tid == 0) flag[0] = 0;
  if (TSMEM)
    for (int e = tid; e < p.table_len; e += 256) table[e] = __ldg(p.code + e);
  __syncthreads();
  if (ntiles > 0) {
    const int nr0 = (int)min((int64_t)TN, r_end - r_begin);
    decode_tile<B, TSMEM>(p, code, r_begin, nr0, xT0, sc, 0, d, true);
  }
  __syncthreads();

  // Thread (j, pq, pn): lane j of queries pq*8.. and records pn*8...  Shared
  // rows are stored permuted per reading lane -- queries by the lane bits
  // (j3 j2 j0), records by j1 -- so register slot a holds query a ^ qmask and
  // slot c record c ^ rhalf.  Each level of the transpose-reduction then keeps
  // the low half of its registers and sends the high half (the partner lane
  // holds the same outputs in the swapped order), with no per-lane select.
  const int j = tid & 15;
  const int pp = tid >> 4;
  const int pq = pp >> 2;
  const int pn = pp & 3;
  const int qmask = (((j >> 3) & 1) << 2) | (((j >> 2) & 1) << 1) | (j & 1);
  const int rhalf = ((j >> 1) & 1) << 2;
  const int qsel = pq * 8 + qmask;  // the query this thread finalizes
  const int rsel = pn * 8 + rhalf;  // its first record
  const int kblocks = d >> 4;

  for (int t = 0; t < ntiles; t++) {
    const int64_t r0 = r_begin + (int64_t)t * TN;
    const int nr = (int)min((int64_t)TN, r_end - r0);
    const float *xT = (t & 1) ? xT1 : xT0;
    const float *scs = sc + (t & 1) * NSC * TN;

    // ---- decode-GEMM in paired f32 FMAs: acc[a][c] = lane j, query a, records 2c,2c+1
    float2 acc[8][4];
#pragma unroll
    for (int a = 0; a < 8; a++)
#pragma unroll
      for (int c = 0; c < 4; c++) acc[a][c] = make_float2(0.0f, 0.0f);
#pragma unroll 2
    for (int b = 0; b < kblocks; b++) {
      const int coord = (b << 4) + j;
      const float *qrow = qT + (size_t)coord * QSTR + pq * 8;
      const float *xrow = xT + (size_t)coord * XSTR + pn * 8;
      const float4 x0 = *(const float4 *)(xrow);
      const float4 x1 = *(const float4 *)(xrow + 4);
      const float4 q0 = *(const float4 *)(qrow);
      const float4 q1 = *(const float4 *)(qrow + 4);
      const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      const float2 xv[4] = {make_float2(x0.x, x0.y), make_float2(x0.z, x0.w),
                            make_float2(x1.x, x1.y), make_float2(x1.z, x1.w)};
#pragma unroll
      for (int a = 0; a < 8; a++) {
        const float2 q2 = make_float2(qv[a], qv[a]);
#pragma unroll
        for (int c = 0; c < 4; c++) acc[a][c] = __ffma2_rn(q2, xv[c], acc[a][c]);
      }
    }

    // ---- transpose-reduction: xor 8, 4, 1 over queries, xor 2 over records.
    // The additions pair lanes (j, j^8), (j, j^4), (j, j^1), (j, j^2):
    // v_j = a_j + a_{j+8}, s_j = v_j + v_{j+4}, (s0+s1), (s2+s3), total --
    // exactly the hsum256 tree of src/simd.rs:251-262.
    float2 l1[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float2 o;
        o.x = __shfl_xor_sync(0xffffffffu, acc[a + 4][c].x, 8);
        o.y = __shfl_xor_sync(0xffffffffu, acc[a + 4][c].y, 8);
        l1[a][c] = __fadd2_rn(acc[a][c], o);
      }
    float2 l2[2][4];
#pragma unroll
    for (int a = 0; a < 2; a++)
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float2 o;
        o.x = __shfl_xor_sync(0xffffffffu, l1[a + 2][c].x, 4);
        o.y = __shfl_xor_sync(0xffffffffu, l1[a + 2][c].y, 4);
        l2[a][c] = __fadd2_rn(l1[a][c], o);
      }
    float2 l3[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
      float2 o;
      o.x = __shfl_xor_sync(0xffffffffu, l2[1][c].x, 1);
      o.y = __shfl_xor_sync(0xffffffffu, l2[1][c].y, 1);
      l3[c] = __fadd2_rn(l2[0][c], o);
    }
    float2 dot2[2];
#pragma unroll
    for (int c = 0; c < 2; c++) {
      float2 o;
      o.x = __shfl_xor_sync(0xffffffffu, l3[c + 2].x, 2);
      o.y = __shfl_xor_sync(0xffffffffu, l3[c + 2].y, 2);
      dot2[c] = __fadd2_rn(l3[c], o);
    }
    float dot4[4] = {dot2[0].x, dot2[0].y, dot2[1].x, dot2[1].y};
    // scalar tail (src/simd.rs:240-243): total += q[i] * book[idx[i]], in order
    for (int t2 = 0; t2 < ntail; t2++) {
      const int i = d8 + t2;
      const float qv = qtail[qsel * 8 + t2];
      const float *xr = xT + (size_t)i * XSTR;
      const int sw = ((i >> 1) & 1) << 2;
#pragma unroll
      for (int c = 0; c < 4; c++) dot4[c] = fadd(dot4[c], fmul(qv, xr[(rsel + c) ^ sw]));
    }

    // ---- estimator (src/trellis.rs:1517), MIPS norm, threshold test ----
    // A cheap bound first: a = qm + dot*(rnorm/rescale) (x norm) differs from
    // the exact score by at most a few roundings (< 5e-7 of its magnitude), so
    // records below theta - 1e-6*|magnitude| cannot enter the top-k and skip
    // the exact IEEE division.  Survivors get the exact score and key.
    if (!degen[qsel]) {
      const uint64_t th = theta[qsel];
      const float ths = theta_s[qsel];
      const int64_t q = q_base + qsel;
      const uint32_t *cis = (const uint32_t *)(scs + 3 * TN);
#pragma unroll
      for (int c = 0; c < 4; c++) {
        const int r = rsel + c;
        const float qm = p.n_centroids > 0 ? p.qc[q * p.n_centroids + cis[r]] : 0.0f;
        const float tt = fmul(dot4[c], scs[4 * TN + r]);
        float a = fadd(qm, tt);
        float mag = fadd(fabsf(qm), fabsf(tt));
        if (p.mips) {
          a = fmul(a, scs[2 * TN + r]);
          mag = fmul(mag, scs[2 * TN + r]);
        }
        const bool maybe = !(a < fsub(fsub(ths, fmul(1e-6f, mag)), 1e-30f));
        if (maybe && r < nr) {
          float sx = fadd(qm, fmul(scs[TN + r], fdiv(dot4[c], scs[r])));
          if (p.mips) sx = fmul(sx, scs[2 * TN + r]);
          if (p.all_key != nullptr) {
            const int64_t rec = r0 + r;
            p.all_key[q * p.n + rec] = score_key32(sx);
            p.all_id[q * p.n + rec] = p.ids ? p.ids[rec] : p.id_base + rec;
          } else {
            const uint64_t key = rank_key(sx, (uint32_t)(r0 - r_begin + r));
            if (key > th) {
              const int pos = atomicAdd(&cnt[qsel], 1);
              buf[(size_t)qsel * BCAP + pos] = key;
              if (pos == BCAP - TN) flag[0] = t + 1;
            }
          }
        }
      }
    }

    // ---- decode the next tile into the other buffer ----
    if (t + 1 < ntiles) {
      const int64_t rn0 = r0 + TN;
      const int nrn = (int)min((int64_t)TN, r_end - rn0);
      float *xn = (t & 1) ? xT0 : xT1;
      float *scn = sc + ((t + 1) & 1) * NSC * TN;
      decode_tile<B, TSMEM>(p, code, rn0, nrn, xn, scn, 0, d, true);
    }
    __syncthreads();

    // ---- merge candidate buffers that could overflow on the next tile ----
    if (flag[0] == t + 1) {
      const int warp = tid >> 5;
      for (int qi = warp; qi < TQ; qi += 8)
        if (cnt[qi] > BCAP - TN)
          flush_query<KCAP, BCAP>(top + (size_t)qi * KCAP, buf + (size_t)qi * BCAP, &cnt[qi], &theta[qi],
                      &theta_s[qi], p.k);
      __syncthreads();
    }
  }

  // ---- final merge and write-out of this split's top-k ----
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int qi = warp; qi < TQ; qi += 8) {
      const int64_t q = q_base + qi;
      if (cnt[qi] > 0)
        flush_query<KCAP, BCAP>(top + (size_t)qi * KCAP, buf + (size_t)qi * BCAP, &cnt[qi], &theta[qi],
                    &theta_s[qi], p.k);
      if (q < p.nq && p.part_key != nullptr) {
        uint32_t *ok = p.part_key + (q * gridDim.y + split) * (int64_t)p.k;
        int64_t *oid = p.part_id + (q * gridDim.y + split) * (int64_t)p.k;
        for (int i = lane; i < p.k; i += 32) {
          const uint64_t key = top[(size_t)qi * KCAP + i];
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

// The flat scan over coset records: p.dim is the row width rounded up to 16
// (the zero lanes of a last 8-wide block add exact zeros, which is how
// simd::dot's 8-wide tail into the first accumulator comes out).
const void *coset_scan_kernel_ptr() { return (const void *)flat_scan_kernel<0, false>; }

const void *flat_scan_kernel_ptr(int bits, bool table_in_smem) {
#define UV_SCAN_CASE(b)                                                                   \
  case b:                                                                                 \
    return table_in_smem ? (const void *)flat_scan_kernel<b, true>                        \
                         : (const void *)flat_scan_kernel<b, false>;
  switch (bits) {
    UV_SCAN_CASE(1)
    UV_SCAN_CASE(2)
    UV_SCAN_CASE(3)
    UV_SCAN_CASE(4)
  }
#undef UV_SCAN_CASE
  return nullptr;
}

// ---------------------------------------------------------------------------
// K-chunked scan: the same tile computation as flat_scan_kernel for rows
// wider than the query tile can hold in shared memory, and for IVF lists.
// Coordinates are processed in chunks of KCH = 128: for each (record tile,
// chunk) step the query chunk and the decoded record chunk are staged in one
// buffer while the previous step's buffer feeds the FMAs, with one barrier
// per step.  The 16-lane accumulators persist across chunks, so the FMA order
// per lane is still ascending blocks -- the same association.
// ---------------------------------------------------------------------------
constexpr int KCH = kScanKChunk;

template <int KC_, int BC_>
struct ChunkLayout {
  static constexpr size_t xT = 0;                                   // 2 x KCH x XSTR f32
  static constexpr size_t qT = xT + 2 * KCH * XSTR * 4;             // 2 x KCH x QSTR f32
  static constexpr size_t top = qT + 2 * KCH * QSTR * 4;            // TQ x KC_ u64
  static constexpr size_t buf = top + TQ * KC_ * 8;                 // TQ x BC_ u64
  static constexpr size_t theta = buf + TQ * BC_ * 8;               // TQ u64
  static constexpr size_t qrow = theta + TQ * 8;                    // TQ i64 (query row)
  static constexpr size_t slot = qrow + TQ * 8;                     // TQ i64 (output slot)
  static constexpr size_t theta_s = slot + TQ * 8;                  // TQ f32
  static constexpr size_t qm = theta_s + TQ * 4;                    // TQ f32
  static constexpr size_t cnt = qm + TQ * 4;                        // TQ i32
  static constexpr size_t degen = cnt + TQ * 4;                     // TQ u32
  static constexpr size_t sc = degen + TQ * 4;                      // 2 x NSC x TN f32
  static constexpr size_t flag = sc + 2 * NSC * TN * 4;             // 4 i32
  static constexpr size_t qtail = flag + 16;                        // TQ x 8 f32
  static constexpr size_t table = qtail + TQ * 8 * 4;
};

template <int B, bool TSMEM, int KC_, int BC_>
__global__ void __launch_bounds__(256, 2) chunked_scan_kernel(const ScanParams p, const ScanWork w) {
  using L = ChunkLayout<KC_, BC_>;
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x;
  const int d = p.dim;
  float *const xT0 = (float *)(sm + L::xT);
  float *const xT1 = xT0 + KCH * XSTR;
  float *const qT0 = (float *)(sm + L::qT);
  float *const qT1 = qT0 + KCH * QSTR;
  uint64_t *top = (uint64_t *)(sm + L::top);
  uint64_t *buf = (uint64_t *)(sm + L::buf);
  uint64_t *theta = (uint64_t *)(sm + L::theta);
  int64_t *qrow = (int64_t *)(sm + L::qrow);
  int64_t *slot = (int64_t *)(sm + L::slot);
  float *theta_s = (float *)(sm + L::theta_s);
  float *qm_s = (float *)(sm + L::qm);
  int *cnt = (int *)(sm + L::cnt);
  uint32_t *degen = (uint32_t *)(sm + L::degen);
  float *sc = (float *)(sm + L::sc);
  int *flag = (int *)(sm + L::flag);
  float *qtail = (float *)(sm + L::qtail);
  float *table = (float *)(sm + L::table);
  const float *code = TSMEM ? table : p.code;
  // coordinates [d8, d8 + ntail) are the scalar tail (dim_data % 8 of them)
  const int d8 = p.dim_data > 0 ? (p.dim_data & ~7) : d;
  const int ntail = p.dim_data > 0 ? p.dim_data - d8 : 0;

  // ---- this CTA's work: record range and up to 32 (query, slot) pairs ----
  int64_t r_begin, r_end;
  int nql;
  if (!w.ivf) {
    const int64_t q_base = (int64_t)blockIdx.x * TQ;
    const int split = blockIdx.y;
    r_begin = p.n * split / gridDim.y;
    r_end = p.n * (split + 1) / gridDim.y;
    nql = (int)min((int64_t)TQ, p.nq - q_base);
    if (tid < TQ) {
      const int64_t q = q_base + tid;
      qrow[tid] = tid < nql ? q : -1;
      slot[tid] = tid < nql ? q * gridDim.y + split : -1;
      qm_s[tid] = 0.0f;
    }
  } else {
    const int item = blockIdx.x;
    if (item >= w.n_items[0]) return;  // before any barrier: the whole CTA leaves
    const int list = w.item_list[item];
    const int pair0 = w.item_pair[item];
    const int range = w.item_range[item];
    nql = w.item_npairs[item];
    const int64_t lo = w.list_off[list], hi = w.list_off[list + 1];
    const int64_t nr = hi - lo <= w.range_size ? 1 : (hi - lo + w.range_size - 1) / w.range_size;
    r_begin = min(hi, lo + (int64_t)range * w.range_size);
    r_end = min(hi, r_begin + w.range_size);
    if (tid < TQ) {
      // output slot: this pair's block of nr range slots, entry `range`
      const int64_t pl = (int64_t)(pair0 + tid) - w.list_pair_off[list];
      qrow[tid] = tid < nql ? (int64_t)w.pair_query[pair0 + tid] : -1;
      slot[tid] = tid < nql ? w.list_rbase[list] + pl * nr + range : -1;
      qm_s[tid] = (tid < nql && w.pair_qm) ? w.pair_qm[pair0 + tid] : 0.0f;
    }
  }
  for (int e = tid; e < TQ * KC_; e += 256) top[e] = kEmptyKey;
  if (tid < TQ) {
    theta[tid] = kEmptyKey;
    theta_s[tid] = -INFINITY;
    cnt[tid] = 0;
  }
  if (tid == 0) flag[0] = 0;
  if (TSMEM)
    for (int e = tid; e < p.table_len; e += 256) table[e] = __ldg(p.code + e);
  __syncthreads();
  if (tid < TQ) degen[tid] = qrow[tid] >= 0 ? p.degenerate[qrow[tid]] : 1u;
  for (int e = tid; e < TQ * 8; e += 256) {
    const int qi = e >> 3, t = e & 7;
    const int64_t q = qrow[qi];
    qtail[e] = (t < ntail && q >= 0) ? __ldg(p.q_r + q * (int64_t)p.q_stride + d8 + t) : 0.0f;
  }

  const int nchunks = (d + KCH - 1) / KCH;
  const int ntiles = (int)((r_end - r_begin + TN - 1) / TN);
  const int64_t steps = (int64_t)ntiles * nchunks;

  // stage the query chunk [k0, k0 + kc) pre-permuted per reading lane
  auto load_q = [&](float *qT, int k0, int kc) {
    for (int e = tid; e < TQ * kc; e += 256) {
      const int qi = e / kc, i = e - qi * kc;
      const int jm = i & 15;
      const int qmk = (((jm >> 3) & 1) << 2) | (((jm >> 2) & 1) << 1) | (jm & 1);
      const int64_t q = qrow[qi];
      qT[(size_t)i * QSTR + (qi ^ qmk)] =
          (q >= 0 && k0 + i < d8) ? __ldg(p.q_r + q * (int64_t)p.q_stride + k0 + i) : 0.0f;
    }
  };
  if (steps > 0) {
    __syncthreads();  // qrow visible
    const int kc0 = min(KCH, d);
    load_q(qT0, 0, kc0);
    decode_tile<B, TSMEM>(p, code, r_begin, (int)min((int64_t)TN, r_end - r_begin), xT0, sc, 0,
                          kc0, true);
  }
  __syncthreads();

  const int j = tid & 15;
  const int pp = tid >> 4;
  const int pq = pp >> 2;
  const int pn = pp & 3;
  const int qmask = (((j >> 3) & 1) << 2) | (((j >> 2) & 1) << 1) | (j & 1);
  const int rhalf = ((j >> 1) & 1) << 2;
  const int qsel = pq * 8 + qmask;
  const int rsel = pn * 8 + rhalf;

  float2 acc[8][4];
  for (int64_t s = 0; s < steps; s++) {
    const int tile = (int)(s / nchunks);
    const int ch = (int)(s - (int64_t)tile * nchunks);
    const int bsel = (int)(s & 1);
    const int64_t r0 = r_begin + (int64_t)tile * TN;
    const int nr = (int)min((int64_t)TN, r_end - r0);
    const int kc = min(KCH, d - ch * KCH);
    if (ch == 0) {
#pragma unroll
      for (int a = 0; a < 8; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) acc[a][c] = make_float2(0.0f, 0.0f);
    }
    {
      const float *xT = bsel ? xT1 : xT0;
      const float *qT = bsel ? qT1 : qT0;
      const int kb = kc >> 4;
#pragma unroll 2
      for (int b = 0; b < kb; b++) {
        const int coord = (b << 4) + j;
        const float *qr = qT + (size_t)coord * QSTR + pq * 8;
        const float *xr = xT + (size_t)coord * XSTR + pn * 8;
        const float4 x0 = *(const float4 *)(xr);
        const float4 x1 = *(const float4 *)(xr + 4);
        const float4 q0 = *(const float4 *)(qr);
        const float4 q1 = *(const float4 *)(qr + 4);
        const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const float2 xv[4] = {make_float2(x0.x, x0.y), make_float2(x0.z, x0.w),
                              make_float2(x1.x, x1.y), make_float2(x1.z, x1.w)};
#pragma unroll
        for (int a = 0; a < 8; a++) {
          const float2 q2 = make_float2(qv[a], qv[a]);
#pragma unroll
          for (int c = 0; c < 4; c++) acc[a][c] = __ffma2_rn(q2, xv[c], acc[a][c]);
        }
      }
    }
    if (ch == nchunks - 1) {
      // transpose-reduction (xor 8, 4, 1, 2) -- see flat_scan_kernel
      float2 l1[4][4];
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          float2 o;
          o.x = __shfl_xor_sync(0xffffffffu, acc[a + 4][c].x, 8);
          o.y = __shfl_xor_sync(0xffffffffu, acc[a + 4][c].y, 8);
          l1[a][c] = __fadd2_rn(acc[a][c], o);
        }
      float2 l2[2][4];
#pragma unroll
      for (int a = 0; a < 2; a++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          float2 o;
          o.x = __shfl_xor_sync(0xffffffffu, l1[a + 2][c].x, 4);
          o.y = __shfl_xor_sync(0xffffffffu, l1[a + 2][c].y, 4);
          l2[a][c] = __fadd2_rn(l1[a][c], o);
        }
      float2 l3[4];
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float2 o;
        o.x = __shfl_xor_sync(0xffffffffu, l2[1][c].x, 1);
        o.y = __shfl_xor_sync(0xffffffffu, l2[1][c].y, 1);
        l3[c] = __fadd2_rn(l2[0][c], o);
      }
      float2 dot2[2];
#pragma unroll
      for (int c = 0; c < 2; c++) {
        float2 o;
        o.x = __shfl_xor_sync(0xffffffffu, l3[c + 2].x, 2);
        o.y = __shfl_xor_sync(0xffffffffu, l3[c + 2].y, 2);
        dot2[c] = __fadd2_rn(l3[c], o);
      }
      float dot4[4] = {dot2[0].x, dot2[0].y, dot2[1].x, dot2[1].y};
      // scalar tail (src/simd.rs:240-243), rows of this last chunk
      for (int t2 = 0; t2 < ntail; t2++) {
        const int i = d8 + t2;
        const float qv = qtail[qsel * 8 + t2];
        const float *xr = (bsel ? xT1 : xT0) + (size_t)(i - ch * KCH) * XSTR;
        const int sw = ((i >> 1) & 1) << 2;
#pragma unroll
        for (int c = 0; c < 4; c++) dot4[c] = fadd(dot4[c], fmul(qv, xr[(rsel + c) ^ sw]));
      }
      const float *scs = sc + (tile & 1) * NSC * TN;
      if (!degen[qsel]) {
        const uint64_t th = theta[qsel];
        const float ths = theta_s[qsel];
        const int64_t q = qrow[qsel];
        const uint32_t *cis = (const uint32_t *)(scs + 3 * TN);
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int r = rsel + c;
          const float qm = w.ivf ? qm_s[qsel]
                                 : (p.n_centroids > 0 ? p.qc[q * p.n_centroids + cis[r]] : 0.0f);
          const float tt = fmul(dot4[c], scs[4 * TN + r]);
          float a = fadd(qm, tt);
          float mag = fadd(fabsf(qm), fabsf(tt));
          if (p.mips) {
            a = fmul(a, scs[2 * TN + r]);
            mag = fmul(mag, scs[2 * TN + r]);
          }
          const bool maybe = !(a < fsub(fsub(ths, fmul(1e-6f, mag)), 1e-30f));
          if (maybe && r < nr) {
            float sx = fadd(qm, fmul(scs[TN + r], fdiv(dot4[c], scs[r])));
            if (p.mips) sx = fmul(sx, scs[2 * TN + r]);
            if (p.all_key != nullptr) {
              const int64_t rec = r0 + r;
              p.all_key[q * p.n + rec] = score_key32(sx);
              p.all_id[q * p.n + rec] = p.ids ? p.ids[rec] : p.id_base + rec;
            } else {
              const uint64_t key = rank_key(sx, (uint32_t)(r0 - r_begin + r));
              if (key > th) {
                const int pos = atomicAdd(&cnt[qsel], 1);
                buf[(size_t)qsel * BC_ + pos] = key;
                if (pos == BC_ - TN) flag[0] = tile + 1;
              }
            }
          }
        }
      }
    }
    // ---- stage the next step into the other buffer ----
    if (s + 1 < steps) {
      const int64_t sn = s + 1;
      const int tn = (int)(sn / nchunks);
      const int chn = (int)(sn - (int64_t)tn * nchunks);
      const int64_t rn0 = r_begin + (int64_t)tn * TN;
      const int kcn = min(KCH, d - chn * KCH);
      load_q(bsel ? qT0 : qT1, chn * KCH, kcn);
      decode_tile<B, TSMEM>(p, code, rn0, (int)min((int64_t)TN, r_end - rn0), bsel ? xT0 : xT1,
                            sc + (tn & 1) * NSC * TN, chn * KCH, kcn, chn == 0);
    }
    __syncthreads();
    if (ch == nchunks - 1 && flag[0] == tile + 1) {
      const int warp = tid >> 5;
      for (int qi = warp; qi < TQ; qi += 8)
        if (cnt[qi] > BC_ - TN)
          flush_query<KC_, BC_>(top + (size_t)qi * KC_, buf + (size_t)qi * BC_, &cnt[qi],
                                &theta[qi], &theta_s[qi], p.k);
      __syncthreads();
    }
  }

  // ---- final merge and write-out ----
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int qi = warp; qi < TQ; qi += 8) {
      if (cnt[qi] > 0)
        flush_query<KC_, BC_>(top + (size_t)qi * KC_, buf + (size_t)qi * BC_, &cnt[qi],
                              &theta[qi], &theta_s[qi], p.k);
      const int64_t sl = slot[qi];
      if (sl >= 0 && p.part_key != nullptr) {
        uint32_t *ok = p.part_key + sl * (int64_t)p.k;
        int64_t *oid = p.part_id + sl * (int64_t)p.k;
        for (int i = lane; i < p.k; i += 32) {
          const uint64_t key = top[(size_t)qi * KC_ + i];
          if (key == kEmptyKey) {
            ok[i] = 0u;
            oid[i] = -1;
          } else {
            const int64_t rec = r_begin + rank_key_index(key);
            ok[i] = (uint32_t)(key >> 32);
            oid[i] = p.ids ? p.ids[rec] : p.id_base + rec;
          }
        }
      }
    }
  }
}

const void *chunked_scan_kernel_ptr(int bits, bool table_in_smem, bool small_k) {
#define UV_CH_CASE(b)                                                                      \
  case b:                                                                                  \
    if (small_k)                                                                           \
      return table_in_smem ? (const void *)chunked_scan_kernel<b, true, 32, 32>            \
                           : (const void *)chunked_scan_kernel<b, false, 32, 32>;          \
    return table_in_smem ? (const void *)chunked_scan_kernel<b, true, 128, 64>             \
                         : (const void *)chunked_scan_kernel<b, false, 128, 64>;
  switch (bits) {
    case 0:  // coset records (decode_tile_coset); no code table
      return small_k ? (const void *)chunked_scan_kernel<0, false, 32, 32>
                     : (const void *)chunked_scan_kernel<0, false, 128, 64>;
    UV_CH_CASE(1)
    UV_CH_CASE(2)
    UV_CH_CASE(3)
    UV_CH_CASE(4)
  }
#undef UV_CH_CASE
  return nullptr;
}

size_t chunked_scan_smem_bytes(int table_len, bool table_in_smem, bool small_k) {
  const size_t base = small_k ? ChunkLayout<32, 32>::table : ChunkLayout<128, 64>::table;
  return base + (table_in_smem ? (size_t)table_len * 4 : 0);
}

// ---------------------------------------------------------------------------
// Top-k merge of n_lists sorted lists per query (one warp per query).
// Elements compare by (score key desc, id asc); empty slots (id < 0) sort
// last.  The lists are already sorted, so an element's place in the merged
// order is its index in its own list plus, for every other list, the number
// of that list's elements that precede it (a binary search; equal elements
// of lower lists precede) -- a k-way merge with no data-dependent loop.
// Only the first min(k_in, k) elements of each list can land in the top k.
// A list that is not sorted by (key, id) -- producers that break exact score
// ties by record position with ids not increasing in position -- sends its
// query to a bitonic sort of all entries instead.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool kid_better(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
  if (ia < 0) return false;
  if (ib < 0) return true;
  return ka > kb || (ka == kb && ia < ib);
}

__global__ void __launch_bounds__(256) merge_topk_kernel(const MergeParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * p.warps + warp;
  int64_t *ids = (int64_t *)sm + (size_t)warp * p.pow2;
  uint32_t *keys = (uint32_t *)((int64_t *)sm + (size_t)p.warps * p.pow2) + (size_t)warp * p.pow2;
  if (q >= p.nq) return;  // whole warp exits together
  // fixed rows: n_lists lists per query; ragged rows: lists [row_off[q], row_off[q+1])
  const int64_t list_stride = p.list_stride > 0 ? p.list_stride : p.k_in;
  const int64_t row_stride = p.row_stride > 0 ? p.row_stride : (int64_t)p.n_lists * p.k_in;
  const int64_t first = p.row_off ? p.row_off[q] * p.k_in : q * row_stride;
  const int nl = p.row_off ? (int)(p.row_off[q + 1] - p.row_off[q]) : p.n_lists;
  const int total = nl * p.k_in;
  const int64_t orow = p.out_row ? (int64_t)p.out_row[q] : q;
  int n = 32;
  while (n < total) n <<= 1;
  bool unsorted = false;
  for (int i = lane; i < n; i += 32) {
    uint32_t key = 0u;
    int64_t id = -1;
    if (i < total) {
      const int l = i / p.k_in, j = i - l * p.k_in;
      const int64_t src = p.row_off ? first + i : first + l * list_stride + j;
      if (p.in_packed) {
        const int32_t *e = p.in_packed + 3 * src;
        id = (int64_t)(((uint64_t)(uint32_t)e[1] << 32) | (uint32_t)e[0]);
        key = score_key32(__int_as_float(e[2]));
      } else {
        id = p.in_id[src];
        key = p.in_key ? p.in_key[src] : 0u;
        if (p.in_score) key = score_key32(p.in_score[src]);
      }
      if (id < 0) key = 0u;
    }
    ids[i] = id;
    keys[i] = key;
  }
  __syncwarp();
  for (int i = lane; i < total; i += 32) {
    const int j = i % p.k_in;
    if (j > 0 && kid_better(keys[i], ids[i], keys[i - 1], ids[i - 1])) unsorted = true;
  }
  unsorted = __any_sync(0xffffffffu, unsorted);
  if (!unsorted) {
    // k-way merge by ranks: at most k entries of each list are placed
    const int kk = min(p.k_in, p.k);
    for (int e = lane; e < nl * kk; e += 32) {
      const int l = e / kk, j = e - l * kk;
      const int i = l * p.k_in + j;
      const int64_t id = ids[i];
      if (id < 0) continue;
      const uint32_t key = keys[i];
      int rank = j;
      for (int l2 = 0; l2 < nl && rank < p.k; l2++) {
        if (l2 == l) continue;
        // elements of list l2 before this one: better, or equal and l2 < l
        const uint32_t *kl = keys + l2 * p.k_in;
        const int64_t *il = ids + l2 * p.k_in;
        int lo = 0, hi = min(p.k_in, p.k);
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          const bool before = kid_better(kl[mid], il[mid], key, id) ||
                              (l2 < l && il[mid] >= 0 && kl[mid] == key && il[mid] == id);
          if (before)
            lo = mid + 1;
          else
            hi = mid;
        }
        rank += lo;
      }
      if (rank < p.k) {
        p.out_id[orow * p.k + rank] = id;
        p.out_score[orow * p.k + rank] = key32_score(key);
      }
    }
    // slots past the valid entries stay unfilled
    int valid = 0;
    for (int i = lane; i < total; i += 32) valid += ids[i] >= 0 && (i % p.k_in) < p.k ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) valid += __shfl_xor_sync(0xffffffffu, valid, o);
    for (int i = valid + lane; i < p.k; i += 32) {
      p.out_id[orow * p.k + i] = -1;
      p.out_score[orow * p.k + i] = -INFINITY;
    }
    return;
  }
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < n / 2; pi += 32) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int jx = i + stride;
        const bool desc = (i & size) == 0;
        const uint32_t ka = keys[i], kb = keys[jx];
        const int64_t ia = ids[i], ib = ids[jx];
        const bool swap = desc ? kid_better(kb, ib, ka, ia) : kid_better(ka, ia, kb, ib);
        if (swap) {
          keys[i] = kb;
          keys[jx] = ka;
          ids[i] = ib;
          ids[jx] = ia;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    const bool ok = i < n && ids[i] >= 0;
    p.out_id[orow * p.k + i] = ok ? ids[i] : -1;
    p.out_score[orow * p.k + i] = ok ? key32_score(keys[i]) : -INFINITY;
  }
}

// The same merge with one CTA per row, for rows of many entries (several
// hundred): the rank searches of a row spread over all 256 threads, so a
// row's latency is a few binary searches per thread instead of a warp's
// dozens.  Same entry order, tie rule and fallback.
__global__ void __launch_bounds__(256) merge_topk_block_kernel(const MergeParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x;
  const int64_t q = blockIdx.x;
  int64_t *ids = (int64_t *)sm;
  uint32_t *keys = (uint32_t *)(ids + p.pow2);
  __shared__ int valid_s;
  if (q >= p.nq) return;  // the whole CTA
  const int64_t list_stride = p.list_stride > 0 ? p.list_stride : p.k_in;
  const int64_t row_stride = p.row_stride > 0 ? p.row_stride : (int64_t)p.n_lists * p.k_in;
  const int64_t first = p.row_off ? p.row_off[q] * p.k_in : q * row_stride;
  const int nl = p.row_off ? (int)(p.row_off[q + 1] - p.row_off[q]) : p.n_lists;
  const int total = nl * p.k_in;
  const int64_t orow = p.out_row ? (int64_t)p.out_row[q] : q;
  int n = 32;
  while (n < total) n <<= 1;
  if (tid == 0) valid_s = 0;
  for (int i = tid; i < n; i += 256) {
    uint32_t key = 0u;
    int64_t id = -1;
    if (i < total) {
      const int l = i / p.k_in, j = i - l * p.k_in;
      const int64_t src = p.row_off ? first + i : first + l * list_stride + j;
      if (p.in_packed) {
        const int32_t *e = p.in_packed + 3 * src;
        id = (int64_t)(((uint64_t)(uint32_t)e[1] << 32) | (uint32_t)e[0]);
        key = score_key32(__int_as_float(e[2]));
      } else {
        id = p.in_id[src];
        key = p.in_key ? p.in_key[src] : 0u;
        if (p.in_score) key = score_key32(p.in_score[src]);
      }
      if (id < 0) key = 0u;
    }
    ids[i] = id;
    keys[i] = key;
  }
  __syncthreads();
  bool unsorted = false;
  int valid = 0;
  for (int i = tid; i < total; i += 256) {
    const int j = i % p.k_in;
    if (j > 0 && kid_better(keys[i], ids[i], keys[i - 1], ids[i - 1])) unsorted = true;
    valid += ids[i] >= 0 && j < p.k ? 1 : 0;
  }
  if (__syncthreads_or(unsorted ? 1 : 0) == 0) {
    atomicAdd(&valid_s, valid);
    const int kk = min(p.k_in, p.k);
    for (int e = tid; e < nl * kk; e += 256) {
      const int l = e / kk, j = e - l * kk;
      const int i = l * p.k_in + j;
      const int64_t id = ids[i];
      if (id < 0) continue;
      const uint32_t key = keys[i];
      int rank = j;
      for (int l2 = 0; l2 < nl && rank < p.k; l2++) {
        if (l2 == l) continue;
        const uint32_t *kl = keys + l2 * p.k_in;
        const int64_t *il = ids + l2 * p.k_in;
        int lo = 0, hi = min(p.k_in, p.k);
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          const bool before = kid_better(kl[mid], il[mid], key, id) ||
                              (l2 < l && il[mid] >= 0 && kl[mid] == key && il[mid] == id);
          if (before)
            lo = mid + 1;
          else
            hi = mid;
        }
        rank += lo;
      }
      if (rank < p.k) {
        p.out_id[orow * p.k + rank] = id;
        p.out_score[orow * p.k + rank] = key32_score(key);
      }
    }
    __syncthreads();
    for (int i = valid_s + tid; i < p.k; i += 256) {
      p.out_id[orow * p.k + i] = -1;
      p.out_score[orow * p.k + i] = -INFINITY;
    }
    return;
  }
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = tid; pi < n / 2; pi += 256) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int jx = i + stride;
        const bool desc = (i & size) == 0;
        const uint32_t ka = keys[i], kb = keys[jx];
        const int64_t ia = ids[i], ib = ids[jx];
        const bool swap = desc ? kid_better(kb, ib, ka, ia) : kid_better(ka, ia, kb, ib);
        if (swap) {
          keys[i] = kb;
          keys[jx] = ka;
          ids[i] = ib;
          ids[jx] = ia;
        }
      }
      __syncthreads();
    }
  }
  for (int i = tid; i < p.k; i += 256) {
    const bool ok = i < n && ids[i] >= 0;
    p.out_id[orow * p.k + i] = ok ? ids[i] : -1;
    p.out_score[orow * p.k + i] = ok ? key32_score(keys[i]) : -INFINITY;
  }
}

// The inverse of topk_pack_kernel.
__global__ void topk_unpack_kernel(const int32_t *packed, int64_t n, int64_t *ids,
                                   float *scores) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t lo = (uint32_t)packed[3 * e], hi = (uint32_t)packed[3 * e + 1];
    ids[e] = (int64_t)(((uint64_t)hi << 32) | lo);
    if (scores != nullptr) scores[e] = __int_as_float(packed[3 * e + 2]);
  }
}

// Pack ids and scores into 12-byte records (id low, id high, score bits):
// one buffer for a single collective of a sharded search's lists.
__global__ void topk_pack_kernel(const int64_t *ids, const float *scores, int64_t n,
                                 int32_t *packed) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t id = (uint64_t)ids[e];
    packed[3 * e] = (int32_t)(uint32_t)id;
    packed[3 * e + 1] = (int32_t)(uint32_t)(id >> 32);
    packed[3 * e + 2] = __float_as_int(scores[e]);
  }
}

}  // namespace uvb

namespace uvb {

// Must match the carve-up at the top of flat_scan_kernel.
size_t scan_smem_bytes(int dim, int img_words, int table_len, bool table_in_smem) {
  (void)img_words;
  size_t b = 0;
  b += 2 * (size_t)dim * XSTR * 4;                      // x-bar tiles
  b += (((size_t)dim * QSTR + 3) & ~(size_t)3) * 4;     // queries
  b += (size_t)TQ * KCAP * 8 + (size_t)TQ * BCAP * 8;   // top-k + buffers
  b += (size_t)TQ * 8 + (size_t)TQ * 4 * 3;             // theta, cnt, degenerate, theta_s
  b += 2 * NSC * (size_t)TN * 4 + 16;                   // scalars, flag
  b += (size_t)TQ * 8 * 4;                              // tail coordinates
  if (table_in_smem) b += (size_t)table_len * 4;
  return b;
}

}  // namespace uvb
