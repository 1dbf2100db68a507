// coset.cu -- the coset trellis encoder (src/coset_trellis.rs): trellis-coded
// vector quantization over the eight cosets of an index-8 sublattice of E8.
//
// A row is encoded in three launches over a batch of rows:
//   coset_prep_kernel     one warp per row: normalize, center on the nearest
//                         centroid, rotate, standardize (src/coset_trellis.rs:
//                         298-318, 322-326) -> u_r and the lattice-space y;
//   coset_nearest_kernel  one thread per (row, 8-wide block, coset): the
//                         nearest kept point of the coset and its squared
//                         distance, by the reference's own search (bisection
//                         seed, then every E8 point within the seed's
//                         distance; 214-278) so that ties resolve alike;
//   coset_viterbi_kernel  one CTA per row: the free-start Viterbi over the
//                         blocks (4 branches per state, 343-368), first
//                         minimum, traceback, emission, rescale and packing
//                         (369-411).
// Every f32 operation is a separately rounded intrinsic, as in the reference.
#include "uv_kernels.h"
#include "uv_team.cuh"

namespace uvb {

namespace {

// three-bit coset label ((R0-R1)/2, (R2-R3)/2, (R4-R5)/2) mod 2
// (src/coset_trellis.rs:73-79); C++ division truncates like Rust's
__device__ __forceinline__ int coset_label(const int *r) {
  return ((((r[0] - r[1]) / 2) & 1) << 2) | ((((r[2] - r[3]) / 2) & 1) << 1) |
         (((r[4] - r[5]) / 2) & 1);
}

// the coset a (state, branch) pair names: parity of the whole state (90-94)
__device__ __forceinline__ int coset_for(uint32_t state, int br) {
  return ((__popc(state) & 1) << 2) | br;
}

__device__ __forceinline__ bool in_key_range(const int *r) {
  bool ok = true;
#pragma unroll
  for (int j = 0; j < 8; j++) ok &= r[j] >= -16 && r[j] <= 15;
  return ok;
}

__device__ __forceinline__ uint64_t e8_key(const int *r) {
  int n = 0;
  uint64_t lex = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    n += r[j] * r[j];
    lex = (lex << 5) | (uint64_t)((r[j] + 16) & 31);
  }
  return ((uint64_t)n << 40) | lex;
}

__device__ __forceinline__ void e8_unkey(uint64_t key, int *r) {
#pragma unroll
  for (int j = 0; j < 8; j++) r[j] = (int)((key >> (5 * (7 - j))) & 31) - 16;
}

// |y - p/2|^2 as the reference sums it: from 0.0, one rounding per op
__device__ __forceinline__ float dist2(const float *y, const int *p) {
  float d = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const float e = fsub(y[j], fmul((float)p[j], 0.5f));
    d = fadd(d, fmul(e, e));
  }
  return d;
}

// nearest point of D8 + offset (src/e8.rs:53-80): round to the offset grid,
// and on an odd coordinate sum move the least confidently rounded coordinate
__device__ __forceinline__ void nearest_d8(const float *y, float off, float *pt) {
  long long isum = 0;
  int worst = 0;
  float werr = -1.0f, wdir = 1.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float s = fsub(y[i], off);
    const float r = roundf(s);  // half away from zero, as f32::round
    pt[i] = fadd(r, off);
    isum += (long long)r;
    const float resid = fsub(s, r);
    const float err = fabsf(resid);
    if (err > werr) {
      werr = err;
      worst = i;
      wdir = resid >= 0.0f ? 1.0f : -1.0f;
    }
  }
  if (isum & 1) {
#pragma unroll
    for (int i = 0; i < 8; i++)
      if (i == worst) pt[i] = fadd(pt[i], wdir);
  }
}

// nearest E8 point (src/e8.rs:37-51)
__device__ __forceinline__ void e8_nearest(const float *y, float *out) {
  float a[8], b[8];
  nearest_d8(y, 0.0f, a);
  nearest_d8(y, 0.5f, b);
  float da = -0.0f, db = -0.0f;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float e = fsub(y[i], a[i]);
    da = fadd(da, fmul(e, e));
  }
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float e = fsub(y[i], b[i]);
    db = fadd(db, fmul(e, e));
  }
  const bool pa = da <= db;
#pragma unroll
  for (int i = 0; i < 8; i++) out[i] = pa ? a[i] : b[i];
}

// position of a key in a coset's sorted book (the key is in the book)
__device__ __forceinline__ int book_index(const uint64_t *book, int len, uint64_t key) {
  int lo = 0, hi = len;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(book + mid) < key)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// A point of coset c is kept iff its key is at most the book's last key: the
// book is the coset's per_coset smallest keys.
struct NearestState {
  float best_d;
  uint64_t best_key;
};

__device__ __forceinline__ void offer(const CosetModel &m, int c, const float *y, const int *p,
                                      NearestState &st) {
  if (!in_key_range(p) || coset_label(p) != c) return;
  const uint64_t key = e8_key(p);
  if (key > m.bound[c]) return;
  const float d = dist2(y, p);
  if (d < st.best_d) {
    st.best_d = d;
    st.best_key = key;
  }
}

// Nearest kept point of coset c to y and its squared distance
// (src/coset_trellis.rs:214-278, and the exhaustive guard 281-296).
__device__ void nearest_in_coset(const CosetModel &m, int c, const float *y, uint32_t *idx_out,
                                 float *d_out) {
  const uint64_t *book = m.books + (size_t)c * m.per_coset;
  int t[8];
  e8_unkey(__ldg(book), t);
  NearestState st;
  st.best_d = dist2(y, t);
  st.best_key = __ldg(book);
  float lo = 0.0f, hi = 1.0f;
  for (int it = 0; it < 12; it++) {
    const float a = fmul(0.5f, fadd(lo, hi));
    float z[8], pt[8];
#pragma unroll
    for (int j = 0; j < 8; j++) z[j] = fsub(fmul(a, y[j]), fmul((float)t[j], 0.5f));
    e8_nearest(z, pt);
    int r[8];
#pragma unroll
    for (int j = 0; j < 8; j++) r[j] = (int)(short)((int)roundf(fmul(pt[j], 2.0f)) + t[j]);
    const bool hit = in_key_range(r) && coset_label(r) == c && e8_key(r) <= m.bound[c];
    if (hit) {
      const float d = dist2(y, r);
      if (d < st.best_d) {
        st.best_d = d;
        st.best_key = e8_key(r);
      }
      lo = a;
    } else {
      hi = a;
    }
  }
  // about pi^4 d^8 / 24 lattice points lie within the seed's distance
  const double bd = (double)st.best_d, bd2 = __dmul_rn(bd, bd);
  const double est = __ddiv_rn(__dmul_rn(m.pi4, __dmul_rn(bd2, bd2)), 24.0);
  if (!isfinite(est) || est > (double)m.per_coset) {
    int best = 0;
    float best_d = INFINITY;
    for (int i = 0; i < m.per_coset; i++) {
      int p[8];
      e8_unkey(__ldg(book + i), p);
      const float d = dist2(y, p);
      if (d < best_d) {
        best_d = d;
        best = i;
      }
    }
    *idx_out = (uint32_t)best;
    *d_out = best_d;
    return;
  }
  // every E8 point within sqrt(budget) of 2y, in the order src/e8.rs:143-203
  // produces them: parity 0 then 1, coordinates in order, values ascending
  float centre[8];
#pragma unroll
  for (int j = 0; j < 8; j++) centre[j] = fmul(y[j], 2.0f);
  const double budget = __dadd_rn(__dmul_rn(__dmul_rn(4.0, bd), 1.0 + 1e-6), 1e-6);
  for (int parity = 0; parity < 2; parity++) {
    int cur[8], rhi[8];
    double left[8];
    int sum[8];
    int pos = 0;
    left[0] = budget;
    sum[0] = 0;
    auto open_level = [&](int ps) {
      const double cc = (double)centre[ps];
      const double span = __dsqrt_rn(left[ps] > 0.0 ? left[ps] : 0.0);
      int r = (int)floor(__dsub_rn(cc, span));
      rhi[ps] = (int)ceil(__dadd_rn(cc, span));
      if ((r & 1) != parity) r++;
      cur[ps] = r;
    };
    open_level(0);
    for (;;) {
      if (cur[pos] > rhi[pos]) {
        if (pos == 0) break;
        pos--;
        cur[pos] += 2;
        continue;
      }
      const double dd = __dsub_rn((double)cur[pos], (double)centre[pos]);
      const double d2 = __dmul_rn(dd, dd);
      if (d2 <= left[pos]) {
        if (pos == 7) {
          if (((sum[7] + cur[7]) & 3) == 0) offer(m, c, y, cur, st);
          cur[7] += 2;
        } else {
          left[pos + 1] = __dsub_rn(left[pos], d2);
          sum[pos + 1] = sum[pos] + cur[pos];
          pos++;
          open_level(pos);
        }
      } else {
        cur[pos] += 2;
      }
    }
  }
  *idx_out = (uint32_t)book_index(book, m.per_coset, st.best_key);
  *d_out = st.best_d;
}

}  // namespace

// ---------------------------------------------------------------------------
// Nearest kept point of every coset for every 8-wide block of every row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) coset_nearest_kernel(const CosetEncParams p) {
  const int nb = p.m.dim >> 3;
  const int64_t total = p.n * nb * 8;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e & 7);
    const int64_t rb = e >> 3;  // row * nb + block
    const float *ys = p.y + rb * 8;
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; j++) y[j] = ys[j];
    uint32_t idx;
    float d;
    nearest_in_coset(p.m, c, y, &idx, &d);
    p.blk_idx[e] = idx;
    p.blk_cost[e] = d;
  }
}

// ---------------------------------------------------------------------------
// The same results for books of up to 8192 points (one and two bits): every
// point of the coset's book is scored against tiles of y-blocks held in
// registers, the book staged in shared memory as eight signed bytes per
// point.  The minimum is exact, so when one point attains it that point is
// the reference's answer too; when several do, the reference's choice among
// them depends on its search order, so that y-block runs nearest_in_coset.
// Grid: (y-block tiles, coset).
// ---------------------------------------------------------------------------
constexpr int kBruteY = kCosetBruteY;

__global__ void __launch_bounds__(256) coset_nearest_brute_kernel(const CosetEncParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const CosetModel &m = p.m;
  const int c = blockIdx.y;
  const int nb = m.dim >> 3;
  const int64_t ny = p.n * nb;
  const uint64_t *book = m.books + (size_t)c * m.per_coset;
  uint2 *pts = (uint2 *)sm;  // per point: raw coordinates as signed bytes
  for (int i = threadIdx.x; i < m.per_coset; i += blockDim.x) {
    const uint64_t key = __ldg(book + i);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t r = (uint32_t)((int)((key >> (5 * (7 - j))) & 31) - 16) & 0xffu;
      if (j < 4)
        lo |= r << (8 * j);
      else
        hi |= r << (8 * (j - 4));
    }
    pts[i] = make_uint2(lo, hi);
  }
  __syncthreads();
  const int64_t y0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kBruteY;
  float y[kBruteY][8];
  float best[kBruteY];
  int bidx[kBruteY];
  bool tie[kBruteY];
#pragma unroll
  for (int u = 0; u < kBruteY; u++) {
    const int64_t e = y0 + u < ny ? y0 + u : ny - 1;
#pragma unroll
    for (int j = 0; j < 8; j++) y[u][j] = p.y[e * 8 + j];
    best[u] = INFINITY;
    bidx[u] = 0;
    tie[u] = false;
  }
  // two y-blocks per paired f32 instruction: y - p/2 is y + (-p/2) exactly
  float2 y2[kBruteY / 2][8];
#pragma unroll
  for (int u = 0; u < kBruteY / 2; u++)
#pragma unroll
    for (int j = 0; j < 8; j++) y2[u][j] = make_float2(y[2 * u][j], y[2 * u + 1][j]);
  for (int i = 0; i < m.per_coset; i++) {
    const uint2 w = pts[i];
    float2 nh[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t word = j < 4 ? w.x : w.y;
      const float h = fmul((float)(int8_t)((word >> (8 * (j & 3))) & 0xffu), -0.5f);
      nh[j] = make_float2(h, h);
    }
#pragma unroll
    for (int u = 0; u < kBruteY / 2; u++) {
      float2 d = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float2 e = __fadd2_rn(y2[u][j], nh[j]);
        d = __fadd2_rn(d, __fmul2_rn(e, e));
      }
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int v = 2 * u + h;
        const float dv = h ? d.y : d.x;
        if (dv < best[v]) {
          best[v] = dv;
          bidx[v] = i;
          tie[v] = false;
        } else if (dv == best[v]) {
          tie[v] = true;
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < kBruteY; u++) {
    const int64_t e = y0 + u;
    if (e >= ny) continue;
    uint32_t idx = (uint32_t)bidx[u];
    float d = best[u];
    if (tie[u] || !(d < INFINITY)) nearest_in_coset(m, c, y[u], &idx, &d);
    p.blk_idx[e * 8 + c] = idx;
    p.blk_cost[e * 8 + c] = d;
  }
}

size_t coset_brute_smem_bytes(int per_coset) { return (size_t)per_coset * 8; }

// ---------------------------------------------------------------------------
// Prep: one warp per row (src/coset_trellis.rs:298-318, 322-326, 335-341).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) coset_prep_kernel(const CosetEncParams p) {
  extern __shared__ __align__(16) float smem[];
  const int d = p.m.dim;
  const int team = threadIdx.x >> 5;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  float *x = smem + (size_t)team * (d + 8);
  float *misc = x + d;
  for (int64_t row = (int64_t)blockIdx.x * 8 + team; row < p.n; row += (int64_t)gridDim.x * 8) {
    const float *src = p.rows + row * d;
    for (int i = tm.t; i < d; i += 32) x[i] = src[i];
    tm.sync();
    if (tm.leader()) misc[0] = fmax_rs(fsqrt(seq_sum_sq(x, d)), kF32Eps);
    tm.sync();
    const float nrm = misc[0];
    for (int i = tm.t; i < d; i += 32) x[i] = fdiv(x[i], nrm);
    tm.sync();
    float rn = 1.0f;
    uint32_t ci = 0;
    if (p.n_centroids > 0) {
      // nearest centroid: first strict minimum of the squared distance
      uint64_t best = ~0ull;
      for (int j = tm.t; j < p.n_centroids; j += 32) {
        const float *c = p.centroids + (size_t)j * d;
        float s = -0.0f;
        for (int i = 0; i < d; i++) {
          const float e = fsub(x[i], c[i]);
          s = fadd(s, fmul(e, e));
        }
        if (s < INFINITY) {
          const uint32_t u = __float_as_uint(s);
          const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
          const uint64_t key = ((uint64_t)k << 32) | (uint32_t)j;
          best = key < best ? key : best;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const uint64_t w = __shfl_xor_sync(0xffffffffu, best, o);
        best = w < best ? w : best;
      }
      ci = best == ~0ull ? 0u : (uint32_t)(best & 0xffffffffu);
      const float *c = p.centroids + (size_t)ci * d;
      for (int i = tm.t; i < d; i += 32) x[i] = fsub(x[i], c[i]);
      tm.sync();
      if (tm.leader()) misc[1] = fmax_rs(fsqrt(seq_sum_sq(x, d)), kF32Eps);
      tm.sync();
      rn = misc[1];
      for (int i = tm.t; i < d; i += 32) x[i] = fdiv(x[i], rn);
      tm.sync();
    }
    team_rotate(x, p.rot, tm, false);
    if (tm.leader()) misc[2] = fmax_rs(seq_std_about_mean(x, d), kF32Eps);
    tm.sync();
    const float scale = misc[2];
    float *ur = p.u_r + row * d;
    float *yy = p.y + row * d;
    for (int i = tm.t; i < d; i += 32) {
      ur[i] = x[i];
      yy[i] = fadd(fmul(fdiv(x[i], scale), p.m.scale_std), p.m.scale_mean);
    }
    if (tm.leader()) {
      p.rnorm[row] = rn;
      p.cidx[row] = ci;
    }
    tm.sync();
  }
}

// ---------------------------------------------------------------------------
// Viterbi + emission: one CTA per row.  State s at block b+1 is reached from
// the four states (ns >> 2) | t << (mem-2), t = 0..3, on branch ns & 3, tried
// in ascending order with a strict `<` exactly as the reference's loop over
// all (state, branch) pairs meets them; the back pointer keeps t (or, at
// mem = 1, the whole window), 255 when no predecessor was finite.
// ---------------------------------------------------------------------------
constexpr int kVitThreads = 256;

size_t coset_viterbi_smem_bytes(int dim, int mem, bool back_smem, bool cost_smem) {
  const size_t nb = (size_t)dim / 8, S = (size_t)1 << mem;
  size_t b = nb * 8 * 4 * 2 + (size_t)dim * 4 + ((nb + 15) & ~(size_t)15) + 32 * 8;
  if (cost_smem) b += 2 * S * 4;
  if (back_smem) b += nb * S;
  return b;
}

__global__ void __launch_bounds__(kVitThreads) coset_viterbi_kernel(const CosetEncParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const CosetModel &m = p.m;
  const int d = m.dim, nb = d >> 3, mem = m.mem;
  const int S = 1 << mem;
  const uint32_t mask = (uint32_t)S - 1;
  const int tid = threadIdx.x;
  float *bc = (float *)sm;                             // nb x 8 costs
  uint32_t *bi = (uint32_t *)(bc + nb * 8);            // nb x 8 indices
  float *ur = (float *)(bi + nb * 8);                  // dim
  uint8_t *branch = (uint8_t *)(ur + d);               // nb (padded to 16)
  uint64_t *red = (uint64_t *)(branch + ((nb + 15) & ~15));  // 32
  uint8_t *tail = (uint8_t *)(red + 32);

  for (int64_t row = blockIdx.x; row < p.n; row += gridDim.x) {
    float *cost0, *cost1;
    uint8_t *back;
    uint8_t *t2 = tail;
    if (p.cost_smem) {
      cost0 = (float *)t2;
      cost1 = cost0 + S;
      t2 += (size_t)2 * S * 4;
    } else {
      cost0 = p.cost + (size_t)blockIdx.x * 2 * S;
      cost1 = cost0 + S;
    }
    back = p.back_smem ? t2 : p.back + (size_t)blockIdx.x * nb * S;

    for (int e = tid; e < nb * 8; e += kVitThreads) {
      bc[e] = p.blk_cost[row * nb * 8 + e];
      bi[e] = p.blk_idx[row * nb * 8 + e];
    }
    for (int i = tid; i < d; i += kVitThreads) ur[i] = p.u_r[row * d + i];
    for (int s = tid; s < S; s += kVitThreads) cost0[s] = 0.0f;
    __syncthreads();

    float *cur = cost0, *nxt = cost1;
    for (int b = 0; b < nb; b++) {
      const float *cb = bc + b * 8;
      uint8_t *bk = back + (size_t)b * S;
      if (mem >= 2) {
        // butterfly of base q: sources q | t << (mem-2) (t = 0..3) feed the
        // four destinations (q << 2) | br; reads are coalesced over q
        const int Q = S >> 2;
        const float c0 = cb[0], c1 = cb[1], c2 = cb[2], c3 = cb[3];
        const float c4 = cb[4], c5 = cb[5], c6 = cb[6], c7 = cb[7];
#pragma unroll 2
        for (int q = tid; q < Q; q += kVitThreads) {
          float best[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
          uint32_t sel = 0xffffffffu;  // four back bytes, 255 = no finite source
#pragma unroll
          for (int t = 0; t < 4; t++) {
            const uint32_t s = (uint32_t)q | ((uint32_t)t << (mem - 2));
            const float cs = cur[s];
            if (cs == INFINITY) continue;
            const bool odd = __popc(s) & 1;
            const float e[4] = {odd ? c4 : c0, odd ? c5 : c1, odd ? c6 : c2, odd ? c7 : c3};
#pragma unroll
            for (int br = 0; br < 4; br++) {
              const float tot = fadd(cs, e[br]);
              if (tot < best[br]) {
                best[br] = tot;
                sel = (sel & ~(0xffu << (8 * br))) | ((uint32_t)t << (8 * br));
              }
            }
          }
          *(float4 *)(nxt + 4 * q) = make_float4(best[0], best[1], best[2], best[3]);
          *(uint32_t *)(bk + 4 * q) = sel;
        }
      } else if (tid < 2) {
        // mem = 1: ns = br & 1; the pairs (s, br) meet it in this order
        const int ns = tid;
        float best = INFINITY;
        int sel = 255;
        for (int s = 0; s < 2; s++) {
          const float cs = cur[s];
          if (cs == INFINITY) continue;
          for (int h = 0; h < 2; h++) {
            const int br = ns + 2 * h;
            const float tot = fadd(cs, cb[coset_for((uint32_t)s, br)]);
            if (tot < best) {
              best = tot;
              sel = (s << 2) | br;
            }
          }
        }
        nxt[ns] = best;
        bk[ns] = (uint8_t)sel;
      }
      __syncthreads();
      float *tt = cur;
      cur = nxt;
      nxt = tt;
    }

    // first minimum under f32::total_cmp
    uint64_t key = ~0ull;
    for (int s = tid; s < S; s += kVitThreads) {
      const uint32_t u = __float_as_uint(cur[s]);
      const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
      const uint64_t kk = ((uint64_t)k << 32) | (uint32_t)s;
      key = kk < key ? kk : key;
    }
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t w = __shfl_xor_sync(0xffffffffu, key, o);
      key = w < key ? w : key;
    }
    if ((tid & 31) == 0) red[tid >> 5] = key;
    __syncthreads();

    if (tid == 0) {
      uint64_t k0 = red[0];
      for (int w = 1; w < kVitThreads / 32; w++) k0 = red[w] < k0 ? red[w] : k0;
      uint32_t s = (uint32_t)(k0 & 0xffffffffu);
      for (int b = nb - 1; b >= 0; b--) {
        const int sel = back[(size_t)b * S + s];
        uint32_t w;
        if (sel == 255)
          w = 0;
        else if (mem >= 2)
          w = ((((s >> 2) | ((uint32_t)sel << (mem - 2)))) << 2) | (s & 3);
        else
          w = (uint32_t)sel;
        branch[b] = (uint8_t)(w & 3);
        s = w >> 2;
      }
      const uint32_t start = s;
      // emission, rescale from the stored reconstruction, packing
      uint8_t *out = p.codes + row * (int64_t)m.code_stride;
      for (int i = 0; i < m.start_bytes; i++) out[i] = (uint8_t)((start >> (8 * i)) & 0xff);
      const int W = 2 + m.m_bits;
      uint64_t buf = 0;
      int inb = 0, o = m.start_bytes;
      float rescale = 0.0f;
      uint32_t st = start;
      for (int b = 0; b < nb; b++) {
        const int br = branch[b];
        const int c = coset_for(st, br);
        const uint32_t idx = bi[b * 8 + c];
        buf = (buf << W) | (((uint64_t)br << m.m_bits) | idx);
        inb += W;
        while (inb >= 8) {
          inb -= 8;
          out[o++] = (uint8_t)((buf >> inb) & 0xff);
        }
        int pt[8];
        e8_unkey(__ldg(m.books + (size_t)c * m.per_coset + idx), pt);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float v = fdiv(fsub(fmul((float)pt[j], 0.5f), m.scale_mean), m.scale_std);
          rescale = fadd(rescale, fmul(v, ur[b * 8 + j]));
        }
        st = ((st << 2) | (uint32_t)br) & mask;
      }
      if (inb > 0) out[o++] = (uint8_t)((buf << (8 - inb)) & 0xff);
      for (; o < m.code_stride; o++) out[o] = 0;
      p.rescale[row] = fmax_rs(rescale, kF32Eps);
    }
    __syncthreads();
  }
}

// out[i] = base + i: the ids of an add_batch (the batch's positions)
__global__ void iota_i64_kernel(int64_t *out, int64_t n, int64_t base) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = base + i;
}

// ---------------------------------------------------------------------------
// Reconstruction (src/coset_trellis.rs:414-434, 521-529): decode a record,
// rotate back, normalize.  One warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) coset_reconstruct_kernel(const CosetEncParams p) {
  extern __shared__ __align__(16) float smem[];
  const CosetModel &m = p.m;
  const int d = m.dim, nb = d >> 3;
  const int team = threadIdx.x >> 5;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  float *x = smem + (size_t)team * (d + 8);
  float *misc = x + d;
  const uint32_t mask = (1u << m.mem) - 1, imask = (1u << m.m_bits) - 1;
  const int W = 2 + m.m_bits;
  for (int64_t row = (int64_t)blockIdx.x * 8 + team; row < p.n; row += (int64_t)gridDim.x * 8) {
    const uint8_t *rec = p.codes + row * (int64_t)m.code_stride;
    if (tm.leader()) {
      uint32_t st = 0;
      for (int i = 0; i < m.start_bytes; i++) st |= (uint32_t)rec[i] << (8 * i);
      for (int b = 0; b < nb; b++) {
        const int bit0 = 8 * m.start_bytes + b * W;
        uint32_t sym = 0;
        for (int k = 0; k < W; k++) {
          const int bit = bit0 + k;
          sym = (sym << 1) | ((rec[bit >> 3] >> (7 - (bit & 7))) & 1u);
        }
        const int br = (int)(sym >> m.m_bits);
        const int c = coset_for(st, br);
        int pt[8];
        e8_unkey(__ldg(m.books + (size_t)c * m.per_coset + (sym & imask)), pt);
        for (int j = 0; j < 8; j++)
          x[b * 8 + j] = fdiv(fsub(fmul((float)pt[j], 0.5f), m.scale_mean), m.scale_std);
        st = ((st << 2) | (uint32_t)br) & mask;
      }
    }
    tm.sync();
    team_rotate(x, p.rot, tm, true);
    if (tm.leader()) misc[0] = fmax_rs(fsqrt(seq_sum_sq(x, d)), kF32Eps);
    tm.sync();
    const float nrm = misc[0];
    for (int i = tm.t; i < d; i += 32) p.recon[row * d + i] = fdiv(x[i], nrm);
    tm.sync();
  }
}

}  // namespace uvb
