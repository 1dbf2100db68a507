// ivf.cu -- the IVF coarse stage and list bookkeeping for sm_100a.
//
//   k-means       bench.rs:298-349 (units, splitmix64 picks, 5 Lloyd rounds,
//                 strict-> argmax, sums in original row order, mean = sum / count)
//   assignment    ivf.rs:405-421 (normalize the row, first strict maximum)
//   probe         ivf.rs:209-223 (exact cosine, lib.rs:240-248, best nprobe)
//   search        ivf.rs:229-239 (each probed list scores its own records;
//                 the per-list top-k are merged)
//   rerank        ivf.rs:248-274 (exact fp32 cosine of the global top-r)
//
// Every dot here is the reference's `a.iter().zip(b).map(|(x, y)| x * y).sum()`:
// a left fold from -0.0 with the product and the sum rounded separately.  The
// tile kernel evaluates one such chain per (row, centroid) pair; 16 chains per
// thread give the ILP.  Products are paired f32x2 multiplies and the fold adds
// are written fma(product, one, acc) with a run-time one: the code generator
// fuses a paired multiply into a following paired add (one rounding instead
// of two), and an fma whose multiplier is 1.0 rounds exactly like the add.
#include "uv_kernels.h"

namespace uvb {

namespace {

constexpr int SD_T = 64;   // rows and centroids per tile
constexpr int SD_K = 32;   // coordinates per staged chunk
constexpr int SD_S = SD_T + 4;

}  // namespace

// C[a][b] = seq_dot(A[a], B[b]) over `dim` terms.  MODE 0: per A row, the
// first strict maximum over b as a 64-bit key (score key, ~b) folded into
// out_key[a] with atomicMax.  MODE 1: cosine(A[a], B[b]) into out[a * nB + b].
template <int MODE>
__global__ void __launch_bounds__(256) seqdot_kernel(const SeqDotParams p) {
  __shared__ __align__(16) float As[SD_K][SD_S];
  __shared__ __align__(16) float Bs[SD_K][SD_S];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int d = p.dim;
  const int64_t b0 = (int64_t)blockIdx.x * SD_T;
  const float2 one2 = p.one2;
  for (int64_t a0 = (int64_t)blockIdx.y * SD_T; a0 < p.nA; a0 += (int64_t)gridDim.y * SD_T) {
    float2 acc[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i][0] = acc[i][1] = make_float2(-0.0f, -0.0f);
    const int lr = tid >> 2, lk = (tid & 3) * 8;
    const int64_t ar = a0 + lr, br = b0 + lr;
    const float *arow = p.A + (ar < p.nA ? ar : 0) * (int64_t)p.lda;
    const float *brow = p.B + (br < p.nB ? br : 0) * (int64_t)p.ldb;
    for (int k0 = 0; k0 < d; k0 += SD_K) {
      const int kc = min(SD_K, d - k0);
      __syncthreads();
#pragma unroll
      for (int e = 0; e < 8; e++) {
        const int k = lk + e;
        As[k][lr] = (k < kc && ar < p.nA) ? __ldg(arow + k0 + k) : 0.0f;
        Bs[k][lr] = (k < kc && br < p.nB) ? __ldg(brow + k0 + k) : 0.0f;
      }
      __syncthreads();
#pragma unroll 4
      for (int k = 0; k < kc; k++) {
        const float4 a4 = *(const float4 *)&As[k][ty * 4];
        const float4 b4 = *(const float4 *)&Bs[k][tx * 4];
        const float2 b01 = make_float2(b4.x, b4.y), b23 = make_float2(b4.z, b4.w);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 ai = make_float2(av[i], av[i]);
          acc[i][0] = __ffma2_rn(__fmul2_rn(ai, b01), one2, acc[i][0]);
          acc[i][1] = __ffma2_rn(__fmul2_rn(ai, b23), one2, acc[i][1]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t a = a0 + ty * 4 + i;
      const float dv[4] = {acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y};
      if (MODE == 0) {
        uint64_t best = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int64_t b = b0 + tx * 4 + j;
          const uint64_t key = b < p.nB ? rank_key(dv[j], (uint32_t)b) : 0ull;
          best = key > best ? key : best;
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) {
          const uint64_t w = __shfl_xor_sync(0xffffffffu, best, o);
          best = w > best ? w : best;
        }
        if (tx == 0 && a < p.nA) atomicMax((unsigned long long *)&p.out_key[a], best);
      } else if (a < p.nA) {
        const float na = p.a_norm[a];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int64_t b = b0 + tx * 4 + j;
          if (b >= p.nB) continue;
          const float nb = p.b_norm[b];
          p.out[a * p.nB + b] =
              (na < kF32Eps || nb < kF32Eps) ? 0.0f : fdiv(dv[j], fmul(na, nb));
        }
      }
    }
  }
}

// Key of the first strict maximum -> its index (rank_key puts ~b low).
__global__ void argmax_index_kernel(const uint64_t *key, int64_t n, uint32_t *out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = rank_key_index(key[i]);
}

// norms[i] = sqrt(seq_sum_sq(row i)) (lib.rs:215-217), one thread per row.
__global__ void row_norms_kernel(const float *rows, int64_t n, int dim, float *norms) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float *r = rows + i * (int64_t)dim;
  float s = -0.0f;
  int t = 0;
  for (; t + 8 <= dim; t += 8) {  // eight loads ahead of the in-order fold
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = __ldg(r + t + u);
#pragma unroll
    for (int u = 0; u < 8; u++) s = fadd(s, fmul(v[u], v[u]));
  }
  for (; t < dim; t++) {
    const float x = __ldg(r + t);
    s = fadd(s, fmul(x, x));
  }
  norms[i] = fsqrt(s);
}

// units[i] = row[i] / max(norm, EPS), elementwise.
__global__ void normalize_rows_kernel(const float *rows, const float *norms, int64_t n, int dim,
                                      float *units) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n * (int64_t)dim) return;
  const int64_t i = e / dim;
  units[e] = fdiv(rows[e], fmax_rs(norms[i], kF32Eps));
}

// cent[j] = units[pick[j]]
__global__ void gather_rows_kernel(const float *src, const int64_t *pick, int nrows, int dim,
                                   float *dst) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)nrows * dim) return;
  const int64_t j = e / dim, t = e - j * dim;
  dst[e] = src[pick[j] * (int64_t)dim + t];
}

// Lloyd update (bench.rs:334-346): per (list, coordinate) the sum of the
// member units in original row order from +0.0, then sum / (count as f32);
// empty lists keep their centroid.  `order` lists rows by list, stable.
__global__ void list_means_kernel(const float *units, const int64_t *order, const int64_t *off,
                                  int nlist, int dim, float *cent) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)nlist * dim) return;
  const int j = (int)(e / dim);
  const int t = (int)(e - (int64_t)j * dim);
  const int64_t lo = off[j], hi = off[j + 1];
  if (hi == lo) return;
  float s = 0.0f;
  for (int64_t m = lo; m < hi; m++) s = fadd(s, units[order[m] * (int64_t)dim + t]);
  cent[e] = fdiv(s, (float)(hi - lo));
}

// Best `np` of each row of an (n x nb) score matrix by (score desc, index
// asc), NaN as -inf (the probe order of ivf.rs:209-223).  One CTA per row,
// bitonic sort of the row's keys in shared memory (pow2 >= nb).
__global__ void __launch_bounds__(256) select_top_kernel(const float *scores, int64_t n, int nb,
                                                         int pow2, int np, int ld_out,
                                                         int32_t *out) {
  extern __shared__ uint64_t keys[];
  for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
    const float *s = scores + row * (int64_t)nb;
    for (int i = threadIdx.x; i < pow2; i += blockDim.x)
      keys[i] = i < nb ? rank_key(s[i], (uint32_t)i) : 0ull;
    __syncthreads();
    for (int size = 2; size <= pow2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int pi = threadIdx.x; pi < pow2 / 2; pi += blockDim.x) {
          const int lo = 2 * pi - (pi & (stride - 1));
          const int hi = lo + stride;
          const bool desc = (lo & size) == 0;
          const uint64_t x = keys[lo], y = keys[hi];
          if ((x < y) == desc) {
            keys[lo] = y;
            keys[hi] = x;
          }
        }
        __syncthreads();
      }
    }
    for (int i = threadIdx.x; i < np; i += blockDim.x)
      out[row * ld_out + i] = (int32_t)rank_key_index(keys[i]);
    __syncthreads();
  }
}

// flags[i] = 1 when norms[i] is below EPS or not finite (the probe's
// tensor-core rows are zero for those)
__global__ void unit_flags_kernel(const float *norms, int64_t n, uint32_t *flags) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) flags[i] = (norms[i] >= kF32Eps && isfinite(norms[i])) ? 0u : 1u;
}

// The probe from tensor-core dots (the same lists as seqdot_kernel<1> +
// select_top_kernel).  approx[q][j] = the fp16 dot of the unit query and the
// unit centroid, within p.bound of the exact f32 cosine (src/lib.rs:240-248:
// the sequential dot over the norms' product, 0 below EPS).  One CTA per
// query: theta = the np-th largest approximate dot; every centroid j with
// approx >= theta - 2 bound can reach the np-th best exact cosine, so its
// exact cosine is computed (sequential f32, as the reference) and the
// candidates are ranked by (cosine desc, index asc, NaN last).  With
// cosine = 0 the score is the plain sequential dot (seqdot_kernel<0>, the
// k-means assignment's first strict maximum at np = 1).
__device__ __forceinline__ uint32_t ord_key(float f) {
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(256) probe_refine_kernel(const ProbeRefineParams p) {
  extern __shared__ __align__(16) uint64_t keys[];       // pow2
  uint32_t *aux = (uint32_t *)(keys + p.pow2);          // nlist: approx keys, then candidates
  float *qs = (float *)(aux + ((p.nlist + 3) & ~3));    // dim: the query row
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[3];
  const int tid = threadIdx.x;
  const int nl = p.nlist;
  for (int64_t q = blockIdx.x; q < p.m; q += gridDim.x) {
    const float *v = p.approx + q * p.ld;
    for (int j = tid; j < nl; j += 256) aux[j] = ord_key(v[j]);
    // radix select of the np-th largest key
    uint32_t prefix = 0, mask = 0, kk = (uint32_t)p.np;
    for (int shift = 24; shift >= 0; shift -= 8) {
      hist[tid] = 0;
      __syncthreads();
      for (int j = tid; j < nl; j += 256) {
        const uint32_t key = aux[j];
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t above = 0;
        int b = 255;
        for (; b > 0; b--) {
          if (above + hist[b] >= kk) break;
          above += hist[b];
        }
        sel[0] = (uint32_t)b;
        sel[1] = above;
      }
      __syncthreads();
      prefix |= sel[0] << shift;
      mask |= 255u << shift;
      kk -= sel[1];
      __syncthreads();
    }
    const float theta = __uint_as_float((prefix & 0x80000000u) ? (prefix & 0x7fffffffu) : ~prefix);
    const float thr = fsub(theta, fmul(2.0001f, p.bound));
    if (tid == 0) sel[2] = 0;
    __syncthreads();
    for (int j = tid; j < nl; j += 256)
      if (v[j] >= thr) aux[atomicAdd(&sel[2], 1u)] = (uint32_t)j;
    __syncthreads();
    const int nc = (int)sel[2];
    int pow2 = 32;
    while (pow2 < nc) pow2 <<= 1;
    const float na = p.cosine ? p.qnorm[q] : 1.0f;
    const float *qa = p.queries + q * (int64_t)p.dim;
    for (int t = tid; t < p.dim; t += 256) qs[t] = qa[t];
    __syncthreads();
    for (int i = tid; i < pow2; i += 256) {
      uint64_t key = 0ull;
      if (i < nc) {
        const int j = (int)aux[i];
        // the centroid row in batches of 32 values, the next batch's eight
        // 16-byte loads in flight while the current batch is folded in the
        // reference order (dim is a multiple of 32 here)
        const float4 *c4 = (const float4 *)(p.cent + (int64_t)j * p.dim);
        const float4 *q4 = (const float4 *)qs;
        float dot = -0.0f;
        float4 b[8];
#pragma unroll
        for (int u = 0; u < 8; u++) b[u] = __ldg(c4 + u);
        for (int t4 = 0; t4 < p.dim / 4; t4 += 8) {
          float4 nb[8];
          const bool more = t4 + 8 < p.dim / 4;
#pragma unroll
          for (int u = 0; u < 8; u++) nb[u] = more ? __ldg(c4 + t4 + 8 + u) : b[u];
#pragma unroll
          for (int u = 0; u < 8; u++) {
            const float4 a = q4[t4 + u];
            dot = fadd(dot, fmul(a.x, b[u].x));
            dot = fadd(dot, fmul(a.y, b[u].y));
            dot = fadd(dot, fmul(a.z, b[u].z));
            dot = fadd(dot, fmul(a.w, b[u].w));
          }
#pragma unroll
          for (int u = 0; u < 8; u++) b[u] = nb[u];
        }
        float cs = dot;  // the k-means assignment ranks the plain dot
        if (p.cosine) {
          const float nb = p.cnorm[j];
          cs = (na < kF32Eps || nb < kF32Eps) ? 0.0f : fdiv(dot, fmul(na, nb));
        }
        key = rank_key(cs, (uint32_t)j);
      }
      keys[i] = key;
    }
    __syncthreads();
    for (int size = 2; size <= pow2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int pi = tid; pi < pow2 / 2; pi += 256) {
          const int lo = 2 * pi - (pi & (stride - 1));
          const int hi = lo + stride;
          const bool desc = (lo & size) == 0;
          const uint64_t x = keys[lo], y = keys[hi];
          if ((x < y) == desc) {
            keys[lo] = y;
            keys[hi] = x;
          }
        }
        __syncthreads();
      }
    }
    for (int i = tid; i < p.np; i += 256) p.out[q * p.ld_out + i] = (int32_t)rank_key_index(keys[i]);
    __syncthreads();
  }
}

// Empty result slots: id -1, score -inf (as the merge writes them).
__global__ void fill_empty_kernel(int64_t *ids, float *scores, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  ids[i] = -1;
  scores[i] = -INFINITY;
}

// ---- (query, list) pairs bucketed by list ----
// Probes of lists that hold no records contribute nothing: they become -1
// (no pair).  A list id outside 0..nlist-1 sets *bad.
__global__ void drop_empty_lists_kernel(int32_t *lists, int64_t npairs, const int64_t *list_off,
                                        int nlist, int *bad) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= npairs) return;
  const int l = lists[i];
  if (l < 0) return;
  if (l >= nlist) {
    atomicExch(bad, 1);
    lists[i] = -1;
    return;
  }
  if (list_off[l + 1] == list_off[l]) lists[i] = -1;
}

__global__ void pair_count_kernel(const int32_t *lists, int64_t npairs, int32_t *cnt) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < npairs && lists[i] >= 0) atomicAdd(&cnt[lists[i]], 1);
}

// Record ranges of a list of `size` records: 1 for short lists, else
// ceil(size / range_size).
__device__ __forceinline__ int64_t list_ranges(int64_t size, int64_t range_size) {
  return size <= range_size ? 1 : (size + range_size - 1) / range_size;
}

// One CTA: exclusive scans over the lists of the pair counts, of the scan
// items (ranges x ceil(pairs / per_item)) and of the range slots (pairs x
// ranges); totals = {items, range slots, pairs}.
__global__ void __launch_bounds__(1024) pair_scan_kernel(const int32_t *cnt,
                                                         const int64_t *list_off, int nlist,
                                                         int64_t range_size, int per_item,
                                                         int32_t *pair_off, int32_t *item_off,
                                                         int64_t *list_rbase, int64_t *totals) {
  __shared__ int64_t sp[1024], si[1024], sr[1024];
  const int t = threadIdx.x;
  const int per = (nlist + 1023) / 1024;
  const int lo = min(nlist, t * per), hi = min(nlist, lo + per);
  int64_t ps = 0, is = 0, rs = 0;
  for (int l = lo; l < hi; l++) {
    const int64_t nr = list_ranges(list_off[l + 1] - list_off[l], range_size);
    ps += cnt[l];
    is += nr * ((cnt[l] + per_item - 1) / per_item);
    rs += nr * cnt[l];
  }
  sp[t] = ps;
  si[t] = is;
  sr[t] = rs;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int64_t a = t >= o ? sp[t - o] : 0, b = t >= o ? si[t - o] : 0,
                  c = t >= o ? sr[t - o] : 0;
    __syncthreads();
    sp[t] += a;
    si[t] += b;
    sr[t] += c;
    __syncthreads();
  }
  int64_t pbase = sp[t] - ps, ibase = si[t] - is, rbase = sr[t] - rs;
  for (int l = lo; l < hi; l++) {
    const int64_t nr = list_ranges(list_off[l + 1] - list_off[l], range_size);
    pair_off[l] = (int32_t)pbase;
    item_off[l] = (int32_t)ibase;
    list_rbase[l] = rbase;
    pbase += cnt[l];
    ibase += nr * ((cnt[l] + per_item - 1) / per_item);
    rbase += nr * cnt[l];
  }
  if (t == 1023) {
    totals[2] = sp[1023];
    totals[0] = si[1023];
    totals[1] = sr[1023];
  }
}

__global__ void pair_scatter_kernel(const int32_t *lists, int64_t nq, int np,
                                    const int32_t *pair_off, int32_t *fill, int32_t *pair_query,
                                    int32_t *pair_slot, int32_t *pair_list) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * np) return;
  const int l = lists[i];
  if (l < 0) return;
  const int pos = pair_off[l] + atomicAdd(&fill[l], 1);
  pair_query[pos] = (int32_t)(i / np);
  pair_slot[pos] = (int32_t)i;
  pair_list[pos] = l;
}

__global__ void item_fill_kernel(const int32_t *cnt, const int32_t *pair_off,
                                 const int32_t *item_off, const int64_t *list_off, int nlist,
                                 int64_t range_size, int per_item, int32_t *item_list,
                                 int32_t *item_pair, int32_t *item_npairs, int32_t *item_range) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= nlist) return;
  const int c = cnt[l];
  const int64_t nr = list_ranges(list_off[l + 1] - list_off[l], range_size);
  int it = item_off[l];
  for (int64_t r = 0; r < nr; r++)
    for (int i = 0; i * per_item < c; i++, it++) {
      item_list[it] = l;
      item_pair[it] = pair_off[l] + i * per_item;
      item_npairs[it] = min(per_item, c - i * per_item);
      item_range[it] = (int32_t)r;
    }
}

// First range slot of every pair (bucketed order) and, at index npairs, the
// total: the ragged rows of the per-pair range merge.
__global__ void pair_rows_kernel(const int32_t *pair_list, const int32_t *pair_off,
                                 const int64_t *list_rbase, const int64_t *list_off,
                                 int64_t range_size, int npairs, int64_t *row_off) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i > npairs) return;
  if (i == npairs) {
    if (npairs == 0) row_off[0] = 0;
    return;
  }
  const int l = pair_list[i];
  const int64_t nr = list_ranges(list_off[l + 1] - list_off[l], range_size);
  row_off[i] = list_rbase[l] + (int64_t)(i - pair_off[l]) * nr;
  if (i == npairs - 1) row_off[npairs] = row_off[i] + nr;
}

// qm of each pair: seq_dot(u_query, centroid_list) (trellis.rs:2120-2183 with
// the list codec's single centroid): one sequential f32 fold per pair, the
// product and the sum rounded separately, from -0.0.  A warp takes 32
// consecutive (bucketed) pairs and stages 32 coordinates at a time in
// shared memory with coalesced loads: the 32 query rows transposed, and the
// centroid chunk once when all 32 pairs are on one list (the usual case:
// a list's pairs are contiguous); lane r then folds row r's 32 products in
// order.  Blocks of kPairQmWarps warps.
__global__ void __launch_bounds__(32 * kPairQmWarps) pair_qm_kernel(
    const float *u, int u_stride, const float *cent, int dim, const int32_t *pair_query,
    const int32_t *pair_list, int npairs, float *qm) {
  __shared__ float su[kPairQmWarps][32][33];
  __shared__ float sc[kPairQmWarps][32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p0 = (blockIdx.x * kPairQmWarps + warp) * 32;
  if (p0 >= npairs) return;  // whole warps; no block barrier below
  const int mine = min(p0 + lane, npairs - 1);
  const int64_t qrow = pair_query[mine];
  const int lrow = pair_list[mine];
  const bool one_list = __all_sync(0xffffffffu, lrow == __shfl_sync(0xffffffffu, lrow, 0));
  float s = -0.0f;
  for (int k0 = 0; k0 < dim; k0 += 32) {
    const int kc = min(32, dim - k0);
    for (int r = 0; r < 32; r++) {
      const int64_t q = __shfl_sync(0xffffffffu, qrow, r);
      if (lane < kc) su[warp][r][lane] = __ldg(u + q * (int64_t)u_stride + k0 + lane);
    }
    if (one_list) {
      if (lane < kc) sc[warp][0][lane] = __ldg(cent + (int64_t)lrow * dim + k0 + lane);
    } else {
      for (int r = 0; r < 32; r++) {
        const int64_t l = __shfl_sync(0xffffffffu, lrow, r);
        if (lane < kc) sc[warp][r][lane] = __ldg(cent + l * dim + k0 + lane);
      }
    }
    __syncwarp();
    const float *cr = one_list ? sc[warp][0] : sc[warp][lane];
    for (int i = 0; i < kc; i++) s = fadd(s, fmul(su[warp][lane][i], cr[i]));
    __syncwarp();  // the chunk is restaged next
  }
  if (p0 + lane < npairs) qm[p0 + lane] = s;
}

// Exact fp32 rerank (ivf.rs:248-274): cosine(query, db[id]) for each of the r
// candidates of a query, then the best k by (cosine desc, id asc).  One warp
// per query; r <= 128.
__global__ void __launch_bounds__(256) rerank_kernel(const RerankParams p) {
  __shared__ uint64_t keys[8][128];
  __shared__ int64_t cid[8][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * 8 + warp;
  if (q >= p.nq) return;
  const float *qv = p.queries + q * (int64_t)p.dim;
  float qs = -0.0f;
  for (int t = 0; t < p.dim; t++) qs = fadd(qs, fmul(qv[t], qv[t]));
  const float na = fsqrt(qs);
  for (int c = lane; c < 128; c += 32) {
    const int64_t id = c < p.r ? p.cand[q * p.r + c] : -1;
    cid[warp][c] = id;
    uint64_t key = 0;
    if (id >= p.n_db) atomicExch(p.err, 1);  // an id that does not index db
    if (id >= 0 && id < p.n_db) {
      const float *x = p.db + id * (int64_t)p.dim;
      float dot = -0.0f, xs = -0.0f;
      for (int t = 0; t < p.dim; t++) {
        const float xv = __ldg(x + t);
        dot = fadd(dot, fmul(qv[t], xv));
        xs = fadd(xs, fmul(xv, xv));
      }
      const float nb = fsqrt(xs);
      const float cs = (na < kF32Eps || nb < kF32Eps) ? 0.0f : fdiv(dot, fmul(na, nb));
      key = ((uint64_t)score_key32(cs) << 32) | (uint32_t)c;
    }
    keys[warp][c] = key;
  }
  __syncwarp();
  // order: key desc, then id asc; ids are compared after the sort below
  for (int size = 2; size <= 128; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < 64; pi += 32) {
        const int lo = 2 * pi - (pi & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = keys[warp][lo], y = keys[warp][hi];
        const int64_t ix = cid[warp][(uint32_t)x], iy = cid[warp][(uint32_t)y];
        const bool x_first = x == 0 ? false
                             : y == 0 ? true
                                      : ((x >> 32) > (y >> 32) || ((x >> 32) == (y >> 32) && ix < iy));
        if (x_first != desc) {
          keys[warp][lo] = y;
          keys[warp][hi] = x;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    const uint64_t key = keys[warp][i];
    const bool ok = i < p.r && key != 0;
    p.out_id[q * p.k + i] = ok ? cid[warp][(uint32_t)key] : -1;
    p.out_score[q * p.k + i] = ok ? key32_score((uint32_t)(key >> 32)) : -INFINITY;
  }
}

template __global__ void seqdot_kernel<0>(const SeqDotParams p);
template __global__ void seqdot_kernel<1>(const SeqDotParams p);

int seqdot_tile() { return SD_T; }

}  // namespace uvb
