// rank.cu -- full ranking of every record for searches whose k exceeds the
// fused top-k capacity of the scan kernels.
//
// The reference's search scores every entry, sorts all of them by score and
// truncates to `limit` (src/trellis.rs:2120-2183); its MIPS harness asks for
// limit = len() and re-ranks the whole list by the row norm
// (src/bench.rs:1029-1045).  Here the scan kernels write every (query,
// record) score key and id (ScanParams::all_key), and this file sorts each
// query's segment of n elements by (score key descending, id ascending):
//   1. rank_tile_sort_kernel: bitonic sort of tiles of kRankTile elements in
//      shared memory;
//   2. rank_merge_kernel: merge passes over pairs of sorted runs (merge path:
//      every thread finds its output diagonal by binary search, then merges
//      eight elements); runs keep only their best `klim` elements, since no
//      later element of a run can reach a query's top k;
//   3. rank_emit_kernel: the first k of each segment (unfilled slots and
//      degenerate queries give id -1 and score -inf).
#include "uv_kernels.h"

namespace uvb {

namespace {

constexpr int kRankThreads = 256;
constexpr int kRankPer = 8;  // outputs per thread of a merge pass

__device__ __forceinline__ bool rk_better(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
  return ka > kb || (ka == kb && ia < ib);
}

}  // namespace

// One CTA sorts tile blockIdx.x of segment blockIdx.y in place.  Padding
// slots hold key 0, which no score reaches (score_key32 of every score,
// -inf included, is above 0), so they sort last and are never written.
__global__ void __launch_bounds__(kRankThreads) rank_tile_sort_kernel(uint32_t *key, int64_t *id,
                                                                      int64_t n) {
  __shared__ uint32_t sk[kRankTile];
  __shared__ int64_t si[kRankTile];
  const int64_t seg = blockIdx.y;
  const int64_t lo = (int64_t)blockIdx.x * kRankTile;
  const int cnt = (int)min((int64_t)kRankTile, n - lo);
  uint32_t *kp = key + seg * n + lo;
  int64_t *ip = id + seg * n + lo;
  for (int i = threadIdx.x; i < kRankTile; i += kRankThreads) {
    const bool ok = i < cnt;
    sk[i] = ok ? kp[i] : 0u;
    si[i] = ok ? ip[i] : INT64_MAX;
  }
  __syncthreads();
  for (int size = 2; size <= kRankTile; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = threadIdx.x; pi < kRankTile / 2; pi += kRankThreads) {
        const int i = ((pi & ~(stride - 1)) << 1) | (pi & (stride - 1));
        const int j = i + stride;
        const bool desc = (i & size) == 0;
        const uint32_t ka = sk[i], kb = sk[j];
        const int64_t ia = si[i], ib = si[j];
        const bool swap = desc ? rk_better(kb, ib, ka, ia) : rk_better(ka, ia, kb, ib);
        if (swap) {
          sk[i] = kb;
          sk[j] = ka;
          si[i] = ib;
          si[j] = ia;
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < cnt; i += kRankThreads) {
    kp[i] = sk[i];
    ip[i] = si[i];
  }
}

// Runs [r*w, (r+1)*w) of every segment are sorted, of which the first
// min(len, klim) elements are valid; merge runs 2p and 2p+1 into run p of
// width 2w (first min(len, klim) elements written).  A CTA covers
// kRankThreads * kRankPer consecutive outputs of one merged run (w is a
// multiple of that span, so no CTA straddles two runs).  Equal elements
// take the first run's first (stable).
__global__ void __launch_bounds__(kRankThreads) rank_merge_kernel(const uint32_t *ik,
                                                                  const int64_t *ii, uint32_t *ok,
                                                                  int64_t *oi, int64_t n,
                                                                  int64_t w, int64_t klim) {
  const int64_t seg = blockIdx.y;
  const int64_t out_lo = (int64_t)blockIdx.x * (kRankThreads * kRankPer);
  const int64_t base = out_lo / (2 * w) * (2 * w);
  const int64_t a1 = min(base + w, n), b1 = min(base + 2 * w, n);
  const int64_t la = min(a1 - base, klim), lb = min(b1 - a1, klim);
  const int64_t total = min(la + lb, klim);
  const int64_t d0 = out_lo - base + (int64_t)threadIdx.x * kRankPer;
  if (d0 >= total) return;
  const uint32_t *ak = ik + seg * n + base;
  const int64_t *ai = ii + seg * n + base;
  const uint32_t *bk = ik + seg * n + a1;
  const int64_t *bi = ii + seg * n + a1;
  // the number of first-run elements among the first d0 outputs: the
  // smallest i whose A[i] is placed after B[d0 - 1 - i]
  int64_t lo = max((int64_t)0, d0 - lb), hi = min(d0, la);
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    const int64_t jb = d0 - 1 - mid;
    if (rk_better(bk[jb], bi[jb], ak[mid], ai[mid]))
      hi = mid;
    else
      lo = mid + 1;
  }
  int64_t ia = lo, ib = d0 - lo;
  uint32_t *okp = ok + seg * n + base;
  int64_t *oip = oi + seg * n + base;
#pragma unroll
  for (int j = 0; j < kRankPer; j++) {
    const int64_t o = d0 + j;
    if (o >= total) break;
    bool take_a;
    if (ia >= la)
      take_a = false;
    else if (ib >= lb)
      take_a = true;
    else
      take_a = !rk_better(bk[ib], bi[ib], ak[ia], ai[ia]);
    if (take_a) {
      okp[o] = ak[ia];
      oip[o] = ai[ia];
      ia++;
    } else {
      okp[o] = bk[ib];
      oip[o] = bi[ib];
      ib++;
    }
  }
}

// Slot i < k of query q: element i of its sorted segment, or an unfilled
// slot (id -1, score -inf) past n, for a degenerate query (degen may be
// null) or for an empty entry (key 0).
__global__ void rank_emit_kernel(const uint32_t *key, const int64_t *id, int64_t n, int64_t nq,
                                 int64_t k, const uint32_t *degen, int64_t *out_id,
                                 float *out_score) {
  const int64_t total = nq * k;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = e / k, i = e - q * k;
    const bool fill = i < n && (degen == nullptr || degen[q] == 0u) && key[q * n + i] != 0u;
    out_id[e] = fill ? id[q * n + i] : -1;
    if (out_score != nullptr) out_score[e] = fill ? key32_score(key[q * n + i]) : -INFINITY;
  }
}

// Row q of a merge (MergeParams layout) as one sort segment of `total`
// entries: keys[q * total + i], ids[q * total + i]; empty entries (id < 0)
// get key 0, below every score.
__global__ void rank_gather_kernel(const MergeParams p, int64_t total, uint32_t *keys,
                                   int64_t *ids) {
  const int64_t list_stride = p.list_stride > 0 ? p.list_stride : p.k_in;
  const int64_t row_stride = p.row_stride > 0 ? p.row_stride : (int64_t)p.n_lists * p.k_in;
  const int64_t all = p.nq * total;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < all;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = e / total, i = e - q * total;
    const int64_t l = i / p.k_in, j = i - l * p.k_in;
    const int64_t src = q * row_stride + l * list_stride + j;
    int64_t id;
    uint32_t key;
    if (p.in_packed) {
      const int32_t *r = p.in_packed + 3 * src;
      id = (int64_t)(((uint64_t)(uint32_t)r[1] << 32) | (uint32_t)r[0]);
      key = score_key32(__int_as_float(r[2]));
    } else {
      id = p.in_id[src];
      key = p.in_key ? p.in_key[src] : score_key32(p.in_score[src]);
    }
    keys[e] = id < 0 ? 0u : key;
    ids[e] = id;
  }
}

__global__ void fill_value_kernel(float *out, int64_t n, float v) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x)
    out[e] = v;
}

int rank_merge_span() { return kRankThreads * kRankPer; }

}  // namespace uvb
