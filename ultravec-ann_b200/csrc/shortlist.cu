// shortlist.cu -- the 1-bit companion shortlist search (src/trellis.rs:841-948;
// the IVF arm IvfCodec::TrellisShortlist, src/ivf.rs:52-60, 111-135).
//
// Stage 1 ranks every entry of a codec by a cheap similarity to the query's
// rotated direction q_r: the Hamming form dim - 2 * popcount(q_bits ^ sign)
// (src/trellis.rs:2251-2266) or the asymmetric masked sum, a sequential fold
// of +-q_r[i] by the entry's sign bits (2271-2279), times the entry's rnorm
// under centering.  The best C = min(max(c, k), len) entries are kept --
// ties go to the lower entry, where the reference's select_nth_unstable
// leaves them unspecified -- and stage 2 scores only those with the search
// estimator qm + rnorm * (dot / rescale) and returns the top k.
//
// One CTA per (query, list) pair (the flat index is one list).  Stage 1
// streams the list 256 entries at a time; an entry whose 64-bit key
// (similarity, then ~entry) beats the running threshold (the C-th best key
// so far) is appended to a shared buffer, which is bitonic-sorted into the
// kept top region when it could overflow.  Stage 2 gives every kept entry a
// thread (record_dot_thread, the reference's FMA association), sorts the
// ranking keys and writes the top k.
#include "uv_common.cuh"
#include "uv_kernels.h"
#include "uv_score_thread.cuh"

namespace uvb {

namespace {

constexpr int kSlThreads = 256;

// descending bitonic sort of keys[0, n), n a power of two
__device__ __forceinline__ void sort_desc(uint64_t *keys, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < n / 2; i += kSlThreads) {
        const int lo = 2 * i - (i & (stride - 1));
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
}

}  // namespace

template <int BITS, bool ASYM>
__global__ void __launch_bounds__(kSlThreads) shortlist_kernel(const ShortlistParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int cp = p.cp;
  uint64_t *keys = (uint64_t *)sm;                             // 2 * cp
  float *qv = (float *)(keys + 2 * cp);                        // q_stride
  uint32_t *qbits = (uint32_t *)(qv + p.q_stride);             // sign_stride / 4
  float *table = (float *)(qbits + p.sign_stride / 4);         // table_len
  __shared__ int app_s, kept_s;
  __shared__ uint64_t thr_s;
  __shared__ float qm_s;

  const int tid = threadIdx.x;
  const int64_t pair = blockIdx.x;
  const int64_t q = pair / p.per_query;
  int64_t r0 = 0, r1 = p.n_flat;
  int list = -1;
  if (p.lists) {
    list = p.lists[pair];
    r0 = list >= 0 ? p.list_off[list] : 0;
    r1 = list >= 0 ? p.list_off[list + 1] : 0;
  }
  const int64_t len = r1 - r0;
  int64_t *oid = p.out_id + pair * p.k;
  float *osc = p.out_score + pair * p.k;
  if (len <= 0 || p.degenerate[q]) {
    for (int i = tid; i < p.k; i += kSlThreads) {
      oid[i] = -1;
      osc[i] = -INFINITY;
    }
    return;
  }
  const int ce = (int)min((int64_t)max(p.cs, p.k), len);

  // ---- query side: q_r, its sign bits, the table, qm of a centered list ----
  const float *qsrc = p.q_r + q * (int64_t)p.q_stride;
  for (int i = tid; i < p.q_stride; i += kSlThreads) qv[i] = qsrc[i];
  for (int i = tid; i < p.table_len; i += kSlThreads) table[i] = __ldg(p.code + i);
  for (int i = tid; i < 2 * cp; i += kSlThreads) keys[i] = kEmptyKey;
  if (tid == 0) {
    app_s = 0;
    kept_s = 0;
    thr_s = kEmptyKey;
    float qm = 0.0f;  // qc.get(0).unwrap_or(0.0): 0 without a centroid
    if (p.u != nullptr && list >= 0) {
      const float *a = p.u + q * (int64_t)p.u_stride;
      const float *c = p.centroids + (int64_t)list * p.dim;
      float s = -0.0f;  // <u, c_list>, the reference's sequential dot
      for (int t = 0; t < p.dim; t++) s = fadd(s, fmul(a[t], __ldg(c + t)));
      qm = s;
    }
    qm_s = qm;
  }
  __syncthreads();
  for (int w = tid; w < p.sign_stride / 4; w += kSlThreads) {
    uint32_t word = 0;  // big-endian bytes of pack_indices(q_r > 0, 1) as loaded
#pragma unroll
    for (int b = 0; b < 4; b++) {
      uint32_t byte = 0;
#pragma unroll
      for (int t = 0; t < 8; t++) {
        const int i = (w * 4 + b) * 8 + t;
        if (i < p.dim && qv[i] > 0.0f) byte |= 0x80u >> t;
      }
      word |= byte << (8 * b);
    }
    qbits[w] = word;
  }
  __syncthreads();

  // ---- stage 1: the C best entries by sign-code similarity ----
  const int swords = (p.dim + 31) >> 5;  // sign words that carry bits
  for (int64_t t0 = 0; t0 < len; t0 += kSlThreads) {
    const int64_t li = t0 + tid;
    if (li < len) {
      const int64_t r = r0 + li;
      const uint32_t *sg = (const uint32_t *)(p.signs + r * (int64_t)p.sign_stride);
      float sim;
      if constexpr (ASYM) {
        float s = 0.0f;
        for (int w = 0; w < swords; w++) {
          const uint32_t word = __byte_perm(__ldg(sg + w), 0, 0x0123);  // bit 31 = entry 32w
          const int nb = min(32, p.dim - 32 * w);
          for (int t = 0; t < nb; t++) {
            const float x = qv[32 * w + t];
            s = fadd(s, ((word >> (31 - t)) & 1u) ? x : -x);
          }
        }
        sim = s;
      } else {
        uint32_t h = 0;
        for (int w = 0; w < swords; w++) h += __popc(__ldg(sg + w) ^ qbits[w]);
        sim = fsub((float)p.dim, fmul(2.0f, (float)h));
      }
      if (p.weight) sim = fmul(p.rnorm ? __ldg(p.rnorm + r) : 1.0f, sim);
      const uint64_t key =
          ((uint64_t)score_key32(sim) << 32) | (uint64_t)(0xffffffffu - (uint32_t)li);
      if (key > thr_s) {
        // at most one append per thread per tile, into a region merged before
        // it can hold more than cp - 256 keys: slot < cp always
        const int slot = atomicAdd(&app_s, 1);
        if (slot < cp) keys[cp + slot] = key;
      }
    }
    __syncthreads();
    const int app = app_s;
    // every thread holds the same count before the next tile appends to it,
    // so the merge below is entered by all threads or by none
    __syncthreads();
    if (app > cp - kSlThreads || (t0 + kSlThreads >= len && app > 0)) {
      sort_desc(keys, 2 * cp);
      if (tid == 0) {
        kept_s = min(cp, kept_s + app);
        app_s = 0;
        if (kept_s >= ce) thr_s = keys[ce - 1];
      }
      for (int i = cp + tid; i < 2 * cp; i += kSlThreads) keys[i] = kEmptyKey;
      __syncthreads();
    }
  }

  // ---- stage 2: the estimator on the kept entries, top k ----
  int cp2 = 32;
  while (cp2 < ce) cp2 <<= 1;
  uint64_t *k2 = keys + cp;
  for (int i = tid; i < cp2; i += kSlThreads) {
    uint64_t key = kEmptyKey;
    if (i < ce) {
      const uint32_t li = 0xffffffffu - (uint32_t)(keys[i] & 0xffffffffu);
      const int64_t r = r0 + li;
      const float dot = record_dot_thread<BITS>(qv, p.codes + r * (int64_t)p.code_stride,
                                                __ldg(p.start + r), p.dim, p.mem,
                                                p.code_stride, table, 1, 0);
      float qm = qm_s;  // IVF: <u, c_list> (0 uncentered)
      if (p.n_centroids > 0) {  // flat centered: qc[cidx] (src/trellis.rs:2153)
        const uint32_t ci = p.cidx ? __ldg(p.cidx + r) : 0u;
        qm = ci < (uint32_t)p.n_centroids ? __ldg(p.qc + q * p.n_centroids + ci) : 0.0f;
      }
      const float rn = p.rnorm ? __ldg(p.rnorm + r) : 1.0f;
      const float s = fadd(qm, fmul(rn, fdiv(dot, __ldg(p.rescale + r))));
      key = rank_key(s, li);
    }
    k2[i] = key;
  }
  __syncthreads();
  sort_desc(k2, cp2);
  for (int i = tid; i < p.k; i += kSlThreads) {
    const uint64_t key = i < cp2 ? k2[i] : kEmptyKey;
    const bool full = key != kEmptyKey;
    const int64_t r = r0 + rank_key_index(key);
    oid[i] = full ? (p.ids ? p.ids[r] : r) : -1;
    osc[i] = full ? key32_score((uint32_t)(key >> 32)) : -INFINITY;
  }
}

const void *shortlist_kernel_ptr(int bits, bool asym) {
#define UV_SL_CASE(b)                                                                 \
  case b:                                                                             \
    return asym ? (const void *)shortlist_kernel<b, true> : (const void *)shortlist_kernel<b, false>;
  switch (bits) {
    UV_SL_CASE(1)
    UV_SL_CASE(2)
    UV_SL_CASE(3)
    UV_SL_CASE(4)
  }
#undef UV_SL_CASE
  return nullptr;
}

size_t shortlist_smem_bytes(int cp, int q_stride, int sign_stride, int table_len) {
  return (size_t)2 * cp * 8 + (size_t)q_stride * 4 + (size_t)sign_stride + (size_t)table_len * 4;
}

}  // namespace uvb
