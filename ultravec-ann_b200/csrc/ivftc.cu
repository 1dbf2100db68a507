// ivftc.cu -- the IVF list scan on the tensor cores (sm_100a).
//
// An IVF search scores, for every probed (query, list) pair, the list's
// records (src/ivf.rs:229-239; trellis.rs:1483-1536): score = qm + rnorm *
// (dot / rescale), qm = <u, c_list> for centered lists.  Scoring every pair
// exactly is FP32-issue bound on the CUDA cores.  Here the certified fp16
// bounds of the flat prefilter (tcscan.cu: record operand rows B' = fp16(g x
// s), bound constants C' in an extra K slice, s a power of two) are taken per
// work item = (posting list, up to 128 of its probing pairs, a range of at
// most 512 of the list's records):
//
//   MMA      D = A . B'^T - C' over the item's pairs (A: the fp16 query rows
//            of the pairs, gathered in bucketed order) and the range's
//            records, 128 x 256 per tile, both tiles of a range held in TMEM
//            (512 columns), so every bound is read from TMEM, never
//            recomputed;
//   lower    lb = fadd_rd(s qm, D) <= s * score: the reference adds qm last
//            (fadd), and D <= s * rnorm * (dot / rescale) (the extra slice);
//   upper    ub = fadd_ru(s qm, fadd_ru(D, 2 C')) >= s * score (D + 2 C' is
//            the MMA's upper bound D + C' formed outside it, rounded up);
//   theta    the k-th largest lb of the range (per pair, a sorted register
//            list): k records of the range reach it;
//   keep     every record with ub >= theta, with its lb and ub, appended to
//            a compact store (one reservation per warp).
//
// ivf_select_kernel then works per query: theta0 = the largest slot
// threshold (a score k records reach), theta_q = the k-th largest lb over
// the query's kept records at or above theta0 (every record with lb >=
// theta0 was kept, so this is the k-th largest lb over all its probed
// records), and the kept records with ub >= theta_q are scored exactly --
// the reference's association and estimator -- and ranked by (score desc,
// id asc).  The exact top k is among them, ties included.  A store or list
// that overflows sends the search to the CUDA-core scan.
//
// tc_ivf_kernel's warps: 0-3 epilogue (TMEM lane quarter w, thread = pair
// row), 4 TMEM allocation and MMA issue, 5 TMA.  Boxes of 32 rows load only
// the rows that hold pairs or records (rows past them keep stale values,
// which reach only accumulator rows and columns that are never read).  No
// cluster multicast; every wait is bounded.
#include <cuda.h>
#include <cuda_fp16.h>

#include "uv_kernels.h"
#include "uv_score_thread.cuh"
#include "uv_tc.cuh"

namespace uvb {

namespace {

constexpr int V_M = kIvfTcRows;           // pair rows per CTA
constexpr int V_N = 256;                  // records per tile
constexpr int V_TILES = kIvfTcRange / V_N;
constexpr int V_STAGES = 4;
constexpr int V_EPI = 4;                  // epilogue warps
constexpr int V_THREADS = (V_EPI + 2) * 32;
constexpr int V_BOX = 32;                 // rows per TMA box
constexpr int V_A = V_M * 128;            // 128 x 64 fp16 query chunk
constexpr int V_B = V_N * 128;            // 256 x 64 fp16 record chunk
constexpr int V_STAGE = V_A + V_B;        // 48 KB
constexpr int V_BARS = V_STAGES * V_STAGE;
constexpr int V_CP = V_BARS + 16 * 8;     // 2 C' of the range's records
constexpr int V_MISC = V_CP + kIvfTcRange * 4;
constexpr int V_TOTAL = V_MISC + 64;
constexpr uint32_t kWaitLimit = 1u << 20;
static_assert(V_STAGE % 1024 == 0 && V_A % 1024 == 0, "stage alignment");
static_assert(2 * V_STAGES + V_TILES + 1 <= 16, "barrier slots");
static_assert(V_TILES * V_N <= 512, "TMEM columns");
static_assert(V_TOTAL <= 227 * 1024, "shared memory");

// the bits of a float as an unsigned key of the same order, and back
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_order(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

}  // namespace

template <int KT>
__global__ void __launch_bounds__(V_THREADS, 1)
    tc_ivf_kernel(const TcIvfParams p, const __grid_constant__ CUtensorMap tmap_a,
                  const __grid_constant__ CUtensorMap tmap_ax,
                  const __grid_constant__ CUtensorMap tmap_b,
                  const __grid_constant__ CUtensorMap tmap_bx) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t *full = (uint64_t *)(sm + V_BARS);  // [V_STAGES]
  uint64_t *empty = full + V_STAGES;           // [V_STAGES]
  uint64_t *accf = empty + V_STAGES;           // [V_TILES]
  uint64_t *drained = accf + V_TILES;          // MMAs done after an abort
  float *c2_s = (float *)(sm + V_CP);          // [kIvfTcRange]
  uint32_t *tbase_s = (uint32_t *)(sm + V_MISC);
  volatile int *abort_s = (volatile int *)(sm + V_MISC + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.x;
  if (item >= *p.n_items) return;  // before any barrier: the whole CTA leaves
  const int l = p.item_list[item];
  const int p0 = p.item_pair[item];
  const int npr = p.item_npairs[item];
  const int rg = p.item_range[item];
  const int64_t L0 = p.list_off[l], L1 = p.list_off[l + 1];
  const int64_t nr = (L1 - L0) <= p.range_size ? 1 : (L1 - L0 + p.range_size - 1) / p.range_size;
  const int64_t lo = min(L1, L0 + (int64_t)rg * p.range_size);
  const int nrec = (int)min((int64_t)kIvfTcRange, min(L1, lo + p.range_size) - lo);
  const int ntiles = (nrec + V_N - 1) / V_N;
  const int steps = p.kchunks + 1;  // K chunks of 64, then the extra slice
  const int na = (npr + V_BOX - 1) / V_BOX;

  if (tid == 0) {
    for (int s = 0; s < V_STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int t = 0; t < V_TILES; t++) tc::mbar_init(&accf[t], 1);
    tc::mbar_init(drained, 1);
    *abort_s = 0;
    tc::mbar_fence_init();
  }
  // 2 C' of the range's records (C' is an fp16 value: doubling it is exact)
  for (int c = tid; c < nrec; c += V_THREADS)
    c2_s[c] = 2.0f * __half2float(__ushort_as_half(__ldg(p.xext + (lo + c) * 16)));
  if (warp == V_EPI) tc::tmem_alloc(tbase_s, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tbase_s;

  if (warp < V_EPI) {
    // ================= epilogue: thread = pair row =================
    const int row = warp * 32 + lane;
    const bool has = row < npr;
    const int pp = p0 + row;
    bool ok = false;
    float sqm_lo = 0.0f, sqm_hi = 0.0f;
    if (has) {
      ok = p.degenerate[p.pair_query[pp]] == 0u;
      if (p.pair_qm != nullptr) {
        const float s = *p.scale, qm = p.pair_qm[pp];
        sqm_lo = __fmul_rd(s, qm);
        sqm_hi = __fmul_ru(s, qm);
      }
    }
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    float tk[KT];  // the KT largest lower bounds so far, descending
#pragma unroll
    for (int i = 0; i < KT; i++) tk[i] = -INFINITY;
    bool alive = true;
    for (int t = 0; t < ntiles; t++) {
      if (!tc::mbar_wait(&accf[t], 0, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (__any_sync(0xffffffffu, *abort_s != 0)) {
        alive = false;
        break;
      }
      tc::tc_fence_after();
      for (int c0 = t * V_N; c0 < min(nrec, (t + 1) * V_N); c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld32(lane_base + (uint32_t)c0, r);
        tc::tmem_ld_wait();
        if (!ok) continue;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          float x = __fadd_rd(sqm_lo, __uint_as_float(r[j]));
          if (c0 + j < nrec && x > tk[KT - 1]) {
#pragma unroll
            for (int i = 0; i < KT; i++) {
              const float top = fmaxf(tk[i], x);
              x = fminf(tk[i], x);
              tk[i] = top;
            }
          }
        }
      }
    }
    // the k-th largest lower bound (-inf when the range holds fewer than k
    // records with finite bounds: every record is then kept)
    float theta = tk[0];
#pragma unroll
    for (int i = 1; i < KT; i++)
      if (i < p.k) theta = tk[i];
    // count, reserve (one atomic per warp), then store
    int cnt = 0;
    if (alive) {
      for (int c0 = 0; c0 < nrec; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld32(lane_base + (uint32_t)c0, r);
        tc::tmem_ld_wait();
        if (!ok) continue;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          if (c0 + j < nrec) {
            const float ub = __fadd_ru(sqm_hi, __fadd_ru(__uint_as_float(r[j]), c2_s[c0 + j]));
            cnt += !(ub < theta) ? 1 : 0;  // a NaN bound (C' = +inf) is kept
          }
        }
      }
    }
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int wtot = __shfl_sync(0xffffffffu, incl, 31);
    unsigned long long wbase = 0ull;
    if (lane == 31 && wtot > 0) wbase = atomicAdd(p.cand_used, (unsigned long long)wtot);
    wbase = __shfl_sync(0xffffffffu, wbase, 31);
    const int64_t base = (int64_t)wbase + (incl - cnt);
    const bool fits = base + cnt <= p.cand_cap;
    if (alive && __any_sync(0xffffffffu, ok && fits && cnt > 0)) {
      int pos = 0;
      for (int c0 = 0; c0 < nrec; c0 += 32) {
        uint32_t r[32];
        tc::tmem_ld32(lane_base + (uint32_t)c0, r);
        tc::tmem_ld_wait();
        if (!ok || !fits) continue;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          if (c0 + j < nrec) {
            const float d = __uint_as_float(r[j]);
            const float ub = __fadd_ru(sqm_hi, __fadd_ru(d, c2_s[c0 + j]));
            if (!(ub < theta)) {
              const int64_t e = base + pos++;
              p.cand_rec[e] = (uint32_t)(lo + c0 + j);
              p.cand_lb[e] = __fadd_rd(sqm_lo, d);
              p.cand_ub[e] = ub;
            }
          }
        }
      }
    }
    if (has) {
      const int64_t slot = p.list_rbase[l] + (int64_t)(pp - p.list_pair_off[l]) * nr + rg;
      p.slot_cnt[slot] = !alive ? -1 : (!ok ? 0 : (fits ? cnt : -1));
      p.slot_base[slot] = base;
      // the query's theta0: the largest slot threshold (a score k records reach)
      if (ok && theta > -INFINITY)
        atomicMax(p.q_theta0 + p.pair_query[pp], order_key(theta));
      if (alive && ok && !fits) atomicOr(p.err, 2);  // the store is full
    }
  } else if (warp == V_EPI) {
    if (lane == 0) {
      // ================= MMA issue =================
      const uint32_t idesc = tc::idesc_f16_f32(V_M, V_N);
      int64_t step = 0;
      for (int t = 0; t < ntiles && !*abort_s; t++) {
        const uint32_t d = tmem + (uint32_t)(t * V_N);
        for (int k = 0; k < steps; k++, step++) {
          const int s = (int)(step % V_STAGES);
          if (!tc::mbar_wait(&full[s], (uint32_t)((step / V_STAGES) & 1), kWaitLimit)) {
            *abort_s = 1;
            atomicExch(p.err, 1);
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_base = tc::smem_u32(sm + s * V_STAGE);
          const uint32_t b_base = a_base + V_A;
          if (k < p.kchunks) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
              const uint32_t off = (uint32_t)(kk * 32);  // 16 fp16 = 32 B per K step
              tc::mma_f16(d, tc::sw128_desc(a_base + off), tc::sw128_desc(b_base + off), idesc,
                          (k > 0 || kk > 0) ? 1u : 0u);
            }
          } else {
            tc::mma_f16(d, tc::sw32_desc(a_base), tc::sw32_desc(b_base), idesc, 1u);
          }
          tc::mma_commit(&empty[s]);
        }
        if (*abort_s) break;
        tc::mma_commit(&accf[t]);
      }
      if (*abort_s) {  // let every issued MMA finish before TMEM is freed
        tc::mma_commit(drained);
        tc::mbar_wait(drained, 0, kWaitLimit);
      }
    }
  } else if (lane == 0) {
    // ================= TMA producer =================
    int64_t step = 0;
    for (int t = 0; t < ntiles && !*abort_s; t++) {
      const int row_b = (int)(lo + (int64_t)t * V_N);
      const int nb = (min(V_N, nrec - t * V_N) + V_BOX - 1) / V_BOX;
      for (int k = 0; k < steps; k++, step++) {
        const int s = (int)(step % V_STAGES);
        if (*abort_s ||
            !tc::mbar_wait(&empty[s], (uint32_t)(((step / V_STAGES) & 1) ^ 1), kWaitLimit)) {
          *abort_s = 1;
          atomicExch(p.err, 1);
          break;
        }
        uint8_t *dst = sm + s * V_STAGE;
        if (k < p.kchunks) {
          // boxes of 32 rows x 64 fp16 (4 KB): the 128-byte swizzle repeats
          // every 1 KB, so boxes at 4 KB offsets make the layout of one tile
          tc::mbar_arrive_expect_tx(&full[s], (uint32_t)((na + nb) * V_BOX * 128));
          for (int b = 0; b < na; b++)
            tc::tma_load_2d(dst + b * V_BOX * 128, &tmap_a, 64 * k, p0 + V_BOX * b, &full[s]);
          for (int b = 0; b < nb; b++)
            tc::tma_load_2d(dst + V_A + b * V_BOX * 128, &tmap_b, 64 * k, row_b + V_BOX * b,
                            &full[s]);
        } else {
          // the extra slices: -1 in element 0 of every pair row (one 128-row
          // box of a constant map), C' of every record row (boxes of 32 x 16)
          tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(V_M * 32 + nb * V_BOX * 32));
          tc::tma_load_2d(dst, &tmap_ax, 0, 0, &full[s]);
          for (int b = 0; b < nb; b++)
            tc::tma_load_2d(dst + V_A + b * V_BOX * 32, &tmap_bx, 0, row_b + V_BOX * b, &full[s]);
        }
      }
    }
    if (*abort_s) tc::drain_stages(full, V_STAGES, step, kWaitLimit);
  }

  // ---- teardown: the epilogue has waited for every MMA ----
  tc::tc_fence_before();
  __syncthreads();
  if (warp == V_EPI) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
    tc::tmem_relinquish();
  }
}

namespace {

// (key desc, id asc): the merges' order (score_key32 keys)
__device__ __forceinline__ bool key_id_before(uint32_t ka, int64_t ia, uint32_t kb, int64_t ib) {
  return ka > kb || (ka == kb && ia < ib);
}

struct SelWarp {
  int n_lb, n_c;
};



// Calls fn(entry, qm) for every kept record of query q's slots, the warp's
// lanes spread over the slots: probes in chunks of 32 (lane j: probe j0 + j,
// its bucketed pair and slot range), then the chunk's slots in turn, each
// lane finding its slot's probe by a bisection over the chunk's prefix.
template <class Fn>
__device__ __forceinline__ void for_each_entry(const IvfSelectParams &p, int64_t q, int lane,
                                               Fn fn) {
  for (int j0 = 0; j0 < p.np; j0 += 32) {
    const int j = j0 + lane;
    int pp = -1;
    if (j < p.np) pp = p.pair_of[q * p.np + j];
    int64_t s0 = 0;
    int ns = 0;
    float qm = 0.0f;
    if (pp >= 0) {
      s0 = p.row_off[pp];
      ns = (int)(p.row_off[pp + 1] - s0);
      if (p.pair_qm != nullptr) qm = p.pair_qm[pp];
    }
    int incl = ns;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int ex = incl - ns;
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    for (int t0 = 0; t0 < total; t0 += 32) {
      const int t = t0 + lane;
      // the last lane whose first slot is at or before t
      int lo = 0, hi = 31;
#pragma unroll
      for (int it = 0; it < 5; it++) {
        const int mid = (lo + hi + 1) >> 1;
        const int v = __shfl_sync(0xffffffffu, ex, mid);
        if (v <= t) lo = mid;
        else hi = mid - 1;
      }
      const int64_t so = __shfl_sync(0xffffffffu, s0, lo);
      const int eo = __shfl_sync(0xffffffffu, ex, lo);
      const float qo = __shfl_sync(0xffffffffu, qm, lo);
      if (t < total) {
        const int64_t slot = so + (t - eo);
        const int c = p.slot_cnt[slot];
        const int64_t b0 = p.slot_base[slot];
        for (int i = 0; i < c; i++) fn(b0 + i, qo);
      }
    }
  }
}

}  // namespace

// One warp per query (kIvfSelWarps per CTA): the query-wide threshold over
// its slots, the exact scores of the kept records that reach it (half a
// warp per record: 16 lanes = the 16 FMA chains of simd.rs:202-262, then the
// hsum256 tree), and the top k.  A query with an overflowed slot or more
// candidates than the per-query store holds is counted in *n_over.
template <int BITS>
__global__ void __launch_bounds__(32 * kIvfSelWarps) ivf_select_kernel(const IvfSelectParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rw = p.code_stride >> 2;
  float *table = (float *)sm;
  const int img_words = (2 * (rw + 1) + 3) & ~3;
  uint8_t *wbase = sm + (((size_t)p.table_len * 4 + 15) & ~(size_t)15) +
                   (size_t)warp * ((size_t)img_words * 4 + kIvfSelLb * 4 + kIvfSelCand * 20 + 16);
  uint32_t *img = (uint32_t *)wbase;                        // 2 x (rw + 1)
  float *lbv = (float *)(img + img_words);                  // kIvfSelLb
  uint32_t *crec = (uint32_t *)(lbv + kIvfSelLb);           // kIvfSelCand
  float *cqm = (float *)(crec + kIvfSelCand);               // kIvfSelCand
  uint32_t *ckey = (uint32_t *)(cqm + kIvfSelCand);         // kIvfSelCand
  int64_t *cid = (int64_t *)(ckey + kIvfSelCand);           // kIvfSelCand
  SelWarp *cw = (SelWarp *)(cid + kIvfSelCand);
  for (int e = tid; e < p.table_len; e += 32 * kIvfSelWarps) table[e] = __ldg(p.code + e);
  __syncthreads();
  const int64_t q = (int64_t)blockIdx.x * kIvfSelWarps + warp;
  if (q >= p.nq) return;  // whole warps, after the only block barrier
  int64_t *out_id = p.out_id + q * p.k;
  float *out_score = p.out_score + q * p.k;
  if (p.degenerate[q]) {
    for (int i = lane; i < p.k; i += 32) {
      out_id[i] = -1;
      out_score[i] = -INFINITY;
    }
    return;
  }
  // theta0: the largest slot threshold (tc_ivf_kernel's atomicMax; key 0:
  // no slot of this query holds k records)
  const uint32_t th0_key = p.q_theta0[q];
  const float th0 = th0_key == 0u ? -INFINITY : key_order(th0_key);
  if (lane == 0) {
    cw->n_lb = 0;
    cw->n_c = 0;
  }
  __syncwarp();
  // theta_q: the k-th largest lower bound at or above theta0 (at least k:
  // the records behind theta0's own slot)
  float thq = -INFINITY;
  if (th0 > -INFINITY) {
    for_each_entry(p, q, lane, [&](int64_t e, float) {
      const float lb = p.cand_lb[e];
      if (lb >= th0) {
        const int pos = atomicAdd(&cw->n_lb, 1);
        if (pos < kIvfSelLb) lbv[pos] = lb;
      }
    });
    __syncwarp();
    const int nlb = cw->n_lb;
    if (nlb > kIvfSelLb) {
      // more than the store holds (long lists split into many ranges, each
      // with its own threshold): a most-significant-digit radix select over
      // the same entries, 8 bits of the ordered key per pass, the 256-bin
      // histogram in lbv
      uint32_t *hist = (uint32_t *)lbv;
      uint32_t prefix = 0u, mask = 0u;
      int kk = p.k;  // rank still to find among the entries matching prefix
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0u;
        __syncwarp();
        for_each_entry(p, q, lane, [&](int64_t e, float) {
          const float lb = p.cand_lb[e];
          const uint32_t key = order_key(lb);
          if (lb >= th0 && (key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        });
        __syncwarp();
        // lane l sums bins 8l .. 8l + 7; suffix sums from the top bin down
        uint32_t mine = 0u;
#pragma unroll
        for (int t = 0; t < 8; t++) mine += hist[8 * lane + t];
        uint32_t suf = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
          if (lane + o < 32) suf += v;
        }
        // the lane whose bins hold the kk-th largest: suffix through it >= kk,
        // suffix above it < kk
        const bool here = suf >= (uint32_t)kk && suf - mine < (uint32_t)kk;
        const int owner = __ffs(__ballot_sync(0xffffffffu, here)) - 1;
        int bin = 0, above = 0;
        if (lane == owner) {
          uint32_t acc = suf - mine;
          for (int t = 7; t >= 0; t--) {
            const uint32_t h = hist[8 * lane + t];
            if (acc + h >= (uint32_t)kk) {
              bin = 8 * lane + t;
              above = (int)acc;
              break;
            }
            acc += h;
          }
        }
        bin = __shfl_sync(0xffffffffu, bin, owner < 0 ? 0 : owner);
        above = __shfl_sync(0xffffffffu, above, owner < 0 ? 0 : owner);
        prefix |= (uint32_t)bin << shift;
        mask |= 255u << shift;
        kk -= above;
        __syncwarp();  // the histogram is cleared for the next pass
      }
      thq = key_order(prefix);
    } else {
      int pow2 = 32;
      while (pow2 < nlb) pow2 <<= 1;
      for (int i = nlb + lane; i < pow2; i += 32) lbv[i] = -INFINITY;
      __syncwarp();
      for (int size = 2; size <= pow2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int pi = lane; pi < pow2 / 2; pi += 32) {
            const int a = 2 * pi - (pi & (stride - 1));
            const int b = a + stride;
            const bool desc = (a & size) == 0;
            const float x = lbv[a], y = lbv[b];
            if ((x < y) == desc) {
              lbv[a] = y;
              lbv[b] = x;
            }
          }
          __syncwarp();
        }
      }
      thq = p.k <= nlb ? lbv[p.k - 1] : th0;
    }
  }
  // the kept records that reach theta_q
  for_each_entry(p, q, lane, [&](int64_t e, float qm) {
    if (!(p.cand_ub[e] < thq)) {
      const int pos = atomicAdd(&cw->n_c, 1);
      if (pos < kIvfSelCand) {
        crec[pos] = p.cand_rec[e];
        cqm[pos] = qm;
      }
    }
  });
  __syncwarp();
  const int nc = cw->n_c;
  if (nc > kIvfSelCand) {
    if (lane == 0) atomicAdd(p.n_over, 1);
    return;
  }
  if (lane == 0 && p.n_cand != nullptr) atomicAdd(p.n_cand, (unsigned long long)nc);
  // exact scores: two records at a time, one per half-warp
  const int W = p.mem + p.bits;
  const int j16 = lane & 15, half = lane >> 4;
  uint32_t *im = img + half * (rw + 1);
  const float *qv = p.q_r + q * (int64_t)p.q_stride;
  for (int i0 = 0; i0 < nc; i0 += 2) {
    const int i = i0 + half;
    const bool okc = i < nc;
    const int64_t rec = (int64_t)crec[okc ? i : i0];
    const uint32_t *cwd = (const uint32_t *)(p.codes + rec * (int64_t)p.code_stride);
    for (int w = j16; w <= rw; w += 16)
      im[w] = w == 0 ? __ldg(p.start + rec) : __byte_perm(__ldg(cwd + w - 1), 0, 0x0123);
    __syncwarp();
    float acc = 0.0f;
    for (int b = 0; b < p.dim / 16; b++) {
      const int c = 16 * b + j16;
      const int pos = 32 + c * BITS - p.mem;
      const int w0 = pos >> 5, sh = pos & 31;
      const uint32_t hi = im[w0];
      const uint32_t lo = w0 + 1 <= rw ? im[w0 + 1] : 0u;
      const uint32_t win = __funnelshift_l(lo, hi, sh) >> (32 - W);
      acc = fmaf(__ldg(qv + c), table[win], acc);
    }
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    if (okc && j16 == 0) {
      const float rs = __ldg(p.rescale + rec);
      const float rn = p.rnorm != nullptr ? __ldg(p.rnorm + rec) : 1.0f;
      const float sx = fadd(cqm[i], fmul(rn, fdiv(acc, rs)));
      ckey[i] = score_key32(sx);
      cid[i] = p.ids != nullptr ? p.ids[rec] : rec;
    }
    __syncwarp();  // the images are rewritten for the next records
  }
  // rank by (score desc, id asc)
  int pow2 = 32;
  while (pow2 < nc) pow2 <<= 1;
  for (int i = nc + lane; i < pow2; i += 32) {
    ckey[i] = 0u;  // below every score key
    cid[i] = -1;
  }
  __syncwarp();
  for (int size = 2; size <= pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < pow2 / 2; pi += 32) {
        const int a = 2 * pi - (pi & (stride - 1));
        const int b = a + stride;
        const bool desc = (a & size) == 0;
        const uint32_t ka = ckey[a], kb = ckey[b];
        const int64_t ia = cid[a], ib = cid[b];
        if (desc ? key_id_before(kb, ib, ka, ia) : key_id_before(ka, ia, kb, ib)) {
          ckey[a] = kb;
          ckey[b] = ka;
          cid[a] = ib;
          cid[b] = ia;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    const bool full = i < nc;
    out_id[i] = full ? cid[i] : -1;
    out_score[i] = full ? key32_score(ckey[i]) : -INFINITY;
  }
}

// The fp16 query operand row of every pair, in bucketed pair order: a copy
// of the query's row of a16 (tc_prepare_queries_kernel), 16 bytes per
// thread.
__global__ void ivf_pair_rows16_kernel(const uint16_t *a16, const int32_t *pair_query,
                                       int64_t npairs, int kpad, uint16_t *pa16) {
  const int cpr = kpad / 8;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < npairs * cpr;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pp = e / cpr;
    const int c = (int)(e - pp * cpr);
    const int64_t q = pair_query[pp];
    ((uint4 *)(pa16 + pp * kpad))[c] = __ldg((const uint4 *)(a16 + q * kpad) + c);
  }
}

// pair_of[q * np + j] = the bucketed pair of probe j of query q
__global__ void ivf_pair_of_kernel(const int32_t *pair_slot, int64_t npairs, int32_t *pair_of) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < npairs) pair_of[pair_slot[i]] = (int32_t)i;
}

// The constant extra slice of the pair rows: 128 rows of (-1, 0, ..., 0).
__global__ void ivf_neg_slice_kernel(uint16_t *ax) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e < kIvfTcRows * 16)
    ax[e] = (e & 15) == 0 ? __half_as_ushort(__float2half_rn(-1.0f)) : (uint16_t)0;
}

// s = 2^-e with gmax * max|code| * s in [2^13, 2^14) (tc_prepare_records_kernel)
__global__ void tc_scale_kernel(const uint32_t *gmax_bits, float code_absmax, float *scale) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const double top = (double)__uint_as_float(*gmax_bits) * (double)code_absmax;
  const int e = top > 0.0 ? (int)ceil(log2(top)) - 14 : 0;
  *scale = (float)ldexp(1.0, -e);
}

const void *tc_ivf_kernel_ptr(int k) {
  if (k <= 16) return (const void *)tc_ivf_kernel<16>;
  if (k <= 32) return (const void *)tc_ivf_kernel<32>;
  return nullptr;
}

size_t tc_ivf_smem_bytes() { return (size_t)V_TOTAL; }
int tc_ivf_threads() { return V_THREADS; }

const void *ivf_select_kernel_ptr(int bits) {
  switch (bits) {
    case 1: return (const void *)ivf_select_kernel<1>;
    case 2: return (const void *)ivf_select_kernel<2>;
    case 3: return (const void *)ivf_select_kernel<3>;
    case 4: return (const void *)ivf_select_kernel<4>;
  }
  return nullptr;
}

size_t ivf_select_smem_bytes(int table_len, int code_stride) {
  const int rw = code_stride / 4;
  const size_t img_words = (size_t)((2 * (rw + 1) + 3) & ~3);
  return (((size_t)table_len * 4 + 15) & ~(size_t)15) +
         (size_t)kIvfSelWarps * (img_words * 4 + kIvfSelLb * 4 + kIvfSelCand * 20 + 16);
}

}  // namespace uvb
