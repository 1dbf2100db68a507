// tcscan.cu -- tensor-core prefilter for the codes-only flat scan (sm_100a).
//
// The exact score of a record (trellis.rs:1483-1536: qm + rnorm * (dot /
// rescale), times the row norm for MIPS) needs the f32 dot in the AVX2
// association of simd.rs:183-262.  Computing every dot that way is FP32-issue
// bound.  Here every (query, record) dot is first computed on the tensor
// cores in fp16 x fp16 -> f32 (tcgen05.mma, 128 queries x 256 records per
// MMA tile), and a rigorous per-record bound turns it into an interval that
// provably contains the exact f32 score:
//
//   |dot_tc - dot_exact| <= beta_r = eps * |q| * |x_r| + small absolute terms
//   eps = 1.5e-3 covers the fp16 rounding of both operands (2 * 2^-11), the
//   tensor-core accumulation (allowed 2^-12 of sum |q_i x_i|) and the f32
//   reference accumulation; |q| <= 1.0001 for a rotated unit query.
//   score in [fma(dot_tc, g_r, -c_r), fma(dot_tc, g_r, c_r)] with
//   g_r = rnorm_r / rescale_r (x norm_r) and c_r = (beta_r + 10u A_r) g_r,
//   A_r = |q| |x_r| + beta_r bounding every f32 rounding of the score.
//
// Pass 1 (MODE 1) writes, per query and 128-record half tile, the largest
// lower bound; the k-th largest of those maxima is a score that at least k
// records reach, so it lower-bounds the exact k-th best (theta).  Pass 2
// (MODE 2) appends every record whose upper bound reaches theta to the
// query's candidate list; the exact top-k is among them, ties included.
// The candidates are then scored exactly (tc_rescore_kernel) and ranked.
//
// Records are first decoded once per search into an fp16 row-major copy
// (tc_prepare_records_kernel, which also computes the bound constants).  The
// scan kernel then streams 256-record tiles of it into shared memory by TMA
// (128-byte swizzle, the K-major operand layout of the MMA).
//
// CTA = one unit of 128 queries x a record range.  Warp roles:
//   warps 0-7  epilogue: warp w reads TMEM lane quarter w % 4 (thread =
//              query) and column half w / 4 (128 records) of each tile
//   warp 8     TMEM allocation; lane 0 issues the MMAs
//   warp 9     lane 0 issues the TMA loads
// Three shared-memory stages and two TMEM accumulators (2 x 256 columns)
// are handed over with mbarriers; every wait is bounded.
#include <cuda.h>

#include "uv_kernels.h"
#include "uv_tc.cuh"

namespace uvb {

namespace {

constexpr int TC_M = 128;      // queries per unit
constexpr int TC_N = 256;      // records per MMA tile
constexpr int TC_D = 128;      // coordinates (K)
constexpr int TC_STAGES = 3;
constexpr int TC_THREADS = 320;
constexpr int TC_EPI = 256;    // epilogue threads
constexpr uint32_t kWaitLimit = 1u << 20;

struct TcLayout {
  static constexpr int a_bytes = TC_M * TC_D * 2;        // 32 KB
  static constexpr int b_bytes = TC_N * TC_D * 2;        // 64 KB per stage
  static constexpr int a = 0;
  static constexpr int b = a + a_bytes;
  static constexpr int bars = b + TC_STAGES * b_bytes;   // 10 mbarriers
  static constexpr int misc = bars + 16 * 8;             // tmem base, abort flag
  static constexpr int total = misc + 64;
};

// 3-input maximum (NaN-ignoring like fmaxf)
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_scan_kernel(const TcScanParams p, const __grid_constant__ CUtensorMap tmap) {
  using L = TcLayout;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t *sa = sm + L::a;
  uint64_t *full = (uint64_t *)(sm + L::bars);  // [3]
  uint64_t *empty = full + 3;                   // [3]
  uint64_t *accf = full + 6;                    // [2]
  uint64_t *acce = full + 8;                    // [2]
  uint32_t *tbase_s = (uint32_t *)(sm + L::misc);
  volatile int *abort_s = (volatile int *)(sm + L::misc + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t q0 = (int64_t)blockIdx.x * TC_M;
  const int64_t t_begin = p.n_tiles * blockIdx.y / gridDim.y;
  const int64_t t_end = p.n_tiles * (blockIdx.y + 1) / gridDim.y;
  const int ntiles = (int)(t_end - t_begin);

  // ---- setup: barriers, TMEM, query tile ----
  if (tid == 0) {
    for (int s = 0; s < TC_STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      tc::mbar_init(&accf[a], 1);
      tc::mbar_init(&acce[a], TC_EPI);
    }
    *abort_s = 0;
    tc::mbar_fence_init();
  }
  if (warp == 8) tc::tmem_alloc(tbase_s, 512);
  // queries -> fp16, swizzled K-major (zeros past nq and for degenerate rows)
  for (int e = tid; e < TC_M * (TC_D / 8); e += TC_THREADS) {
    const int r = e / (TC_D / 8), c = e - r * (TC_D / 8);
    const int64_t q = q0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q < p.nq && !p.degenerate[q]) {
      const float4 *src = (const float4 *)(p.q_r + q * (int64_t)p.q_stride + c * 8);
      const float4 x0 = __ldg(src), x1 = __ldg(src + 1);
      __half2 h0 = __floats2half2_rn(x0.x, x0.y), h1 = __floats2half2_rn(x0.z, x0.w);
      __half2 h2 = __floats2half2_rn(x1.x, x1.y), h3 = __floats2half2_rn(x1.z, x1.w);
      v = make_uint4(*(uint32_t *)&h0, *(uint32_t *)&h1, *(uint32_t *)&h2, *(uint32_t *)&h3);
    }
    *(uint4 *)(sa + tc::sw128_chunk_offset(r, c, TC_M)) = v;
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tbase_s;

  if (warp < 8) {
    // ================= epilogue =================
    const int quarter = warp & 3, half = warp >> 2;
    const int64_t q = q0 + quarter * 32 + lane;
    const bool qok = q < p.nq && !p.degenerate[q];
    const float theta = (MODE == 2 && qok) ? p.theta[q] : INFINITY;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 128);
    for (int it = 0; it < ntiles; it++) {
      const int a = it & 1;
      const int64_t tile = t_begin + it;
      const int64_t rec0 = tile * TC_N + half * 128;
      const float4 *gc = (const float4 *)(p.gc + rec0);  // (g, c) of two records
      if (!tc::mbar_wait(&accf[a], (it >> 1) & 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      tc::tc_fence_after();
      const uint32_t base = lane_base + (uint32_t)(a * TC_N);
      float best = -INFINITY;
      uint32_t mask0 = 0u, mask1 = 0u, mask2 = 0u, mask3 = 0u;
      uint32_t ra[32], rb[32];
      // bound of every record of 32-column chunk c, its max, and (pass 2)
      // the mask of records that can reach theta
      auto chunk = [&](const uint32_t(&cur)[32], int c) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float4 g4 = __ldg(gc + (32 * c + j) / 2);
          const float2 dd = make_float2(__uint_as_float(cur[j]), __uint_as_float(cur[j + 1]));
          const float2 g2 = make_float2(g4.x, g4.z);
          const float2 c2 = MODE == 1 ? make_float2(-g4.y, -g4.w) : make_float2(g4.y, g4.w);
          const float2 t2 = __ffma2_rn(dd, g2, c2);
          v[j] = t2.x;
          v[j + 1] = t2.y;
        }
        float m = max3(v[0], v[1], v[2]);
#pragma unroll
        for (int j = 3; j < 31; j += 2) m = max3(m, v[j], v[j + 1]);
        m = fmaxf(m, v[31]);
        if (MODE == 1) {
          best = fmaxf(best, m);
        } else if (qok && !(m < theta)) {
          uint32_t mk = 0;
#pragma unroll
          for (int j = 0; j < 32; j++) mk |= (!(v[j] < theta) ? 1u : 0u) << j;
          // selects, not an indexed store: the masks stay in registers
          mask0 = c == 0 ? mk : mask0;
          mask1 = c == 1 ? mk : mask1;
          mask2 = c == 2 ? mk : mask2;
          mask3 = c == 3 ? mk : mask3;
        }
      };
      // TMEM -> registers two chunks at a time: the next load is in flight
      // while the current chunk is processed
      tc::tmem_ld32(base, ra);
      tc::tmem_ld_wait();
#pragma unroll 1
      for (int c = 0; c < 4; c += 2) {
        tc::tmem_ld32(base + (uint32_t)(32 * (c + 1)), rb);
        chunk(ra, c);
        tc::tmem_ld_wait();
        if (c + 2 < 4) tc::tmem_ld32(base + (uint32_t)(32 * (c + 2)), ra);
        chunk(rb, c + 1);
        if (c + 2 < 4) tc::tmem_ld_wait();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&acce[a]);
      if (MODE == 1 && q < p.nq)
        p.tmax[q * p.n_groups + 2 * tile + half] = qok ? best : -INFINITY;
      if (MODE == 2) {
        uint32_t mask[4] = {mask0, mask1, mask2, mask3};
        // one reservation per thread and tile for all of its candidates
        if (rec0 + 128 > p.n) {
          const int64_t lim = p.n - rec0;  // records past n are padding
#pragma unroll
          for (int c = 0; c < 4; c++) {
            const int64_t room = lim - 32 * c;
            mask[c] &= room >= 32 ? 0xffffffffu : (room <= 0 ? 0u : ((1u << room) - 1u));
          }
        }
        const int cnt = __popc(mask[0]) + __popc(mask[1]) + __popc(mask[2]) + __popc(mask[3]);
        if (cnt > 0) {
          int pos = atomicAdd(&p.cand_cnt[q], cnt);
          uint32_t *dst = p.cand + q * (int64_t)p.cand_cap;
#pragma unroll
          for (int c = 0; c < 4; c++) {
            uint32_t mk = mask[c];
            while (mk != 0u) {
              const int j = __ffs(mk) - 1;
              mk &= mk - 1u;
              if (pos < p.cand_cap) dst[pos] = (uint32_t)(rec0 + 32 * c + j);
              pos++;
            }
          }
        }
      }
    }
  } else if (warp == 8) {
    if (lane == 0) {
      // ================= MMA issue =================
      const uint32_t idesc = tc::idesc_f16_f32(TC_M, TC_N);
      const uint32_t a_base = tc::smem_u32(sa);
      for (int it = 0; it < ntiles; it++) {
        const int s = it % TC_STAGES, a = it & 1;
        if (!tc::mbar_wait(&full[s], (it / TC_STAGES) & 1, kWaitLimit) ||
            !tc::mbar_wait(&acce[a], ((it >> 1) & 1) ^ 1, kWaitLimit)) {
          *abort_s = 1;
          atomicExch(p.err, 1);
        }
        if (*abort_s) break;
        tc::tc_fence_after();
        const uint32_t b_base = tc::smem_u32(sm + L::b + s * L::b_bytes);
#pragma unroll
        for (int k = 0; k < TC_D / 16; k++) {
          const uint32_t off = (uint32_t)((k & 3) * 32);  // 16 fp16 = 32 B per K step
          const uint64_t ad = tc::sw128_desc(a_base + (k >> 2) * TC_M * 128 + off);
          const uint64_t bd = tc::sw128_desc(b_base + (k >> 2) * TC_N * 128 + off);
          tc::mma_f16(tmem + (uint32_t)(a * TC_N), ad, bd, idesc, k > 0 ? 1u : 0u);
        }
        tc::mma_commit(&empty[s]);
        tc::mma_commit(&accf[a]);
      }
    }
  } else if (lane == 0) {
    // ================= TMA producer =================
    for (int it = 0; it < ntiles; it++) {
      const int s = it % TC_STAGES;
      if (!tc::mbar_wait(&empty[s], ((it / TC_STAGES) & 1) ^ 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      uint8_t *dst = sm + L::b + s * L::b_bytes;
      const int row = (int)((t_begin + it) * TC_N);
      tc::mbar_arrive_expect_tx(&full[s], (uint32_t)L::b_bytes);
      tc::tma_load_2d(dst, &tmap, 0, row, &full[s]);
      tc::tma_load_2d(dst + TC_N * 128, &tmap, 64, row, &full[s]);
    }
  }

  // ---- teardown: the epilogue has waited for every MMA ----
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
    tc::tmem_relinquish();
  }
}

// ---------------------------------------------------------------------------
// Per record: the fp16 row of decoded code values (the scan kernel's MMA
// operand; padded rows are zero) and the bound constants (g, c): score in
// [fma(dot_tc, g, -c), fma(dot_tc, g, c)] with g = (rnorm / rescale) [x norm].
// Non-finite g or c (NaN or infinite sidecars) gives g = 0, c = +inf: never
// pruned, never a lower bound.
// ---------------------------------------------------------------------------
__global__ void tc_prepare_records_kernel(const TcPrepareParams p) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= p.n_pad) return;
  uint4 *xrow = (uint4 *)(p.x16 + r * TC_D);
  if (r >= p.n) {
    for (int c = 0; c < TC_D / 8; c++) xrow[c] = make_uint4(0, 0, 0, 0);
    p.gc[r] = make_float2(0.0f, INFINITY);
    return;
  }
  const int W = p.mem + p.bits;
  const uint32_t *cw = (const uint32_t *)(p.codes + r * (int64_t)p.code_stride);
  const uint32_t st = __ldg(p.start + r);
  const int rw = p.code_stride >> 2;
  double xs = 0.0;
  for (int c = 0; c < TC_D / 8; c++) {
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 8; h++) {
      const int i = 8 * c + h;
      const int pos = 32 + i * p.bits - p.mem;
      const int w0 = pos >> 5, sh = pos & 31;
      const uint32_t hi = w0 == 0 ? st : (w0 <= rw ? __byte_perm(__ldg(cw + w0 - 1), 0, 0x0123) : 0u);
      const uint32_t lo = w0 + 1 <= rw ? __byte_perm(__ldg(cw + w0), 0, 0x0123) : 0u;
      const uint32_t win = __funnelshift_l(lo, hi, sh) >> (32 - W);
      const float x = __ldg(p.code + win);
      xs += (double)x * (double)x;
      const uint32_t hx = __half_as_ushort(__float2half_rn(x));
      if (h & 1) o[h >> 1] |= hx << 16;
      else o[h >> 1] = hx;
    }
    xrow[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  const float rs = __ldg(p.rescale + r);
  const float rn = p.rnorm ? __ldg(p.rnorm + r) : 1.0f;
  float g = fdiv(rn, rs);
  if (p.mips) g = fmul(g, __ldg(p.norms + r));
  const double u = 5.9604644775390625e-8;  // 2^-24
  const double qn = 1.0001;                // |q_r| of a rotated unit query
  const double xn = sqrt(xs) * (1.0 + 1e-12);
  const double beta =
      p.eps * qn * xn + u * sqrt((double)TC_D) * (xn * (1.0 + 4.8828125e-4) + qn) + 1e-30;
  const double A = qn * xn + beta;
  const double cd = (beta + 10.0 * u * A) * (double)g * (1.0 + 1e-6);
  float c = __double2float_ru(cd);
  if (!isfinite(g) || !isfinite(c) || g < 0.0f) {
    g = 0.0f;
    c = INFINITY;
  }
  p.gc[r] = make_float2(g, c);
}

// ---------------------------------------------------------------------------
// theta[q] = k-th largest of the query's tile maxima (radix select on
// order-preserving keys, four 8-bit rounds).  Fewer than k tiles: -inf.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t fkey(float f) {
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__global__ void __launch_bounds__(256) tc_theta_kernel(const float *tmax, int64_t n_tiles,
                                                        int64_t nq, int k, float *theta) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[2];
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  const float *v = tmax + q * n_tiles;
  if (n_tiles < k) {
    if (threadIdx.x == 0) theta[q] = -INFINITY;
    return;
  }
  uint32_t prefix = 0, mask = 0, kk = (uint32_t)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n_tiles; i += 256) {
      const uint32_t key = fkey(v[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
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
  if (threadIdx.x == 0) theta[q] = fkey_inv(prefix);
}

// ---------------------------------------------------------------------------
// Exact scores of the candidates (simd.rs:183-262 association: 16 FMA chains
// over 16-wide blocks, then the hsum256 tree; trellis.rs:1517 estimator) and
// the query's top-k by (score desc, record asc).  One CTA per query; two
// candidates per warp at a time, one per half-warp.  A query whose list
// overflowed is recorded for the exact fallback scan.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) tc_rescore_kernel(const TcRescoreParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint64_t *keys = (uint64_t *)sm;                    // cap (power of two)
  float *qv = (float *)(keys + p.cap);                // dim
  float *table = qv + p.dim;                          // table_len (optional)
  const int64_t q = blockIdx.x;
  if (q >= p.nq) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cnt_raw = p.cand_cnt[q];
  if (cnt_raw > p.cap) {
    if (tid == 0) p.over_list[atomicAdd(p.n_over, 1)] = (int32_t)q;
    return;
  }
  const int cnt = p.degenerate[q] ? 0 : cnt_raw;
  if (tid == 0) atomicAdd(p.n_cand, (unsigned long long)cnt);
  int pow2 = 32;
  while (pow2 < cnt) pow2 <<= 1;
  for (int i = tid; i < p.dim; i += 256) qv[i] = p.q_r[q * (int64_t)p.q_stride + i];
  if (p.table_in_smem)
    for (int i = tid; i < p.table_len; i += 256) table[i] = __ldg(p.code + i);
  for (int i = tid; i < pow2; i += 256) keys[i] = kEmptyKey;
  __syncthreads();
  const float *code = p.table_in_smem ? table : p.code;
  const int W = p.mem + p.bits;
  const int rw = p.code_stride >> 2;
  const int j = lane & 15, half = lane >> 4;
  const uint32_t *cand = p.cand + q * (int64_t)p.cap;
  for (int i0 = warp * 2; i0 < cnt; i0 += 16) {
    const int i = i0 + half;
    const bool ok = i < cnt;
    const int64_t rec = ok ? (int64_t)cand[i] : 0;
    const uint32_t *cw = (const uint32_t *)(p.codes + rec * (int64_t)p.code_stride);
    const uint32_t st = __ldg(p.start + rec);
    float acc = 0.0f;
    for (int b = 0; b < p.dim / 16; b++) {
      const int c = 16 * b + j;
      const int pos = 32 + c * p.bits - p.mem;
      const int w0 = pos >> 5, sh = pos & 31;
      const uint32_t hi = w0 == 0 ? st : (w0 <= rw ? __byte_perm(__ldg(cw + w0 - 1), 0, 0x0123) : 0u);
      const uint32_t lo = w0 + 1 <= rw ? __byte_perm(__ldg(cw + w0), 0, 0x0123) : 0u;
      const uint32_t win = __funnelshift_l(lo, hi, sh) >> (32 - W);
      acc = fmaf(qv[c], code[win], acc);
    }
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
    acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
    if (ok && j == 0) {
      const float rs = __ldg(p.rescale + rec);
      const float rn = p.rnorm ? __ldg(p.rnorm + rec) : 1.0f;
      float sx = fadd(0.0f, fmul(rn, fdiv(acc, rs)));
      if (p.mips) sx = fmul(sx, __ldg(p.norms + rec));
      keys[i] = rank_key(sx, (uint32_t)rec);
    }
  }
  __syncthreads();
  // bitonic sort, descending
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
  for (int i = tid; i < p.k; i += 256) {
    const uint64_t key = i < pow2 ? keys[i] : kEmptyKey;
    const bool full = key != kEmptyKey;
    const int64_t rec = rank_key_index(key);
    p.out_id[q * p.k + i] = full ? (p.ids ? p.ids[rec] : rec) : -1;
    p.out_score[q * p.k + i] = full ? key32_score((uint32_t)(key >> 32)) : -INFINITY;
  }
}

size_t tc_scan_smem_bytes() { return (size_t)TcLayout::total; }

const void *tc_scan_kernel_ptr(int mode) {
  return mode == 1 ? (const void *)tc_scan_kernel<1> : (const void *)tc_scan_kernel<2>;
}

int tc_threads() { return TC_THREADS; }
int tc_tile_records() { return TC_N; }
int tc_tile_queries() { return TC_M; }
int tc_dim() { return TC_D; }

}  // namespace uvb
