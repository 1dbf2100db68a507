// tcscan.cu -- tensor-core prefilter for the codes-only flat scan (sm_100a).
//
// The exact score of a record (trellis.rs:1483-1536: qm + rnorm * (dot /
// rescale), times the row norm for MIPS) needs the f32 dot in the AVX2
// association of simd.rs:183-262.  Computing every dot that way is FP32-issue
// bound.  Here every (query, record) dot is first computed on the tensor
// cores in fp16 x fp16 -> f32 (tcgen05.mma, 128 queries x 192 records per
// MMA), and a rigorous per-record bound turns it into an interval that
// provably contains the exact f32 score:
//
//   |dot_tc - dot_exact| <= beta_r = eps * |q| * |x_r| + small absolute terms
//   eps = 1.5e-3 covers the fp16 rounding of both operands (2 * 2^-11), the
//   tensor-core accumulation (allowed 2^-12 of sum |q_i x_i|) and the f32
//   reference accumulation; |q| <= 1.0001 for a rotated unit query.
//   score in [g_r dot_tc - c_r, g_r dot_tc + c_r] with g_r = rnorm_r /
//   rescale_r (x norm_r) and c_r = g_r beta_r plus the f32 roundings of the
//   score; the epilogue forms both bounds from the MMA's g_r dot_tc (below).
//
// Pass 1 (MODE 1) writes, per query and 96-record half tile, a lower bound
// of its best record's score; the k-th largest of those maxima is a score that at least k
// records reach, so it lower-bounds the exact k-th best (theta).  Pass 2
// (MODE 2) appends every record whose upper bound reaches theta to the
// query's candidate list; the exact top-k is among them, ties included.
// The candidates are then scored exactly (tc_rescore_kernel) and ranked.
//
// Records are first turned into fp16 operand rows plus their bound
// constants (tc_prepare_records_kernel; kept between searches):
//   main  B'_r,i = fp16(g_r * x_r,i * s)             128 coordinates
//   ext   C'_r   = fp16 rounded up of c_r * s         one extra K slice of 16
// with s = 2^-e a power of two that keeps every |B'| below 2^14, and the
// largest C' of every 16-record chunk (tc_chunk_cmax_kernel).  The MMA runs
// over the 128 coordinates only (K = 128: the extra slice would cost a ninth
// more tensor work and record bytes per tile); the epilogue turns
// s * g * dot into bounds with the chunk's largest C', rounded outwards
// (bounds_run_cmax in uv_tc_epilogue.cuh).  Record tiles stream in by TMA (128-byte swizzle).
//
// CTA = one unit of 128 queries x a record range, streaming 192-record
// tiles.  Warp roles:
//   warps 0-15 epilogue: warp w reads TMEM lane quarter w % 4 (thread =
//              query) and column slice w / 4 (48 records) of each tile;
//              sixteen warps, because pass 2's epilogue, not the MMA, sets
//              the tile rate (four per scheduler hide its latency).  Pass 1
//              has no candidate path and uses warps 0-7 on half tiles.
//   warp 16    TMEM allocation; lane 0 issues the MMAs
//   warp 17    lane 0 issues the TMA loads
// The query tile (A) sits in TMEM (default; the MMA reads it there) or in
// shared memory.  Four (three) shared-memory stages and two TMEM
// accumulators of 192 columns are handed over with mbarriers; every wait is
// bounded.
#include <cuda.h>

#include "uv_kernels.h"
#include "uv_tc.cuh"
#include "uv_tc_epilogue.cuh"
#include "uv_score_thread.cuh"

namespace uvb {

namespace {

constexpr int TC_M = 128;      // queries per MMA (TMEM lanes)
constexpr int TC_D = 128;      // coordinates (K) of the main rows
constexpr int TC_X = 16;       // the extra K slice (bound constant + zeros)
constexpr int TC_EPI_WARPS = 16;                   // epilogue warps
constexpr int TC_THREADS = (TC_EPI_WARPS + 2) * 32;  // + MMA warp + TMA warp
constexpr uint32_t kWaitLimit = 1u << 20;

// CTA shapes.  S = 1: the queries (A) in shared memory, three stages.
// S = 3 (the default): A held in TMEM next to the accumulators (tcgen05.mma
// reads A from TMEM and B from shared memory), which takes A's reads off the
// shared-memory port the MMAs and the TMA writes share and frees its 32 KB
// for a fourth stage.  TMEM: two accumulators of 192 columns (+ 64 columns
// of A for S = 3).
template <int S>
struct TcShape {
  static constexpr bool A_TMEM = S == 3;
  static constexpr int TN = 192;                       // records per tile
  static constexpr int STAGES = A_TMEM ? 4 : 3;
  static constexpr int SLICES = TC_EPI_WARPS / 4;      // column slices of a tile
  static constexpr int CW = TN / SLICES;               // accumulator columns per epilogue warp
  static constexpr int NC = CW / 16;                   // 16-column TMEM loads (chunks) per warp
  static constexpr int a_tile = A_TMEM ? 0 : TC_M * TC_D * 2;   // 32 KB
  static constexpr int bm_bytes = TN * 128;            // one 64-wide atom column of records
  static constexpr int b_bytes = 2 * bm_bytes;
  static constexpr int a = 0;
  static constexpr int b = a + a_tile;
  static constexpr int bars = b + STAGES * b_bytes;   // 2 * STAGES + 4 mbarriers
  static constexpr int misc = bars + 16 * 8;          // tmem base, abort flag
  static constexpr int total = misc + 64;
  static constexpr uint32_t a_col = 2 * TN;           // first TMEM column of A (S = 3)
};
static_assert(TcShape<1>::b % 1024 == 0 && TcShape<1>::b_bytes % 1024 == 0, "stage alignment");
static_assert(TcShape<3>::b % 1024 == 0 && TcShape<3>::b_bytes % 1024 == 0, "stage alignment");
static_assert(TcShape<1>::total <= 227 * 1024 && TcShape<3>::total <= 227 * 1024, "shared memory");
static_assert(TcShape<3>::a_col + TC_D / 2 <= 512, "TMEM columns");

// registers -> TMEM: 32 lanes x 8 columns
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&w)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(
                   taddr),
               "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]),
               "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// D (+)= A B with A in TMEM (row i in lane i, K pairs packed low-first in
// 32-bit columns) and B by shared-memory descriptor
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :
      : "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}


}  // namespace

template <int MODE, int S>
__global__ void __launch_bounds__(TC_THREADS, 1)
    tc_scan_kernel(const TcScanParams p, const __grid_constant__ CUtensorMap tmap_main) {
  using L = TcShape<S>;
  constexpr int TN = L::TN, STAGES = L::STAGES, NC = L::NC, SLICES = L::SLICES;
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t *sa = sm + L::a;
  uint64_t *full = (uint64_t *)(sm + L::bars);  // [STAGES]
  uint64_t *empty = full + STAGES;              // [STAGES]
  uint64_t *accf = empty + STAGES;              // [2]
  uint64_t *acce = accf + 2;                    // [2]
  uint64_t *drained = acce + 2;                 // MMAs done after an abort
  uint32_t *tbase_s = (uint32_t *)(sm + L::misc);
  volatile int *abort_s = (volatile int *)(sm + L::misc + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t q0 = (int64_t)blockIdx.x * TC_M;
  const int64_t t_begin = p.n_tiles * blockIdx.y / gridDim.y;
  const int64_t t_end = p.n_tiles * (blockIdx.y + 1) / gridDim.y;
  const int ntiles = (int)(t_end - t_begin);

  // ---- setup: barriers, TMEM, query tile ----
  if (tid == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      tc::mbar_init(&accf[a], 1);
      tc::mbar_init(&acce[a], MODE == 1 ? 8 : TC_EPI_WARPS);  // one arrival per epilogue warp
    }
    tc::mbar_init(drained, 1);
    *abort_s = 0;
    tc::mbar_fence_init();
  }
  if (warp == TC_EPI_WARPS) tc::tmem_alloc(tbase_s, 512);
  if constexpr (L::A_TMEM) {
    // queries -> fp16 rows in TMEM: warp w < 4 writes lanes 32w..32w+31, one
    // query per lane; 64 columns of coordinate pairs
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    if (warp < 4) {
      const int64_t q = q0 + warp * 32 + lane;
      const bool ok = q < p.nq && !p.degenerate[q];
      const float *src = p.q_r + (ok ? q : 0) * (int64_t)p.q_stride;
      const uint32_t ta = *tbase_s + ((uint32_t)(warp * 32) << 16) + L::a_col;
#pragma unroll
      for (int g = 0; g < TC_D / 16; g++) {
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float2 x = ok ? __ldg((const float2 *)(src + 16 * g + 2 * j)) : make_float2(0.f, 0.f);
          const __half2 h = __floats2half2_rn(x.x, x.y);  // .x in the low half
          w[j] = *(const uint32_t *)&h;
        }
        tmem_st8(ta + 8 * g, w);
      }
      tmem_st_wait();
    }
  } else {
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
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tbase_s;

  if (MODE == 1 && warp < 8) {
    // ================= pass-1 epilogue =================
    // No candidate path, so eight warps keep up: warp w reads TMEM lane
    // quarter w % 4 (thread = query) and column half w / 4 (96 records, two
    // loads of 48), and writes one lower bound per (query, half tile), the
    // best over the half's 16-record chunks of max(dot) - cmax rounded down.
    const int quarter = warp & 3, half = warp >> 2;
    constexpr int HC = TN / 2 / 16;  // chunks per half tile
    const int64_t q = q0 + quarter * 32 + lane;
    const bool qok = q < p.nq && !p.degenerate[q];
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * TN / 2);
    float cm_next[HC];
    auto load_cm = [&](int it, float(&c)[HC]) {
      const int64_t r0 = (t_begin + it) * p.tile_stride * TN + half * TN / 2;
#pragma unroll
      for (int l = 0; l < HC; l++) c[l] = __ldg(p.cmax + (r0 >> 4) + l);
    };
    if (ntiles > 0) load_cm(0, cm_next);
    for (int it = 0; it < ntiles; it++) {
      const int a = it & 1;
      const int64_t tile = t_begin + it;
      const int64_t rec0 = tile * p.tile_stride * TN + half * TN / 2;
      float cm[HC];
#pragma unroll
      for (int l = 0; l < HC; l++) cm[l] = cm_next[l];
      if (it + 1 < ntiles) load_cm(it + 1, cm_next);
      if (!tc::mbar_wait(&accf[a], (it >> 1) & 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      tc::tc_fence_after();
      const uint32_t base = lane_base + (uint32_t)(a * TN);
      float m = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        uint32_t r[HC / 2][16];
#pragma unroll
        for (int l = 0; l < HC / 2; l++) tc::tmem_ld16(base + 16 * (h * HC / 2 + l), r[l]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int l = 0; l < HC / 2; l++) {
          const int64_t c0 = rec0 + 16 * (h * HC / 2 + l);
          float mc = tcep::chunk_max16(r[l]);
          if (c0 + 16 > p.n) {  // the last tile: padding rows stay out of the maximum
            mc = -INFINITY;
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (c0 + j < p.n) mc = fmaxf(mc, __uint_as_float(r[l][j]));
          }
          m = fmaxf(m, __fsub_rd(mc, cm[h * HC / 2 + l]));
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[a]);
      if (q < p.nq) p.tmax[q * p.n_groups + 2 * tile + half] = qok ? m : -INFINITY;
    }
  } else if (MODE == 2 && warp < TC_EPI_WARPS) {
    // ================= pass-2 epilogue =================
    // warp w: TMEM lane quarter w % 4 (thread = query), column slice w / 4
    const int quarter = warp & 3, slice = warp >> 2;
    const int64_t q = q0 + quarter * 32 + lane;
    const bool qok = q < p.nq && !p.degenerate[q];
    const float theta = (MODE == 2 && qok) ? p.theta[q] : INFINITY;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(slice * L::CW);
    // pass 2: this thread's segment of the query's candidate list
    const int region = (int)blockIdx.y * SLICES + slice;
    uint32_t *seg = MODE == 2 ? p.cand + q * (int64_t)p.cand_cap + (int64_t)region * p.region_cap
                              : nullptr;
    int seg_cnt = 0;
    // the chunk constants of a tile are loaded one tile ahead, so their
    // latency overlaps the wait for the accumulator
    float cm_next[NC];
    auto load_cm = [&](int it, float(&c)[NC]) {
      const int64_t r0 = (t_begin + it) * p.tile_stride * TN + slice * L::CW;
#pragma unroll
      for (int l = 0; l < NC; l++) c[l] = __ldg(p.cmax + (r0 >> 4) + l);
    };
    if (ntiles > 0) load_cm(0, cm_next);
    for (int it = 0; it < ntiles; it++) {
      const int a = it & 1;
      const int64_t tile = t_begin + it;  // group index; records of tile * tile_stride
      const int64_t rec0 = tile * p.tile_stride * TN + slice * L::CW;
      float cm[NC];
#pragma unroll
      for (int l = 0; l < NC; l++) cm[l] = cm_next[l];
      if (it + 1 < ntiles) load_cm(it + 1, cm_next);
      if (!tc::mbar_wait(&accf[a], (it >> 1) & 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      tc::tc_fence_after();
      const uint32_t base = lane_base + (uint32_t)(a * TN);
      uint32_t r[NC][16];
#pragma unroll
      for (int l = 0; l < NC; l++) tc::tmem_ld16(base + 16 * l, r[l]);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[a]);  // the warp's accumulator part is in registers
      tcep::bounds_run_cmax<MODE, NC>(p, r, cm, q, qok, theta, SLICES * tile + slice, rec0,
                                      seg, &seg_cnt);
      // reconverge before the next poll: lanes that found no candidate
      // would otherwise sit in mbarrier.try_wait (which may suspend them
      // until the next accumulator is ready) while the others append
      __syncwarp();
    }
    if (MODE == 2 && q < p.nq) p.cand_cnt[q * p.regions + region] = seg_cnt;
  } else if (warp == TC_EPI_WARPS) {
    if (lane == 0) {
      // ================= MMA issue =================
      const uint32_t idesc = tc::idesc_f16_f32(TC_M, TN);
      for (int it = 0; it < ntiles; it++) {
        const int s = it % STAGES, a = it & 1;
        if (!tc::mbar_wait(&full[s], (it / STAGES) & 1, kWaitLimit) ||
            !tc::mbar_wait(&acce[a], ((it >> 1) & 1) ^ 1, kWaitLimit)) {
          *abort_s = 1;
          atomicExch(p.err, 1);
        }
        if (*abort_s) break;
        tc::tc_fence_after();
        const uint32_t b_base = tc::smem_u32(sm + L::b + s * L::b_bytes);
        const uint32_t d = tmem + (uint32_t)(a * TN);
        if constexpr (L::A_TMEM) {
          const uint32_t at = tmem + L::a_col;
#pragma unroll
          for (int k = 0; k < TC_D / 16; k++) {
            const uint32_t off = (uint32_t)((k & 3) * 32);  // 16 fp16 = 32 B per K step
            const uint64_t bd = tc::sw128_desc(b_base + (k >> 2) * L::bm_bytes + off);
            mma_f16_ts(d, at + 8 * k, bd, idesc, k > 0 ? 1u : 0u);
          }
        } else {
          const uint32_t a_base = tc::smem_u32(sa);
#pragma unroll
          for (int k = 0; k < TC_D / 16; k++) {
            const uint32_t off = (uint32_t)((k & 3) * 32);
            const uint64_t ad = tc::sw128_desc(a_base + (k >> 2) * TC_M * 128 + off);
            const uint64_t bd = tc::sw128_desc(b_base + (k >> 2) * L::bm_bytes + off);
            tc::mma_f16(d, ad, bd, idesc, k > 0 ? 1u : 0u);
          }
        }
        tc::mma_commit(&empty[s]);
        tc::mma_commit(&accf[a]);
      }
      if (*abort_s) {  // let every issued MMA finish before TMEM is freed
        tc::mma_commit(drained);
        tc::mbar_wait(drained, 0, kWaitLimit);
      }
    }
  } else if (warp == TC_EPI_WARPS + 1 && lane == 0) {
    // ================= TMA producer =================
    int64_t issued = 0;
    for (int it = 0; it < ntiles; it++, issued++) {
      const int s = it % STAGES;
      if (!tc::mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      uint8_t *dst = sm + L::b + s * L::b_bytes;
      const int row = (int)((t_begin + it) * p.tile_stride * TN);
      tc::mbar_arrive_expect_tx(&full[s], (uint32_t)L::b_bytes);
      tc::tma_load_2d(dst, &tmap_main, 0, row, &full[s]);
      tc::tma_load_2d(dst + L::bm_bytes, &tmap_main, 64, row, &full[s]);
    }
    if (*abort_s) tc::drain_stages(full, STAGES, issued, kWaitLimit);
  }

  // ---- teardown: the epilogue has waited for every MMA ----
  tc::tc_fence_before();
  __syncthreads();
  if (warp == TC_EPI_WARPS) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
    tc::tmem_relinquish();
  }
}

// ---------------------------------------------------------------------------
// g_r = (rnorm / rescale) [x norm] of every record and the largest finite one
// (as the bits of a non-negative float, which order like the float).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float record_g(const TcPrepareParams &p, int64_t r) {
  const float rs = __ldg(p.rescale + r);
  const float rn = p.rnorm ? __ldg(p.rnorm + r) : 1.0f;
  float g = fdiv(rn, rs);
  if (p.mips) g = fmul(g, __ldg(p.norms + r));
  return g;
}

__global__ void tc_gmax_kernel(const TcPrepareParams p) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  float g = 0.0f;
  if (r < p.n) {
    g = record_g(p, r);
    if (!isfinite(g) || g < 0.0f) g = 0.0f;
  }
  for (int o = 16; o > 0; o >>= 1) g = fmaxf(g, __shfl_xor_sync(0xffffffffu, g, o));
  if ((threadIdx.x & 31) == 0 && g > 0.0f) atomicMax(p.gmax_bits, __float_as_uint(g));
}

// ---------------------------------------------------------------------------
// The operand rows of every record (padded rows are zero, with C' = +inf so
// that they never bound theta from below):
//   B'_i = fp16(g * x_i * s),  C' = fp16 rounded up of
//   c = s * g * eps * |q| * |x| + 2^-23 sqrt(d) (|q| + s * g * |x|)
// eps = 1.5e-3 covers 2 x 2^-11 (fp16 rounding of q and of g x s), 2^-12 of
// sum |terms| for the tensor-core accumulation, the f32 reference dot and
// the five roundings of the score (two in g, three in the estimator); the
// absolute term covers fp16 subnormals.  |q| <= 1.0001 for a rotated unit
// query.  Non-finite or negative g: zero row, C' = +inf (never pruned).
// ---------------------------------------------------------------------------
__global__ void tc_prepare_records_kernel(const TcPrepareParams p) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= p.n_pad) return;
  uint4 *xrow = (uint4 *)(p.x16 + r * p.kpad);
  uint4 *xext = (uint4 *)(p.xext + r * TC_X);
  const uint32_t hinf = 0x7C00u;  // fp16 +inf
  float g = r < p.n ? record_g(p, r) : 0.0f;
  const bool bad = r >= p.n || !isfinite(g) || g < 0.0f;
  // s = 2^-e with gmax * max|code| * s in [2^13, 2^14)
  const float gmax = __uint_as_float(*p.gmax_bits);
  const double top = (double)gmax * (double)p.code_absmax;
  const int e = top > 0.0 ? (int)ceil(log2(top)) - 14 : 0;
  const double s = ldexp(1.0, -e);
  if (bad) {
    for (int c = 0; c < p.kpad / 8; c++) xrow[c] = make_uint4(0, 0, 0, 0);
    xext[0] = make_uint4(hinf, 0, 0, 0);
    xext[1] = make_uint4(0, 0, 0, 0);
    return;
  }
  const int W = p.mem + p.bits;
  const uint32_t *cw = (const uint32_t *)(p.codes + r * (int64_t)p.code_stride);
  const uint32_t st = __ldg(p.start + r);
  const int rw = p.code_stride >> 2;
  const float gs = (float)((double)g * s);  // exact: s is a power of two
  double xs = 0.0;
  for (int c = 0; c < p.kpad / 8; c++) {
    uint32_t o[4];
    if (8 * c >= p.dim) {  // zero padding up to kpad
      xrow[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
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
      const uint32_t hx = __half_as_ushort(__float2half_rn(fmul(gs, x)));
      if (h & 1) o[h >> 1] |= hx << 16;
      else o[h >> 1] = hx;
    }
    xrow[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  const double qn = 1.0001;
  const double xn = sqrt(xs) * (1.0 + 1e-12);
  const double sg = s * (double)g;
  const double cd = (sg * p.eps * qn * xn + 1.1920928955078125e-7 * sqrt((double)p.dim) *
                                                (qn + sg * xn)) * (1.0 + 1e-6);
  const uint32_t hc = __half_as_ushort(__float2half_ru(__double2float_ru(cd)));
  xext[0] = make_uint4(hc, 0, 0, 0);
  xext[1] = make_uint4(0, 0, 0, 0);
}

// The same rows for widths 1, 2 and 4 with the code table in shared memory:
// each record's code is read 16 bytes at a time and its windows are cut with
// shifts known at compile time (code rows are padded to 16 bytes); one
// thread per record.
//
// F32SUM (the default): the conversions of tc_prepare_records_kernel run on
// the SM's conversion (XU) pipe, which bounds this kernel together with the
// table lookups, so |x|^2 is summed in f32 (one fma per coordinate, no
// widening to f64) and each pair of B' values is rounded to fp16 by one
// paired conversion (the same round-to-nearest bits).  Every term is
// non-negative, so with at most dim roundings of relative size 2^-24 the
// exact sum is at most the computed one times (1 + (dim + 64) 2^-23); terms
// below the f32 normal range lose at most 2^-149 each, far inside the
// bound's absolute term.  C' may then exceed the f64 sum's by a unit of its
// last fp16 place; both are valid bounds, and B' is the same bits.
// !F32SUM: the f64 sum and per-value conversions of tc_prepare_records_kernel.
template <int BITS, bool F32SUM>
__global__ void __launch_bounds__(256) tc_prepare_records_fast_kernel(const TcPrepareParams p) {
  extern __shared__ float tab[];
  for (int i = threadIdx.x; i < (1 << (p.mem + BITS)); i += blockDim.x) tab[i] = __ldg(p.code + i);
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= p.n_pad) return;
  uint4 *xrow = (uint4 *)(p.x16 + r * p.kpad);
  uint4 *xext = (uint4 *)(p.xext + r * TC_X);
  const uint32_t hinf = 0x7C00u;  // fp16 +inf
  float g = r < p.n ? record_g(p, r) : 0.0f;
  const bool bad = r >= p.n || !isfinite(g) || g < 0.0f;
  const float gmax = __uint_as_float(*p.gmax_bits);
  const double top = (double)gmax * (double)p.code_absmax;
  const int e = top > 0.0 ? (int)ceil(log2(top)) - 14 : 0;
  const double s = ldexp(1.0, -e);
  if (bad) {
    for (int c = 0; c < p.kpad / 8; c++) xrow[c] = make_uint4(0, 0, 0, 0);
    xext[0] = make_uint4(hinf, 0, 0, 0);
    xext[1] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint32_t wmask = (1u << (p.mem + BITS)) - 1u;
  const uint4 *cw4 = (const uint4 *)(p.codes + r * (int64_t)p.code_stride);
  const float gs = (float)((double)g * s);  // exact: s is a power of two
  double xs = 0.0;
  float xs32 = 0.0f;
  constexpr int CPC = 128 / BITS;  // coordinates per 16-byte chunk
  uint32_t prev = __ldg(p.start + r);
  const int nchunks = (p.dim + CPC - 1) / CPC;
  for (int k = 0; k < nchunks; k++) {
    const uint4 raw = __ldg(cw4 + k);
    const uint32_t w[4] = {__byte_perm(raw.x, 0, 0x0123), __byte_perm(raw.y, 0, 0x0123),
                           __byte_perm(raw.z, 0, 0x0123), __byte_perm(raw.w, 0, 0x0123)};
#pragma unroll
    for (int g8 = 0; g8 < CPC / 8; g8++) {
      const int c0 = k * CPC + g8 * 8;
      if (c0 >= p.dim) break;
      uint32_t o[4];
      float xv[8];
#pragma unroll
      for (int h = 0; h < 8; h++) {
        const int e2 = (g8 * 8 + h + 1) * BITS;  // chunk bits consumed through this window
        const int wi = (e2 - 1) >> 5;
        const int sh = 31 - ((e2 - 1) & 31);
        const uint32_t hiw = wi == 0 ? prev : w[wi > 0 ? wi - 1 : 0];
        const uint64_t v = ((uint64_t)hiw << 32) | w[wi];
        const float x = tab[(uint32_t)(v >> sh) & wmask];
        xv[h] = x;
        if (F32SUM) {
          xs32 = __fmaf_rn(x, x, xs32);
        } else {
          xs += (double)x * (double)x;
          const uint32_t hx = __half_as_ushort(__float2half_rn(fmul(gs, x)));
          if (h & 1)
            o[h >> 1] |= hx << 16;
          else
            o[h >> 1] = hx;
        }
      }
      if (F32SUM) {
#pragma unroll
        for (int h = 0; h < 4; h++) {
          // low half: the even coordinate
          const __half2 pr = __floats2half2_rn(fmul(gs, xv[2 * h]), fmul(gs, xv[2 * h + 1]));
          memcpy(&o[h], &pr, sizeof(uint32_t));
        }
      }
      xrow[c0 / 8] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    prev = w[3];
  }
  for (int c = (p.dim + 7) / 8; c < p.kpad / 8; c++) xrow[c] = make_uint4(0, 0, 0, 0);
  if (F32SUM) xs = (double)xs32 * (1.0 + (double)(p.dim + 64) * 0x1p-23);
  const double qn = 1.0001;
  const double xn = sqrt(xs) * (1.0 + 1e-12);
  const double sg = s * (double)g;
  const double cd = (sg * p.eps * qn * xn + 1.1920928955078125e-7 * sqrt((double)p.dim) *
                                                (qn + sg * xn)) * (1.0 + 1e-6);
  const uint32_t hc = __half_as_ushort(__float2half_ru(__double2float_ru(cd)));
  xext[0] = make_uint4(hc, 0, 0, 0);
  xext[1] = make_uint4(0, 0, 0, 0);
}

// ---------------------------------------------------------------------------
// The first pass's sample.  The k-th largest lower bound of any set of
// distinct records is a score k records reach, so pass 1 may bound any
// subset of the records; the tighter the threshold, the fewer candidates
// pass 2 admits.  Instead of every S-th tile, pass 1 bounds the n/S records
// of largest score scale g (rnorm / rescale, times the row norm for MIPS):
// the records whose scores spread widest, which hold most of every query's
// best scores when the norms vary (the heavy-tailed MIPS corpora).  They are
// chosen by a two-level 12-bit histogram of g's bits (positive floats order
// as unsigned integers) and copied, operand rows and bound constants, into
// a compact sample that pass 1 streams like the full rows.  Records past the
// sample's capacity are dropped and unfilled slots are padding rows (zero,
// bound constant +inf), so any outcome is a subset of distinct records.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t hot_key(const TcPrepareParams &p, int64_t r) {
  const float g = record_g(p, r);
  return (isfinite(g) && g > 0.0f) ? __float_as_uint(g) : 0u;
}

// The keys, and the level-0 histogram (key >> 20).  Lanes that meet in one
// bin add once (__match_any_sync): the scales of a corpus fall in a few
// bins, and plain shared atomics would serialize on them.
__global__ void __launch_bounds__(256) tc_hot_keys_kernel(const TcPrepareParams p, uint32_t *keys,
                                                          uint32_t *hist) {
  __shared__ uint32_t h[4096];
  for (int i = threadIdx.x; i < 4096; i += 256) h[i] = 0u;
  __syncthreads();
  const int64_t stride = (int64_t)gridDim.x * 256;
  const int64_t n_round = (p.n + 255) / 256 * 256;  // whole warps in every round
  for (int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x; r < n_round; r += stride) {
    const uint32_t key = r < p.n ? hot_key(p, r) : 0u;
    if (r < p.n) keys[r] = key;
    const uint32_t bin = key >> 20;
    const uint32_t peers = __match_any_sync(0xffffffffu, bin);
    if (key != 0u && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&h[bin], __popc(peers));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 4096; i += 256)
    if (h[i] != 0u) atomicAdd(&hist[i], h[i]);
}

// Level 1: histogram of (key >> 8) & 4095 over the keys in bin sel[0].
__global__ void __launch_bounds__(256) tc_hot_hist_kernel(const uint32_t *keys, int64_t n,
                                                          const uint32_t *sel, uint32_t *hist) {
  __shared__ uint32_t h[4096];
  for (int i = threadIdx.x; i < 4096; i += 256) h[i] = 0u;
  __syncthreads();
  const uint32_t b0 = sel[0];
  const int64_t stride = (int64_t)gridDim.x * 256;
  const int64_t n_round = (n + 255) / 256 * 256;
  for (int64_t r = (int64_t)blockIdx.x * 256 + threadIdx.x; r < n_round; r += stride) {
    const uint32_t key = r < n ? keys[r] : 0u;
    const bool in = key != 0u && (key >> 20) == b0 && sel[3] == 0u;
    const uint32_t bin = in ? (key >> 8) & 4095u : 0xffffffffu;
    const uint32_t peers = __match_any_sync(0xffffffffu, bin);
    if (in && (threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&h[bin], __popc(peers));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 4096; i += 256)
    if (h[i] != 0u) atomicAdd(&hist[i], h[i]);
}

// One CTA of 256 threads: the highest bin at which the count from the top
// reaches `want` (level 0: sel[0] = bin, sel[1] = records in higher bins;
// level 1: sel[2] = the sample's smallest key, (sel[0] << 20) | (bin << 8);
// a base with fewer keyed records than `want` takes all of them, key 1).
__global__ void __launch_bounds__(256) tc_hot_pick_kernel(const uint32_t *hist, int64_t want,
                                                          int level, uint32_t *sel) {
  __shared__ unsigned long long part[256];
  const int t = threadIdx.x;
  // thread t holds bins [4080 - 16 t, 4096 - 16 t): higher bins on lower t
  unsigned long long mine = 0;
  for (int b = 4095 - 16 * t; b > 4095 - 16 * (t + 1); b--) mine += hist[b];
  part[t] = mine;
  __syncthreads();
  if (t == 0) {
    const unsigned long long above = (level == 1) ? sel[1] : 0ull;
    if (level == 1 && sel[3] != 0u) return;
    unsigned long long acc = above;
    int tt = 0;
    for (; tt < 256; tt++) {
      if (acc + part[tt] >= (unsigned long long)want) break;
      acc += part[tt];
    }
    int b = -1;
    if (tt < 256) {
      for (b = 4095 - 16 * tt; b > 4095 - 16 * (tt + 1); b--) {
        acc += hist[b];
        if (acc >= (unsigned long long)want) break;
      }
    }
    if (level == 0) {
      if (b < 0) {  // every keyed record fits
        sel[0] = 0u;
        sel[1] = 0u;
        sel[2] = 1u;
        sel[3] = 1u;
        return;
      }
      sel[0] = (uint32_t)b;
      sel[1] = (uint32_t)(acc - hist[b]);
      sel[3] = 0u;
    } else {
      sel[2] = (sel[0] << 20) | ((uint32_t)(b < 0 ? 0 : b) << 8);
    }
  }
}

// The sample in record order: tc_hot_count_kernel counts each CTA's sample
// records (CTA c covers records [c * span, (c + 1) * span)),
// tc_hot_scan_kernel turns the counts into offsets, tc_hot_gather_kernel
// copies every sample record's operand row and bound constants to its slot
// (slots at or past cap are dropped).  Deterministic: the same index gives
// the same sample, whatever the order the threads run in.
__global__ void __launch_bounds__(256) tc_hot_count_kernel(const uint32_t *keys, int64_t n,
                                                           int64_t span, const uint32_t *sel,
                                                           uint32_t *counts) {
  __shared__ uint32_t c;
  if (threadIdx.x == 0) c = 0u;
  __syncthreads();
  const uint32_t t = sel[2];
  const int64_t lo = (int64_t)blockIdx.x * span, hi = min(n, lo + span);
  uint32_t mine = 0;
  for (int64_t r = lo + threadIdx.x; r < hi; r += 256) mine += (keys[r] != 0u && keys[r] >= t);
  atomicAdd(&c, mine);
  __syncthreads();
  if (threadIdx.x == 0) counts[blockIdx.x] = c;
}

__global__ void __launch_bounds__(1024) tc_hot_scan_kernel(uint32_t *counts, int blocks) {
  __shared__ uint32_t s[1024];
  const int t = threadIdx.x;
  // up to 1024 x 4 blocks: each thread sums (then offsets) 4 consecutive counts
  uint32_t v[4], tot = 0;
  for (int j = 0; j < 4; j++) {
    const int b = 4 * t + j;
    v[j] = b < blocks ? counts[b] : 0u;
    tot += v[j];
  }
  s[t] = tot;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const uint32_t x = t >= o ? s[t - o] : 0u;
    __syncthreads();
    s[t] += x;
    __syncthreads();
  }
  uint32_t ex = s[t] - tot;
  for (int j = 0; j < 4; j++) {
    const int b = 4 * t + j;
    if (b < blocks) counts[b] = ex;
    ex += v[j];
  }
}

__global__ void __launch_bounds__(256) tc_hot_gather_kernel(const TcPrepareParams p,
                                                            const uint32_t *keys, int64_t span,
                                                            const uint32_t *sel,
                                                            const uint32_t *offs, int64_t cap,
                                                            uint16_t *x16_hot,
                                                            uint16_t *xext_hot) {
  __shared__ uint32_t warp_tot[8];
  __shared__ uint32_t base_s;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t t = sel[2];
  const int64_t lo = (int64_t)blockIdx.x * span, hi = min(p.n, lo + span);
  if (tid == 0) base_s = offs[blockIdx.x];
  __syncthreads();
  for (int64_t r0 = lo; r0 < hi; r0 += 256) {
    const int64_t r = r0 + tid;
    const bool in = r < hi && keys[r] != 0u && keys[r] >= t;
    const uint32_t ball = __ballot_sync(0xffffffffu, in);
    if (lane == 0) warp_tot[warp] = __popc(ball);
    __syncthreads();
    uint32_t before = base_s;
    for (int w = 0; w < warp; w++) before += warp_tot[w];
    const uint32_t j = before + __popc(ball & ((1u << lane) - 1u));
    if (in && (int64_t)j < cap) {
      const uint4 *src = (const uint4 *)(p.x16 + r * p.kpad);
      uint4 *dst = (uint4 *)(x16_hot + (int64_t)j * p.kpad);
      for (int c = 0; c < p.kpad / 8; c++) dst[c] = __ldg(src + c);
      const uint4 *se = (const uint4 *)(p.xext + r * TC_X);
      uint4 *de = (uint4 *)(xext_hot + (int64_t)j * TC_X);
      de[0] = __ldg(se);
      de[1] = __ldg(se + 1);
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t add = 0;
      for (int w = 0; w < 8; w++) add += warp_tot[w];
      base_s += add;
    }
    __syncthreads();
  }
}

// Unfilled sample slots: padding rows (zero row, bound constant +inf).
// offs_end is the scanned offset past the last CTA (the sample's size).
__global__ void tc_hot_pad_kernel(const uint32_t *offs_end, int64_t cap, int kpad,
                                  uint16_t *x16_hot, uint16_t *xext_hot) {
  const int64_t filled = min((int64_t)*offs_end, cap);
  for (int64_t j = filled + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < cap;
       j += (int64_t)gridDim.x * blockDim.x) {
    uint4 *dst = (uint4 *)(x16_hot + j * kpad);
    for (int c = 0; c < kpad / 8; c++) dst[c] = make_uint4(0, 0, 0, 0);
    uint4 *de = (uint4 *)(xext_hot + j * TC_X);
    de[0] = make_uint4(0x7C00u, 0, 0, 0);
    de[1] = make_uint4(0, 0, 0, 0);
  }
}

__global__ void __launch_bounds__(256)
    tc_chunk_cmax_kernel(const uint16_t *xext, int64_t n, int64_t n_pad, float *cmax) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_pad) return;  // whole warps: n_pad % 32 == 0
  float c = r < n ? __half2float(__ushort_as_half(xext[r * TC_X])) : 0.0f;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) c = fmaxf(c, __shfl_xor_sync(0xffffffffu, c, o));
  if ((threadIdx.x & 15) == 0) cmax[r >> 4] = c;
}

const void *tc_prepare_records_fast_ptr(int bits, bool f32sum) {
  switch (bits) {
    case 1: return f32sum ? (const void *)tc_prepare_records_fast_kernel<1, true>
                          : (const void *)tc_prepare_records_fast_kernel<1, false>;
    case 2: return f32sum ? (const void *)tc_prepare_records_fast_kernel<2, true>
                          : (const void *)tc_prepare_records_fast_kernel<2, false>;
    case 4: return f32sum ? (const void *)tc_prepare_records_fast_kernel<4, true>
                          : (const void *)tc_prepare_records_fast_kernel<4, false>;
  }
  return nullptr;
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
                                                        int64_t nq, int k, float *theta,
                                                        int lists) {
  extern __shared__ uint32_t keys_s[];  // n_tiles keys when they fit (see the launch)
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel[2];
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  // one list: query q's n_tiles values at tmax[q * n_tiles + i]; several
  // (gathered shard-major, lists x nq x per): value i is element i % per of
  // list i / per
  const int64_t per = n_tiles / lists;
  const float *v1 = tmax + q * n_tiles;
  auto at = [&](int64_t i) -> float {
    if (lists == 1) return v1[i];
    const int64_t l = i / per;
    return tmax[(l * nq + q) * per + (i - l * per)];
  };
  if (n_tiles < k) {
    if (threadIdx.x == 0) theta[q] = -INFINITY;
    return;
  }
  // the four radix passes read the maxima from shared memory when they fit
  const bool staged = n_tiles <= kThetaSmemKeys;
  if (staged)
    for (int64_t i = threadIdx.x; i < n_tiles; i += 256) keys_s[i] = fkey(at(i));
  uint32_t prefix = 0, mask = 0, kk = (uint32_t)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    hist[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < n_tiles; i += 256) {
      const uint32_t key = staged ? keys_s[i] : fkey(at(i));
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

// A shard's contribution to a threshold shared by several shards: the k
// largest group lower bounds of each query as a multiset (any order) -- the
// values above the query's k-th largest (theta, from tc_theta_kernel), then
// theta repeated up to k (-inf when the query has fewer than k groups).
// Every value is reached by a distinct record of the shard.
__global__ void __launch_bounds__(256) tc_bounds_kernel(const float *tmax, int64_t n_groups,
                                                        int64_t nq, int k, const float *theta,
                                                        float *bounds) {
  __shared__ int cnt;
  const int64_t q = blockIdx.x;
  if (q >= nq) return;
  if (threadIdx.x == 0) cnt = 0;
  __syncthreads();
  const float th = theta[q];
  const uint32_t tk = fkey(th);
  const float *v = tmax + q * n_groups;
  float *out = bounds + q * (int64_t)k;
  for (int64_t i = threadIdx.x; i < n_groups; i += 256) {
    const float x = v[i];
    if (fkey(x) > tk) {
      const int pos = atomicAdd(&cnt, 1);
      if (pos < k) out[pos] = x;
    }
  }
  __syncthreads();
  for (int i = min(cnt, k) + threadIdx.x; i < k; i += 256) out[i] = th;
}

// The same k-th largest value for up to kThetaWarpKeys values per query, one
// warp per query with the keys in registers: the answer's bits are fixed
// from the top, each by counting the keys at or above the candidate (a
// ballot-free count and one warp reduction per bit), with no shared-memory
// histogram and no block barrier.
template <int NJ>
__global__ void __launch_bounds__(256) tc_theta_warp_kernel(const float *tmax, int64_t n_tiles,
                                                            int64_t nq, int k, float *theta,
                                                            int lists) {
  const int lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (q >= nq) return;  // whole warps
  if (n_tiles < k) {
    if (lane == 0) theta[q] = -INFINITY;
    return;
  }
  const int64_t per = n_tiles / lists;
  uint32_t v[NJ];
#pragma unroll
  for (int j = 0; j < NJ; j++) {
    const int64_t i = lane + 32 * j;
    float x = -INFINITY;
    if (i < n_tiles) {
      if (lists == 1) {
        x = tmax[q * n_tiles + i];
      } else {
        const int64_t l = i / per;
        x = tmax[(l * nq + q) * per + (i - l * per)];
      }
    }
    v[j] = i < n_tiles ? fkey(x) : 0u;
  }
  uint32_t prefix = 0u;
  for (int bit = 31; bit >= 0; bit--) {
    const uint32_t cand = prefix | (1u << bit);
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < NJ; j++) c += v[j] >= cand ? 1u : 0u;
    c = __reduce_add_sync(0xffffffffu, c);
    if (c >= (uint32_t)k) prefix = cand;
  }
  if (lane == 0) theta[q] = fkey_inv(prefix);
}

const void *tc_theta_warp_kernel_ptr(int64_t n_tiles) {
  if (n_tiles <= 32 * 8) return (const void *)tc_theta_warp_kernel<8>;
  if (n_tiles <= 32 * 16) return (const void *)tc_theta_warp_kernel<16>;
  if (n_tiles <= 32 * 32) return (const void *)tc_theta_warp_kernel<32>;
  if (n_tiles <= 32 * 64) return (const void *)tc_theta_warp_kernel<64>;
  return nullptr;
}

// ---------------------------------------------------------------------------
// Exact scores of the candidates (simd.rs:183-262 association: 16 FMA chains
// over 16-wide blocks, then the hsum256 tree; trellis.rs:1517 estimator) and
// the query's top-k by (score desc, record asc).  One CTA per query; two
// candidates per warp at a time, one per half-warp.  A query whose list
// overflowed is recorded for the exact fallback scan.
// ---------------------------------------------------------------------------
template <int BITS, bool PER_THREAD>
__global__ void __launch_bounds__(256) tc_rescore_kernel(const TcRescoreParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint64_t *keys = (uint64_t *)sm;                    // cap (power of two)
  uint32_t *cidx = (uint32_t *)(keys + p.cap);        // cap gathered candidates
  int *roff = (int *)(cidx + p.cap);                  // regions + 1 segment offsets
  float *qv = (float *)(roff + ((p.regions + 4) & ~3));  // dim
  float *table = qv + p.dim;                          // table_len (optional)
  // every query, or those the warp kernel left (a device count: CTAs past
  // it leave at once)
  if (p.big_list != nullptr && (int)blockIdx.x >= *p.n_big) return;
  const int64_t q = p.big_list != nullptr ? (int64_t)p.big_list[blockIdx.x] : (int64_t)blockIdx.x;
  if (q >= p.nq) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // gather the segments pass 2 wrote (one per record split and column slice);
  // a full segment or more than cap candidates in all sends the query to
  // the exact scan
  if (warp == 0) {
    // lane l owns regions [l*per, (l+1)*per); an exclusive scan gives offsets
    const int per = (p.regions + 31) >> 5;  // <= 8
    int c_loc[8];
    int tot = 0;
    bool over = false;
#pragma unroll
    for (int t = 0; t < 8; t++) {
      const int r = lane * per + t;
      int c = (t < per && r < p.regions) ? p.cand_cnt[q * p.regions + r] : 0;
      over |= c > p.region_cap;
      c = min(c, p.region_cap);
      c_loc[t] = c;
      tot += c;
    }
    int incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int ex = incl - tot;
#pragma unroll
    for (int t = 0; t < 8; t++) {
      const int r = lane * per + t;
      if (t < per && r < p.regions) roff[r] = ex;
      ex += c_loc[t];
    }
    const bool any_over = __any_sync(0xffffffffu, over);
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) roff[p.regions] = (any_over || total > p.cap) ? -1 : total;
  }
  __syncthreads();
  const int cnt_raw = roff[p.regions];
  if (cnt_raw < 0) {
    if (tid == 0) p.over_list[atomicAdd(p.n_over, 1)] = (int32_t)q;
    return;
  }
  // every entry at once: its region is the last r with roff[r] <= i (a
  // non-empty one, since i < roff[regions]), found by bisection
  for (int i = tid; i < cnt_raw; i += 256) {
    int lo = 0, hi = p.regions - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (roff[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    cidx[i] = p.cand[q * p.cand_stride + (int64_t)lo * p.region_cap + (i - roff[lo])];
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
  if constexpr (!PER_THREAD) {
    // few candidates: half a warp per candidate, 16 lanes over the
    // coordinates (the 16 FMA chains), its record image staged in shared
    // memory by one coalesced load per lane
    const int W = p.mem + p.bits;
    const int rw = p.code_stride >> 2;
    const int j = lane & 15, half = lane >> 4;
    uint32_t *img = (uint32_t *)(table + (p.table_in_smem ? p.table_len : 0)) +
                    (warp * 2 + half) * (rw + 1);
    for (int i0 = warp * 2; i0 < cnt; i0 += 16) {
      const int i = i0 + half;
      const bool ok = i < cnt;
      const int64_t rec = ok ? (int64_t)cidx[i] : 0;
      const uint32_t *cw = (const uint32_t *)(p.codes + rec * (int64_t)p.code_stride);
      for (int w = j; w <= rw; w += 16)
        img[w] = w == 0 ? __ldg(p.start + rec) : __byte_perm(__ldg(cw + w - 1), 0, 0x0123);
      float rs = 1.0f, rn = 1.0f, nm = 1.0f;
      if (ok && j == 0) {
        rs = __ldg(p.rescale + rec);
        if (p.rnorm) rn = __ldg(p.rnorm + rec);
        if (p.mips) nm = __ldg(p.norms + rec);
      }
      __syncwarp();
      float acc = 0.0f;
      for (int b = 0; b < p.dim / 16; b++) {
        const int c = 16 * b + j;
        const int pos = 32 + c * p.bits - p.mem;
        const int w0 = pos >> 5, sh = pos & 31;
        const uint32_t hi = img[w0];
        const uint32_t lo = w0 + 1 <= rw ? img[w0 + 1] : 0u;
        const uint32_t win = __funnelshift_l(lo, hi, sh) >> (32 - W);
        acc = fmaf(qv[c], code[win], acc);
      }
      acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
      acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
      acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
      acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
      if (ok && j == 0) {
        float sx = fadd(0.0f, fmul(rn, fdiv(acc, rs)));
        if (p.mips) sx = fmul(sx, nm);
        keys[i] = rank_key(sx, (uint32_t)rec);
      }
      __syncwarp();  // the image is rewritten for the next candidate
    }
  } else {
    // many candidates: one thread per candidate, the whole record dot in
    // registers (record_dot_thread, the same association), many candidates
    // in flight per SM
    for (int i = tid; i < cnt; i += 256) {
      const int64_t rec = (int64_t)cidx[i];
      const uint8_t *rc = p.codes + rec * (int64_t)p.code_stride;
      const uint32_t st = __ldg(p.start + rec);
      const float rs = __ldg(p.rescale + rec);
      const float rn = p.rnorm ? __ldg(p.rnorm + rec) : 1.0f;
      const float acc = record_dot_thread<BITS>(qv, rc, st, p.dim, p.mem, p.code_stride, code, 1, 0);
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

// The same exact rescoring, one warp per query, for queries whose candidate
// list holds at most kRescoreWarpCap entries and no full segment (the others
// are listed for tc_rescore_kernel, launched after this one).
// Many short lists are the multi-GPU case, where a shared threshold leaves
// each shard a few dozen candidates per query: a CTA per query would spend
// most of its time on set-up and block-wide barriers.  The code table sits
// in kRescoreCopies interleaved copies (entry w of copy c at w * copies + c,
// lane l reading copy l % copies), so the candidates' random lookups rarely
// meet in one bank.
template <int BITS>
__global__ void __launch_bounds__(32 * kRescoreWarps, 2) tc_rescore_warp_kernel(
    const TcRescoreParams p) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int CAP = kRescoreWarpCap, NC = kRescoreCopies;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float *table = (float *)sm;
  const size_t roff_words = ((size_t)p.regions + 4) & ~(size_t)3;
  const size_t per_warp = (size_t)CAP * 12 + (size_t)kRescoreWarpDim * 4 + roff_words * 4;
  uint8_t *wb = sm + (size_t)p.table_len * NC * 4 + (size_t)warp * per_warp;
  uint64_t *keys = (uint64_t *)wb;
  uint32_t *cidx = (uint32_t *)(keys + CAP);
  float *qv = (float *)(cidx + CAP);
  int *roff = (int *)(qv + kRescoreWarpDim);
  for (int e = tid; e < p.table_len * NC; e += 32 * kRescoreWarps)
    table[e] = __ldg(p.code + e / NC);
  __syncthreads();
  const int64_t q = (int64_t)blockIdx.x * kRescoreWarps + warp;
  if (q >= p.nq) return;  // whole warps leave, after the only block barrier
  // segment counts and offsets (as tc_rescore_kernel's warp 0)
  const int per = (p.regions + 31) >> 5;  // <= 8
  int c_loc[8];
  int tot = 0;
  bool over = false;
#pragma unroll
  for (int t = 0; t < 8; t++) {
    const int r = lane * per + t;
    int c = (t < per && r < p.regions) ? p.cand_cnt[q * p.regions + r] : 0;
    over |= c > p.region_cap;
    c = min(c, p.region_cap);
    c_loc[t] = c;
    tot += c;
  }
  int incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int ex = incl - tot;
#pragma unroll
  for (int t = 0; t < 8; t++) {
    const int r = lane * per + t;
    if (t < per && r < p.regions) roff[r] = ex;
    ex += c_loc[t];
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (__any_sync(0xffffffffu, over) || total > CAP) {
    // a long list or a full segment: tc_rescore_kernel takes the query
    if (lane == 0) p.big_list[atomicAdd(p.n_big, 1)] = (int32_t)q;
    return;
  }
  __syncwarp();
  for (int i = lane; i < total; i += 32) {
    int lo = 0, hi = p.regions - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (roff[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    cidx[i] = p.cand[q * p.cand_stride + (int64_t)lo * p.region_cap + (i - roff[lo])];
  }
  const int cnt = p.degenerate[q] ? 0 : total;
  if (lane == 0) atomicAdd(p.n_cand, (unsigned long long)cnt);
  int pow2 = 32;
  while (pow2 < cnt) pow2 <<= 1;
  for (int i = lane; i < p.dim; i += 32) qv[i] = p.q_r[q * (int64_t)p.q_stride + i];
  for (int i = lane; i < pow2; i += 32) keys[i] = kEmptyKey;
  __syncwarp();
  for (int i = lane; i < cnt; i += 32) {
    const int64_t rec = (int64_t)cidx[i];
    const uint8_t *rc = p.codes + rec * (int64_t)p.code_stride;
    const uint32_t st = __ldg(p.start + rec);
    const float rs = __ldg(p.rescale + rec);
    const float rn = p.rnorm ? __ldg(p.rnorm + rec) : 1.0f;
    const float acc =
        record_dot_thread<BITS>(qv, rc, st, p.dim, p.mem, p.code_stride, table, NC, lane % NC);
    float sx = fadd(0.0f, fmul(rn, fdiv(acc, rs)));
    if (p.mips) sx = fmul(sx, __ldg(p.norms + rec));
    keys[i] = rank_key(sx, (uint32_t)rec);
  }
  __syncwarp();
  // bitonic sort of the warp's keys, descending
  for (int size = 2; size <= pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int pi = lane; pi < pow2 / 2; pi += 32) {
        const int lo = 2 * pi - (pi & (stride - 1));
        const int hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = keys[lo], y = keys[hi];
        if ((x < y) == desc) {
          keys[lo] = y;
          keys[hi] = x;
        }
      }
      __syncwarp();
    }
  }
  for (int i = lane; i < p.k; i += 32) {
    const uint64_t key = i < pow2 ? keys[i] : kEmptyKey;
    const bool full = key != kEmptyKey;
    const int64_t rec = rank_key_index(key);
    p.out_id[q * p.k + i] = full ? (p.ids ? p.ids[rec] : rec) : -1;
    p.out_score[q * p.k + i] = full ? key32_score((uint32_t)(key >> 32)) : -INFINITY;
  }
}

const void *tc_rescore_warp_kernel_ptr(int bits) {
  switch (bits) {
    case 1: return (const void *)tc_rescore_warp_kernel<1>;
    case 2: return (const void *)tc_rescore_warp_kernel<2>;
    case 3: return (const void *)tc_rescore_warp_kernel<3>;
    case 4: return (const void *)tc_rescore_warp_kernel<4>;
  }
  return nullptr;
}

size_t tc_rescore_warp_smem_bytes(int table_len, int regions) {
  const size_t roff_words = ((size_t)regions + 4) & ~(size_t)3;
  const size_t per_warp = (size_t)kRescoreWarpCap * 12 + (size_t)kRescoreWarpDim * 4 +
                          roff_words * 4;
  return (size_t)table_len * kRescoreCopies * 4 + per_warp * kRescoreWarps;
}

size_t tc_scan_smem_bytes(int shape) {
  return shape == 3 ? (size_t)TcShape<3>::total : (size_t)TcShape<1>::total;
}

const void *tc_scan_kernel_ptr(int mode, int shape) {
  if (shape == 3)
    return mode == 1 ? (const void *)tc_scan_kernel<1, 3> : (const void *)tc_scan_kernel<2, 3>;
  return mode == 1 ? (const void *)tc_scan_kernel<1, 1> : (const void *)tc_scan_kernel<2, 1>;
}

const void *tc_rescore_kernel_ptr(int bits, bool per_thread) {
#define UV_RS_CASE(b)                                                              \
  case b:                                                                          \
    return per_thread ? (const void *)tc_rescore_kernel<b, true>                   \
                      : (const void *)tc_rescore_kernel<b, false>;
  switch (bits) {
    UV_RS_CASE(1)
    UV_RS_CASE(2)
    UV_RS_CASE(3)
    UV_RS_CASE(4)
  }
#undef UV_RS_CASE
  return nullptr;
}

int tc_threads() { return TC_THREADS; }
int tc_groups_per_tile() { return TcShape<3>::SLICES; }
int tc_tile_records() { return TcShape<1>::TN; }
int tc_tile_queries() { return TC_M; }
int tc_dim() { return TC_D; }

}  // namespace uvb
