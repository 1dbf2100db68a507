// tcwide.cu -- the tensor-core prefilter for rows of any width (sm_100a).
//
// The same certified bounds as tcscan.cu (lower bounds in pass 1, upper
// bounds in pass 2, both produced by the MMA through the extra K slice), for
// dimensions other than 128: the query rows and the record rows are both
// streamed through shared memory in K chunks of 64 (a pipeline step = one
// chunk of one 192-record tile: a 128 x 64 query chunk and a 192 x 64 record
// chunk, 40 KB, 128-byte swizzle; the tile's last step carries the 16-wide
// extra slices, 32-byte swizzle).  Four MMAs of 128 x 192 x 16 per chunk
// accumulate into one of two TMEM accumulators; the epilogue (the bounds of
// uv_tc_epilogue.cuh) runs when a tile's last step has been committed.
//
// Warp roles as in tcscan.cu: warps 0-7 epilogue (TMEM lane quarter w % 4,
// column half w / 4), warp 8 TMEM allocation and MMA issue, warp 9 TMA.  Five
// 40 KB stages; every wait is bounded.  No cluster multicast.
#include <cuda.h>

#include "uv_kernels.h"
#include "uv_tc.cuh"
#include "uv_tc_epilogue.cuh"

namespace uvb {

namespace {

constexpr int W_M = 128;        // queries per CTA
constexpr int W_N = 192;        // records per tile
constexpr int W_STAGES = 5;
constexpr int W_THREADS = 320;
constexpr int W_A = W_M * 128;  // 128 x 64 fp16 query chunk
constexpr int W_B = W_N * 128;  // 192 x 64 fp16 record chunk
constexpr int W_STAGE = W_A + W_B;        // 40 KB
constexpr int W_AX = W_M * 32;            // extra slices (16 fp16 per row)
constexpr int W_BX = W_N * 32;
constexpr int W_BARS = W_STAGES * W_STAGE;
constexpr int W_MISC = W_BARS + 16 * 8;
constexpr int W_TOTAL = W_MISC + 64;
constexpr uint32_t kWaitLimit = 1u << 20;
static_assert(W_STAGE % 1024 == 0 && W_A % 1024 == 0, "stage alignment");
static_assert(W_TOTAL <= 227 * 1024, "shared memory");

}  // namespace

template <int MODE>
__global__ void __launch_bounds__(W_THREADS, 1)
    tc_wide_kernel(const TcScanParams p, int kchunks,
                   const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_ax,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_bx) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t *full = (uint64_t *)(sm + W_BARS);  // [W_STAGES]
  uint64_t *empty = full + W_STAGES;           // [W_STAGES]
  uint64_t *accf = empty + W_STAGES;           // [2]
  uint64_t *acce = accf + 2;                   // [2]
  uint64_t *drained = acce + 2;                // MMAs done after an abort
  uint32_t *tbase_s = (uint32_t *)(sm + W_MISC);
  volatile int *abort_s = (volatile int *)(sm + W_MISC + 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t q0 = (int64_t)blockIdx.x * W_M;
  const int64_t t_begin = p.n_tiles * blockIdx.y / gridDim.y;
  const int64_t t_end = p.n_tiles * (blockIdx.y + 1) / gridDim.y;
  const int ntiles = (int)(t_end - t_begin);
  const int steps = kchunks + 1;  // K chunks of 64, then the extra slice

  if (tid == 0) {
    for (int s = 0; s < W_STAGES; s++) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; a++) {
      tc::mbar_init(&accf[a], 1);
      tc::mbar_init(&acce[a], 8);  // one arrival per epilogue warp
    }
    tc::mbar_init(drained, 1);
    *abort_s = 0;
    tc::mbar_fence_init();
  }
  if (warp == 8) tc::tmem_alloc(tbase_s, 512);
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
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(half * 96);
    // pass 2: this thread's segment of the query's candidate list
    const int region = (int)blockIdx.y * 2 + half;
    uint32_t *seg = MODE == 2 ? p.cand + q * (int64_t)p.cand_cap + (int64_t)region * p.region_cap
                              : nullptr;
    int seg_cnt = 0;
    for (int it = 0; it < ntiles; it++) {
      const int a = it & 1;
      const int64_t tile = t_begin + it;
      if (!tc::mbar_wait(&accf[a], (it >> 1) & 1, kWaitLimit)) {
        *abort_s = 1;
        atomicExch(p.err, 1);
      }
      if (*abort_s) break;
      tc::tc_fence_after();
      const uint32_t base = lane_base + (uint32_t)(a * W_N);
      uint32_t r[3][32];
#pragma unroll
      for (int l = 0; l < 3; l++) tc::tmem_ld32(base + 32 * l, r[l]);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[a]);
      tcep::bounds_run<MODE, 3>(p, r, q, qok, theta, 2 * tile + half,
                                tile * p.tile_stride * W_N + half * 96, seg, &seg_cnt);
    }
    if (MODE == 2 && q < p.nq) p.cand_cnt[q * p.regions + region] = seg_cnt;
  } else if (warp == 8) {
    if (lane == 0) {
      // ================= MMA issue =================
      const uint32_t idesc = tc::idesc_f16_f32(W_M, W_N);
      int64_t step = 0;
      for (int it = 0; it < ntiles && !*abort_s; it++) {
        const int a = it & 1;
        if (!tc::mbar_wait(&acce[a], ((it >> 1) & 1) ^ 1, kWaitLimit)) {
          *abort_s = 1;
          atomicExch(p.err, 1);
          break;
        }
        const uint32_t d = tmem + (uint32_t)(a * W_N);
        for (int k = 0; k < steps; k++, step++) {
          const int s = (int)(step % W_STAGES);
          if (!tc::mbar_wait(&full[s], (uint32_t)((step / W_STAGES) & 1), kWaitLimit)) {
            *abort_s = 1;
            atomicExch(p.err, 1);
            break;
          }
          tc::tc_fence_after();
          const uint32_t a_base = tc::smem_u32(sm + s * W_STAGE);
          const uint32_t b_base = a_base + W_A;
          if (k < kchunks) {
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
        tc::mma_commit(&accf[a]);
      }
      if (*abort_s) {  // let every issued MMA finish before TMEM is freed
        tc::mma_commit(drained);
        tc::mbar_wait(drained, 0, kWaitLimit);
      }
    }
  } else if (lane == 0) {
    // ================= TMA producer =================
    int64_t step = 0;
    for (int it = 0; it < ntiles && !*abort_s; it++) {
      const int row = (int)((t_begin + it) * p.tile_stride * W_N);
      for (int k = 0; k < steps; k++, step++) {
        const int s = (int)(step % W_STAGES);
        if (*abort_s ||
            !tc::mbar_wait(&empty[s], (uint32_t)(((step / W_STAGES) & 1) ^ 1), kWaitLimit)) {
          *abort_s = 1;
          atomicExch(p.err, 1);
          break;
        }
        uint8_t *dst = sm + s * W_STAGE;
        if (k < kchunks) {
          tc::mbar_arrive_expect_tx(&full[s], (uint32_t)W_STAGE);
          tc::tma_load_2d(dst, &tmap_a, 64 * k, (int)q0, &full[s]);
          tc::tma_load_2d(dst + W_A, &tmap_b, 64 * k, row, &full[s]);
        } else {
          tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(W_AX + W_BX));
          tc::tma_load_2d(dst, &tmap_ax, 0, (int)q0, &full[s]);
          tc::tma_load_2d(dst + W_A, &tmap_bx, 0, row, &full[s]);
        }
      }
    }
    if (*abort_s) tc::drain_stages(full, W_STAGES, step, kWaitLimit);
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

// queries -> fp16 operand rows (zeros past dim, past nq and for degenerate
// queries) and the extra slices: -1 (pass 1) / +1 (pass 2) in element 0
__global__ void tc_prepare_queries_kernel(const float *q_r, int q_stride, const uint32_t *degen,
                                          int64_t nq, int64_t nq_pad, int dim, int kpad,
                                          uint16_t *a16, uint16_t *aext_lo, uint16_t *aext_hi) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one 8-element chunk
  const int cpr = kpad / 8;
  if (e >= nq_pad * cpr) return;
  const int64_t q = e / cpr;
  const int c = (int)(e - q * cpr);
  const bool ok = q < nq && !degen[q];
  uint32_t o[4] = {0, 0, 0, 0};
  if (ok && 8 * c < dim) {
    const float4 *src = (const float4 *)(q_r + q * (int64_t)q_stride + 8 * c);
    const float4 x0 = __ldg(src), x1 = __ldg(src + 1);
    const __half2 h0 = __floats2half2_rn(x0.x, x0.y), h1 = __floats2half2_rn(x0.z, x0.w);
    const __half2 h2 = __floats2half2_rn(x1.x, x1.y), h3 = __floats2half2_rn(x1.z, x1.w);
    o[0] = *(const uint32_t *)&h0;
    o[1] = *(const uint32_t *)&h1;
    o[2] = *(const uint32_t *)&h2;
    o[3] = *(const uint32_t *)&h3;
  }
  *(uint4 *)(a16 + q * (int64_t)kpad + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
  if (c < 2) {
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    if (c == 0 && ok) {
      lo.x = (uint32_t)__half_as_ushort(__float2half_rn(-1.0f));
      hi.x = (uint32_t)__half_as_ushort(__float2half_rn(1.0f));
    }
    *(uint4 *)(aext_lo + q * 16 + 8 * c) = lo;
    *(uint4 *)(aext_hi + q * 16 + 8 * c) = hi;
  }
}

const void *tc_wide_kernel_ptr(int mode) {
  if (mode == 3) return (const void *)tc_wide_kernel<3>;
  return mode == 1 ? (const void *)tc_wide_kernel<1> : (const void *)tc_wide_kernel<2>;
}

size_t tc_wide_smem_bytes() { return (size_t)W_TOTAL; }

int tc_wide_threads() { return W_THREADS; }

}  // namespace uvb
