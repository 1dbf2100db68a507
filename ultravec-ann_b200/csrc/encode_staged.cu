// encode_staged.cu -- the trellis encoder for every shape the resident
// encoders (encode.cu: one team per row; encode_cluster.cu: one thread-block
// cluster per row) do not hold: window widths mem + bits of 15 and more at 3
// or 4 bits, widths above 18, and the reference's general pass for mem <
// bits (src/trellis.rs:1348-1387).
//
// A batch of R rows advances through the trellis one step at a time: one
// launch per step updates every state of every row of the batch, with the
// path costs of all rows in global memory (ping-pong) and the back-pointers
// of every (row, step, state) kept there for the traceback.  A thread owns
// one next state and a few rows; its 2^bits windows' table values stay in
// registers across those rows.
//
//   staged_prep_kernel    one warp per row: unit row, centering, rotation,
//                         standardization (uv_encode_row.cuh)
//   staged_step_kernel    mem >= bits: the V=1 fast path's add-compare-select
//                         (src/trellis.rs:1688-1751) -- candidates k = 0..2^b-1
//                         of next state ns are the windows w = ns + k * 2^mem
//                         from predecessor w >> bits, the minimum of the
//                         separately rounded metric + cost, first k on ties
//   staged_general_kernel mem < bits: the scalar triple loop (src/trellis.rs:
//                         1349-1378) -- every (state s, emission e) in s-major
//                         order, window w = (s << bits) | e into next state
//                         w & (2^mem - 1), replaced only on a strictly smaller
//                         cost; the back-pointer is the window itself
//   staged_final_kernel   one warp per row: total_cmp argmin (first state on
//                         ties), traceback, rescale and packing
// The arithmetic is that of encode.cu, so records are bit-identical.
#include "uv_encode_row.cuh"
#include "uv_kernels.h"

namespace uvb {

namespace {

constexpr int kStagedRowsPerThread = 8;
constexpr int kStagedWarps = 4;  // rows per CTA of the prep and final kernels

}  // namespace

__global__ void __launch_bounds__(32 * kStagedWarps) staged_prep_kernel(const EncodeParams p,
                                                                        int64_t row0, int64_t R,
                                                                        float *u_rs, float *u_r,
                                                                        float *misc_out) {
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5;
  const int d = p.dim;
  float *xbuf = smem + (size_t)warp * (2 * p.dim_pad + 80);
  float *ubuf = xbuf + p.dim_pad;
  float *misc = ubuf + p.dim_pad;            // 16 words
  uint64_t *red = (uint64_t *)(misc + 16);   // 32 u64
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kStagedWarps + warp;
  if (r >= R) return;  // whole warps; the kernel has no block barrier
  encode_row_prep(p, row0 + r, xbuf, ubuf, misc, red, tm);
  tm.sync();
  for (int i = tm.t; i < d; i += 32) {
    u_rs[r * d + i] = ubuf[i];
    u_r[r * p.dim_pad + i] = xbuf[i];
  }
  if (tm.t < 8) misc_out[r * 8 + tm.t] = misc[tm.t];
}

__global__ void staged_init_kernel(float *cost, int64_t total, int n_states, uint32_t free_states) {
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x)
    cost[e] = (uint32_t)(e % n_states) < free_states ? 0.0f : INFINITY;
}

template <int B>
__global__ void __launch_bounds__(256) staged_step_kernel(const EncodeParams p, const float *u_rs,
                                                          int step, int64_t R, const float *cur,
                                                          float *nxt, uint8_t *back) {
  constexpr int NE = 1 << B;
  const int NS = p.n_states;
  const int ns = blockIdx.x * blockDim.x + threadIdx.x;
  if (ns >= NS) return;
  const int d = p.dim;
  const int GS = NS >> B;
  const int g = ns >> B;
  // negated table values of this state's windows: xi - c == xi + (-c)
  float ncode[NE];
#pragma unroll
  for (int k = 0; k < NE; k++) ncode[k] = -__ldg(p.code + ns + k * NS);
  const bool aniso = p.lambda != 0.0f;
  const int64_t r0 = (int64_t)blockIdx.y * kStagedRowsPerThread;
  for (int rr = 0; rr < kStagedRowsPerThread; rr++) {
    const int64_t r = r0 + rr;
    if (r >= R) break;
    const float xi = u_rs[r * d + step];
    const float wi = aniso ? fadd(1.0f, fmul(fmul(p.lambda, xi), xi)) : 1.0f;
    const float *cr = cur + r * NS;
    float cv[NE];
#pragma unroll
    for (int k = 0; k < NE; k++) {
      const float dd = fadd(xi, ncode[k]);
      const float m = aniso ? fmul(fmul(wi, dd), dd) : fmul(dd, dd);
      cv[k] = fadd(cr[g + k * GS], m);
    }
    // the minimum (NaN only when every candidate is NaN), then the first k
    // that does not exceed it: the reference's strict-< scan from k = 0
    float mn = cv[0];
#pragma unroll
    for (int k = 1; k < NE; k++) mn = fminf(mn, cv[k]);
    uint32_t bk = NE - 1;
#pragma unroll
    for (int k = NE - 2; k >= 0; k--) bk = (cv[k] > mn) ? bk : (uint32_t)k;
    nxt[r * NS + ns] = mn;
    back[(r * d + step) * (int64_t)NS + ns] = (uint8_t)bk;
  }
}

// mem < bits: next state ns is reached from every state s by the emissions
// e = ns + j * 2^mem (j < 2^(bits - mem)); the reference walks s, then e, in
// ascending order and keeps the first strictly smaller cost (an infinite
// predecessor never wins).  The stored back-pointer is the window
// (s << bits) | e (0 when no candidate is finite, as the reference's zeroed
// buffer).
__global__ void __launch_bounds__(256) staged_general_kernel(const EncodeParams p, int bits,
                                                             const float *u_rs, int step,
                                                             int64_t R, const float *cur,
                                                             float *nxt, uint32_t *back) {
  const int NS = p.n_states;
  const int64_t e_all = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e_all >= R * NS) return;
  const int64_t r = e_all / NS;
  const int ns = (int)(e_all - r * NS);
  const int d = p.dim;
  const int n_emit = 1 << bits;
  const float xi = u_rs[r * d + step];
  const float wi = fadd(1.0f, fmul(fmul(p.lambda, xi), xi));
  float best = INFINITY;
  uint32_t bw = 0;
  for (int s = 0; s < NS; s++) {
    const float cs = cur[r * NS + s];
    if (cs == INFINITY) continue;
    for (int e = ns; e < n_emit; e += NS) {
      const uint32_t w = ((uint32_t)s << bits) | (uint32_t)e;
      const float dd = fsub(xi, __ldg(p.code + w));
      const float d2 = fadd(0.0f, fmul(fmul(wi, dd), dd));
      const float c = fadd(cs, d2);
      if (c < best) {
        best = c;
        bw = w;
      }
    }
  }
  nxt[r * NS + ns] = best;
  back[(r * d + step) * (int64_t)NS + ns] = bw;
}

template <int B>
__global__ void __launch_bounds__(32 * kStagedWarps) staged_final_kernel(
    const EncodeParams p, int64_t row0, int64_t R, const float *u_r, const float *misc_in,
    const float *cost, const uint8_t *back8, const uint32_t *back32) {
  extern __shared__ __align__(16) float smem[];
  const int warp = threadIdx.x >> 5;
  const int d = p.dim;
  const int NS = p.n_states;
  float *xbuf = smem + (size_t)warp * (2 * p.dim_pad + 16);
  uint32_t *wv = (uint32_t *)(xbuf + p.dim_pad);
  float *misc = xbuf + 2 * p.dim_pad;  // 16 words
  uint32_t *misc_u = (uint32_t *)misc;
  Team tm;
  tm.T = 32;
  tm.cta = false;
  tm.t = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * kStagedWarps + warp;
  if (r >= R) return;  // whole warps; the kernel has no block barrier
  // argmin under total_cmp, first state on ties (src/trellis.rs:1783-1802)
  uint64_t bkey = 0;
  for (int s = tm.t; s < NS; s += 32) {
    const uint32_t k32 = (uint32_t)total_key(cost[r * NS + s]) ^ 0x80000000u;
    const uint64_t key = ((uint64_t)(~k32) << 32) | (uint32_t)(~(uint32_t)s);
    bkey = key > bkey ? key : bkey;
  }
  bkey = team_max_u64(bkey, tm, nullptr);
  for (int i = tm.t; i < d; i += 32) xbuf[i] = u_r[r * p.dim_pad + i];
  if (tm.t < 8) misc[tm.t] = misc_in[r * 8 + tm.t];
  if (tm.leader()) {
    uint32_t s = ~(uint32_t)(bkey & 0xffffffffu);
    for (int step = d - 1; step >= 0; step--) {
      const int64_t at = (r * d + step) * (int64_t)NS + s;
      const uint32_t w = back32 != nullptr ? __ldcg(back32 + at)
                                           : s + (uint32_t)__ldcg(back8 + at) * (uint32_t)NS;
      wv[step] = w;
      s = w >> B;
    }
    misc_u[5] = s;
  }
  tm.sync();
  encode_row_finalize<B>(p, row0 + r, true, wv, xbuf, misc, tm);
}

// ---------------------------------------------------------------------------
// Planning and launch.
// ---------------------------------------------------------------------------

int staged_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why) {
  if (bits < 1 || bits > 4) {
    *why = "bits must be 1..4";
    return 1;
  }
  plan->B = bits;
  plan->WPT = 1 << bits;
  plan->T = 32;
  plan->n_states = 1 << mem;
  plan->dim_pad = (dim + 3) & ~3;
  plan->teams_per_cta = 1;
  plan->threads = 256;
  plan->cluster = 0;
  plan->staged = mem < bits ? 2 : 1;
  plan->back_smem = false;
  plan->back_words_team = 0;
  plan->team_smem_words = 0;
  plan->smem_bytes = 0;
  plan->kernel = nullptr;
  const size_t prep_smem = (size_t)kStagedWarps * (2 * plan->dim_pad + 80) * 4;
  if (prep_smem > 227 * 1024) {
    *why = "staged encoder row buffers exceed shared memory";
    return 2;
  }
  return 0;
}

int64_t staged_rows_per_batch(const EncodePlan &plan, int dim, int64_t n) {
  // the back-pointers of a batch (one byte, or a 4-byte window for the
  // general pass, per row, step and state) within about 512 MiB
  const int64_t per_row =
      (int64_t)dim * plan.n_states * (plan.staged == 2 ? 4 : 1) + 2 * (int64_t)plan.n_states * 4;
  const int64_t r = std::max<int64_t>(1, ((int64_t)512 << 20) / std::max<int64_t>(per_row, 1));
  return std::min<int64_t>(std::min<int64_t>(r, n), 65535 * (int64_t)kStagedRowsPerThread);
}

size_t staged_scratch_bytes(const EncodePlan &plan, int dim, int64_t R, size_t *offs) {
  // u_rs, u_r, misc, cost0, cost1, back (256-byte aligned sections)
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t sizes[6] = {
      (size_t)R * dim * 4, (size_t)R * plan.dim_pad * 4, (size_t)R * 8 * 4,
      (size_t)R * plan.n_states * 4, (size_t)R * plan.n_states * 4,
      (size_t)R * dim * plan.n_states * (plan.staged == 2 ? 4 : 1)};
  size_t off = 0;
  for (int i = 0; i < 6; i++) {
    offs[i] = off;
    off += al(sizes[i]);
  }
  return off;
}

cudaError_t encode_staged_launch(const EncodePlan &plan, EncodeParams p, int64_t row0, int64_t R,
                                 uint8_t *scratch, const size_t *offs, cudaStream_t st) {
  p.n_states = plan.n_states;
  p.dim_pad = plan.dim_pad;
  const int d = p.dim;
  const int NS = plan.n_states;
  float *u_rs = (float *)(scratch + offs[0]);
  float *u_r = (float *)(scratch + offs[1]);
  float *misc = (float *)(scratch + offs[2]);
  float *cost0 = (float *)(scratch + offs[3]);
  float *cost1 = (float *)(scratch + offs[4]);
  uint8_t *back = scratch + offs[5];
  const unsigned row_ctas = (unsigned)((R + kStagedWarps - 1) / kStagedWarps);
  const size_t prep_smem = (size_t)kStagedWarps * (2 * plan.dim_pad + 80) * 4;
  cudaError_t e = cudaFuncSetAttribute(staged_prep_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)prep_smem);
  if (e != cudaSuccess) return e;
  staged_prep_kernel<<<row_ctas, 32 * kStagedWarps, prep_smem, st>>>(p, row0, R, u_rs, u_r, misc);
  const int64_t total = R * NS;
  staged_init_kernel<<<(unsigned)std::min<int64_t>((total + 255) / 256, 4096), 256, 0, st>>>(
      cost0, total, NS, (uint32_t)(p.start_bits >= 31 ? 0xffffffffu : (1u << p.start_bits)));
  float *cur = cost0, *nxt = cost1;
  for (int step = 0; step < d; step++) {
    if (plan.staged == 2) {
      staged_general_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
          p, plan.B, u_rs, step, R, cur, nxt, (uint32_t *)back);
    } else {
      const int threads = std::min(NS, 256);
      const dim3 grid((unsigned)((NS + threads - 1) / threads),
                      (unsigned)((R + kStagedRowsPerThread - 1) / kStagedRowsPerThread));
      switch (plan.B) {
        case 1: staged_step_kernel<1><<<grid, threads, 0, st>>>(p, u_rs, step, R, cur, nxt, back); break;
        case 2: staged_step_kernel<2><<<grid, threads, 0, st>>>(p, u_rs, step, R, cur, nxt, back); break;
        case 3: staged_step_kernel<3><<<grid, threads, 0, st>>>(p, u_rs, step, R, cur, nxt, back); break;
        default: staged_step_kernel<4><<<grid, threads, 0, st>>>(p, u_rs, step, R, cur, nxt, back); break;
      }
    }
    float *t = cur;
    cur = nxt;
    nxt = t;
  }
  const size_t fin_smem = (size_t)kStagedWarps * (2 * plan.dim_pad + 16) * 4;
  const void *fk = plan.B == 1 ? (const void *)staged_final_kernel<1>
                 : plan.B == 2 ? (const void *)staged_final_kernel<2>
                 : plan.B == 3 ? (const void *)staged_final_kernel<3>
                               : (const void *)staged_final_kernel<4>;
  e = cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fin_smem);
  if (e != cudaSuccess) return e;
  const uint8_t *b8 = plan.staged == 2 ? nullptr : back;
  const uint32_t *b32 = plan.staged == 2 ? (const uint32_t *)back : nullptr;
  void *args[] = {&p, &row0, &R, &u_r, &misc, &cur, &b8, &b32};
  e = cudaLaunchKernel(fk, dim3(row_ctas), dim3(32 * kStagedWarps), args, fin_smem, st);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace uvb
