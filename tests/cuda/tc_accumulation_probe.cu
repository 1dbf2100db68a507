// Accumulation error of the tensor cores, the one property of the hardware
// that the scan's prefilter bound assumes (an allowance of 2^-12 of
// sum |a_i b_i|).  One CTA computes D[128 x 256] = A[128 x 128] . B[256 x
// 128]^T with tcgen05 (fp16 operands, f32 accumulator); the host compares
// every D with the exact sum of the fp16 products (in double) and prints the
// largest error relative to sum |a_i b_i|, per scenario:
//   random      mixed magnitudes (1e-3, 1, 30)
//   dominant    one product of about 2^14 among 127 of about 2^-14
//   cancel      alternating signs of nearly equal products (sum near 0)
//   crossing    partial sums that change exponent between K slices of 16
//               (+2^10, then -2^10 + 1, then values of 2^-4)
//   subnormal   fp16 subnormal operands (2^-24 .. 2^-14): whole rows of them,
//               and rows mixed with normal ones
//   large       operands near the fp16 maximum mixed with tiny ones
//   slices      every K slice of 16 scaled by its own power of two in
//               [2^-12, 2^12]
// Uses the library's own tcgen05 wrappers (uv_tc.cuh).
#include <cstdio>
#include <cstdlib>
#include <cstdint>
#include <vector>
#include <cmath>
#include "uv_tc.cuh"
using namespace uvb::tc;

constexpr int M = 128, N = 256, K = 128;

__global__ void __launch_bounds__(128) probe(const __half *A, const __half *B, float *D, int *err) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint8_t *sa = sm;                      // 128 x 128 fp16 = 32 KB
  uint8_t *sb = sm + M * K * 2;          // 256 x 128 fp16 = 64 KB
  uint64_t *bar = (uint64_t *)(sm + (M + N) * K * 2);
  uint32_t *tbase = (uint32_t *)(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (warp == 0) tmem_alloc(tbase, 512);
  if (tid == 0) { mbar_init(bar, 1); mbar_fence_init(); }
  // fill A and B (16-byte chunks)
  for (int e = tid; e < M * (K / 8); e += 128) {
    int r = e / (K / 8), c = e % (K / 8);
    *(uint4 *)(sa + sw128_chunk_offset(r, c, M)) = *(const uint4 *)(A + r * K + c * 8);
  }
  for (int e = tid; e < N * (K / 8); e += 128) {
    int r = e / (K / 8), c = e % (K / 8);
    *(uint4 *)(sb + sw128_chunk_offset(r, c, N)) = *(const uint4 *)(B + r * K + c * 8);
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tbase;
  if (tid == 0) {
    const uint32_t idesc = idesc_f16_f32(M, N);
    for (int s = 0; s < K / 16; s++) {
      const int atom = s >> 2, within = (s & 3) * 32;
      uint64_t ad = sw128_desc(smem_u32(sa + atom * M * 128 + within));
      uint64_t bd = sw128_desc(smem_u32(sb + atom * N * 128 + within));
      mma_f16(tmem, ad, bd, idesc, s > 0 ? 1u : 0u);
    }
    mma_commit(bar);
  }
  __syncwarp();
  if (!mbar_wait(bar, 0, 1u << 20)) { if (lane == 0) atomicExch(err, 1); }
  tc_fence_after();
  for (int c0 = 0; c0 < N; c0 += 32) {
    uint32_t r[32];
    tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, r);
    tmem_ld_wait();
    for (int j = 0; j < 32; j++) D[(warp * 32 + lane) * N + c0 + j] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) { tmem_dealloc(tmem, 512); tmem_relinquish(); }
}

static double gauss() {
  double u = (rand() + 0.5) / (RAND_MAX + 1.0), v = (rand() + 0.5) / (RAND_MAX + 1.0);
  return sqrt(-2 * log(u)) * cos(6.283185307179586 * v);
}

// value k of row r of operand `which` (0: A, 1: B) in a scenario
static double scenario_value(int sc, int which, int r, int k) {
  const double g = gauss();
  switch (sc) {
    case 0: {
      const int i = r * K + k + which;
      return g * ((i % 5 == 0) ? 1e-3 : ((i % 7 == 0) ? 30.0 : 1.0));
    }
    case 1:  // the dominant product sits at k = r % K in A and every B row
      return (k == (which == 0 ? r % K : (r / 2) % K)) ? 128.0 * (1.0 + 0.1 * g)
                                                       : g * (1.0 / 128.0);
    case 2:  // a ~ 1, b ~ (-1)^k: products cancel pairwise
      return which == 0 ? 1.0 + 1e-3 * g : ((k & 1) ? -1.0 : 1.0) * (1.0 + 1e-3 * g);
    case 3: {  // slice sums +2^10, -2^10 + 1, then 2^-4 (b ~ 1)
      if (which == 1) return 1.0 + 1e-3 * g;
      if (k < 16) return 64.0 * (1.0 + 1e-2 * g);
      if (k < 32) return -64.0 * (1.0 + 1e-2 * g) + 1.0 / 16;
      return (1.0 / 16) * g;
    }
    case 4:  // fp16 subnormals: every a of even rows, and every other a of odd
             // rows, in [2^-24, 2^-14) with random sign; b normal
      if (which == 0 && (r % 2 == 0 || (k & 1)))
        return (g > 0 ? 1.0 : -1.0) * ldexp(1.0 + 0.5 * fabs(g) / 4.0, -24 + (rand() % 10));
      return g;
    case 5:  // near 65504 mixed with 2^-10
      return (k % 9 == 0) ? (g > 0 ? 1.0 : -1.0) * (60000.0 - 1000.0 * fabs(g)) / 64.0
                          : g / 1024.0;
    default: {  // every slice of 16 at its own power of two
      const int e = ((k / 16) * 7 + r * 3 + which * 5) % 25 - 12;
      return ldexp(g, e / 2);
    }
  }
}

int main() {
  const char *names[] = {"random", "dominant", "cancel", "crossing", "subnormal", "large",
                         "slices"};
  const int n_sc = 7;
  std::vector<__half> A(M * K), B(N * K);
  std::vector<float> Af(M * K), Bf(N * K);
  __half *dA, *dB; float *dD; int *derr;
  cudaMalloc(&dA, M * K * 2); cudaMalloc(&dB, N * K * 2); cudaMalloc(&dD, M * N * 4); cudaMalloc(&derr, 4);
  const int smem = (M + N) * K * 2 + 64;
  cudaFuncSetAttribute(probe, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  double worst_all = 0;
  long bad_all = 0, total = 0;
  int herr_all = 0;
  cudaError_t e_all = cudaSuccess;
  srand(3);
  for (int sc = 0; sc < n_sc; sc++) {
    for (int i = 0; i < M * K; i++) {
      A[i] = __float2half((float)scenario_value(sc, 0, i / K, i % K));
      Af[i] = __half2float(A[i]);
    }
    for (int i = 0; i < N * K; i++) {
      B[i] = __float2half((float)scenario_value(sc, 1, i / K, i % K));
      Bf[i] = __half2float(B[i]);
    }
    cudaMemcpy(dA, A.data(), M * K * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dB, B.data(), N * K * 2, cudaMemcpyHostToDevice);
    cudaMemset(dD, 0, M * N * 4); cudaMemset(derr, 0, 4);
    probe<<<1, 128, smem>>>(dA, dB, dD, derr);
    cudaError_t e = cudaDeviceSynchronize();
    std::vector<float> D(M * N); int herr = 0;
    cudaMemcpy(D.data(), dD, M * N * 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    double worst = 0, sum_rel = 0; long bad = 0;
    for (int i = 0; i < M; i++) for (int j = 0; j < N; j++) {
      double want = 0, l1 = 0;
      for (int k = 0; k < K; k++) { double t = (double)Af[i * K + k] * (double)Bf[j * K + k]; want += t; l1 += fabs(t); }
      double rel = fabs((double)D[i * N + j] - want) / (l1 > 0 ? l1 : 1);
      if (rel > worst) worst = rel;
      sum_rel += rel;
      if (rel > 1.0 / 4096) bad++;
    }
    printf("scenario %-9s max |tc-exact|/sum|ab| = %.3e (= 2^%.2f), mean %.3e, above 2^-12: %ld of %d\n",
           names[sc], worst, log2(worst > 0 ? worst : 1e-30), sum_rel / (M * N), bad, M * N);
    if (worst > worst_all) worst_all = worst;
    bad_all += bad;
    total += M * N;
    herr_all |= herr;
    if (e != cudaSuccess) e_all = e;
    if (e != cudaSuccess) break;
  }
  printf("status %s timeout %d  max |tc-exact|/sum|ab| = %.3e (= 2^%.2f), above 2^-12: %ld of %ld\n",
         cudaGetErrorString(e_all), herr_all, worst_all, log2(worst_all > 0 ? worst_all : 1e-30),
         bad_all, total);
  return e_all != cudaSuccess || herr_all;
}
