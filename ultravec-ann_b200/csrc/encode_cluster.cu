// encode_cluster.cu -- the trellis encoder for large state counts (sm_100a).
//
// At mem + bits >= 15 a row's trellis needs more than 512 threads (32
// windows per thread: 2^(mem+bits) / 32 threads), beyond one CTA of the
// single-CTA encoder (encode.cu).  Here one thread-block cluster of C CTAs
// of 512 threads encodes a row:
//
//   * CTA c owns the contiguous states [c*NS/C, (c+1)*NS/C) and their path
//     costs (ping-pong arrays in its shared memory); each thread owns whole
//     state groups (the 2^b states that share their 2^b predecessors), so
//     its next-cost stores stay local;
//   * the predecessors of group g are g + k*2^(mem-bits): read from the
//     owning CTA's shared memory through the cluster's distributed shared
//     memory (no other GPU's memory, no TMA);
//   * one cluster barrier per step (hardware barrier, every thread arrives);
//   * back-pointers go to a per-cluster global slot; CTA 0 takes the
//     total_cmp argmin over the cluster, walks the traceback and finalizes.
//
// The arithmetic and the tie rules are those of encode.cu (trellis.rs:
// 1246-1387, 1688-1802, 1878-2001): separately rounded metric, 3-input-min
// add-compare-select with the first-not-greater choice, total_cmp argmin.
#include <cooperative_groups.h>

#include "uv_encode_row.cuh"
#include "uv_kernels.h"

namespace cg = cooperative_groups;

namespace uvb {

namespace {

constexpr int CL_TB = 512;  // threads per CTA

__device__ __forceinline__ float cl_min3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace

template <int B>
__global__ void __launch_bounds__(CL_TB, 1) encode_cluster_kernel(const EncodeParams p) {
  constexpr int NE = 1 << B;
  constexpr int WPT = 32;
  constexpr int SPT = WPT / NE;   // states per thread
  constexpr int GPT = SPT / NE;   // whole groups per thread
  constexpr int BPS = SPT * B;    // back-pointer bits per thread per step
  constexpr int SPW = 32 / BPS;   // steps per word
  constexpr uint32_t EMASK = NE - 1;
  static_assert(GPT >= 1, "the cluster encoder needs whole groups per thread");

  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int c = (int)cluster.block_rank();
  const int tt = threadIdx.x;
  const int d = p.dim;
  const int NS = p.n_states;
  const int T = C * CL_TB;             // team size
  const int t = c * CL_TB + tt;         // rank in the team
  const int NSC = NS / C;               // states per CTA
  const int GC = NSC / NE;              // groups per CTA (= GPT * CL_TB)
  const int GS = NS >> B;               // group count = predecessor stride

  extern __shared__ __align__(16) float smem[];
  float *xbuf = smem;
  float *ubuf = xbuf + p.dim_pad;
  float *cost0 = ubuf + p.dim_pad;
  float *cost1 = cost0 + NSC;
  float *misc = cost1 + NSC;                   // 16 words
  uint64_t *red = (uint64_t *)(misc + 16);     // 32 u64
  uint64_t *ckeys = red + 32;                  // 16 u64: per-CTA argmin keys (on CTA 0)
  uint32_t *misc_u = (uint32_t *)misc;

  Team tm;
  tm.T = CL_TB;
  tm.cta = true;
  tm.t = tt;

  // owned groups (global indices) and their windows' negated table values
  int grp[GPT];
#pragma unroll
  for (int i = 0; i < GPT; i++) grp[i] = c * GC + tt + i * CL_TB;
  float2 ncode[SPT][NE / 2];
#pragma unroll
  for (int j = 0; j < SPT; j++) {
    const int ns = (grp[j / NE] << B) + (j % NE);
#pragma unroll
    for (int k = 0; k < NE; k += 2)
      ncode[j][k / 2] =
          make_float2(-__ldg(p.code + ns + k * NS), -__ldg(p.code + ns + (k + 1) * NS));
  }

  const int64_t cluster_id = blockIdx.x / C;
  const int64_t n_clusters = gridDim.x / C;
  uint32_t *backg = p.back_global + cluster_id * p.back_words_team;
  const int64_t iters = (p.n + n_clusters - 1) / n_clusters;
  const bool aniso = p.lambda != 0.0f;
  const uint32_t free_states = 1u << p.start_bits;

  for (int64_t it = 0; it < iters; it++) {
    const int64_t v = cluster_id + it * n_clusters;
    const bool valid = v < p.n;
    const int64_t vv = valid ? v : p.n - 1;

    // ---- prep (every CTA computes the same u_rs) ----
    encode_row_prep(p, vv, xbuf, ubuf, misc, red, tm);
    for (int i = tt; i < NSC; i += CL_TB)
      cost0[i] = ((uint32_t)(c * NSC + i) < free_states) ? 0.0f : INFINITY;
    cluster.sync();

    // ---- forward: one cluster barrier per step ----
    float *cur = cost0, *nxt = cost1;
    float last[SPT];
    for (int step0 = 0; step0 < d; step0 += SPW) {
      uint32_t word = 0;
#pragma unroll
      for (int sub = 0; sub < SPW; sub++) {
        const int step = step0 + sub;
        if (step >= d) break;
        const float xi = ubuf[step];
        const float2 xi2 = make_float2(xi, xi);
        const float wi = aniso ? fadd(1.0f, fmul(fmul(p.lambda, xi), xi)) : 1.0f;
        const float2 wi2 = make_float2(wi, wi);
        // predecessor costs of the owned groups, from their owning CTAs
        float2 cp[GPT][NE / 2];
#pragma unroll
        for (int i = 0; i < GPT; i++) {
          float pv[NE];
#pragma unroll
          for (int k = 0; k < NE; k++) {
            const int s = grp[i] + k * GS;
            const float *src = cluster.map_shared_rank(cur, s / NSC);
            pv[k] = src[s % NSC];
          }
#pragma unroll
          for (int k = 0; k < NE; k += 2) cp[i][k / 2] = make_float2(pv[k], pv[k + 1]);
        }
        float best[SPT];
#pragma unroll
        for (int j = 0; j < SPT; j++) {
          const int i = j / NE;
          float cv[NE];
#pragma unroll
          for (int k = 0; k < NE; k += 2) {
            const float2 dd = __fadd2_rn(xi2, ncode[j][k / 2]);
            const float2 m = aniso ? __fmul2_rn(__fmul2_rn(wi2, dd), dd) : __fmul2_rn(dd, dd);
            const float2 cc = __ffma2_rn(m, p.one2, cp[i][k / 2]);
            cv[k] = cc.x;
            cv[k + 1] = cc.y;
          }
          float mn;
          if (NE == 2) {
            mn = fminf(cv[0], cv[1]);
          } else {
            mn = cl_min3(cv[0], cv[1], cv[2]);
#pragma unroll
            for (int k = 3; k < NE; k += 2)
              mn = (k + 1 < NE) ? cl_min3(mn, cv[k], cv[k + 1]) : fminf(mn, cv[k]);
          }
          uint32_t bk = NE - 1;
#pragma unroll
          for (int k = NE - 2; k >= 0; k--) bk = (cv[k] > mn) ? bk : (uint32_t)k;
          best[j] = mn;
          last[j] = mn;
          word |= bk << (sub * BPS + j * B);
        }
#pragma unroll
        for (int i = 0; i < GPT; i++) {
          float *dst = nxt + ((grp[i] << B) - c * NSC);
          if (NE == 2) {
            *(float2 *)dst = make_float2(best[i * NE], best[i * NE + 1]);
          } else {
            *(float4 *)dst = make_float4(best[i * NE], best[i * NE + 1], best[i * NE + 2],
                                         best[i * NE + 3]);
          }
        }
        float *tmp = cur;
        cur = nxt;
        nxt = tmp;
        cluster.sync();
      }
      backg[(int64_t)(step0 / SPW) * T + t] = word;
    }

    // ---- argmin under total_cmp over the cluster, first index on ties ----
    uint64_t bkey = 0;
#pragma unroll
    for (int j = 0; j < SPT; j++) {
      const uint32_t k32 = (uint32_t)total_key(last[j]) ^ 0x80000000u;
      const uint32_t st = (uint32_t)((grp[j / NE] << B) + (j % NE));
      const uint64_t key = ((uint64_t)(~k32) << 32) | (uint32_t)(~st);
      bkey = key > bkey ? key : bkey;
    }
    bkey = team_max_u64(bkey, tm, red);
    if (tt == 0) {
      uint64_t *dst = cluster.map_shared_rank(ckeys, 0);
      dst[c] = bkey;
    }
    cluster.sync();

    // ---- traceback and finalize on CTA 0 ----
    if (c == 0) {
      uint32_t *wv = (uint32_t *)ubuf;
      if (tt == 0) {
        uint64_t best = 0;
        for (int r = 0; r < C; r++) best = ckeys[r] > best ? ckeys[r] : best;
        uint32_t s = ~(uint32_t)(best & 0xffffffffu);
        for (int step = d - 1; step >= 0; step--) {
          // owner of state s: CTA, thread and slot of the back-pointer
          const uint32_t g = s >> B;
          const uint32_t oc = g / (uint32_t)GC, lg = g % (uint32_t)GC;
          const uint32_t ot = oc * CL_TB + lg % CL_TB;
          const uint32_t slot = (lg / CL_TB) * NE + (s & EMASK);
          const uint32_t wd = __ldcg(backg + (int64_t)(step / SPW) * T + ot);
          const uint32_t k = (wd >> ((step % SPW) * BPS + slot * B)) & EMASK;
          const uint32_t w = s + k * (uint32_t)NS;
          wv[step] = w;
          s = w >> B;
        }
        misc_u[5] = s;
      }
      tm.sync();
      encode_row_finalize<B>(p, vv, valid, wv, xbuf, misc, tm);
    }
  }
  cluster.sync();  // no CTA leaves while a peer may still read its memory
}

// ---------------------------------------------------------------------------
// Planning and launch of the cluster encoder.
// ---------------------------------------------------------------------------
int encode_cluster_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why) {
  if (bits > 2) {
    *why = "2^(mem+bits) > 16384 windows with bits > 2 is not built";
    return 2;
  }
  const int64_t nw = (int64_t)1 << (mem + bits);
  const int64_t T = nw / 32;
  const int64_t C = T / CL_TB;
  if (C < 2 || C > 16) {
    *why = "mem + bits above 18 needs a cluster of more than 16 CTAs";
    return 2;
  }
  const int spt = 32 >> bits;
  const int spw = 32 / (spt * bits);
  plan->B = bits;
  plan->WPT = 32;
  plan->T = (int)T;
  plan->n_states = 1 << mem;
  plan->dim_pad = (dim + 3) & ~3;
  plan->teams_per_cta = 1;
  plan->threads = CL_TB;
  plan->cluster = (int)C;
  plan->back_smem = false;
  plan->back_words_team = (int64_t)((dim + spw - 1) / spw) * T;
  const int64_t words = 2 * (int64_t)plan->dim_pad + 2 * (plan->n_states / C) + 16 + 64 + 32;
  plan->team_smem_words = (int)words;
  plan->smem_bytes = (size_t)words * 4;
  if (plan->smem_bytes > 227 * 1024) {
    *why = "cluster encoder working set exceeds shared memory";
    return 2;
  }
  plan->kernel = bits == 1 ? (const void *)encode_cluster_kernel<1>
                           : (const void *)encode_cluster_kernel<2>;
  return 0;
}

cudaError_t encode_cluster_grid(const EncodePlan &plan, int64_t n, int *grid) {
  cudaError_t e = cudaFuncSetAttribute(plan.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)plan.smem_bytes);
  if (e != cudaSuccess) return e;
  if (plan.cluster > 8) {
    e = cudaFuncSetAttribute(plan.kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.cluster);
  cfg.blockDim = dim3(plan.threads);
  cfg.dynamicSmemBytes = plan.smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, plan.kernel, &cfg);
  if (e != cudaSuccess) return e;
  if (clusters < 1) return cudaErrorInvalidConfiguration;
  *grid = (int)(plan.cluster * std::max<int64_t>(1, std::min<int64_t>(n, clusters)));
  return cudaSuccess;
}

cudaError_t encode_cluster_launch(const EncodePlan &plan, EncodeParams p, int grid,
                                  cudaStream_t st) {
  p.T = plan.T;
  p.teams_per_cta = 1;
  p.team_smem_words = plan.team_smem_words;
  p.n_states = plan.n_states;
  p.dim_pad = plan.dim_pad;
  p.back_words_team = plan.back_words_team;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(plan.threads);
  cfg.dynamicSmemBytes = plan.smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = plan.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void *args[] = {&p};
  return cudaLaunchKernelExC(&cfg, plan.kernel, args);
}

}  // namespace uvb
