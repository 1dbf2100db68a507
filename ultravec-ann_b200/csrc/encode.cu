// encode.cu -- batched free-start Viterbi trellis encoder for sm_100a.
//
// One team of T threads encodes one row at a time (persistent grid, teams
// stride over rows).  Per row, fully on device:
//   prep        unit row (or unit residual to its centroid), src/trellis.rs:1144-1160
//   rotation    R x (sign flip, normalized FWHT), src/lib.rs:472-484
//   standardize u_rs = u_r / max(std(u_r), EPS), src/trellis.rs:1172-1176
//   forward     2^M-state add-compare-select over the dim steps,
//               src/trellis.rs:1296-1332, 1688-1751, 1878-2001
//   traceback   from the total_cmp argmin, src/trellis.rs:1783-1802
//   finalize    rescale = sum code[w_i] * u_r[i] and MSB-first packing,
//               src/trellis.rs:1009-1133, src/lib.rs:610-627
//
// Thread mapping of the trellis.  The window of state ns and candidate k is
// w = ns + k*2^M, whose predecessor is s = w >> B = (ns >> B) + k*2^(M-B): the
// 2^B states that share ns >> B (a "group") share their 2^B predecessors.  A
// thread owns SPT consecutive states, i.e. whole groups (or a slice of one
// group when 2^B > SPT), so every min over k is thread-local.  Its WPT =
// SPT*2^B windows are fixed for the whole encode, so their table values live
// in registers.  Path costs are exchanged through shared memory (ping-pong,
// one team barrier per step) and each thread packs its SPT back-pointer k's
// (B bits each) into 32-bit words: shared memory when the whole back-pointer
// array fits, otherwise a per-team global scratch slot that the traceback
// reads back in coalesced chunks.
//
// Tie rule (src/trellis.rs:1724-1750): the k = 0 candidate seeds the minimum,
// later k replace it only when strictly smaller, so the smallest k (smallest
// predecessor) wins an exact tie.  Every f32 op is a separately rounded
// intrinsic, matching the reference bit for bit.
#include "uv_kernels.h"
#include "uv_encode_row.cuh"

namespace uvb {

// 3-input minimum (NaN-ignoring like fminf; NaN only when all three are).
__device__ __forceinline__ float min3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int B, int WPT, bool BACK_SMEM>
__global__ void __launch_bounds__(512) encode_kernel(const EncodeParams p) {
  constexpr int NE = 1 << B;
  constexpr int SPT = WPT / NE;                 // states per thread
  constexpr int GPT = SPT >= NE ? SPT / NE : 1;  // groups per thread
  constexpr int BPS = SPT * B;                  // back-pointer bits per thread per step
  constexpr int SPW = 32 / BPS;                 // steps per 32-bit word
  constexpr uint32_t EMASK = NE - 1;
  static_assert(SPT >= 1 && BPS <= 32, "bad trellis tiling");

  extern __shared__ __align__(16) float smem[];
  const int T = p.T;
  Team tm;
  tm.T = T;
  tm.cta = T > 32;
  const int team = threadIdx.x / T;
  tm.t = threadIdx.x - team * T;

  float *ts = smem + (size_t)team * p.team_smem_words;
  const int d = p.dim;
  const int NS = p.n_states;
  const int GS = NS >> B;
  float *xbuf = ts;                                // row -> unit -> u_r
  float *ubuf = ts + p.dim_pad;                    // u_rs, then windows
  float *cost0 = ubuf + p.dim_pad;
  float *cost1 = cost0 + NS;
  float *misc = cost1 + NS;                        // 16 words
  uint64_t *red = (uint64_t *)(misc + 16);         // 32 u64
  uint32_t *backs = (uint32_t *)(misc + 80);       // back-pointers or a traceback chunk
  uint32_t *misc_u = (uint32_t *)misc;

  // State ownership.  Whole groups (SPT >= 2^B): thread t owns groups
  // t, t+T, t+2T, ... so that at every step the predecessor loads and the
  // next-cost stores of a warp touch consecutive words (no bank conflicts).
  // Partial groups (SPT < 2^B): thread t owns states t*SPT .. t*SPT+SPT-1.
  auto state_of = [&](int j) -> int {
    if (SPT >= NE) return ((tm.t + (j / NE) * T) << B) + (j % NE);
    return tm.t * SPT + j;
  };
  auto group_of = [&](int g) -> int {
    if (SPT >= NE) return tm.t + g * T;
    return (tm.t * SPT) >> B;
  };

  // negated table values of the owned windows: xi - c == xi + (-c) exactly
  float2 ncode[SPT][NE / 2];
#pragma unroll
  for (int j = 0; j < SPT; j++) {
    const int ns = state_of(j);
#pragma unroll
    for (int k = 0; k < NE; k += 2)
      ncode[j][k / 2] = make_float2(-__ldg(p.code + ns + k * NS), -__ldg(p.code + ns + (k + 1) * NS));
  }

  const int64_t slot = (int64_t)blockIdx.x * p.teams_per_cta + team;
  uint32_t *backg = BACK_SMEM ? nullptr : p.back_global + slot * p.back_words_team;
  const int64_t team_stride = (int64_t)gridDim.x * p.teams_per_cta;
  const int64_t iters = (p.n + team_stride - 1) / team_stride;
  const bool aniso = p.lambda != 0.0f;
  const uint32_t free_states = 1u << p.start_bits;

  for (int64_t it = 0; it < iters; it++) {
    const int64_t v = slot + it * team_stride;
    const bool valid = v < p.n;
    const int64_t vv = valid ? v : p.n - 1;

    // ---- prep: load, normalize, center, rotate, standardize ----
    encode_row_prep(p, vv, xbuf, ubuf, misc, red, tm);
    for (int s = tm.t; s < NS; s += T) cost0[s] = ((uint32_t)s < free_states) ? 0.0f : INFINITY;
    tm.sync();

    // ---- forward: add-compare-select over d steps ----
    // metric (xi - c)^2 as paired IEEE ops: (xi + (-c)) then d*d, then the
    // predecessor cost added -- three roundings per window, as the reference.
    // A paired multiply whose only use is a paired add is fused into one
    // paired FMA by the code generator even from the .rn forms (one rounding
    // instead of two, measured on sm_100a).  The add is therefore written as
    // fma(m, one, cost) with `one` a run-time 1.0f (a kernel parameter, read
    // as an operand from the constant bank): m * 1 is exact, so the result is
    // round(cost + m) and nothing is left to contract.
    float *cur = cost0, *nxt = cost1;
    float last[SPT];
    // Add-compare-select.  The reference keeps the first candidate and
    // replaces it only on a strictly smaller cost, i.e. it picks the first k
    // whose cost equals the minimum.  Here the minimum comes from 3-input
    // min instructions and the choice is the first k with !(c_k > min): the
    // same k and the same value (costs are never -0; within one step either
    // every candidate is NaN -- then min is NaN, no c_k > NaN holds and k = 0
    // as in the reference -- or none is).  The step loop is unrolled by the
    // steps per back-pointer word so that the word's shifts are constants.
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
        float2 cp[GPT][NE / 2];
#pragma unroll
        for (int g = 0; g < GPT; g++) {
          const int q = group_of(g);
#pragma unroll
          for (int k = 0; k < NE; k += 2)
            cp[g][k / 2] = make_float2(cur[q + k * GS], cur[q + (k + 1) * GS]);
        }
        float best[SPT];
#pragma unroll
        for (int j = 0; j < SPT; j++) {
          const int g = (SPT >= NE) ? j / NE : 0;
          float cv[NE];
#pragma unroll
          for (int k = 0; k < NE; k += 2) {
            const float2 dd = __fadd2_rn(xi2, ncode[j][k / 2]);
            const float2 m = aniso ? __fmul2_rn(__fmul2_rn(wi2, dd), dd) : __fmul2_rn(dd, dd);
            const float2 c = __ffma2_rn(m, p.one2, cp[g][k / 2]);
            cv[k] = c.x;
            cv[k + 1] = c.y;
          }
          float mn;
          if (NE == 2) {
            mn = fminf(cv[0], cv[1]);
          } else {
            mn = min3(cv[0], cv[1], cv[2]);
#pragma unroll
            for (int k = 3; k < NE; k += 2) mn = (k + 1 < NE) ? min3(mn, cv[k], cv[k + 1]) : fminf(mn, cv[k]);
          }
          uint32_t bk = NE - 1;
#pragma unroll
          for (int k = NE - 2; k >= 0; k--) bk = (cv[k] > mn) ? bk : (uint32_t)k;
          best[j] = mn;
          last[j] = mn;
          word |= bk << (sub * BPS + j * B);
        }
        // next-cost stores: one vector store per owned run of states
        if (SPT >= NE) {
#pragma unroll
          for (int g = 0; g < GPT; g++) {
            float *dst = nxt + (group_of(g) << B);
            if (NE == 2) {
              *(float2 *)dst = make_float2(best[g * NE], best[g * NE + 1]);
            } else {
#pragma unroll
              for (int e = 0; e < NE; e += 4)
                *(float4 *)(dst + e) = make_float4(best[g * NE + e], best[g * NE + e + 1],
                                                   best[g * NE + e + 2], best[g * NE + e + 3]);
            }
          }
        } else {
          float *dst = nxt + tm.t * SPT;
          if (SPT == 2) {
            *(float2 *)dst = make_float2(best[0], best[1]);
          } else {
#pragma unroll
            for (int e = 0; e < SPT; e += 4)
              *(float4 *)(dst + e) = make_float4(best[e], best[e + 1], best[e + 2], best[e + 3]);
          }
        }
        float *tmp = cur;
        cur = nxt;
        nxt = tmp;
        tm.sync();
      }
      const int widx = (step0 / SPW) * T + tm.t;
      if (BACK_SMEM)
        backs[widx] = word;
      else
        backg[widx] = word;
    }

    // ---- argmin under total_cmp, first index on ties ----
    uint64_t bkey = 0;
#pragma unroll
    for (int j = 0; j < SPT; j++) {
      uint32_t k32 = (uint32_t)total_key(last[j]) ^ 0x80000000u;
      uint64_t key = ((uint64_t)(~k32) << 32) | (uint32_t)(~(uint32_t)state_of(j));
      bkey = key > bkey ? key : bkey;
    }
    bkey = team_max_u64(bkey, tm, red);
    uint32_t s = ~(uint32_t)(bkey & 0xffffffffu);

    // ---- traceback: windows w_i into ubuf ----
    // owner of state s and its slot j in that thread's back-pointer field
    auto owner_thread = [&](uint32_t st) -> int {
      if (SPT >= NE) return (int)((st >> B) % (uint32_t)T);
      return (int)(st / SPT);
    };
    auto owner_slot = [&](uint32_t st) -> int {
      if (SPT >= NE) return (int)(((st >> B) / (uint32_t)T) * NE + (st & EMASK));
      return (int)(st % SPT);
    };
    uint32_t *wv = (uint32_t *)ubuf;
    if (BACK_SMEM) {
      if (tm.leader()) {
        for (int step = d - 1; step >= 0; step--) {
          const uint32_t wd = backs[(step / SPW) * T + owner_thread(s)];
          const uint32_t k = (wd >> ((step % SPW) * BPS + owner_slot(s) * B)) & EMASK;
          const uint32_t w = s + k * (uint32_t)NS;
          wv[step] = w;
          s = w >> B;
        }
        misc_u[5] = s;
      }
    } else {
      constexpr int CH = 64;  // steps per traceback chunk (a multiple of SPW)
      const int nch = (d + CH - 1) / CH;
      for (int c = nch - 1; c >= 0; c--) {
        const int lo = c * CH, hi = min(d, lo + CH);
        const int wlo = (lo / SPW) * T, whi = ((hi - 1) / SPW + 1) * T;
        for (int i = wlo + tm.t; i < whi; i += T) backs[i - wlo] = backg[i];
        tm.sync();
        if (tm.leader()) {
          for (int step = hi - 1; step >= lo; step--) {
            const uint32_t wd = backs[(step / SPW) * T - wlo + owner_thread(s)];
            const uint32_t k = (wd >> ((step % SPW) * BPS + owner_slot(s) * B)) & EMASK;
            const uint32_t w = s + k * (uint32_t)NS;
            wv[step] = w;
            s = w >> B;
          }
          misc_u[5] = s;
        }
        tm.sync();
      }
    }
    tm.sync();

    // ---- finalize: rescale (leader, sequential) and packing (team) ----
    encode_row_finalize<B>(p, vv, valid, wv, xbuf, misc, tm);
  }
}

// ---------------------------------------------------------------------------
// Host-side launch planning.
// ---------------------------------------------------------------------------
namespace {

template <int B, int WPT, bool SM>
const void *kernel_ptr() {
  return (const void *)encode_kernel<B, WPT, SM>;
}

const void *pick_kernel(int B, int WPT, bool smem_back) {
#define UV_CASE(b, w)                                                           \
  if (B == b && WPT == w) return smem_back ? kernel_ptr<b, w, true>() : kernel_ptr<b, w, false>();
  UV_CASE(1, 4)
  UV_CASE(1, 8)
  UV_CASE(1, 16)
  UV_CASE(1, 32)
  UV_CASE(2, 16)
  UV_CASE(2, 32)
  UV_CASE(3, 32)
  UV_CASE(4, 32)
#undef UV_CASE
  return nullptr;
}

}  // namespace

std::atomic<int> g_encode_staged{0};  // uv_set_tuning("encode_staged")
std::atomic<int> g_encode_back_mode{0};  // uv_set_tuning("encode_back"): 0 auto, 1 global, 2 shared

int encode_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why) {
  if (bits < 1 || bits > 4) {
    *why = "bits must be 1..4";
    return 1;
  }
  // mem < bits: the reference's general pass (encode_staged.cu)
  if (mem < bits) return staged_plan(dim, bits, mem, plan, why);
  const int64_t nw = (int64_t)1 << (mem + bits);
  const int wpt = nw >= 32 ? 32 : (int)nw;
  const int64_t T = nw / wpt;
  if (T > 512) {
    // one cluster per row where it is built, else batches of rows stepped
    // through the trellis (encode_staged.cu)
    if (g_encode_staged.load() == 1) return staged_plan(dim, bits, mem, plan, why);
    const int rc = encode_cluster_plan(dim, bits, mem, plan, why);
    if (rc != 2) return rc;
    return staged_plan(dim, bits, mem, plan, why);
  }
  const int spt = wpt >> bits;
  const int bps = spt * bits;
  const int spw = 32 / bps;
  plan->B = bits;
  plan->WPT = wpt;
  plan->T = (int)T;
  plan->n_states = 1 << mem;
  plan->dim_pad = (dim + 3) & ~3;
  const int64_t back_words = (int64_t)((dim + spw - 1) / spw) * T;
  const int64_t chunk_words = (int64_t)((64 + spw - 1) / spw + 1) * T;
  const int64_t base_words = 2 * (int64_t)plan->dim_pad + 2 * (int64_t)plan->n_states + 80;
  plan->back_words_team = back_words;
  // Shared-memory back-pointers when at least 8 warps per SM still fit.
  const int64_t budget = 200 * 1024;
  // a team larger than a warp is the whole CTA; smaller teams pack 256 threads
  int tpc_warp = T >= 32 ? 1 : (int)(32 / T);  // teams per warp
  int tpc = T > 32 ? 1 : (int)(256 / T);
  auto fits = [&](int64_t team_words, int teams) { return team_words * 4 * teams <= budget; };
  int64_t team_words_smem = (base_words + back_words + 3) & ~3LL;
  int64_t team_words_glob = (base_words + chunk_words + 3) & ~3LL;
  bool smem = false;
  int teams = tpc;
  // largest team count (whole warps) that fits
  const int back_mode = g_encode_back_mode.load();
  for (int tc = tpc; tc >= tpc_warp && tc >= 1 && back_mode != 1; tc -= tpc_warp) {
    if (fits(team_words_smem, tc)) {
      const int64_t cta_bytes = team_words_smem * 4 * tc;
      const int threads = (int)(tc * T);
      const int ctas = (int)std::min<int64_t>(228 * 1024 / std::max<int64_t>(cta_bytes, 1), 2048 / threads);
      if ((int64_t)ctas * threads >= 256 || back_mode == 2) {
        smem = true;
        teams = tc;
      }
      break;
    }
  }
  if (!smem) {
    teams = tpc;
    while (teams > tpc_warp && !fits(team_words_glob, teams)) teams -= tpc_warp;
    if (!fits(team_words_glob, teams)) {
      *why = "encode working set exceeds shared memory";
      return 2;
    }
  }
  plan->back_smem = smem;
  plan->teams_per_cta = teams;
  plan->threads = teams * (int)T;
  plan->team_smem_words = (int)(smem ? team_words_smem : team_words_glob);
  plan->smem_bytes = (size_t)plan->team_smem_words * 4 * teams;
  plan->kernel = pick_kernel(bits, wpt, smem);
  if (plan->kernel == nullptr) {
    *why = "no encoder instantiation for this (bits, window) shape";
    return 2;
  }
  return 0;
}

cudaError_t encode_launch(const EncodePlan &plan, EncodeParams p, int grid, cudaStream_t st) {
  if (plan.cluster > 0) return encode_cluster_launch(plan, p, grid, st);
  p.T = plan.T;
  p.teams_per_cta = plan.teams_per_cta;
  p.team_smem_words = plan.team_smem_words;
  p.n_states = plan.n_states;
  p.dim_pad = plan.dim_pad;
  p.back_words_team = plan.back_words_team;
  cudaError_t e = cudaFuncSetAttribute(plan.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)plan.smem_bytes);
  if (e != cudaSuccess) return e;
  void *args[] = {&p};
  return cudaLaunchKernel(plan.kernel, dim3(grid), dim3(plan.threads), args, plan.smem_bytes, st);
}

cudaError_t encode_grid(const EncodePlan &plan, int64_t n, int *grid) {
  if (plan.cluster > 0) return encode_cluster_grid(plan, n, grid);
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(plan.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)plan.smem_bytes);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan.kernel, plan.threads,
                                                    plan.smem_bytes);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  const int64_t need = (n + plan.teams_per_cta - 1) / plan.teams_per_cta;
  *grid = (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sms * per_sm));
  return cudaSuccess;
}

}  // namespace uvb
