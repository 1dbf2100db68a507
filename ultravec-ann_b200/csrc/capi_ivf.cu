// capi_ivf.cu -- the IVF index behind the C ABI (ivf.rs, bench.rs:298-349).
//
// Device layout: the posting lists are one list-major SoA (codes at the
// codec's padded stride, start, rescale, rnorm, ids) with list offsets, so a
// probed list is one contiguous record range for the scan kernel.  Build and
// search never leave the device except for the stable bucketing of rows by
// list (a counting sort of n u32 on the host, the reference's bucket loop).
#include <cmath>

#include "capi_internal.h"

using namespace uvcapi;

namespace {

unsigned blocks(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

int seqdot_launch(int mode, const float *A, int64_t nA, const float *B, int64_t nB, int dim,
                  uint64_t *out_key, float *out, const float *a_norm, const float *b_norm,
                  cudaStream_t st) {
  if (nA == 0 || nB == 0) return UV_OK;
  uvb::SeqDotParams p;
  std::memset(&p, 0, sizeof(p));
  p.dim = dim;
  p.lda = dim;
  p.ldb = dim;
  p.nA = nA;
  p.nB = nB;
  p.A = A;
  p.B = B;
  p.one2 = make_float2(1.0f, 1.0f);
  p.out_key = out_key;
  p.out = out;
  p.a_norm = a_norm;
  p.b_norm = b_norm;
  const int T = uvb::seqdot_tile();
  const dim3 grid(blocks(nB, T), (unsigned)std::min<int64_t>((nA + T - 1) / T, 65535));
  void *args[] = {&p};
  const void *fn = mode == 0 ? (const void *)uvb::seqdot_kernel<0> : (const void *)uvb::seqdot_kernel<1>;
  ProfScope ps(mode == 0 ? "ivf_argmax" : "ivf_cosine", st);
  UV_CK(cudaLaunchKernel(fn, grid, dim3(256), args, 0, st));
  return UV_OK;
}

// units = rows / max(|row|, EPS) (device)
int units_launch(const float *rows, int64_t n, int dim, float *norms, float *units,
                 cudaStream_t st) {
  if (n == 0) return UV_OK;
  uvb::row_norms_kernel<<<blocks(n, 128), 128, 0, st>>>(rows, n, dim, norms);
  UV_CK(cudaGetLastError());
  uvb::normalize_rows_kernel<<<blocks(n * dim, 256), 256, 0, st>>>(rows, norms, n, dim, units);
  UV_CK(cudaGetLastError());
  return UV_OK;
}

// the tensor-core paths (below): at least this many centroids
constexpr int kProbeMinLists = 256;
int tc_argmax(const float *units, int64_t n, int dim, const float *cent, int nlist,
              uint32_t *asg, cudaStream_t st, Scratch &sc, bool *used);

// asg[i] = first strict maximum of <units[i], c_j> (device in and out)
int argmax_launch(const float *units, int64_t n, int dim, const float *cent, int nlist,
                  uint64_t *keys, uint32_t *asg, cudaStream_t st) {
  if (n == 0) return UV_OK;
  {
    Scratch sc(st);
    bool used = false;
    UV_TRY(tc_argmax(units, n, dim, cent, nlist, asg, st, sc, &used));
    if (used) return UV_OK;
  }
  UV_CK(cudaMemsetAsync(keys, 0, sizeof(uint64_t) * n, st));
  UV_TRY(seqdot_launch(0, units, n, cent, nlist, dim, keys, nullptr, nullptr, nullptr, st));
  uvb::argmax_index_kernel<<<blocks(n, 256), 256, 0, st>>>(keys, n, asg);
  UV_CK(cudaGetLastError());
  return UV_OK;
}

// ivf.rs:405-421 over raw device rows, in row chunks that bound the scratch.
int assign_device(const float *rows, int64_t n, int dim, const float *cent, int nlist,
                  uint32_t *asg, cudaStream_t st, Scratch &sc) {
  const int64_t chunk = std::max<int64_t>(64, std::min<int64_t>(n, ((int64_t)256 << 20) / (4 * dim)));
  float *units = nullptr, *norms = nullptr;
  uint64_t *keys = nullptr;
  UV_TRY(sc.alloc(&units, (size_t)chunk * dim));
  UV_TRY(sc.alloc(&norms, (size_t)chunk));
  UV_TRY(sc.alloc(&keys, (size_t)chunk));
  for (int64_t r0 = 0; r0 < n; r0 += chunk) {
    const int64_t m = std::min(chunk, n - r0);
    UV_TRY(units_launch(rows + r0 * dim, m, dim, norms, units, st));
    UV_TRY(argmax_launch(units, m, dim, cent, nlist, keys, asg + r0, st));
  }
  return UV_OK;
}

// Stable bucketing of rows by list (ivf.rs:179-183): order = rows grouped by
// list, input order inside a list; off has nlist + 1 entries.
int bucket_host(const std::vector<uint32_t> &asg, int nlist, std::vector<int64_t> &order,
                std::vector<int64_t> &off) {
  off.assign((size_t)nlist + 1, 0);
  for (uint32_t a : asg) {
    if (a >= (uint32_t)nlist) return fail(UV_EINVAL, "assignment outside 0..nlist-1");
    off[a + 1]++;
  }
  for (int j = 0; j < nlist; j++) off[j + 1] += off[j];
  std::vector<int64_t> fill(off.begin(), off.end() - 1);
  order.resize(asg.size());
  for (size_t i = 0; i < asg.size(); i++) order[(size_t)fill[asg[i]]++] = (int64_t)i;
  return UV_OK;
}

int copy_to_host(void *dst, const void *src, size_t bytes, cudaStream_t st) {
  UV_CK(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, st));
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

template <class T>
int upload(const std::vector<T> &h, Scratch &sc, T **d, cudaStream_t st) {
  UV_TRY(sc.alloc(d, h.size()));
  if (!h.empty()) UV_CK(cudaMemcpyAsync(*d, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice, st));
  return UV_OK;
}

void free_lists(uv_ivf *ix) {
  cudaFree(ix->codes);
  cudaFree(ix->start);
  cudaFree(ix->rescale);
  cudaFree(ix->rnorm);
  cudaFree(ix->ids);
  cudaFree(ix->d_off);
  cudaFree(ix->signs);
  ix->signs = nullptr;
  ix->codes = nullptr;
  ix->start = nullptr;
  ix->rescale = ix->rnorm = nullptr;
  ix->ids = nullptr;
  ix->d_off = nullptr;
  ix->n = 0;
  // the tensor-core list scan's rows were made from these lists
  cudaFree(ix->list_rows.x16);
  cudaFree(ix->list_rows.xext);
  cudaFree(ix->list_scale);
  if (ix->list_rows.ready != nullptr) cudaEventDestroy(ix->list_rows.ready);
  ix->list_rows = TcRows();
  ix->list_scale = nullptr;
}

// Per row of a (m x d): the np best of nlist centroids by exact score, via
// the fp16 dots of tcwide.cu (mode 3; B = c16 / cext, ldc rows, kpad wide)
// and probe_refine_kernel.  With a_norm the rows are raw and the score is the
// cosine (the fp16 side uses a / |a|); without it the rows are used as they
// are and the score is the plain dot.  bound: |fp16 dot - exact score|.
int tc_rank_rows(const float *a, const float *a_norm, int64_t m_total, int d, const uint16_t *c16,
                 const uint16_t *cext, int64_t ldc, const float *cent, const float *cnorm,
                 int nlist, int np, float bound, int32_t *out, int ld_out, int dev,
                 cudaStream_t st, Scratch &sc, int *err_defer = nullptr) {
  const int kpad = (d + 63) / 64 * 64;
  const int TN = 192, TM = 128;
  const int64_t n_tiles = ldc / TN;
  const int64_t chunk = std::max<int64_t>(
      TM,
      std::min<int64_t>((m_total + TM - 1) / TM * TM, ((int64_t)256 << 20) / (4 * ldc) / TM * TM));
  float *approx = nullptr, *u = nullptr;
  uint32_t *aflag = nullptr;
  uint16_t *a16 = nullptr, *ax = nullptr;
  int *err = nullptr;
  UV_TRY(sc.alloc(&approx, (size_t)chunk * ldc));
  if (a_norm != nullptr) UV_TRY(sc.alloc(&u, (size_t)chunk * d));
  UV_TRY(sc.alloc(&aflag, (size_t)chunk));
  UV_TRY(sc.alloc(&a16, (size_t)chunk * kpad));
  UV_TRY(sc.alloc(&ax, (size_t)chunk * 16 * 2));
  if (err_defer != nullptr) {
    err = err_defer;  // the caller zeroed it and reads it later
  } else {
    UV_TRY(sc.alloc(&err, 1));
    UV_CK(cudaMemsetAsync(err, 0, sizeof(int), st));
  }
  if (a_norm == nullptr) UV_CK(cudaMemsetAsync(aflag, 0, sizeof(uint32_t) * chunk, st));
  CUtensorMap tmap_b, tmap_bx;
  UV_TRY(fp16_tensor_map(&tmap_b, c16, ldc, kpad, 64, TN, true));
  UV_TRY(fp16_tensor_map(&tmap_bx, cext, ldc, 16, 16, TN, false));
  const size_t wsmem = uvb::tc_wide_smem_bytes();
  const void *wk = uvb::tc_wide_kernel_ptr(3);
  UV_CK(cudaFuncSetAttribute(wk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem));
  int pow2 = 32;
  while (pow2 < nlist) pow2 <<= 1;
  const size_t rsmem = (size_t)pow2 * 8 + (size_t)((nlist + 3) & ~3) * 4 + (size_t)d * 4;
  UV_CK(cudaFuncSetAttribute(uvb::probe_refine_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem));
  const int64_t slots = sm_count(dev);
  for (int64_t q0 = 0; q0 < m_total; q0 += chunk) {
    const int64_t m = std::min(chunk, m_total - q0);
    const int64_t m_pad = (m + TM - 1) / TM * TM;
    {
      ProfScope ps("ivf_cosine", st);
      const float *rows16 = a + q0 * d;
      if (a_norm != nullptr) {
        uvb::normalize_rows_kernel<<<blocks(m * d, 256), 256, 0, st>>>(a + q0 * d, a_norm + q0, m,
                                                                        d, u);
        uvb::unit_flags_kernel<<<blocks(m, 256), 256, 0, st>>>(a_norm + q0, m, aflag);
        rows16 = u;
      }
      const int64_t chunks = m_pad * (kpad / 8);
      uvb::tc_prepare_queries_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
          rows16, d, aflag, m, m_pad, d, kpad, a16, ax, ax + m_pad * 16);
      UV_CK(cudaGetLastError());
      CUtensorMap tmap_a, tmap_ax;
      UV_TRY(fp16_tensor_map(&tmap_a, a16, m_pad, kpad, 64, TM, true));
      UV_TRY(fp16_tensor_map(&tmap_ax, ax, m_pad, 16, 16, TM, false));
      uvb::TcScanParams tp;
      std::memset(&tp, 0, sizeof(tp));
      tp.nq = m;
      tp.n = nlist;
      tp.n_tiles = n_tiles;
      tp.n_groups = ldc;  // leading dimension of approx
      tp.tile_stride = 1;
      tp.degenerate = aflag;
      tp.tmax = approx;
      tp.err = err;
      // record splits filling whole waves of one CTA per SM
      const int64_t qtiles = m_pad / TM;
      int64_t splits = 1;
      double best_eff = 0.0;
      for (int64_t s2 = 1; s2 <= std::min<int64_t>(n_tiles, 64); s2++) {
        const int64_t ctas = qtiles * s2;
        const int64_t waves = (ctas + slots - 1) / slots;
        const double eff = (double)ctas / (double)(waves * slots) - 0.002 * (double)waves;
        if (eff > best_eff + 1e-9) {
          best_eff = eff;
          splits = s2;
        }
      }
      int kchunks = kpad / 64;
      void *wargs[] = {&tp, &kchunks, &tmap_a, &tmap_ax, &tmap_b, &tmap_bx};
      UV_CK(cudaLaunchKernel(wk, dim3((unsigned)qtiles, (unsigned)splits),
                             dim3(uvb::tc_wide_threads()), wargs, wsmem, st));
    }
    {
      ProfScope ps("ivf_select", st);
      uvb::ProbeRefineParams rp;
      std::memset(&rp, 0, sizeof(rp));
      rp.m = m;
      rp.nlist = nlist;
      rp.np = np;
      rp.dim = d;
      rp.pow2 = pow2;
      rp.ld_out = ld_out;
      rp.cosine = a_norm != nullptr ? 1 : 0;
      rp.ld = ldc;
      rp.bound = bound;
      rp.approx = approx;
      rp.queries = a + q0 * d;
      rp.qnorm = a_norm != nullptr ? a_norm + q0 : nullptr;
      rp.cent = cent;
      rp.cnorm = cnorm;
      rp.out = out + q0 * ld_out;
      void *rargs[] = {&rp};
      UV_CK(cudaLaunchKernel((const void *)uvb::probe_refine_kernel,
                             dim3((unsigned)std::min<int64_t>(m, 65535)), dim3(256), rargs, rsmem,
                             st));
    }
  }
  if (err_defer != nullptr) return UV_OK;
  int h_err = 0;
  UV_CK(cudaMemcpyAsync(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  if (h_err) return fail(UV_ETIMEDOUT, "a tensor-core probe wait timed out");
  return UV_OK;
}

// The k-means / build assignment on the tensor cores: the first strict
// maximum of <unit row, c_j> (as seqdot_kernel<0>) through tc_rank_rows with
// the raw centroids as fp16 rows and np = 1.  Same shape limits as the probe;
// also off when a centroid norm is not finite or above 1e4 (fp16 range).
// Bound: as the probe's, times the largest centroid norm (rows are units).
int tc_argmax(const float *units, int64_t n, int dim, const float *cent, int nlist,
              uint32_t *asg, cudaStream_t st, Scratch &sc, bool *used) {
  *used = false;
  if (g_ivf_tc_probe == 1 || dim % 32 != 0 || dim > 4096 || nlist < kProbeMinLists ||
      nlist > 8192 || n < 1024)
    return UV_OK;
  // both sides are read 16 bytes at a time: a caller's unaligned buffer
  // takes the CUDA-core path
  if (((uintptr_t)cent & 15) != 0 || ((uintptr_t)units & 15) != 0) return UV_OK;
  int dev = 0;
  UV_CK(cudaGetDevice(&dev));
  float *cn = nullptr;
  UV_TRY(sc.alloc(&cn, (size_t)nlist));
  uvb::row_norms_kernel<<<blocks(nlist, 128), 128, 0, st>>>(cent, nlist, dim, cn);
  UV_CK(cudaGetLastError());
  std::vector<float> hn(nlist);
  UV_CK(cudaMemcpyAsync(hn.data(), cn, sizeof(float) * nlist, cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  double maxc = 0.0;
  for (float v : hn) {
    if (!std::isfinite(v)) return UV_OK;
    maxc = std::max(maxc, (double)v);
  }
  if (maxc > 1e4) return UV_OK;
  *used = true;
  const int TN = 192;
  const int kpad = (dim + 63) / 64 * 64;
  const int64_t c_pad = (nlist + TN - 1) / TN * TN;
  uint16_t *c16 = nullptr, *cext = nullptr;
  uint32_t *zf = nullptr;
  UV_TRY(sc.alloc(&c16, (size_t)c_pad * kpad));
  UV_TRY(sc.alloc(&cext, (size_t)c_pad * 16));
  UV_TRY(sc.alloc(&zf, (size_t)nlist));
  UV_CK(cudaMemsetAsync(zf, 0, sizeof(uint32_t) * nlist, st));
  const int64_t chunks = c_pad * (kpad / 8);
  uvb::tc_prepare_queries_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
      cent, dim, zf, nlist, c_pad, dim, kpad, c16, cext, cext);
  UV_CK(cudaGetLastError());
  UV_CK(cudaMemsetAsync(cext, 0, sizeof(uint16_t) * (size_t)c_pad * 16, st));
  const float bound = (float)(1.25 * (std::ldexp(1.0, -10) + std::ldexp(1.0, -12) +
                                      4.0 * dim * std::ldexp(1.0, -24)) *
                              std::max(1.0, maxc));
  return tc_rank_rows(units, nullptr, n, dim, c16, cext, c_pad, cent, nullptr, nlist, 1, bound,
                      (int32_t *)asg, 1, dev, st, sc);
}

// The probe on the tensor cores: every (query, centroid) dot of the unit
// rows in fp16 (tcwide.cu, mode 3), then per query the exact cosines of the
// centroids that can still reach the np-th best (probe_refine_kernel) --
// the same lists as the exact path below.  Sets *used = false outside the
// shapes it is built for (rows a multiple of 32 up to 4096 wide, 256 to
// 8192 centroids) and when a centroid norm is not finite.
//
// Bound: with u = 2^-24 and unit rows, the fp16 dot differs from the exact
// cosine by at most 2^-10 (two fp16 roundings) + 2^-12 (tensor-core
// accumulation, as the flat prefilter's bound) + 4 d u (the f32 norms and
// divisions of both sides, fp16 subnormals, and the reference's sequential
// f32 dot); the kernel uses 1.25 times that.
int tc_probe(const uv_ivf *ix, const float *d_q, const float *qn, int64_t nq, int np, int ld,
             int32_t *lists, cudaStream_t st, Scratch &sc, bool *used, int *err_defer = nullptr) {
  *used = false;
  const int d = ix->codec->cfg.dim;
  const int nlist = ix->nlist;
  if (g_ivf_tc_probe == 1 || d % 32 != 0 || d > 4096 || nlist < kProbeMinLists || np > nlist ||
      nlist > 8192)
    return UV_OK;
  const int kpad = (d + 63) / 64 * 64;
  const int TN = 192, TM = 128;
  {
    std::lock_guard<std::mutex> lk(ix->tc_mu);
    if (ix->tc_state == 0) {
      std::vector<float> hn(nlist);
      UV_CK(cudaMemcpyAsync(hn.data(), ix->cnorm, sizeof(float) * nlist, cudaMemcpyDeviceToHost,
                            st));
      UV_CK(cudaStreamSynchronize(st));
      bool finite = true;
      for (float v : hn) finite &= std::isfinite(v);
      if (!finite) {
        ix->tc_state = -1;
      } else {
        const int64_t c_pad = (nlist + TN - 1) / TN * TN;
        UV_CK(cudaMalloc((void **)&ix->c16, sizeof(uint16_t) * (size_t)c_pad * kpad));
        UV_CK(cudaMalloc((void **)&ix->cext, sizeof(uint16_t) * (size_t)c_pad * 16));
        float *units = nullptr;
        uint32_t *flags = nullptr;
        UV_TRY(sc.alloc(&units, (size_t)nlist * d));
        UV_TRY(sc.alloc(&flags, (size_t)nlist));
        uvb::normalize_rows_kernel<<<blocks((int64_t)nlist * d, 256), 256, 0, st>>>(
            ix->centroids, ix->cnorm, nlist, d, units);
        uvb::unit_flags_kernel<<<blocks(nlist, 256), 256, 0, st>>>(ix->cnorm, nlist, flags);
        const int64_t chunks = c_pad * (kpad / 8);
        uvb::tc_prepare_queries_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
            units, d, flags, nlist, c_pad, d, kpad, ix->c16, ix->cext, ix->cext);
        UV_CK(cudaGetLastError());
        UV_CK(cudaMemsetAsync(ix->cext, 0, sizeof(uint16_t) * (size_t)c_pad * 16, st));
        UV_CK(cudaStreamSynchronize(st));
        ix->c_pad = c_pad;
        ix->tc_state = 1;
      }
    }
    if (ix->tc_state < 0) return UV_OK;
  }
  *used = true;
  const float bound = (float)(1.25 * (std::ldexp(1.0, -10) + std::ldexp(1.0, -12) +
                                      4.0 * d * std::ldexp(1.0, -24)));
  return tc_rank_rows(d_q, qn, nq, d, ix->c16, ix->cext, ix->c_pad, ix->centroids, ix->cnorm,
                      nlist, np, bound, lists, ld, ix->device, st, sc, err_defer);
}

// Probe on device: lists (nq x ld, first np columns) of the best np lists by
// exact cosine of the raw queries.
// err_defer (device, zeroed): the tensor-core probe's timeout flag is left
// there for the caller to read with its next host read, instead of a wait.
int probe_device(const uv_ivf *ix, const float *d_q, int64_t nq, int np, int ld, int32_t *lists,
                 cudaStream_t st, Scratch &sc, int *err_defer = nullptr) {
  const int d = ix->codec->cfg.dim;
  if (np == 0 || nq == 0) return UV_OK;
  int pow2 = 32;
  while (pow2 < ix->nlist) pow2 <<= 1;
  if (pow2 > 16384) return fail(UV_EUNSUPPORTED, "probe supports nlist <= 16384");
  float *qn = nullptr, *cos = nullptr;
  UV_TRY(sc.alloc(&qn, (size_t)nq));
  uvb::row_norms_kernel<<<blocks(nq, 128), 128, 0, st>>>(d_q, nq, d, qn);
  UV_CK(cudaGetLastError());
  bool used = false;
  UV_TRY(tc_probe(ix, d_q, qn, nq, np, ld, lists, st, sc, &used, err_defer));
  if (used) return UV_OK;
  const int64_t chunk =
      std::max<int64_t>(1, std::min<int64_t>(nq, ((int64_t)256 << 20) / (4 * (int64_t)ix->nlist)));
  UV_TRY(sc.alloc(&cos, (size_t)chunk * ix->nlist));
  const size_t smem = (size_t)pow2 * 8;
  UV_CK(cudaFuncSetAttribute(uvb::select_top_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem));
  for (int64_t q0 = 0; q0 < nq; q0 += chunk) {
    const int64_t m = std::min(chunk, nq - q0);
    UV_TRY(seqdot_launch(1, d_q + q0 * d, m, ix->centroids, ix->nlist, d, nullptr, cos, qn + q0,
                         ix->cnorm, st));
    ProfScope ps("ivf_select", st);
    uvb::select_top_kernel<<<(unsigned)std::min<int64_t>(m, 65535), 256, smem, st>>>(
        cos, m, ix->nlist, pow2, np, ld, lists + q0 * ld);
    UV_CK(cudaGetLastError());
  }
  return UV_OK;
}

// The records' fp16 operand rows and bound constants for the tensor-core
// list scan (tc_prepare_records*_kernel with g = rnorm / rescale, or 1 /
// rescale for uncentered lists, as the list scan scores them) and their
// power-of-two scale s; made on the first search that uses them, kept until
// the lists change (free_lists).  Later searches on other streams wait for
// the event recorded after they were made.
int list_rows(const uv_ivf *ix, cudaStream_t st, Scratch &sc, const TcRows **out,
              const float **scale) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int kpad = (d + 63) / 64 * 64;
  const int64_t n = ix->n;
  const int64_t n_pad = (n + 255) / 256 * 256;
  std::lock_guard<std::mutex> lk(ix->tc_mu);
  TcRows &r = ix->list_rows;
  if (r.x16 == nullptr) {
    UV_CK(cudaMalloc((void **)&r.x16, sizeof(uint16_t) * (size_t)n_pad * kpad));
    UV_CK(cudaMalloc((void **)&r.xext, sizeof(uint16_t) * (size_t)n_pad * 16));
    UV_CK(cudaMalloc((void **)&ix->list_scale, sizeof(float)));
    uint32_t *gmax = nullptr;
    UV_TRY(sc.alloc(&gmax, 1));
    UV_CK(cudaMemsetAsync(gmax, 0, sizeof(uint32_t), st));
    uvb::TcPrepareParams pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.mem = c->cfg.mem;
    pp.bits = c->cfg.bits;
    pp.code_stride = c->code_stride;
    pp.mips = 0;
    pp.dim = d;
    pp.kpad = kpad;
    pp.n = n;
    pp.n_pad = n_pad;
    pp.eps = 1.5e-3;
    pp.code_absmax = c->code_absmax;
    pp.codes = ix->codes;
    pp.start = ix->start;
    pp.code = c->d_table;
    pp.rescale = ix->rescale;
    pp.rnorm = ix->centered ? ix->rnorm : nullptr;
    pp.gmax_bits = gmax;
    pp.x16 = r.x16;
    pp.xext = r.xext;
    void *args[] = {&pp};
    ProfScope ps("ivf_tc_prepare", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::tc_gmax_kernel, dim3((unsigned)((n + 255) / 256)),
                           dim3(256), args, 0, st));
    uvb::tc_scale_kernel<<<1, 32, 0, st>>>(gmax, c->code_absmax, ix->list_scale);
    const void *fk = uvb::tc_prepare_records_fast_ptr(c->cfg.bits, g_tc_prepare.load() != 2);
    const size_t tsm = (size_t)4 << (c->cfg.mem + c->cfg.bits);
    if (fk != nullptr && tsm <= 64 * 1024 && g_tc_prepare != 1) {
      UV_CK(cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm));
      UV_CK(cudaLaunchKernel(fk, dim3((unsigned)((n_pad + 255) / 256)), dim3(256), args, tsm, st));
    } else {
      UV_CK(cudaLaunchKernel((const void *)uvb::tc_prepare_records_kernel,
                             dim3((unsigned)((n_pad + 127) / 128)), dim3(128), args, 0, st));
    }
    UV_CK(cudaGetLastError());
    if (r.ready == nullptr) UV_CK(cudaEventCreateWithFlags(&r.ready, cudaEventDisableTiming));
    UV_CK(cudaEventRecord(r.ready, st));
    r.cap = r.n_pad = n_pad;
    r.kpad = kpad;
  } else {
    UV_CK(cudaStreamWaitEvent(st, r.ready, 0));
  }
  *out = &r;
  *scale = ix->list_scale;
  return UV_OK;
}

// The bucketed pairs of one search, as search_device makes them.
struct PairBuckets {
  int64_t npairs = 0;   // bucketed pairs (probes of lists with records here)
  int64_t nprobes = 0;  // nq x nprobe
  int64_t n_items = 0, n_rslots = 0, range_size = 0;
  const int32_t *pair_query = nullptr, *pair_slot = nullptr, *pair_off = nullptr;
  const int64_t *list_rbase = nullptr, *row_off = nullptr;
  const float *pair_qm = nullptr;
  const int32_t *item_list = nullptr, *item_pair = nullptr, *item_npairs = nullptr,
                *item_range = nullptr, *n_items_dev = nullptr;
};

// Whether the tensor-core list scan takes a search (tuning key ivf_tc: 0
// automatic -- rows of at least 256 coordinates --, 1 never, 2 whenever it
// can): k <= 32, width a multiple of 16 (the exact rescoring runs 16 FMA
// chains without a scalar tail), and the rescoring's shared memory.
bool use_tc_scan(const uv_ivf *ix, int k) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int mode = g_ivf_tc.load();
  if (mode == 1 || k > 32 || d % 16 != 0 || ix->n > INT32_MAX - 1024) return false;
  if (uvb::ivf_select_smem_bytes(c->table_len, c->code_stride) > 200 * 1024) return false;
  return mode == 2 || d >= 256;
}

// The tensor-core list scan (ivftc.cu) over the bucketed pairs: per-slot
// thresholds and kept records (tc_ivf_kernel), then per query the shared
// threshold, the exact scores and the top k (ivf_select_kernel), written to
// d_ids / d_scores.  *fallback is set when a store overflowed; the caller
// then runs the CUDA-core scan, whose results replace everything written.
int tc_list_scan(const uv_ivf *ix, int64_t nq, int k, int np, const float *q_r, int q_stride,
                 const uint32_t *degen, const PairBuckets &b, int64_t *d_ids, float *d_scores,
                 cudaStream_t st, Scratch &sc, bool *fallback) {
  *fallback = false;
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const TcRows *rows = nullptr;
  const float *scale = nullptr;
  UV_TRY(list_rows(ix, st, sc, &rows, &scale));
  const int kpad = rows->kpad;
  // the pairs' fp16 query rows (bucketed order; at least one box of rows)
  const int64_t rows_a = std::max<int64_t>(b.npairs, uvb::kIvfTcRows);
  uint16_t *pa16 = nullptr, *ax = nullptr;
  int32_t *pair_of = nullptr;
  UV_TRY(sc.alloc(&pa16, (size_t)rows_a * kpad));
  UV_TRY(sc.alloc(&ax, (size_t)uvb::kIvfTcRows * 16));
  UV_TRY(sc.alloc(&pair_of, (size_t)b.nprobes));
  UV_CK(cudaMemsetAsync(pair_of, 0xff, sizeof(int32_t) * (size_t)b.nprobes, st));  // -1: no pair
  // the queries' fp16 rows (zero past d and for degenerate queries), once
  uint16_t *a16 = nullptr, *axq = nullptr;
  UV_TRY(sc.alloc(&a16, (size_t)nq * kpad));
  UV_TRY(sc.alloc(&axq, (size_t)nq * 32));
  {
    ProfScope ps("ivf_tc_pairs", st);
    const int64_t qchunks = nq * (kpad / 8);
    uvb::tc_prepare_queries_kernel<<<(unsigned)((qchunks + 255) / 256), 256, 0, st>>>(
        q_r, q_stride, degen, nq, nq, d, kpad, a16, axq, axq + nq * 16);
    const int64_t chunks = b.npairs * (kpad / 8);
    uvb::ivf_pair_rows16_kernel<<<(unsigned)std::max<int64_t>(
                                      1, std::min<int64_t>((chunks + 255) / 256, 148 * 32)),
                                  256, 0, st>>>(a16, b.pair_query, b.npairs, kpad, pa16);
    uvb::ivf_neg_slice_kernel<<<(uvb::kIvfTcRows * 16 + 255) / 256, 256, 0, st>>>(ax);
    if (b.npairs > 0)
      uvb::ivf_pair_of_kernel<<<blocks(b.npairs, 256), 256, 0, st>>>(b.pair_slot, b.npairs,
                                                                      pair_of);
    UV_CK(cudaGetLastError());
  }
  alignas(64) CUtensorMap tmap_a, tmap_ax, tmap_b, tmap_bx;
  UV_TRY(fp16_tensor_map(&tmap_a, pa16, rows_a, kpad, 64, 32, true));
  UV_TRY(fp16_tensor_map(&tmap_ax, ax, uvb::kIvfTcRows, 16, 16, uvb::kIvfTcRows, false));
  UV_TRY(fp16_tensor_map(&tmap_b, rows->x16, rows->n_pad, kpad, 64, 32, true));
  UV_TRY(fp16_tensor_map(&tmap_bx, rows->xext, rows->n_pad, 16, 16, 32, false));
  // per-slot thresholds and the store of kept records
  const int64_t nslots = std::max<int64_t>(b.n_rslots, 1);
  const int64_t cand_cap = b.n_rslots * (int64_t)(k + 16) + 65536;
  float *cand_lb = nullptr, *cand_ub = nullptr;
  uint32_t *q_theta0 = nullptr;
  int32_t *slot_cnt = nullptr;
  int64_t *slot_base = nullptr;
  uint32_t *cand_rec = nullptr;
  // kept-record count, scored count, err | queries over the candidate store
  unsigned long long *flags = nullptr;
  UV_TRY(sc.alloc(&q_theta0, (size_t)nq));
  UV_CK(cudaMemsetAsync(q_theta0, 0, sizeof(uint32_t) * (size_t)nq, st));
  UV_TRY(sc.alloc(&slot_cnt, (size_t)nslots));
  UV_TRY(sc.alloc(&slot_base, (size_t)nslots));
  UV_TRY(sc.alloc(&cand_rec, (size_t)cand_cap));
  UV_TRY(sc.alloc(&cand_lb, (size_t)cand_cap));
  UV_TRY(sc.alloc(&cand_ub, (size_t)cand_cap));
  UV_TRY(sc.alloc(&flags, 4));
  UV_CK(cudaMemsetAsync(flags, 0, sizeof(unsigned long long) * 4, st));
  int *err = (int *)(flags + 2), *n_over = err + 1;
  if (b.n_items > 0) {
    uvb::TcIvfParams tp;
    std::memset(&tp, 0, sizeof(tp));
    tp.k = k;
    tp.kchunks = kpad / 64;
    tp.range_size = b.range_size;
    tp.n_items = b.n_items_dev;
    tp.item_list = b.item_list;
    tp.item_pair = b.item_pair;
    tp.item_npairs = b.item_npairs;
    tp.item_range = b.item_range;
    tp.list_off = ix->d_off;
    tp.list_pair_off = b.pair_off;
    tp.list_rbase = b.list_rbase;
    tp.pair_query = b.pair_query;
    tp.pair_qm = b.pair_qm;
    tp.degenerate = degen;
    tp.scale = scale;
    tp.xext = rows->xext;
    tp.q_theta0 = q_theta0;
    tp.slot_cnt = slot_cnt;
    tp.slot_base = slot_base;
    tp.cand_rec = cand_rec;
    tp.cand_lb = cand_lb;
    tp.cand_ub = cand_ub;
    tp.cand_used = flags;
    tp.cand_cap = cand_cap;
    tp.err = err;
    const void *kfn = uvb::tc_ivf_kernel_ptr(k);
    if (kfn == nullptr) return fail(UV_EUNSUPPORTED, "no tensor-core list scan for this k");
    const size_t smem = uvb::tc_ivf_smem_bytes();
    UV_CK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    void *args[] = {&tp, &tmap_a, &tmap_ax, &tmap_b, &tmap_bx};
    ProfScope ps("ivf_tc_scan", st);
    UV_CK(cudaLaunchKernel(kfn, dim3((unsigned)b.n_items), dim3(uvb::tc_ivf_threads()), args, smem,
                           st));
  }
  {
    uvb::IvfSelectParams sp;
    std::memset(&sp, 0, sizeof(sp));
    sp.dim = d;
    sp.mem = c->cfg.mem;
    sp.bits = c->cfg.bits;
    sp.code_stride = c->code_stride;
    sp.q_stride = q_stride;
    sp.k = k;
    sp.np = np;
    sp.table_len = c->table_len;
    sp.nq = nq;
    sp.q_r = q_r;
    sp.degenerate = degen;
    sp.pair_of = pair_of;
    sp.row_off = b.row_off;
    sp.pair_qm = b.pair_qm;
    sp.q_theta0 = q_theta0;
    sp.slot_cnt = slot_cnt;
    sp.slot_base = slot_base;
    sp.cand_rec = cand_rec;
    sp.cand_lb = cand_lb;
    sp.cand_ub = cand_ub;
    sp.codes = ix->codes;
    sp.start = ix->start;
    sp.code = c->d_table;
    sp.rescale = ix->rescale;
    sp.rnorm = ix->centered ? ix->rnorm : nullptr;
    sp.ids = ix->ids;
    sp.out_id = d_ids;
    sp.out_score = d_scores;
    sp.n_over = n_over;
    sp.n_cand = flags + 1;
    const void *kfn = uvb::ivf_select_kernel_ptr(c->cfg.bits);
    if (kfn == nullptr) return fail(UV_EUNSUPPORTED, "no rescoring kernel for these bits");
    const size_t smem = uvb::ivf_select_smem_bytes(c->table_len, c->code_stride);
    UV_CK(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    void *args[] = {&sp};
    ProfScope ps("ivf_tc_select", st);
    UV_CK(cudaLaunchKernel(kfn, dim3((unsigned)((nq + uvb::kIvfSelWarps - 1) / uvb::kIvfSelWarps)),
                           dim3(32 * uvb::kIvfSelWarps), args, smem, st));
  }
  unsigned long long h[4] = {0, 0, 0, 0};
  UV_CK(cudaMemcpyAsync(h, flags, sizeof(h), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  // err (1: a wait timed out, 2: the kept-record store was full) | queries
  // with more candidates than the per-query store holds
  const int h_err = (int)(h[2] & 0xffffffffull), h_cand = (int)(h[2] >> 32);
  g_tc_last_candidates = (int64_t)h[1];
  g_ivf_tc_overflow = ((int64_t)((h_err & 2) ? 1 : 0) << 32) | (int64_t)h_cand;
  *fallback = h_err != 0 || h_cand != 0;
  return UV_OK;
}

// ivf.rs:229-239 on device: per-list top-k of every probed (query, list)
// pair, merged per query.  Device inputs and outputs.
// given_lists (device, nq x np, -1 = no list) replaces the probe: lists
// chosen elsewhere, e.g. by another rank with the same centroids.
int search_device(const uv_ivf *ix, const float *d_q, int64_t nq, int k, int np, int64_t *d_ids,
                  float *d_scores, cudaStream_t st, Scratch &sc, bool allow_tc = true,
                  const int32_t *given_lists = nullptr) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  if (np == 0 || ix->n == 0) {
    // no list probed, or no records: every slot empty
    uvb::fill_empty_kernel<<<blocks(nq * k, 256), 256, 0, st>>>(d_ids, d_scores, nq * k);
    UV_CK(cudaGetLastError());
    return UV_OK;
  }
  const int dim_pad = (d + 3) & ~3;
  float *q_r = nullptr, *qc = nullptr, *u = nullptr;
  uint32_t *degen = nullptr;
  UV_TRY(sc.alloc(&q_r, (size_t)nq * dim_pad));
  UV_TRY(sc.alloc(&qc, 1));
  UV_TRY(sc.alloc(&degen, (size_t)nq));
  if (ix->centered) UV_TRY(sc.alloc(&u, (size_t)nq * dim_pad));
  UV_TRY(prep_launch(c, d_q, nq, nullptr, 0, q_r, qc, degen, u, st));
  // probe
  const int64_t npairs = nq * np;
  if (npairs > INT32_MAX) return fail(UV_EINVAL, "nq * nprobe exceeds 2^31 - 1");
  int32_t *lists = nullptr;
  UV_TRY(sc.alloc(&lists, (size_t)npairs));
  // [0] a list id outside 0..nlist-1, [1] the tensor-core probe timed out:
  // read with the bucket totals below
  int *bad = nullptr;
  UV_TRY(sc.alloc(&bad, 2));
  UV_CK(cudaMemsetAsync(bad, 0, sizeof(int) * 2, st));
  if (given_lists != nullptr) {
    UV_CK(cudaMemcpyAsync(lists, given_lists, sizeof(int32_t) * (size_t)npairs,
                          cudaMemcpyDeviceToDevice, st));
  } else {
    // the shortlist path below reads no totals: its probe waits for its own flag
    UV_TRY(probe_device(ix, d_q, nq, np, np, lists, st, sc, ix->sl_c > 0 ? nullptr : bad + 1));
  }
  // bucket the (query, list) pairs by list; a scan item is one record range
  // (at most range_size records: long lists are split for load balance) of
  // one list for up to 32 of its pairs
  const int nlist = ix->nlist;
  int64_t max_list = 0;
  for (int l = 0; l < nlist; l++) max_list = std::max(max_list, ix->off[l + 1] - ix->off[l]);
  if (ix->sl_c > 0) {
    // IvfCodec::TrellisShortlist (src/ivf.rs:52-60): every probed list runs
    // search_shortlist(query, k, c) (src/trellis.rs:854-948), then the
    // per-list results merge per query (src/ivf.rs:229-239)
    int64_t *pid = nullptr;
    float *psc = nullptr;
    UV_TRY(sc.alloc(&pid, (size_t)npairs * k));
    UV_TRY(sc.alloc(&psc, (size_t)npairs * k));
    UV_TRY(shortlist_launch(c, ix->sl_c, ix->sl_asym, ix->sl_weight && ix->centered, k, npairs,
                            np, lists, ix->d_off, max_list, 0, q_r, ix->centered ? u : nullptr,
                            ix->centroids, nullptr, 0, degen, ix->codes, ix->signs, ix->start,
                            nullptr, ix->rescale, ix->centered ? ix->rnorm : nullptr, ix->ids,
                            pid, psc, st));
    return merge_launch(nq, np, k, k, nullptr, psc, pid, d_ids, d_scores, st);
  }
  // probes of lists without records here (a list owned by another shard,
  // or empty) make no pair
  uvb::drop_empty_lists_kernel<<<blocks(npairs, 256), 256, 0, st>>>(lists, npairs, ix->d_off,
                                                                    nlist, bad);
  UV_CK(cudaGetLastError());
  // the tensor-core list scan: items of up to kIvfTcRows pairs and ranges
  // of kIvfTcRange records; the CUDA-core scan: items of kScanTQ pairs, and
  // ranges such that a pair's ranges merge in one pass of about 1024 entries
  const bool tc = allow_tc && use_tc_scan(ix, k);
  const int per_item = tc ? uvb::kIvfTcRows : uvb::kScanTQ;
  const int64_t range_size =
      tc ? (int64_t)uvb::kIvfTcRange : std::max<int64_t>(1024, (max_list * k + 1023) / 1024);
  int32_t *cnt = nullptr, *fill = nullptr, *pair_off = nullptr, *item_off = nullptr,
          *pair_query = nullptr, *pair_slot = nullptr, *pair_list = nullptr;
  int64_t *list_rbase = nullptr, *totals = nullptr;
  UV_TRY(sc.alloc(&cnt, (size_t)nlist * 2));
  fill = cnt + nlist;
  UV_TRY(sc.alloc(&pair_off, (size_t)nlist));
  UV_TRY(sc.alloc(&item_off, (size_t)nlist));
  UV_TRY(sc.alloc(&list_rbase, (size_t)nlist));
  UV_TRY(sc.alloc(&totals, 3));
  UV_TRY(sc.alloc(&pair_query, (size_t)npairs));
  UV_TRY(sc.alloc(&pair_slot, (size_t)npairs));
  UV_TRY(sc.alloc(&pair_list, (size_t)npairs));
  UV_CK(cudaMemsetAsync(cnt, 0, sizeof(int32_t) * nlist * 2, st));
  {
    ProfScope ps("ivf_bucket", st);
    uvb::pair_count_kernel<<<blocks(npairs, 256), 256, 0, st>>>(lists, npairs, cnt);
    uvb::pair_scan_kernel<<<1, 1024, 0, st>>>(cnt, ix->d_off, nlist, range_size, per_item,
                                                pair_off, item_off, list_rbase, totals);
    uvb::pair_scatter_kernel<<<blocks(npairs, 256), 256, 0, st>>>(lists, nq, np, pair_off, fill,
                                                                  pair_query, pair_slot, pair_list);
    UV_CK(cudaGetLastError());
  }
  int64_t h_tot[3] = {0, 0, 0};
  int h_bad[2] = {0, 0};
  UV_CK(cudaMemcpyAsync(h_tot, totals, sizeof(h_tot), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaMemcpyAsync(h_bad, bad, sizeof(h_bad), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  const int64_t n_items = h_tot[0], n_rslots = h_tot[1];
  if (h_bad[1]) return fail(UV_ETIMEDOUT, "a tensor-core probe wait timed out");
  if (h_bad[0]) return fail(UV_EINVAL, "a probe list id is outside 0..nlist-1");
  // the bucketed pairs: probes of lists with records here
  const int64_t npv = h_tot[2];
  if (n_items > INT32_MAX) return fail(UV_EINVAL, "too many scan items");
  int32_t *item_list = nullptr, *item_pair = nullptr, *item_npairs = nullptr,
          *item_range = nullptr, *d_n_items = nullptr;
  int64_t *row_off = nullptr;
  UV_TRY(sc.alloc(&item_list, (size_t)n_items));
  UV_TRY(sc.alloc(&item_pair, (size_t)n_items));
  UV_TRY(sc.alloc(&item_npairs, (size_t)n_items));
  UV_TRY(sc.alloc(&item_range, (size_t)n_items));
  UV_TRY(sc.alloc(&d_n_items, 1));
  UV_TRY(sc.alloc(&row_off, (size_t)npairs + 1));
  {
    // the item count as the kernels read it: the low half of the device
    // total (n_items < 2^31, little-endian), no host copy to wait for
    UV_CK(cudaMemcpyAsync(d_n_items, totals, sizeof(int32_t), cudaMemcpyDeviceToDevice, st));
    ProfScope ps("ivf_bucket", st);
    uvb::item_fill_kernel<<<blocks(nlist, 256), 256, 0, st>>>(
        cnt, pair_off, item_off, ix->d_off, nlist, range_size, per_item, item_list, item_pair,
        item_npairs, item_range);
    uvb::pair_rows_kernel<<<blocks(npv + 1, 256), 256, 0, st>>>(
        pair_list, pair_off, list_rbase, ix->d_off, range_size, (int)npv, row_off);
    UV_CK(cudaGetLastError());
  }
  float *pair_qm = nullptr;
  if (ix->centered) {
    UV_TRY(sc.alloc(&pair_qm, (size_t)std::max<int64_t>(npv, 1)));
    ProfScope ps("ivf_pair_qm", st);
    if (npv > 0)
      uvb::pair_qm_kernel<<<(unsigned)((npv + 32 * uvb::kPairQmWarps - 1) /
                                       (32 * uvb::kPairQmWarps)),
                            32 * uvb::kPairQmWarps, 0, st>>>(u, dim_pad, ix->centroids, d,
                                                             pair_query, pair_list, (int)npv,
                                                             pair_qm);
    UV_CK(cudaGetLastError());
  }
  if (tc) {
    PairBuckets b;
    b.npairs = npv;
    b.nprobes = npairs;
    b.n_items = n_items;
    b.n_rslots = n_rslots;
    b.range_size = range_size;
    b.pair_query = pair_query;
    b.pair_slot = pair_slot;
    b.pair_off = pair_off;
    b.list_rbase = list_rbase;
    b.row_off = row_off;
    b.pair_qm = pair_qm;
    b.item_list = item_list;
    b.item_pair = item_pair;
    b.item_npairs = item_npairs;
    b.item_range = item_range;
    b.n_items_dev = d_n_items;
    bool fallback = false;
    UV_TRY(tc_list_scan(ix, nq, k, np, q_r, dim_pad, degen, b, d_ids, d_scores, st, sc,
                        &fallback));
    if (!fallback) return UV_OK;
    // a store overflowed: the CUDA-core scan, from the probe on
    return search_device(ix, d_q, nq, k, np, d_ids, d_scores, st, sc, false, given_lists);
  }
  // scan every item: one top-k per (pair, range) slot
  uint32_t *part_key = nullptr;
  int64_t *part_id = nullptr;
  UV_TRY(sc.alloc(&part_key, (size_t)std::max<int64_t>(n_rslots, 1) * k));
  UV_TRY(sc.alloc(&part_id, (size_t)std::max<int64_t>(n_rslots, 1) * k));
  const bool table_smem = (size_t)c->table_len * 4 <= 16 * 1024;
  const bool small_k = k <= 32;
  const size_t smem = uvb::chunked_scan_smem_bytes(c->table_len, table_smem, small_k);
  const void *scan_k = uvb::chunked_scan_kernel_ptr(c->cfg.bits, table_smem, small_k);
  if (scan_k == nullptr) return fail(UV_EUNSUPPORTED, "no scan kernel for these bits");
  UV_CK(cudaFuncSetAttribute(scan_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int rw = c->code_stride / 4;
  int img_words = 4 + rw + 3;
  if ((img_words & 1) == 0) img_words++;
  uvb::ScanParams sp;
  std::memset(&sp, 0, sizeof(sp));
  // rows of any width: the decode-GEMM over width d rounded up to 16, then
  // the reference's scalar tail over the last d % 8 coordinates
  sp.dim = (d + 15) & ~15;
  sp.dim_data = sp.dim != d ? d : 0;
  sp.mem = c->cfg.mem;
  sp.bits = c->cfg.bits;
  sp.nq = nq;
  sp.n = ix->n;
  sp.q_r = q_r;
  sp.q_stride = dim_pad;
  sp.qc = qc;
  sp.n_centroids = 0;
  sp.degenerate = degen;
  sp.codes = ix->codes;
  sp.code_stride = c->code_stride;
  sp.start = ix->start;
  sp.rescale = ix->rescale;
  sp.rnorm = ix->centered ? ix->rnorm : nullptr;
  sp.norms = nullptr;
  sp.cidx = nullptr;
  sp.code = c->d_table;
  sp.table_len = c->table_len;
  sp.table_in_smem = table_smem ? 1 : 0;
  sp.img_words = img_words;
  sp.mips = 0;
  sp.k = k;
  sp.ids = ix->ids;
  sp.id_base = 0;
  sp.part_key = part_key;
  sp.part_id = part_id;
  uvb::ScanWork work;
  std::memset(&work, 0, sizeof(work));
  work.ivf = 1;
  work.item_list = item_list;
  work.item_pair = item_pair;
  work.item_npairs = item_npairs;
  work.item_range = item_range;
  work.list_off = ix->d_off;
  work.list_pair_off = pair_off;
  work.list_rbase = list_rbase;
  work.range_size = range_size;
  work.pair_query = pair_query;
  work.pair_qm = pair_qm;
  work.n_items = d_n_items;
  if (n_items > 0) {
    void *args[] = {&sp, &work};
    ProfScope ps("ivf_scan", st);
    UV_CK(cudaLaunchKernel(scan_k, dim3((unsigned)n_items), dim3(256), args, smem, st));
  }
  // each pair's ranges -> its (query, probe) slot; then the probes per query
  const int max_ranges = (int)((max_list + range_size - 1) / range_size) + 1;
  uint32_t *pk = nullptr;
  int64_t *pid = nullptr;
  float *psc = nullptr;
  UV_TRY(sc.alloc(&pid, (size_t)npairs * k));
  UV_TRY(sc.alloc(&psc, (size_t)npairs * k));
  (void)pk;
  if (npv < npairs) {  // probes without a pair: empty lists for the per-query merge
    uvb::fill_empty_kernel<<<blocks(npairs * k, 256), 256, 0, st>>>(pid, psc, npairs * k);
    UV_CK(cudaGetLastError());
  }
  if (npv > 0)
    UV_TRY(merge_launch(npv, max_ranges, k, k, part_key, nullptr, part_id, pid, psc, st, row_off,
                        pair_slot));
  return merge_launch(nq, np, k, k, nullptr, psc, pid, d_ids, d_scores, st);
}

}  // namespace

extern "C" {

int uv_kmeans(int32_t device, const float *rows, int64_t n, int32_t dim, int32_t nlist,
              uint64_t seed, int32_t iters, float *centroids_out, void *stream) {
  if (rows == nullptr || centroids_out == nullptr) return fail(UV_EINVAL, "null argument");
  if (n < 1 || dim < 1 || nlist < 1 || iters < 0) return fail(UV_EINVAL, "bad size");
  DeviceGuard g(device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_rows = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * dim, device, sc, &d_rows));
  float *cent = nullptr, *units = nullptr, *norms = nullptr;
  UV_TRY(outs.stage(centroids_out, (size_t)nlist * dim, device, sc, &cent));
  UV_TRY(sc.alloc(&units, (size_t)n * dim));
  UV_TRY(sc.alloc(&norms, (size_t)n));
  UV_TRY(units_launch(d_rows, n, dim, norms, units, st));
  // seeded init: units[splitmix64 % n], with replacement (bench.rs:307-310)
  std::vector<int64_t> pick((size_t)nlist);
  uint64_t state = seed;
  for (int j = 0; j < nlist; j++) pick[j] = (int64_t)(uvb::splitmix64(&state) % (uint64_t)n);
  int64_t *d_pick = nullptr;
  UV_TRY(upload(pick, sc, &d_pick, st));
  uvb::gather_rows_kernel<<<blocks((int64_t)nlist * dim, 256), 256, 0, st>>>(units, d_pick, nlist,
                                                                           dim, cent);
  UV_CK(cudaGetLastError());
  uint64_t *keys = nullptr;
  uint32_t *asg = nullptr;
  int64_t *d_order = nullptr, *d_off = nullptr;
  UV_TRY(sc.alloc(&keys, (size_t)n));
  UV_TRY(sc.alloc(&asg, (size_t)n));
  UV_TRY(sc.alloc(&d_order, (size_t)n));
  UV_TRY(sc.alloc(&d_off, (size_t)nlist + 1));
  std::vector<uint32_t> h_asg((size_t)n);
  std::vector<int64_t> order, off;
  for (int it = 0; it < iters; it++) {
    UV_TRY(argmax_launch(units, n, dim, cent, nlist, keys, asg, st));
    UV_TRY(copy_to_host(h_asg.data(), asg, sizeof(uint32_t) * n, st));
    UV_TRY(bucket_host(h_asg, nlist, order, off));
    UV_CK(cudaMemcpyAsync(d_order, order.data(), sizeof(int64_t) * n, cudaMemcpyHostToDevice, st));
    UV_CK(cudaMemcpyAsync(d_off, off.data(), sizeof(int64_t) * (nlist + 1), cudaMemcpyHostToDevice,
                          st));
    ProfScope ps("ivf_means", st);
    uvb::list_means_kernel<<<blocks((int64_t)nlist * dim, 256), 256, 0, st>>>(units, d_order, d_off,
                                                                            nlist, dim, cent);
    UV_CK(cudaGetLastError());
    UV_CK(cudaStreamSynchronize(st));  // host order/off are reused next round
  }
  return outs.finish(st);
}

int uv_ivf_assign(int32_t device, const float *rows, int64_t n, int32_t dim,
                  const float *centroids, int32_t nlist, uint32_t *assign_out, void *stream) {
  if (rows == nullptr || centroids == nullptr || assign_out == nullptr)
    return fail(UV_EINVAL, "null argument");
  if (n < 0 || dim < 1 || nlist < 1) return fail(UV_EINVAL, "bad size");
  if (n == 0) return UV_OK;
  DeviceGuard g(device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_rows = nullptr, *d_cent = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * dim, device, sc, &d_rows));
  UV_TRY(stage_in(centroids, (size_t)nlist * dim, device, sc, &d_cent));
  uint32_t *asg = nullptr;
  UV_TRY(outs.stage(assign_out, (size_t)n, device, sc, &asg));
  UV_TRY(assign_device(d_rows, n, dim, d_cent, nlist, asg, st, sc));
  return outs.finish(st);
}

int uv_ivf_create(const uv_codec *codec, const float *centroids, int32_t nlist, int32_t centered,
                  uv_ivf **out) {
  if (codec == nullptr || centroids == nullptr || out == nullptr)
    return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  if (nlist < 1) return fail(UV_EINVAL, "nlist must be positive");
  const int d = codec->cfg.dim;
  DeviceGuard g(codec->cfg.device);
  uv_ivf *ix = new (std::nothrow) uv_ivf();
  if (ix == nullptr) return fail(UV_ENOMEM, "host allocation failed");
  ix->codec = codec;
  ix->device = codec->cfg.device;
  ix->nlist = nlist;
  ix->centered = centered ? 1 : 0;
  ix->off.assign((size_t)nlist + 1, 0);
  cudaError_t e = cudaMalloc(&ix->centroids, sizeof(float) * (size_t)nlist * d);
  if (e == cudaSuccess) e = cudaMalloc(&ix->cnorm, sizeof(float) * (size_t)nlist);
  if (e == cudaSuccess)
    e = cudaMemcpy(ix->centroids, centroids, sizeof(float) * (size_t)nlist * d, cudaMemcpyDefault);
  if (e == cudaSuccess) {
    uvb::row_norms_kernel<<<blocks(nlist, 128), 128>>>(ix->centroids, nlist, d, ix->cnorm);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ix->centroids);
    cudaFree(ix->cnorm);
    delete ix;
    return fail(e == cudaErrorMemoryAllocation ? UV_ENOMEM : UV_ECUDA,
                std::string("ivf create: ") + cudaGetErrorString(e));
  }
  *out = ix;
  return UV_OK;
}

int uv_ivf_destroy(uv_ivf *ix) {
  if (ix == nullptr) return UV_OK;
  {
    DeviceGuard g(ix->device);
    free_lists(ix);
    cudaFree(ix->centroids);
    cudaFree(ix->cnorm);
    cudaFree(ix->c16);
    cudaFree(ix->cext);
  }
  delete ix;
  return UV_OK;
}

int uv_ivf_build(uv_ivf *ix, const float *rows, int64_t n, const uint32_t *assign,
                 const int64_t *ids, void *stream) {
  if (ix == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  UV_CK(cudaStreamSynchronize(st));
  free_lists(ix);
  ix->off.assign((size_t)ix->nlist + 1, 0);
  Scratch sc(st);
  const float *d_rows = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * d, dev, sc, &d_rows));
  // assignment and stable bucketing
  std::vector<uint32_t> h_asg((size_t)n);
  if (assign != nullptr) {
    if (n > 0) UV_TRY(copy_to_host(h_asg.data(), assign, sizeof(uint32_t) * n, st));
  } else if (n > 0) {
    uint32_t *asg = nullptr;
    UV_TRY(sc.alloc(&asg, (size_t)n));
    UV_TRY(assign_device(d_rows, n, d, ix->centroids, ix->nlist, asg, st, sc));
    UV_TRY(copy_to_host(h_asg.data(), asg, sizeof(uint32_t) * n, st));
  }
  std::vector<int64_t> order, off;
  UV_TRY(bucket_host(h_asg, ix->nlist, order, off));
  std::vector<int64_t> h_ids((size_t)n);
  if (ids != nullptr && n > 0) {
    std::vector<int64_t> in((size_t)n);
    UV_TRY(copy_to_host(in.data(), ids, sizeof(int64_t) * n, st));
    for (int64_t i = 0; i < n; i++) h_ids[i] = in[(size_t)order[i]];
  } else {
    for (int64_t i = 0; i < n; i++) h_ids[i] = order[i];
  }
  std::vector<uint32_t> row_list((size_t)n);
  for (int j = 0; j < ix->nlist; j++)
    for (int64_t i = off[j]; i < off[j + 1]; i++) row_list[(size_t)i] = (uint32_t)j;
  // device lists
  const int64_t cap = std::max<int64_t>(n, 1);
  UV_CK(cudaMalloc(&ix->codes, (size_t)cap * c->code_stride));
  UV_CK(cudaMalloc(&ix->start, sizeof(uint32_t) * cap));
  UV_CK(cudaMalloc(&ix->rescale, sizeof(float) * cap));
  UV_CK(cudaMalloc(&ix->rnorm, sizeof(float) * cap));
  UV_CK(cudaMalloc(&ix->ids, sizeof(int64_t) * cap));
  UV_CK(cudaMalloc(&ix->d_off, sizeof(int64_t) * (ix->nlist + 1)));
  if (ix->sl_c > 0) UV_CK(cudaMalloc(&ix->signs, (size_t)cap * c->sign_stride));
  UV_CK(cudaMemcpyAsync(ix->d_off, off.data(), sizeof(int64_t) * (ix->nlist + 1),
                        cudaMemcpyHostToDevice, st));
  if (n > 0) {
    UV_CK(cudaMemcpyAsync(ix->ids, h_ids.data(), sizeof(int64_t) * n, cudaMemcpyHostToDevice, st));
    int64_t *d_order = nullptr;
    uint32_t *d_list = nullptr;
    UV_TRY(upload(order, sc, &d_order, st));
    UV_TRY(upload(row_list, sc, &d_list, st));
    UV_TRY(encode_device(c, d_rows, n, nullptr, 0, false, ix->codes, ix->start, ix->rescale,
                         ix->rnorm, nullptr, nullptr, st, sc,
                         ix->centered ? ix->centroids : nullptr, d_list, d_order, ix->signs));
  }
  UV_CK(cudaStreamSynchronize(st));  // the host vectors above end with this call
  ix->off = off;
  ix->n = n;
  return UV_OK;
}

int uv_ivf_len(const uv_ivf *ix, int64_t *len) {
  if (ix == nullptr || len == nullptr) return fail(UV_EINVAL, "null argument");
  *len = ix->n;
  return UV_OK;
}

int uv_ivf_nlist(const uv_ivf *ix, int32_t *nlist) {
  if (ix == nullptr || nlist == nullptr) return fail(UV_EINVAL, "null argument");
  *nlist = ix->nlist;
  return UV_OK;
}

int uv_ivf_mem_bytes(const uv_ivf *ix, int64_t *bytes) {
  if (ix == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  int32_t cb = 0, sb = 0, rb = 0;
  uv_codec_record_bytes(ix->codec, &cb, &sb, &rb);
  const int64_t sign = ix->sl_c > 0 ? ix->codec->sign_bytes : 0;  // src/trellis.rs:2196
  *bytes = ix->n * (int64_t)(cb + sb + rb + (ix->centered ? 4 : 0) + sign);
  return UV_OK;
}

// IvfCodec::TrellisShortlist{c, asym, rnorm} (src/ivf.rs:52-60, 111-135):
// set before build, which writes the sign codes.
int uv_ivf_set_shortlist(uv_ivf *ix, int32_t c, int32_t asym, int32_t rnorm) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  if (c < 0 || (asym != 0 && asym != 1) || (rnorm != 0 && rnorm != 1))
    return fail(UV_EINVAL, "shortlist: c >= 0, asym and rnorm 0 or 1");
  if (ix->n > 0 && (c > 0) != (ix->sl_c > 0))
    return fail(UV_EINVAL, "shortlist: switch it on or off before build");
  ix->sl_c = c;
  ix->sl_asym = asym;
  ix->sl_weight = rnorm;
  return UV_OK;
}

int uv_ivf_export_signs(const uv_ivf *ix, uint8_t *signs, void *stream) {
  if (ix == nullptr || signs == nullptr) return fail(UV_EINVAL, "null argument");
  if (ix->sl_c == 0) return fail(UV_EINVAL, "the shortlist is off: no sign codes");
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  if (ix->n == 0) return UV_OK;
  UV_CK(cudaMemcpy2DAsync(signs, c->sign_bytes, ix->signs, c->sign_stride, c->sign_bytes, ix->n,
                          cudaMemcpyDefault, st));
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

int uv_ivf_probe(const uv_ivf *ix, const float *queries, int64_t nq, int32_t nprobe,
                 int32_t *lists_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || lists_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0 || nprobe < 0) return fail(UV_EINVAL, "negative size");
  if (nq == 0 || nprobe == 0) return UV_OK;
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * ix->codec->cfg.dim, dev, sc, &d_q));
  int32_t *lists = nullptr;
  UV_TRY(outs.stage(lists_out, (size_t)nq * nprobe, dev, sc, &lists));
  const int np = std::min(nprobe, ix->nlist);
  if (np < nprobe) UV_CK(cudaMemsetAsync(lists, 0xff, sizeof(int32_t) * nq * nprobe, st));
  UV_TRY(probe_device(ix, d_q, nq, np, nprobe, lists, st, sc));
  return outs.finish(st);
}

int uv_ivf_search(const uv_ivf *ix, const float *queries, int64_t nq, int32_t k, int32_t nprobe,
                  int64_t *ids_out, float *scores_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0 || nprobe < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1 || k > uvb::kScanKCap) return fail(UV_EINVAL, "k must be 1..128");
  if (nq == 0) return UV_OK;
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * ix->codec->cfg.dim, dev, sc, &d_q));
  int64_t *d_ids = nullptr;
  float *d_scores = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, sc, &d_scores));
  } else {
    UV_TRY(sc.alloc(&d_scores, (size_t)nq * k));
  }
  UV_TRY(search_device(ix, d_q, nq, k, std::min(nprobe, ix->nlist), d_ids, d_scores, st, sc));
  return outs.finish(st);
}

int uv_ivf_search_lists(const uv_ivf *ix, const float *queries, int64_t nq, int32_t k,
                        int32_t nprobe, const int32_t *lists, int64_t *ids_out, float *scores_out,
                        void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr ||
                                   (nprobe > 0 && lists == nullptr))))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0 || nprobe < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1 || k > uvb::kScanKCap) return fail(UV_EINVAL, "k must be 1..128");
  if (nq == 0) return UV_OK;
  if (nq * (int64_t)nprobe > INT32_MAX) return fail(UV_EINVAL, "nq * nprobe exceeds 2^31 - 1");
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  const int32_t *d_lists = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * ix->codec->cfg.dim, dev, sc, &d_q));
  if (nprobe > 0) UV_TRY(stage_in(lists, (size_t)nq * nprobe, dev, sc, &d_lists));
  int64_t *d_ids = nullptr;
  float *d_scores = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, sc, &d_scores));
  } else {
    UV_TRY(sc.alloc(&d_scores, (size_t)nq * k));
  }
  UV_TRY(search_device(ix, d_q, nq, k, nprobe, d_ids, d_scores, st, sc, true, d_lists));
  return outs.finish(st);
}

int uv_ivf_search_rerank(const uv_ivf *ix, const float *queries, int64_t nq, int32_t k,
                         int32_t nprobe, int32_t rdepth, const float *db, int64_t n_db,
                         int64_t *ids_out, float *scores_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr || db == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0 || nprobe < 0 || n_db < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1 || k > uvb::kScanKCap) return fail(UV_EINVAL, "k must be 1..128");
  const int r = std::max(rdepth, k);
  if (r > uvb::kScanKCap) return fail(UV_EUNSUPPORTED, "rerank depth above 128");
  if (nq == 0) return UV_OK;
  const int d = ix->codec->cfg.dim;
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr, *d_db = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * d, dev, sc, &d_q));
  UV_TRY(stage_in(db, (size_t)n_db * d, dev, sc, &d_db));
  int64_t *d_ids = nullptr, *cand = nullptr;
  float *d_scores = nullptr, *cand_s = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, sc, &d_scores));
  } else {
    UV_TRY(sc.alloc(&d_scores, (size_t)nq * k));
  }
  UV_TRY(sc.alloc(&cand, (size_t)nq * r));
  UV_TRY(sc.alloc(&cand_s, (size_t)nq * r));
  UV_TRY(search_device(ix, d_q, nq, r, std::min(nprobe, ix->nlist), cand, cand_s, st, sc));
  int *err = nullptr;
  UV_TRY(sc.alloc(&err, 1));
  UV_CK(cudaMemsetAsync(err, 0, sizeof(int), st));
  uvb::RerankParams rp;
  std::memset(&rp, 0, sizeof(rp));
  rp.nq = nq;
  rp.dim = d;
  rp.r = r;
  rp.k = k;
  rp.queries = d_q;
  rp.db = d_db;
  rp.n_db = n_db;
  rp.err = err;
  rp.cand = cand;
  rp.out_id = d_ids;
  rp.out_score = d_scores;
  {
    void *args[] = {&rp};
    ProfScope ps("ivf_rerank", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::rerank_kernel, dim3(blocks(nq, 8)), dim3(256), args,
                           0, st));
  }
  int h_err = 0;
  UV_TRY(copy_to_host(&h_err, err, sizeof(int), st));
  if (h_err) return fail(UV_EINVAL, "a candidate id does not index db (id >= n_db)");
  return outs.finish(st);
}

int uv_ivf_export(const uv_ivf *ix, int64_t *list_off, int64_t *ids, uint8_t *codes,
                  uint32_t *start, float *rescale, float *rnorm, void *stream) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = ix->n;
  if (list_off)
    UV_CK(cudaMemcpyAsync(list_off, ix->off.data(), sizeof(int64_t) * (ix->nlist + 1),
                          cudaMemcpyDefault, st));
  if (n > 0) {
    if (codes)
      UV_CK(cudaMemcpy2DAsync(codes, c->code_bytes, ix->codes, c->code_stride, c->code_bytes, n,
                              cudaMemcpyDefault, st));
    if (ids) UV_CK(cudaMemcpyAsync(ids, ix->ids, 8 * n, cudaMemcpyDefault, st));
    if (start) UV_CK(cudaMemcpyAsync(start, ix->start, 4 * n, cudaMemcpyDefault, st));
    if (rescale) UV_CK(cudaMemcpyAsync(rescale, ix->rescale, 4 * n, cudaMemcpyDefault, st));
    if (rnorm) UV_CK(cudaMemcpyAsync(rnorm, ix->rnorm, 4 * n, cudaMemcpyDefault, st));
  }
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

int uv_ivf_digest(const uv_ivf *ix, uint64_t *digest, void *stream) {
  if (ix == nullptr || digest == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  *digest = 0;
  if (ix->n == 0) return UV_OK;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  unsigned long long *d_acc = nullptr;
  UV_TRY(sc.alloc(&d_acc, 1));
  UV_CK(cudaMemsetAsync(d_acc, 0, sizeof(unsigned long long), st));
  UV_CK(uvb::launch_digest(ix->codes, c->code_stride, c->code_bytes, ix->start, ix->n, d_acc, st));
  unsigned long long h = 0;
  UV_TRY(copy_to_host(&h, d_acc, sizeof(h), st));
  *digest = h;
  return UV_OK;
}

}  // extern "C"
