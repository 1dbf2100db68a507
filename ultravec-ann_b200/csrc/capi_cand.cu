// capi_cand.cu -- the batched CandidateScorer / PreparedQuery entry points
// (src/lib.rs:83-102, impl src/trellis.rs:2003-2086) over a flat index, and
// the launcher of the 1-bit shortlist search (src/trellis.rs:841-948).
#include "capi_internal.h"

using namespace uvcapi;

namespace uvcapi {

int shortlist_launch(const uv_codec *c, int cs, int asym, int weight, int k, int64_t npairs,
                     int per_query, const int32_t *lists, const int64_t *list_off,
                     int64_t max_len, int64_t n_flat, const float *q_r, const float *u,
                     const float *centroids, const float *qc, int n_centroids,
                     const uint32_t *degen, const uint8_t *codes, const uint8_t *signs,
                     const uint32_t *start, const uint32_t *cidx, const float *rescale,
                     const float *rnorm, const int64_t *ids, int64_t *out_id, float *out_score,
                     cudaStream_t st) {
  if (npairs == 0) return UV_OK;
  if (npairs > INT32_MAX) return fail(UV_EINVAL, "shortlist: too many (query, list) pairs");
  const int d = c->cfg.dim;
  const int64_t ce_max = std::min<int64_t>(std::max(cs, k), std::max<int64_t>(max_len, 1));
  int cp = 256;
  while (cp < ce_max) cp <<= 1;
  if (cp > 4096) return fail(UV_EUNSUPPORTED, "shortlist: C above 4096 is not built");
  const int q_stride = (d + 3) & ~3;
  const size_t smem = uvb::shortlist_smem_bytes(cp, q_stride, c->sign_stride, c->table_len);
  if (smem > 227 * 1024)
    return fail(UV_EUNSUPPORTED, "shortlist: code table and buffers exceed shared memory");
  uvb::ShortlistParams p;
  std::memset(&p, 0, sizeof(p));
  p.dim = d;
  p.mem = c->cfg.mem;
  p.bits = c->cfg.bits;
  p.code_stride = c->code_stride;
  p.sign_stride = c->sign_stride;
  p.q_stride = q_stride;
  p.u_stride = q_stride;
  p.cs = cs;
  p.k = k;
  p.cp = cp;
  p.weight = weight;
  p.table_len = c->table_len;
  p.n_centroids = n_centroids;
  p.per_query = per_query;
  p.npairs = npairs;
  p.n_flat = n_flat;
  p.lists = lists;
  p.list_off = list_off;
  p.q_r = q_r;
  p.u = u;
  p.centroids = centroids;
  p.qc = qc;
  p.degenerate = degen;
  p.codes = codes;
  p.signs = signs;
  p.start = start;
  p.cidx = cidx;
  p.code = c->d_table;
  p.rescale = rescale;
  p.rnorm = rnorm;
  p.ids = ids;
  p.out_id = out_id;
  p.out_score = out_score;
  const void *kern = uvb::shortlist_kernel_ptr(c->cfg.bits, asym != 0);
  if (kern == nullptr) return fail(UV_EUNSUPPORTED, "shortlist: bits must be 1..4");
  UV_CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void *args[] = {&p};
  ProfScope ps("shortlist", st);
  UV_CK(cudaLaunchKernel(kern, dim3((unsigned)npairs), dim3(256), args, smem, st));
  return UV_OK;
}

}  // namespace uvcapi

// A batch of prepared queries: the hoists prepare() makes once per query
// (unit query, rotated q_r, per-centroid qc, the degenerate flag), resident
// on the index's GPU.  Scoring reads the index's arrays at call time.
struct uv_prepared {
  const uv_index *index = nullptr;
  int device = 0;  // destroy touches nothing of the index, which may be gone
  int64_t nq = 0;
  float *q_r = nullptr;  // nq x dim_pad
  float *qc = nullptr;   // nq x max(1, n_centroids)
  uint32_t *degen = nullptr;
  int n_centroids = 0;
};

namespace {

int prepared_free(uv_prepared *p) {
  if (p->q_r) cudaFree(p->q_r);
  if (p->qc) cudaFree(p->qc);
  if (p->degen) cudaFree(p->degen);
  delete p;
  return UV_OK;
}

// Score candidates [0, n) of a CSR batch against prepared queries.  Returns
// UV_EINVAL (after the launch) when a position lies outside the index or a
// candidate falls outside [offsets[0], offsets[nq]).
int score_launch(const uv_index *ix, int64_t nq, const float *q_r, const float *qc,
                 const uint32_t *degen, int n_centroids, const int64_t *d_off,
                 const int64_t *d_pos, int64_t n, float *d_out, cudaStream_t st, Scratch &sc) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  int *d_bad = nullptr;
  UV_TRY(sc.alloc(&d_bad, 1));
  UV_CK(cudaMemsetAsync(d_bad, 0, sizeof(int), st));
  uvb::CandParams p;
  std::memset(&p, 0, sizeof(p));
  p.dim = d;
  p.mem = c->cfg.mem;
  p.bits = c->cfg.bits;
  p.code_stride = c->code_stride;
  p.q_stride = (d + 3) & ~3;
  p.n_centroids = n_centroids;
  p.table_len = c->table_len;
  p.table_in_smem = (size_t)c->table_len * 4 <= 32 * 1024;
  p.nq = nq;
  p.n = n;
  p.n_records = ix->n;
  p.offsets = d_off;
  p.positions = d_pos;
  p.q_r = q_r;
  p.qc = qc;
  p.degenerate = degen;
  p.codes = ix->codes;
  p.start = ix->start;
  p.cidx = ix->cidx;
  p.code = c->d_table;
  p.rescale = ix->rescale;
  p.rnorm = ix->rnorm;
  p.out = d_out;
  p.n_bad = d_bad;
  void *args[] = {&p};
  const void *lane_k = g_cand_kernel == 1 ? nullptr : uvb::score_candidates_lane_kernel_ptr(c->cfg.bits);
  if (lane_k != nullptr) {
    // one thread per candidate; the table replicated R times (bank-private
    // copies at R = 32) within 160 KB of shared memory, else read from global
    int rep = 32;
    while (rep > 0 && (size_t)c->table_len * 4 * rep > 160 * 1024) rep >>= 1;
    p.table_rep = rep;
    const size_t smem = (size_t)c->table_len * 4 * rep;
    UV_CK(cudaFuncSetAttribute(lane_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t blocks = (n + 1023) / 1024;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(blocks, (int64_t)sm_count(c->cfg.device)));
    ProfScope ps("score_candidates", st);
    UV_CK(cudaLaunchKernel(lane_k, dim3(grid), dim3(1024), args, smem, st));
  } else {
    const size_t smem = p.table_in_smem ? (size_t)c->table_len * 4 : 0;
    UV_CK(cudaFuncSetAttribute(uvb::score_candidates_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int64_t blocks = (n + 15) / 16;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(blocks, (int64_t)sm_count(c->cfg.device) * 8));
    ProfScope ps("score_candidates", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::score_candidates_kernel, dim3(grid), dim3(256),
                           args, smem, st));
  }
  int bad = 0;
  UV_CK(cudaMemcpyAsync(&bad, d_bad, sizeof(int), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  if (bad != 0)
    return fail(UV_EINVAL, std::to_string(bad) +
                               " candidates lie outside the index or outside the offsets");
  return UV_OK;
}

// Host-side check of CSR offsets (device offsets are checked by the kernel).
int check_offsets(const int64_t *off, int64_t nq, int64_t n, int dev) {
  bool on_dev = false;
  UV_TRY(classify(off, dev, &on_dev));
  if (on_dev) return UV_OK;
  if (off[0] != 0 || off[nq] != n) return fail(UV_EINVAL, "offsets must run from 0 to n");
  for (int64_t q = 0; q < nq; q++)
    if (off[q + 1] < off[q]) return fail(UV_EINVAL, "offsets must not decrease");
  return UV_OK;
}

}  // namespace

extern "C" {

int uv_index_prepare(const uv_index *ix, const float *queries, int64_t nq, uv_prepared **out,
                     void *stream) {
  if (ix == nullptr || out == nullptr || (nq > 0 && queries == nullptr))
    return fail(UV_EINVAL, "null argument");
  if (nq < 1) return fail(UV_EINVAL, "nq must be at least 1");
  *out = nullptr;
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  uv_prepared *p = new (std::nothrow) uv_prepared;
  if (p == nullptr) return fail(UV_ENOMEM, "out of host memory");
  p->index = ix;
  p->device = dev;
  p->nq = nq;
  p->n_centroids = ix->n_centroids;
  const size_t dim_pad = (size_t)((d + 3) & ~3);
  cudaError_t e = cudaMalloc((void **)&p->q_r, sizeof(float) * (size_t)nq * dim_pad);
  if (e == cudaSuccess)
    e = cudaMalloc((void **)&p->qc, sizeof(float) * (size_t)nq * std::max(1, ix->n_centroids));
  if (e == cudaSuccess) e = cudaMalloc((void **)&p->degen, sizeof(uint32_t) * (size_t)nq);
  if (e != cudaSuccess) {
    cudaGetLastError();
    prepared_free(p);
    return fail(e == cudaErrorMemoryAllocation ? UV_ENOMEM : UV_ECUDA,
                std::string("prepare: ") + cudaGetErrorString(e));
  }
  int rc;
  {
    Scratch sc(st);
    const float *d_q = nullptr;
    rc = stage_in(queries, (size_t)nq * d, dev, sc, &d_q);
    if (rc == UV_OK)
      rc = prep_launch(c, d_q, nq, ix->centroids, ix->n_centroids, p->q_r, p->qc, p->degen,
                       nullptr, st);
    if (rc == UV_OK && cudaStreamSynchronize(st) != cudaSuccess)
      rc = fail(UV_ECUDA, std::string("prepare: ") + cudaGetErrorString(cudaGetLastError()));
  }
  if (rc != UV_OK) {
    prepared_free(p);
    return rc;
  }
  *out = p;
  return UV_OK;
}

int uv_prepared_destroy(uv_prepared *p) {
  if (p == nullptr) return UV_OK;
  DeviceGuard g(p->device);
  return prepared_free(p);
}

int uv_prepared_len(const uv_prepared *p, int64_t *nq) {
  if (p == nullptr || nq == nullptr) return fail(UV_EINVAL, "null argument");
  *nq = p->nq;
  return UV_OK;
}

int uv_prepared_score(const uv_prepared *p, const int64_t *offsets, const int64_t *positions,
                      int64_t n, float *scores_out, void *stream) {
  if (p == nullptr || (n > 0 && (positions == nullptr || scores_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (offsets == nullptr && p->nq != 1)
    return fail(UV_EINVAL, "offsets are required for more than one prepared query");
  if (p->n_centroids != p->index->n_centroids)
    return fail(UV_EINVAL, "the index's centroids changed since prepare");
  const uv_index *ix = p->index;
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  if (offsets != nullptr) UV_TRY(check_offsets(offsets, p->nq, n, dev));
  if (n == 0) return UV_OK;
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const int64_t *d_off = nullptr, *d_pos = nullptr;
  if (offsets != nullptr) UV_TRY(stage_in(offsets, (size_t)p->nq + 1, dev, sc, &d_off));
  UV_TRY(stage_in(positions, (size_t)n, dev, sc, &d_pos));
  float *d_out = nullptr;
  UV_TRY(outs.stage(scores_out, (size_t)n, dev, sc, &d_out));
  UV_TRY(score_launch(ix, p->nq, p->q_r, p->qc, p->degen, p->n_centroids, d_off, d_pos, n, d_out,
                      st, sc));
  return outs.finish(st);
}

int uv_index_score_candidates(const uv_index *ix, const float *query, const int64_t *positions,
                              int64_t n, float *scores_out, void *stream) {
  if (ix == nullptr || query == nullptr || (n > 0 && (positions == nullptr || scores_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  const int64_t *d_pos = nullptr;
  UV_TRY(stage_in(query, (size_t)d, dev, sc, &d_q));
  UV_TRY(stage_in(positions, (size_t)n, dev, sc, &d_pos));
  float *d_out = nullptr;
  UV_TRY(outs.stage(scores_out, (size_t)n, dev, sc, &d_out));
  float *q_r = nullptr, *qc = nullptr;
  uint32_t *degen = nullptr;
  UV_TRY(sc.alloc(&q_r, (size_t)((d + 3) & ~3)));
  UV_TRY(sc.alloc(&qc, (size_t)std::max(1, ix->n_centroids)));
  UV_TRY(sc.alloc(&degen, 1));
  UV_TRY(prep_launch(c, d_q, 1, ix->centroids, ix->n_centroids, q_r, qc, degen, nullptr, st));
  UV_TRY(score_launch(ix, 1, q_r, qc, degen, ix->n_centroids, nullptr, d_pos, n, d_out, st, sc));
  return outs.finish(st);
}

int uv_index_scorer_model_bytes(const uv_index *ix, int64_t *bytes) {
  if (ix == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  *bytes = (int64_t)c->table_len * 4 + (int64_t)c->rot_host.signs.size() * 4 +
           (int64_t)ix->n_centroids * c->cfg.dim * 4;
  return UV_OK;
}

}  // extern "C"
