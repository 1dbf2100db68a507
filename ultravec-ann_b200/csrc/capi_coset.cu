// capi_coset.cu -- the coset trellis index (src/coset_trellis.rs), the
// research arm the reference enables with ULTRAVEC_COSET_TRELLIS=1: handle,
// books, encode (coset.cu) and search (the flat scan's decode-GEMM over
// coset records, scan.cu).
#include <cmath>
#include <functional>
#include <map>
#include <memory>

#include "capi_internal.h"

using namespace uvcapi;

namespace {

// Books of one bit width (src/coset_trellis.rs:131-186), shared by every
// handle: per coset its 2^(8b-3) lowest points by (norm, lex) as sorted
// 64-bit keys, and the unit-variance scaling over their union.
struct CosetBooks {
  int bits = 0, per_coset = 0;
  std::vector<uint64_t> keys;  // 8 x per_coset
  float mean = 0.0f, sd = 0.0f;
};

uint64_t key_of(const int *r) {
  int64_t n = 0;
  uint64_t lex = 0;
  for (int j = 0; j < 8; j++) {
    n += (int64_t)r[j] * r[j];
    lex = (lex << 5) | (uint64_t)((r[j] + 16) & 31);
  }
  return ((uint64_t)n << 40) | lex;
}

int label_of(const int *r) {
  return ((((r[0] - r[1]) / 2) & 1) << 2) | ((((r[2] - r[3]) / 2) & 1) << 1) |
         (((r[4] - r[5]) / 2) & 1);
}

// every E8 point with sum R^2 <= budget in raw doubled coordinates: one
// parity for all coordinates, coordinate sum 0 mod 4 (src/e8.rs:82-141)
template <class F>
void enumerate_e8(int64_t budget, F &&fn) {
  int cur[8];
  for (int parity = 0; parity < 2; parity++) {
    std::function<void(int, int64_t, int64_t)> rec = [&](int pos, int64_t left, int64_t sum) {
      if (pos == 8) {
        if (((sum % 4) + 4) % 4 == 0) fn(cur);
        return;
      }
      const int64_t bound = (int64_t)std::floor(std::sqrt((double)left));
      int64_t r = -bound;
      while (((r % 2) + 2) % 2 != parity) r++;
      for (; r <= bound; r += 2)
        if (r * r <= left) {
          cur[pos] = (int)r;
          rec(pos + 1, left - r * r, sum + r);
        }
    };
    rec(0, budget, 0);
  }
}

std::shared_ptr<const CosetBooks> build_books(int bits) {
  auto b = std::make_shared<CosetBooks>();
  b->bits = bits;
  b->per_coset = 1 << (8 * bits - 3);
  // grow r2 = 2, 4, ... until every coset holds per_coset points
  float r2 = 2.0f;
  for (;;) {
    int64_t counts[8] = {0};
    enumerate_e8((int64_t)std::floor(4.0f * r2), [&](const int *r) { counts[label_of(r)]++; });
    bool ok = true;
    for (int k = 0; k < 8; k++) ok &= counts[k] >= b->per_coset;
    if (ok) break;
    r2 += 2.0f;
  }
  std::vector<uint64_t> all;
  enumerate_e8((int64_t)std::floor(4.0f * r2), [&](const int *r) { all.push_back(key_of(r)); });
  std::sort(all.begin(), all.end());
  b->keys.assign((size_t)8 * b->per_coset, 0);
  int64_t fill[8] = {0};
  for (uint64_t key : all) {
    int r[8];
    for (int j = 0; j < 8; j++) r[j] = (int)((key >> (5 * (7 - j))) & 31) - 16;
    const int k = label_of(r);
    if (fill[k] < b->per_coset) b->keys[(size_t)k * b->per_coset + fill[k]++] = key;
  }
  double sum = 0.0, sumsq = 0.0, cnt = 0.0;
  for (uint64_t key : b->keys)
    for (int j = 0; j < 8; j++) {
      const double x = (double)((int)((key >> (5 * (7 - j))) & 31) - 16) / 2.0;
      sum += x;
      sumsq += x * x;
      cnt += 1.0;
    }
  const double mean = sum / cnt;
  const double var = sumsq / cnt - mean * mean;
  b->mean = (float)mean;
  b->sd = (float)std::sqrt(var > 1e-12 ? var : 1e-12);
  return b;
}

std::shared_ptr<const CosetBooks> books_for(int bits) {
  static std::mutex mu;
  static std::map<int, std::shared_ptr<const CosetBooks>> cache;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(bits);
  if (it != cache.end()) return it->second;
  auto b = build_books(bits);
  cache[bits] = b;
  return b;
}

}  // namespace

struct uv_coset {
  int device = 0, dim = 0, bits = 0, mem = 0;
  std::shared_ptr<const CosetBooks> books;
  uvb::CosetModel m;  // device pointers
  uvb::RotationHost rot_host;
  uvb::RotParams rot;
  float *d_signs = nullptr;
  uint64_t *d_books = nullptr;
  float *d_xval = nullptr;
  float *centroids = nullptr;
  int n_centroids = 0;
  int64_t n = 0, cap = 0;
  uint8_t *codes = nullptr;
  float *rescale = nullptr, *rnorm = nullptr;
  uint32_t *cidx = nullptr;
  int64_t *ids = nullptr;
};

namespace {

// Encode n device rows into records (coset.cu): prep, nearest point of every
// coset per block, Viterbi + emission; in chunks that bound the scratch.
int coset_encode(const uv_coset *ix, const float *d_rows, int64_t n, uint8_t *codes,
                 float *rescale, float *rnorm, uint32_t *cidx, cudaStream_t st, Scratch &sc) {
  if (n == 0) return UV_OK;
  const int d = ix->dim, nb = d / 8, dev = ix->device;
  const int64_t S = (int64_t)1 << ix->mem;
  const int sms = sm_count(dev);
  const int64_t chunk = std::min<int64_t>(
      n, std::max<int64_t>(1024, std::min<int64_t>(262144, (512ll << 20) / (16ll * d))));
  float *u_r = nullptr, *y = nullptr, *bcost = nullptr;
  uint32_t *bidx = nullptr;
  UV_TRY(sc.alloc(&u_r, (size_t)chunk * d));
  UV_TRY(sc.alloc(&y, (size_t)chunk * d));
  UV_TRY(sc.alloc(&bcost, (size_t)chunk * nb * 8));
  UV_TRY(sc.alloc(&bidx, (size_t)chunk * nb * 8));
  // Viterbi placement: costs in shared memory up to 2^13 states, back
  // pointers while the whole CTA footprint stays under 200 KB
  const bool cost_smem = 2 * S * 4 <= 64 * 1024;
  const bool back_smem = uvb::coset_viterbi_smem_bytes(d, ix->mem, true, cost_smem) <= 200 * 1024;
  const size_t vsmem = uvb::coset_viterbi_smem_bytes(d, ix->mem, back_smem, cost_smem);
  UV_CK(cudaFuncSetAttribute(uvb::coset_viterbi_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)vsmem));
  int per_sm = 1;
  UV_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, uvb::coset_viterbi_kernel, 256,
                                                      vsmem));
  int64_t vgrid = std::min<int64_t>(chunk, (int64_t)sms * std::max(per_sm, 1));
  const int64_t per_cta = (back_smem ? 0 : (int64_t)nb * S) + (cost_smem ? 0 : 8 * S);
  if (per_cta > 0) vgrid = std::max<int64_t>(1, std::min<int64_t>(vgrid, (1ll << 30) / per_cta));
  uint8_t *back = nullptr;
  float *cost = nullptr;
  if (!back_smem) UV_TRY(sc.alloc(&back, (size_t)vgrid * nb * S));
  if (!cost_smem) UV_TRY(sc.alloc(&cost, (size_t)vgrid * 2 * S));
  const size_t psmem = (size_t)8 * (d + 8) * 4;
  UV_CK(cudaFuncSetAttribute(uvb::coset_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)psmem));
  const bool brute = g_coset_nearest != 1 && ix->m.per_coset <= 8192;
  const size_t bsmem = uvb::coset_brute_smem_bytes(ix->m.per_coset);
  if (brute)
    UV_CK(cudaFuncSetAttribute(uvb::coset_nearest_brute_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsmem));
  for (int64_t done = 0; done < n; done += chunk) {
    const int64_t rows = std::min(chunk, n - done);
    uvb::CosetEncParams p;
    std::memset(&p, 0, sizeof(p));
    p.m = ix->m;
    p.n = rows;
    p.rows = d_rows + done * d;
    p.rot = ix->rot;
    p.centroids = ix->centroids;
    p.n_centroids = ix->n_centroids;
    p.u_r = u_r;
    p.y = y;
    p.blk_idx = bidx;
    p.blk_cost = bcost;
    p.back = back;
    p.cost = cost;
    p.back_smem = back_smem ? 1 : 0;
    p.cost_smem = cost_smem ? 1 : 0;
    p.codes = codes + done * ix->m.code_stride;
    p.rescale = rescale + done;
    p.rnorm = rnorm + done;
    p.cidx = cidx + done;
    void *args[] = {&p};
    {
      ProfScope ps("coset_prep", st);
      const int pgrid = (int)std::min<int64_t>((rows + 7) / 8, (int64_t)sms * 16);
      UV_CK(cudaLaunchKernel((const void *)uvb::coset_prep_kernel, dim3(pgrid), dim3(256), args,
                             psmem, st));
    }
    {
      ProfScope ps("coset_nearest", st);
      if (brute) {
        // every book point against tiles of y-blocks (books of <= 8192 points)
        const int64_t ny = rows * nb;
        const int64_t per_cta = 256 * uvb::kCosetBruteY;
        UV_CK(cudaLaunchKernel((const void *)uvb::coset_nearest_brute_kernel,
                               dim3((unsigned)((ny + per_cta - 1) / per_cta), 8), dim3(256), args,
                               bsmem, st));
      } else {
        const int64_t items = rows * nb * 8;
        const int ngrid = (int)std::min<int64_t>((items + 255) / 256, (int64_t)sms * 64);
        UV_CK(cudaLaunchKernel((const void *)uvb::coset_nearest_kernel, dim3(ngrid), dim3(256),
                               args, 0, st));
      }
    }
    {
      ProfScope ps("coset_viterbi", st);
      UV_CK(cudaLaunchKernel((const void *)uvb::coset_viterbi_kernel,
                             dim3((unsigned)std::min(vgrid, rows)), dim3(256), args, vsmem, st));
    }
  }
  return UV_OK;
}

template <class T>
int grow_to(T **buf, int64_t n_old, int64_t cap, size_t per, cudaStream_t st) {
  T *nb = nullptr;
  UV_CK(cudaMallocAsync((void **)&nb, (size_t)std::max<int64_t>(cap, 1) * per * sizeof(T), st));
  if (*buf != nullptr && n_old > 0)
    UV_CK(cudaMemcpyAsync(nb, *buf, (size_t)n_old * per * sizeof(T), cudaMemcpyDeviceToDevice, st));
  if (*buf != nullptr) cudaFreeAsync(*buf, st);
  *buf = nb;
  return UV_OK;
}

}  // namespace

extern "C" {

int uv_coset_create(int32_t dim, int32_t bits, int32_t mem, uint64_t rotation_seed,
                    int32_t rotation_rounds, int32_t device, uv_coset **out) {
  if (out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  if (dim <= 0 || dim % 8 != 0) return fail(UV_EINVAL, "coset trellis requires dim % 8 == 0");
  // one warp stages eight rows of the prep and reconstruction in 227 KB
  if (dim > 4096) return fail(UV_EUNSUPPORTED, "coset trellis rows wider than 4096 are not built");
  if (bits < 1 || bits > 3) return fail(UV_EINVAL, "coset trellis supports bits in 1..3");
  if (mem < 1 || mem > 20) return fail(UV_EINVAL, "mem must be 1..20");
  int ndev = 0;
  UV_CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(UV_EINVAL, "no such CUDA device");
  std::unique_ptr<uv_coset> ix(new (std::nothrow) uv_coset());
  if (!ix) return fail(UV_ENOMEM, "host allocation failed");
  ix->device = device;
  ix->dim = dim;
  ix->bits = bits;
  ix->mem = mem;
  ix->rot_host = uvb::build_rotation(dim, rotation_seed, std::max(rotation_rounds, 1));
  if ((int)ix->rot_host.blk_off.size() > uvb::kMaxBlocks)
    return fail(UV_EUNSUPPORTED, "dimension splits into too many power-of-two blocks");
  ix->books = books_for(bits);
  const CosetBooks &bk = *ix->books;
  DeviceGuard g(device);
  // x-bar of a raw coordinate R: (R/2 - mean) / std (src/coset_trellis.rs:430);
  // R/2 is exact, so the host expression rounds like the reference's
  float xval[32];
  for (int i = 0; i < 32; i++) xval[i] = ((float)(i - 16) * 0.5f - bk.mean) / bk.sd;
  auto cleanup = [&]() {
    cudaFree(ix->d_signs);
    cudaFree(ix->d_books);
    cudaFree(ix->d_xval);
  };
  cudaError_t e = cudaMalloc(&ix->d_signs, sizeof(float) * ix->rot_host.signs.size());
  if (e == cudaSuccess) e = cudaMalloc(&ix->d_books, sizeof(uint64_t) * bk.keys.size());
  if (e == cudaSuccess) e = cudaMalloc(&ix->d_xval, sizeof(float) * 32);
  if (e == cudaSuccess)
    e = cudaMemcpy(ix->d_signs, ix->rot_host.signs.data(),
                   sizeof(float) * ix->rot_host.signs.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(ix->d_books, bk.keys.data(), sizeof(uint64_t) * bk.keys.size(),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(ix->d_xval, xval, sizeof(xval), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cleanup();
    return fail(e == cudaErrorMemoryAllocation ? UV_ENOMEM : UV_ECUDA,
                std::string("coset upload: ") + cudaGetErrorString(e));
  }
  uvb::RotParams &r = ix->rot;
  std::memset(&r, 0, sizeof(r));
  r.dim = dim;
  r.rounds = ix->rot_host.rounds;
  r.n_blocks = (int)ix->rot_host.blk_off.size();
  for (int b = 0; b < r.n_blocks; b++) {
    r.blk_off[b] = ix->rot_host.blk_off[b];
    r.blk_len[b] = ix->rot_host.blk_len[b];
    r.blk_inv[b] = ix->rot_host.blk_inv[b];
  }
  r.signs = ix->d_signs;
  uvb::CosetModel &m = ix->m;
  std::memset(&m, 0, sizeof(m));
  m.dim = dim;
  m.mem = mem;
  m.m_bits = 8 * bits - 3;
  m.per_coset = bk.per_coset;
  m.start_bytes = (mem + 7) / 8;
  m.code_len = m.start_bytes + ((dim / 8) * (2 + m.m_bits) + 7) / 8;
  m.code_stride = (m.code_len + 15) & ~15;
  m.books = ix->d_books;
  for (int k = 0; k < 8; k++) m.bound[k] = bk.keys[(size_t)k * bk.per_coset + bk.per_coset - 1];
  m.scale_mean = bk.mean;
  m.scale_std = bk.sd;
  m.pi4 = std::pow(3.14159265358979323846, 4.0);
  m.xval = ix->d_xval;
  *out = ix.release();
  return UV_OK;
}

int uv_coset_destroy(uv_coset *ix) {
  if (ix == nullptr) return UV_OK;
  {
    DeviceGuard g(ix->device);
    cudaDeviceSynchronize();
    cudaFree(ix->d_signs);
    cudaFree(ix->d_books);
    cudaFree(ix->d_xval);
    cudaFree(ix->centroids);
    cudaFree(ix->codes);
    cudaFree(ix->rescale);
    cudaFree(ix->rnorm);
    cudaFree(ix->cidx);
    cudaFree(ix->ids);
  }
  delete ix;
  return UV_OK;
}

// with_centroids (src/coset_trellis.rs:192-196): before the first add.
int uv_coset_set_centroids(uv_coset *ix, const float *centroids, int32_t n_centroids) {
  if (ix == nullptr || (n_centroids > 0 && centroids == nullptr))
    return fail(UV_EINVAL, "null argument");
  if (n_centroids < 0) return fail(UV_EINVAL, "negative centroid count");
  if (ix->n > 0) return fail(UV_EINVAL, "centroids must be set before the first add");
  DeviceGuard g(ix->device);
  cudaFree(ix->centroids);
  ix->centroids = nullptr;
  ix->n_centroids = 0;
  if (n_centroids == 0) return UV_OK;
  const size_t bytes = sizeof(float) * (size_t)n_centroids * ix->dim;
  UV_CK(cudaMalloc(&ix->centroids, bytes));
  UV_CK(cudaMemcpy(ix->centroids, centroids, bytes, cudaMemcpyDefault));
  ix->n_centroids = n_centroids;
  return UV_OK;
}

int uv_coset_len(const uv_coset *ix, int64_t *n) {
  if (ix == nullptr || n == nullptr) return fail(UV_EINVAL, "null argument");
  *n = ix->n;
  return UV_OK;
}

int uv_coset_shape(const uv_coset *ix, int32_t *code_len, int32_t *per_coset) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  if (code_len) *code_len = ix->m.code_len;
  if (per_coset) *per_coset = ix->m.per_coset;
  return UV_OK;
}

// The books: 8 x per_coset keys, host memory.
int uv_coset_books(const uv_coset *ix, uint64_t *keys, float *scale) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  if (keys) std::memcpy(keys, ix->books->keys.data(), sizeof(uint64_t) * ix->books->keys.size());
  if (scale) {
    scale[0] = ix->books->mean;
    scale[1] = ix->books->sd;
  }
  return UV_OK;
}

// mem_bytes (src/coset_trellis.rs:498-504, src/lib.rs:229-237).
int uv_coset_mem_bytes(const uv_coset *ix, int64_t *bytes) {
  if (ix == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  int64_t center = 0;
  if (ix->n_centroids == 1) {
    center = 4;
  } else if (ix->n_centroids > 1) {
    int bitsn = 0;
    uint64_t v = (uint64_t)(ix->n_centroids - 1);
    while (v) {
      bitsn++;
      v >>= 1;
    }
    center = 4 + (bitsn + 7) / 8;
  }
  *bytes = ix->n * ((int64_t)ix->m.code_len + 4 + center);
  return UV_OK;
}

// memory_breakdown().model_bytes (src/coset_trellis.rs:505-517): rotation
// signs, 16 bytes per book point, centroids.
int uv_coset_model_bytes(const uv_coset *ix, int64_t *bytes) {
  if (ix == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = (int64_t)ix->rot_host.signs.size() * 4 + (int64_t)ix->books->keys.size() * 16 +
           (int64_t)ix->n_centroids * ix->dim * 4;
  return UV_OK;
}

}  // extern "C"

extern "C" {

// add (ids given) / add_batch (ids null: the batch's positions 0..n-1, as
// src/coset_trellis.rs:454-469 assigns them).  Rows: n x dim f32.
int uv_coset_add(uv_coset *ix, const int64_t *ids, const float *rows, int64_t n, void *stream) {
  if (ix == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  if (ix->n + n > INT32_MAX) return fail(UV_EUNSUPPORTED, "more than 2^31 - 1 records");
  DeviceGuard g(ix->device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  const float *d_rows = nullptr;
  const int64_t *d_ids = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * ix->dim, ix->device, sc, &d_rows));
  UV_TRY(stage_in(ids, (size_t)n, ix->device, sc, &d_ids));
  const int64_t need = ix->n + n;
  if (need > ix->cap) {
    const int64_t cap = std::max<int64_t>(need, ix->cap + ix->cap / 2);
    UV_TRY(grow_to(&ix->codes, ix->n, cap, (size_t)ix->m.code_stride, st));
    UV_TRY(grow_to(&ix->rescale, ix->n, cap, 1, st));
    UV_TRY(grow_to(&ix->rnorm, ix->n, cap, 1, st));
    UV_TRY(grow_to(&ix->cidx, ix->n, cap, 1, st));
    UV_TRY(grow_to(&ix->ids, ix->n, cap, 1, st));
    ix->cap = cap;
  }
  const int64_t base = ix->n;
  UV_TRY(coset_encode(ix, d_rows, n, ix->codes + base * ix->m.code_stride, ix->rescale + base,
                      ix->rnorm + base, ix->cidx + base, st, sc));
  if (d_ids != nullptr) {
    UV_CK(cudaMemcpyAsync(ix->ids + base, d_ids, sizeof(int64_t) * n, cudaMemcpyDeviceToDevice, st));
  } else {
    uvb::iota_i64_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 65535), 256, 0, st>>>(
        ix->ids + base, n, 0);
    UV_CK(cudaGetLastError());
  }
  ix->n = need;
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

// search (src/coset_trellis.rs:471-497): nq x k ids and scores, score
// descending then insertion position ascending; slots past len() hold id -1
// and score -inf.  Queries, outputs: host or device memory.
int uv_coset_search(const uv_coset *ix, const float *queries, int64_t nq, int32_t k,
                    int64_t *ids_out, float *scores_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1) return fail(UV_EINVAL, "k must be at least 1");
  if (nq == 0) return UV_OK;
  const int d = ix->dim, dev = ix->device;
  const int d16 = (d + 15) & ~15;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * d, dev, sc, &d_q));
  int64_t *d_ids = nullptr;
  float *d_scores = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, sc, &d_scores));
  } else {
    UV_TRY(sc.alloc(&d_scores, (size_t)nq * k));
  }
  // queries: q/|q| (|q| clamped at EPS), <q, c_j>, rotation; rows padded to 16
  float *q_r = nullptr, *qc = nullptr;
  uint32_t *degen = nullptr;
  UV_TRY(sc.alloc(&q_r, (size_t)nq * d16));
  UV_TRY(sc.alloc(&qc, (size_t)nq * std::max(1, ix->n_centroids)));
  UV_TRY(sc.alloc(&degen, (size_t)nq));
  UV_CK(cudaMemsetAsync(q_r, 0, sizeof(float) * nq * d16, st));
  {
    uvb::PrepParams pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.dim = d;
    pp.dim_pad = d16;
    pp.nq = nq;
    pp.queries = d_q;
    pp.rot = ix->rot;
    pp.centroids = ix->centroids;
    pp.n_centroids = ix->n_centroids;
    pp.q_r = q_r;
    pp.qc = qc;
    pp.degenerate = degen;
    pp.clamp_norm = 1;
    pp.teams = uvb::prep_teams(pp.dim);
    const size_t smem = (size_t)(d16 + 4) * 4 * pp.teams;
    UV_CK(cudaFuncSetAttribute(uvb::prep_queries_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((nq + pp.teams - 1) / pp.teams, INT32_MAX));
    void *args[] = {&pp};
    ProfScope ps("prep_queries", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::prep_queries_kernel, dim3(grid), dim3(256), args,
                           smem, st));
  }
  // the decode-GEMM scan over coset records with a per-split top-k
  const int64_t n = ix->n;
  const int64_t qtiles = (nq + uvb::kScanTQ - 1) / uvb::kScanTQ;
  const bool chunked = uvb::scan_smem_bytes(d16, 0, 0, false) > 227 * 1024;
  const bool small_k = k <= 32 || k > uvb::kScanKCap;
  const size_t smem = chunked ? uvb::chunked_scan_smem_bytes(0, false, small_k)
                              : uvb::scan_smem_bytes(d16, 0, 0, false);
  const void *scan_k =
      chunked ? uvb::chunked_scan_kernel_ptr(0, false, small_k) : uvb::coset_scan_kernel_ptr();
  UV_CK(cudaFuncSetAttribute(scan_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  UV_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_k, 256, smem));
  const int64_t slots = (int64_t)sm_count(dev) * std::max(per_sm, 1);
  const int64_t max_splits =
      std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(2048 / k, 32), n / 1024));
  int64_t splits = 1;
  double best_eff = 0.0;
  for (int64_t s = 1; s <= max_splits; s++) {
    const int64_t ctas = qtiles * s;
    const int64_t waves = (ctas + slots - 1) / slots;
    const double eff = (double)ctas / (double)(waves * slots);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      splits = s;
    }
    if (eff >= 0.9) break;
  }
  uvb::ScanParams sp;
  std::memset(&sp, 0, sizeof(sp));
  sp.dim = d16;
  sp.mem = ix->mem;
  sp.bits = 0;
  sp.nq = nq;
  sp.n = n;
  sp.q_r = q_r;
  sp.q_stride = d16;
  sp.qc = qc;
  sp.n_centroids = ix->n_centroids;
  sp.degenerate = degen;
  sp.codes = ix->codes;
  sp.code_stride = ix->m.code_stride;
  sp.rescale = ix->rescale;
  sp.rnorm = ix->rnorm;
  sp.cidx = ix->cidx;
  sp.k = k;
  sp.ids = ix->ids;
  sp.coset = ix->m;
  if (k > uvb::kScanKCap) {
    // any k: every score, sorted per query (the reference sorts all, then
    // truncates, src/coset_trellis.rs:471-497)
    UV_TRY(rank_all_scores(sp, scan_k, smem, nq, k, d_ids, d_scores, dev, st, sc));
    return outs.finish(st);
  }
  uint32_t *part_key = nullptr;
  int64_t *part_id = nullptr;
  UV_TRY(sc.alloc(&part_key, (size_t)nq * splits * k));
  UV_TRY(sc.alloc(&part_id, (size_t)nq * splits * k));
  if (n == 0) {
    UV_CK(cudaMemsetAsync(part_key, 0, sizeof(uint32_t) * nq * splits * k, st));
    UV_CK(cudaMemsetAsync(part_id, 0xff, sizeof(int64_t) * nq * splits * k, st));
  } else {
    sp.part_key = part_key;
    sp.part_id = part_id;
    uvb::ScanWork work;
    std::memset(&work, 0, sizeof(work));
    void *args[] = {&sp, &work};
    ProfScope ps("coset_scan", st);
    UV_CK(cudaLaunchKernel(scan_k, dim3((unsigned)qtiles, (unsigned)splits), dim3(256), args,
                           smem, st));
  }
  UV_TRY(merge_launch(nq, (int)splits, k, k, part_key, nullptr, part_id, d_ids, d_scores, st));
  return outs.finish(st);
}

// The records as the reference stores them: n x code_len bytes (start state
// then packed symbols), rescale, rnorm, cidx, ids.  Any output may be null.
int uv_coset_export(const uv_coset *ix, uint8_t *codes, float *rescale, float *rnorm,
                    uint32_t *cidx, int64_t *ids, void *stream) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  const int64_t n = ix->n;
  if (n == 0) return UV_OK;
  DeviceGuard g(ix->device);
  cudaStream_t st = (cudaStream_t)stream;
  if (codes)
    UV_CK(cudaMemcpy2DAsync(codes, ix->m.code_len, ix->codes, ix->m.code_stride, ix->m.code_len,
                            n, cudaMemcpyDefault, st));
  if (rescale) UV_CK(cudaMemcpyAsync(rescale, ix->rescale, 4 * n, cudaMemcpyDefault, st));
  if (rnorm) UV_CK(cudaMemcpyAsync(rnorm, ix->rnorm, 4 * n, cudaMemcpyDefault, st));
  if (cidx) UV_CK(cudaMemcpyAsync(cidx, ix->cidx, 4 * n, cudaMemcpyDefault, st));
  if (ids) UV_CK(cudaMemcpyAsync(ids, ix->ids, 8 * n, cudaMemcpyDefault, st));
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

// reconstruct_unit (src/coset_trellis.rs:521-529) of n rows: encode, decode,
// rotate back, normalize.  n x dim in and out, host or device memory.
int uv_coset_reconstruct(const uv_coset *ix, const float *rows, int64_t n, float *out,
                         void *stream) {
  if (ix == nullptr || (n > 0 && (rows == nullptr || out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  const int d = ix->dim, dev = ix->device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_rows = nullptr;
  float *d_out = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * d, dev, sc, &d_rows));
  UV_TRY(outs.stage(out, (size_t)n * d, dev, sc, &d_out));
  uint8_t *codes = nullptr;
  float *rs = nullptr, *rn = nullptr;
  uint32_t *ci = nullptr;
  UV_TRY(sc.alloc(&codes, (size_t)n * ix->m.code_stride));
  UV_TRY(sc.alloc(&rs, (size_t)n));
  UV_TRY(sc.alloc(&rn, (size_t)n));
  UV_TRY(sc.alloc(&ci, (size_t)n));
  UV_TRY(coset_encode(ix, d_rows, n, codes, rs, rn, ci, st, sc));
  uvb::CosetEncParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = ix->m;
  p.n = n;
  p.rot = ix->rot;
  p.codes = codes;
  p.recon = d_out;
  const size_t smem = (size_t)8 * (d + 8) * 4;
  UV_CK(cudaFuncSetAttribute(uvb::coset_reconstruct_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void *args[] = {&p};
  const int grid = (int)std::min<int64_t>((n + 7) / 8, (int64_t)sm_count(dev) * 16);
  UV_CK(cudaLaunchKernel((const void *)uvb::coset_reconstruct_kernel, dim3(grid), dim3(256), args,
                         smem, st));
  return outs.finish(st);
}

}  // extern "C"
