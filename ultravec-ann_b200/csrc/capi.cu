// capi.cpp -- the extern "C" boundary (include/ultravec_b200.h).
//
// Owns the handles, decides where each caller buffer lives (host or device),
// stages host buffers through stream-ordered device allocations, plans and
// launches the kernels, and turns every failure into a status code plus a
// thread-local message.  No exception or abort crosses the ABI.
#include "capi_internal.h"

#include <atomic>
#include <cmath>

#include <cuda.h>

namespace uvcapi {

thread_local std::string g_err;
std::mutex g_prof_mu;
// Tuning knobs (uv_set_tuning): atomics, so that a thread that tunes while
// others search is not a data race; every search reads each knob once.
std::atomic<int64_t> g_scan_splits{0};
std::atomic<int> g_tc_mode{0};
std::atomic<int> g_cand_kernel{0};
std::atomic<int> g_tc_shape{0};
std::atomic<int> g_tc_cache{1};
std::atomic<int> g_coset_nearest{0};
std::atomic<int> g_tc_sample{0};
std::atomic<int> g_tc_prepare{0};
std::atomic<int> g_ivf_tc_probe{0};
std::atomic<int> g_ivf_tc{0};
std::atomic<int> g_rescore_warp{0};
std::atomic<int> g_tc_hot{0};
std::atomic<int64_t> g_tc_last_candidates{0};
std::atomic<int64_t> g_ivf_tc_overflow{0};
std::atomic<int64_t> g_tc_last_sample{1};  // pass-1 tile stride of the last prefilter search
std::atomic<bool> g_prof_on{false};
std::vector<ProfRec> g_prof;

cudaMemPool_t scratch_pool() {
  static std::mutex mu;
  static std::vector<cudaMemPool_t> pools;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if ((int)pools.size() <= dev) pools.resize(dev + 1, nullptr);
  if (pools[dev] == nullptr) {
    cudaMemPoolProps props;
    std::memset(&props, 0, sizeof(props));
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = ~0ull;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    pools[dev] = pool;
  }
  return pools[dev];
}

}  // namespace uvcapi

using namespace uvcapi;

extern "C" {

int uv_abi_version(void) { return UV_ABI_VERSION; }

const char *uv_last_error(void) { return g_err.c_str(); }

void uv_config_default(uv_config *cfg, int32_t dim, int32_t bits, int32_t mem) {
  if (cfg == nullptr) return;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->dim = dim;
  cfg->bits = bits;
  cfg->mem = mem;
  cfg->rotation_rounds = 3;
  cfg->rotation_seed = 42;
  cfg->start_bits = mem;
  cfg->rescale_bits = 0;
  cfg->branch_lambda = 0.0f;
  cfg->device = 0;
}

int uv_codec_create(const uv_config *cfg, uv_codec **out) {
  if (cfg == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  if (cfg->dim <= 0) return fail(UV_EINVAL, "dim must be positive");
  if (cfg->bits < 1 || cfg->bits > 4) return fail(UV_EINVAL, "bits must be 1..4");
  if (cfg->mem < 1 || cfg->mem + cfg->bits > 24)
    return fail(UV_EINVAL, "mem must be >= 1 with mem + bits <= 24");
  if (cfg->rescale_bits < 0 || cfg->rescale_bits > 24)
    return fail(UV_EINVAL, "rescale_bits must be 0..24");
  int ndev = 0;
  UV_CK(cudaGetDeviceCount(&ndev));
  if (cfg->device < 0 || cfg->device >= ndev) return fail(UV_EINVAL, "no such CUDA device");
  uv_codec *c = new (std::nothrow) uv_codec();
  if (c == nullptr) return fail(UV_ENOMEM, "host allocation failed");
  c->cfg = *cfg;
  c->cfg.start_bits = std::min(std::max(cfg->start_bits, 0), cfg->mem);
  c->cfg.rotation_rounds = std::max(cfg->rotation_rounds, 1);
  c->code_bytes = (cfg->dim * cfg->bits + 7) / 8;
  c->code_stride = (c->code_bytes + 15) & ~15;
  c->sign_bytes = (cfg->dim + 7) / 8;
  c->sign_stride = (c->sign_bytes + 15) & ~15;
  c->h_table = uvb::build_code_table(cfg->mem, cfg->bits);
  c->table_len = (int)c->h_table.size();
  for (float v : c->h_table) c->code_absmax = std::max(c->code_absmax, std::fabs(v));
  c->rot_host = uvb::build_rotation(cfg->dim, cfg->rotation_seed, c->cfg.rotation_rounds);
  if ((int)c->rot_host.blk_off.size() > uvb::kMaxBlocks) {
    delete c;
    return fail(UV_EUNSUPPORTED, "dimension splits into too many power-of-two blocks");
  }
  DeviceGuard g(cfg->device);
  cudaError_t e = cudaMalloc(&c->d_table, sizeof(float) * c->h_table.size());
  if (e == cudaSuccess) e = cudaMalloc(&c->d_signs, sizeof(float) * c->rot_host.signs.size());
  if (e == cudaSuccess)
    e = cudaMemcpy(c->d_table, c->h_table.data(), sizeof(float) * c->h_table.size(),
                   cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(c->d_signs, c->rot_host.signs.data(), sizeof(float) * c->rot_host.signs.size(),
                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(c->d_table);
    cudaFree(c->d_signs);
    delete c;
    return fail(UV_ECUDA, std::string("codec upload: ") + cudaGetErrorString(e));
  }
  uvb::RotParams &r = c->rot;
  std::memset(&r, 0, sizeof(r));
  r.dim = cfg->dim;
  r.rounds = c->rot_host.rounds;
  r.n_blocks = (int)c->rot_host.blk_off.size();
  for (int b = 0; b < r.n_blocks; b++) {
    r.blk_off[b] = c->rot_host.blk_off[b];
    r.blk_len[b] = c->rot_host.blk_len[b];
    r.blk_inv[b] = c->rot_host.blk_inv[b];
  }
  r.signs = c->d_signs;
  c->plan_status = uvb::encode_plan(cfg->dim, cfg->bits, cfg->mem, &c->plan, &c->plan_why);
  *out = c;
  return UV_OK;
}

int uv_codec_destroy(uv_codec *c) {
  if (c == nullptr) return UV_OK;
  {
    DeviceGuard g(c->cfg.device);
    cudaFree(c->d_table);
    cudaFree(c->d_signs);
  }
  delete c;
  return UV_OK;
}

int uv_codec_code_table_bits(const uv_codec *c, uint32_t *out, int64_t capacity) {
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  if (capacity < c->table_len) return fail(UV_EINVAL, "capacity below 2^(mem+bits)");
  std::memcpy(out, c->h_table.data(), sizeof(float) * c->table_len);
  return UV_OK;
}

int uv_codec_rotation_sign_rounds(const uv_codec *c, float *out, int64_t capacity) {
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  if (capacity < (int64_t)c->rot_host.signs.size()) return fail(UV_EINVAL, "capacity below rounds*dim");
  std::memcpy(out, c->rot_host.signs.data(), sizeof(float) * c->rot_host.signs.size());
  return UV_OK;
}

int uv_codec_memory_bits(const uv_codec *c, int32_t *mem) {
  if (c == nullptr || mem == nullptr) return fail(UV_EINVAL, "null argument");
  *mem = c->cfg.mem;
  return UV_OK;
}

int uv_codec_record_bytes(const uv_codec *c, int32_t *code_bytes, int32_t *start_bytes,
                          int32_t *rescale_bytes) {
  if (c == nullptr) return fail(UV_EINVAL, "null argument");
  if (code_bytes) *code_bytes = c->code_bytes;
  if (start_bytes) *start_bytes = (std::min(c->cfg.start_bits, c->cfg.mem) + 7) / 8;
  if (rescale_bytes) *rescale_bytes = c->cfg.rescale_bits > 0 ? (c->cfg.rescale_bits + 7) / 8 : 4;
  return UV_OK;
}

}  // extern "C"

namespace uvcapi {

// Encode rows already on the device into device outputs (codes at
// code_stride).  The common core of uv_encode, uv_encode_rotated,
// uv_index_add and the IVF build (list centroids, rows read through
// row_index in list-major order).
int encode_device(const uv_codec *c, const float *rows, int64_t n, const float *centroids,
                  int n_centroids, bool rotated, uint8_t *codes, uint32_t *start, float *rescale,
                  float *rnorm, uint32_t *cidx, float *norms, cudaStream_t st, Scratch &sc,
                  const float *list_centroids, const uint32_t *row_list,
                  const int64_t *row_index, uint8_t *signs) {
  if (c->plan_status == 1) return fail(UV_EINVAL, c->plan_why);
  if (c->plan_status != 0) return fail(UV_EUNSUPPORTED, c->plan_why);
  if (n == 0) return UV_OK;
  uvb::EncodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.dim = c->cfg.dim;
  p.n = n;
  p.rows = rows;
  p.code = c->d_table;
  p.rot = c->rot;
  p.lambda = c->cfg.branch_lambda;
  p.one2 = make_float2(1.0f, 1.0f);
  p.start_bits = c->cfg.start_bits;
  p.rescale_bits = c->cfg.rescale_bits;
  p.centroids = centroids;
  p.n_centroids = n_centroids;
  p.codes = codes;
  p.code_stride = c->code_stride;
  p.code_bytes = c->code_bytes;
  p.start = start;
  p.rescale = rescale;
  p.rnorm = rnorm;
  p.cidx = cidx;
  p.norms = norms;
  p.rotated_input = rotated ? 1 : 0;
  p.list_centroids = list_centroids;
  p.row_list = row_list;
  p.row_index = row_index;
  p.signs = signs;
  p.sign_stride = c->sign_stride;
  if (c->plan.staged > 0) {
    // batches of rows stepped through the trellis together
    const int64_t R = uvb::staged_rows_per_batch(c->plan, c->cfg.dim, n);
    size_t offs[6];
    const size_t bytes = uvb::staged_scratch_bytes(c->plan, c->cfg.dim, R, offs);
    uint8_t *scratch = nullptr;
    UV_TRY(sc.alloc(&scratch, bytes));
    ProfScope ps("encode", st);
    for (int64_t row0 = 0; row0 < n; row0 += R)
      UV_CK(uvb::encode_staged_launch(c->plan, p, row0, std::min(R, n - row0), scratch, offs, st));
    return UV_OK;
  }
  int grid = 0;
  UV_CK(uvb::encode_grid(c->plan, n, &grid));
  if (!c->plan.back_smem) {
    // one back-pointer slot per team (per cluster for the cluster encoder)
    const size_t teams = c->plan.cluster > 0 ? (size_t)(grid / c->plan.cluster)
                                             : (size_t)grid * c->plan.teams_per_cta;
    const size_t words = teams * (size_t)c->plan.back_words_team;
    UV_TRY(sc.alloc(&p.back_global, words));
  }
  {
    ProfScope ps("encode", st);
    UV_CK(uvb::encode_launch(c->plan, p, grid, st));
  }
  UV_CK(cudaGetLastError());
  return UV_OK;
}

}  // namespace uvcapi

extern "C" {

static int encode_common(const uv_codec *c, const float *rows, int64_t n, const float *centroids,
                         int32_t n_centroids, bool rotated, uint8_t *codes, uint32_t *start,
                         float *rescale, float *rnorm, uint32_t *cidx, void *stream) {
  if (c == nullptr || (rows == nullptr && n > 0)) return fail(UV_EINVAL, "null argument");
  if (n < 0 || n_centroids < 0) return fail(UV_EINVAL, "negative size");
  if (n_centroids > 0 && centroids == nullptr) return fail(UV_EINVAL, "null centroids");
  if (n == 0) return UV_OK;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const int dev = c->cfg.device;
  const int d = c->cfg.dim;
  const float *d_rows = nullptr, *d_cen = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * d, dev, sc, &d_rows));
  UV_TRY(stage_in(centroids, (size_t)n_centroids * d, dev, sc, &d_cen));
  uint32_t *d_start = nullptr, *d_cidx = nullptr;
  float *d_rescale = nullptr, *d_rnorm = nullptr;
  UV_TRY(outs.stage(start, (size_t)n, dev, sc, &d_start));
  if (!rotated) {
    UV_TRY(outs.stage(rescale, (size_t)n, dev, sc, &d_rescale));
    UV_TRY(outs.stage(rnorm, (size_t)n, dev, sc, &d_rnorm));
    UV_TRY(outs.stage(cidx, (size_t)n, dev, sc, &d_cidx));
  }
  // codes: written at the padded stride, then compacted into the caller's
  // dense layout unless the two coincide on the device.
  bool codes_dev = false;
  UV_TRY(classify(codes, dev, &codes_dev));
  uint8_t *d_codes = nullptr;
  const bool direct = codes_dev && c->code_stride == c->code_bytes;
  if (direct) {
    d_codes = codes;
  } else if (codes != nullptr) {
    UV_TRY(sc.alloc(&d_codes, (size_t)n * c->code_stride));
  }
  UV_TRY(encode_device(c, d_rows, n, d_cen, n_centroids, rotated, d_codes, d_start, d_rescale,
                       d_rnorm, d_cidx, nullptr, st, sc));
  if (codes != nullptr && !direct) {
    UV_CK(cudaMemcpy2DAsync(codes, c->code_bytes, d_codes, c->code_stride, c->code_bytes, n,
                            codes_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
    if (!codes_dev) UV_CK(cudaStreamSynchronize(st));
  }
  return outs.finish(st);
}

int uv_encode(const uv_codec *c, const float *rows, int64_t n, const float *centroids,
              int32_t n_centroids, uint8_t *codes, uint32_t *start, float *rescale, float *rnorm,
              uint32_t *cidx, void *stream) {
  return encode_common(c, rows, n, centroids, n_centroids, false, codes, start, rescale, rnorm,
                       cidx, stream);
}

int uv_encode_rotated(const uv_codec *c, const float *u_r, int64_t n, uint8_t *codes,
                      uint32_t *start, void *stream) {
  return encode_common(c, u_r, n, nullptr, 0, true, codes, start, nullptr, nullptr, nullptr,
                       stream);
}

int uv_rotate(const uv_codec *c, const float *rows, int64_t n, float *out, void *stream) {
  if (c == nullptr || rows == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  if (n <= 0) return n == 0 ? UV_OK : fail(UV_EINVAL, "negative size");
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_rows = nullptr;
  float *d_out = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * c->cfg.dim, c->cfg.device, sc, &d_rows));
  UV_TRY(outs.stage(out, (size_t)n * c->cfg.dim, c->cfg.device, sc, &d_out));
  UV_CK(uvb::launch_rotate(d_rows, n, c->rot, d_out, st));
  return outs.finish(st);
}

int uv_windows(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
               uint32_t *out, void *stream) {
  if (c == nullptr || codes == nullptr || start == nullptr || out == nullptr)
    return fail(UV_EINVAL, "null argument");
  if (n <= 0) return n == 0 ? UV_OK : fail(UV_EINVAL, "negative size");
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const uint8_t *d_codes = nullptr;
  const uint32_t *d_start = nullptr;
  uint32_t *d_out = nullptr;
  UV_TRY(stage_in(codes, (size_t)n * c->code_bytes, c->cfg.device, sc, &d_codes));
  UV_TRY(stage_in(start, (size_t)n, c->cfg.device, sc, &d_start));
  UV_TRY(outs.stage(out, (size_t)n * c->cfg.dim, c->cfg.device, sc, &d_out));
  UV_CK(uvb::launch_windows(d_codes, c->code_bytes, c->code_bytes, d_start, n, c->cfg.dim,
                            c->cfg.mem, c->cfg.bits, d_out, st));
  return outs.finish(st);
}

int uv_decode(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
              float *out, void *stream) {
  if (c == nullptr || codes == nullptr || start == nullptr || out == nullptr)
    return fail(UV_EINVAL, "null argument");
  if (n <= 0) return n == 0 ? UV_OK : fail(UV_EINVAL, "negative size");
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const uint8_t *d_codes = nullptr;
  const uint32_t *d_start = nullptr;
  uint32_t *d_win = nullptr;
  float *d_out = nullptr;
  UV_TRY(stage_in(codes, (size_t)n * c->code_bytes, c->cfg.device, sc, &d_codes));
  UV_TRY(stage_in(start, (size_t)n, c->cfg.device, sc, &d_start));
  UV_TRY(sc.alloc(&d_win, (size_t)n * c->cfg.dim));
  UV_TRY(outs.stage(out, (size_t)n * c->cfg.dim, c->cfg.device, sc, &d_out));
  UV_CK(uvb::launch_windows(d_codes, c->code_bytes, c->code_bytes, d_start, n, c->cfg.dim,
                            c->cfg.mem, c->cfg.bits, d_win, st));
  UV_CK(uvb::launch_decode(d_win, c->d_table, n, c->rot, d_out, st));
  return outs.finish(st);
}

int uv_digest(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
              uint64_t *digest, void *stream) {
  if (c == nullptr || digest == nullptr || (n > 0 && (codes == nullptr || start == nullptr)))
    return fail(UV_EINVAL, "null argument");
  *digest = 0;
  if (n <= 0) return n == 0 ? UV_OK : fail(UV_EINVAL, "negative size");
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  const uint8_t *d_codes = nullptr;
  const uint32_t *d_start = nullptr;
  unsigned long long *d_acc = nullptr;
  UV_TRY(stage_in(codes, (size_t)n * c->code_bytes, c->cfg.device, sc, &d_codes));
  UV_TRY(stage_in(start, (size_t)n, c->cfg.device, sc, &d_start));
  UV_TRY(sc.alloc(&d_acc, 1));
  UV_CK(cudaMemsetAsync(d_acc, 0, sizeof(unsigned long long), st));
  UV_CK(uvb::launch_digest(d_codes, c->code_bytes, c->code_bytes, d_start, n, d_acc, st));
  unsigned long long h = 0;
  UV_CK(cudaMemcpyAsync(&h, d_acc, sizeof(h), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  *digest = h;
  return UV_OK;
}

// ---------------------------------------------------------------------------
// flat index
// ---------------------------------------------------------------------------

int uv_index_create(const uv_codec *c, uv_index **out) {
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  uv_index *ix = new (std::nothrow) uv_index();
  if (ix == nullptr) return fail(UV_ENOMEM, "host allocation failed");
  ix->codec = c;
  ix->device = c->cfg.device;
  *out = ix;
  return UV_OK;
}

int uv_index_destroy(uv_index *ix) {
  if (ix == nullptr) return UV_OK;
  {
    DeviceGuard g(ix->device);
    cudaDeviceSynchronize();
    cudaFree(ix->codes);
    cudaFree(ix->start);
    cudaFree(ix->rescale);
    cudaFree(ix->rnorm);
    cudaFree(ix->norms);
    cudaFree(ix->cidx);
    cudaFree(ix->ids);
    cudaFree(ix->centroids);
    cudaFree(ix->signs);
    for (auto &t : ix->tc_rows) {
      cudaFree(t.x16);
      cudaFree(t.xext);
      cudaFree(t.cmax);
      if (t.ready != nullptr) cudaEventDestroy(t.ready);
    }
  }
  delete ix;
  return UV_OK;
}

int uv_index_set_centroids(uv_index *ix, const float *centroids, int32_t n_centroids) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  if (n_centroids < 0 || (n_centroids > 0 && centroids == nullptr))
    return fail(UV_EINVAL, "bad centroids");
  if (ix->n > 0) return fail(UV_EINVAL, "centroids must be set before the first add");
  ix->version++;
  DeviceGuard g(ix->codec->cfg.device);
  cudaFree(ix->centroids);
  ix->centroids = nullptr;
  ix->n_centroids = 0;
  if (n_centroids == 0) return UV_OK;
  const size_t bytes = sizeof(float) * (size_t)n_centroids * ix->codec->cfg.dim;
  UV_CK(cudaMalloc(&ix->centroids, bytes));
  UV_CK(cudaMemcpy(ix->centroids, centroids, bytes, cudaMemcpyDefault));
  ix->n_centroids = n_centroids;
  return UV_OK;
}

static int index_ensure(uv_index *ix, int64_t need, cudaStream_t st) {
  if (need <= ix->cap) return UV_OK;
  int64_t cap = std::max<int64_t>(need, ix->cap * 2);
  const uv_codec *c = ix->codec;
  UV_TRY(grow(&ix->codes, ix->n * c->code_stride, cap * c->code_stride, st));
  UV_TRY(grow(&ix->start, ix->n, cap, st));
  UV_TRY(grow(&ix->rescale, ix->n, cap, st));
  UV_TRY(grow(&ix->rnorm, ix->n, cap, st));
  UV_TRY(grow(&ix->norms, ix->n, cap, st));
  UV_TRY(grow(&ix->cidx, ix->n, cap, st));
  UV_TRY(grow(&ix->ids, ix->n, cap, st));
  if (ix->sl_c > 0) UV_TRY(grow(&ix->signs, ix->n * c->sign_stride, cap * c->sign_stride, st));
  ix->cap = cap;
  return UV_OK;
}

// with_shortlist(c) / with_shortlist_asym / with_shortlist_rnorm
// (src/trellis.rs:803-839): sign codes are written as records are added, so
// the shortlist is switched on while the index is empty.
int uv_index_set_shortlist(uv_index *ix, int32_t c, int32_t asym, int32_t rnorm) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  if (c < 0 || (asym != 0 && asym != 1) || (rnorm != 0 && rnorm != 1))
    return fail(UV_EINVAL, "shortlist: c >= 0, asym and rnorm 0 or 1");
  if (ix->n > 0 && (c > 0) != (ix->sl_c > 0))
    return fail(UV_EINVAL, "shortlist: switch it on or off while the index is empty");
  DeviceGuard g(ix->codec->cfg.device);
  if (c > 0 && ix->signs == nullptr && ix->cap > 0)
    UV_CK(cudaMalloc(&ix->signs, (size_t)ix->cap * ix->codec->sign_stride));
  if (c == 0 && ix->signs != nullptr) {
    UV_CK(cudaDeviceSynchronize());
    cudaFree(ix->signs);
    ix->signs = nullptr;
  }
  ix->sl_c = c;
  ix->sl_asym = asym;
  ix->sl_weight = rnorm;
  return UV_OK;
}

int uv_index_clear(uv_index *ix) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  ix->n = 0;
  ix->version++;
  return UV_OK;
}

int uv_index_reserve(uv_index *ix, int64_t additional) {
  if (ix == nullptr || additional < 0) return fail(UV_EINVAL, "bad argument");
  DeviceGuard g(ix->codec->cfg.device);
  UV_TRY(index_ensure(ix, ix->n + additional, 0));
  UV_CK(cudaStreamSynchronize(0));
  return UV_OK;
}

namespace {
__global__ void iota_ids(int64_t *ids, int64_t n) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) ids[i] = i;
}
}  // namespace

static int index_add_impl(uv_index *ix, const int64_t *ids, const float *rows, int64_t n,
                          void *stream) {
  if (ix == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  const float *d_rows = nullptr;
  UV_TRY(stage_in(rows, (size_t)n * c->cfg.dim, c->cfg.device, sc, &d_rows));
  UV_TRY(index_ensure(ix, ix->n + n, st));
  const int64_t o = ix->n;
  if (ids != nullptr) {
    UV_CK(cudaMemcpyAsync(ix->ids + o, ids, sizeof(int64_t) * n, cudaMemcpyDefault, st));
  } else {
    iota_ids<<<(int)((n + 255) / 256), 256, 0, st>>>(ix->ids + o, n);
    UV_CK(cudaGetLastError());
  }
  UV_TRY(encode_device(c, d_rows, n, ix->centroids, ix->n_centroids, false,
                       ix->codes + o * c->code_stride, ix->start + o, ix->rescale + o,
                       ix->rnorm + o, ix->cidx + o, ix->norms + o, st, sc, nullptr, nullptr,
                       nullptr, ix->sl_c > 0 ? ix->signs + o * c->sign_stride : nullptr));
  ix->n += n;
  ix->version++;
  bool rows_dev = false;
  classify(rows, c->cfg.device, &rows_dev);
  if (!rows_dev) UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

int uv_index_add(uv_index *ix, const int64_t *ids, const float *rows, int64_t n, void *stream) {
  if (ids == nullptr && n > 0) return fail(UV_EINVAL, "null ids");
  return index_add_impl(ix, ids, rows, n, stream);
}

int uv_index_add_batch(uv_index *ix, const float *rows, int64_t n, void *stream) {
  return index_add_impl(ix, nullptr, rows, n, stream);
}

int uv_index_len(const uv_index *ix, int64_t *len) {
  if (ix == nullptr || len == nullptr) return fail(UV_EINVAL, "null argument");
  *len = ix->n;
  return UV_OK;
}

int uv_index_dimensions(const uv_index *ix, int32_t *dim) {
  if (ix == nullptr || dim == nullptr) return fail(UV_EINVAL, "null argument");
  *dim = ix->codec->cfg.dim;
  return UV_OK;
}

// mem_bytes (src/trellis.rs:2184-2201): codes + rescale + start (+ the
// centering bytes of src/lib.rs:229-237) per record.
int uv_index_mem_bytes(const uv_index *ix, int64_t *bytes) {
  if (ix == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  int32_t cb = 0, sb = 0, rb = 0;
  uv_codec_record_bytes(ix->codec, &cb, &sb, &rb);
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
  // + the sign code when the shortlist is on (src/trellis.rs:2196)
  const int64_t sign = ix->sl_c > 0 ? ix->codec->sign_bytes : 0;
  *bytes = ix->n * (int64_t)(cb + sb + rb + center + sign);
  return UV_OK;
}

// The shortlist's sign codes, n x ceil(dim/8) (host or device).
int uv_index_export_signs(const uv_index *ix, uint8_t *signs, void *stream) {
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

int uv_index_export(const uv_index *ix, uint8_t *codes, uint32_t *start, float *rescale,
                    float *rnorm, float *norms, int64_t *ids, void *stream) {
  if (ix == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = ix->n;
  if (n == 0) return UV_OK;
  if (codes)
    UV_CK(cudaMemcpy2DAsync(codes, c->code_bytes, ix->codes, c->code_stride, c->code_bytes, n,
                            cudaMemcpyDefault, st));
  if (start) UV_CK(cudaMemcpyAsync(start, ix->start, 4 * n, cudaMemcpyDefault, st));
  if (rescale) UV_CK(cudaMemcpyAsync(rescale, ix->rescale, 4 * n, cudaMemcpyDefault, st));
  if (rnorm) UV_CK(cudaMemcpyAsync(rnorm, ix->rnorm, 4 * n, cudaMemcpyDefault, st));
  if (norms) UV_CK(cudaMemcpyAsync(norms, ix->norms, 4 * n, cudaMemcpyDefault, st));
  if (ids) UV_CK(cudaMemcpyAsync(ids, ix->ids, 8 * n, cudaMemcpyDefault, st));
  UV_CK(cudaStreamSynchronize(st));
  return UV_OK;
}

int uv_index_digest(const uv_index *ix, uint64_t *digest, void *stream) {
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
  UV_CK(cudaMemcpyAsync(&h, d_acc, sizeof(h), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  *digest = h;
  return UV_OK;
}

}  // extern "C"

namespace uvcapi {

int merge_launch(int64_t nq, int n_lists, int k_in, int k, const uint32_t *in_key,
                 const float *in_score, const int64_t *in_id, int64_t *out_id, float *out_score,
                 cudaStream_t st, const int64_t *row_off, const int32_t *out_row) {
  uvb::MergeParams m;
  std::memset(&m, 0, sizeof(m));
  m.nq = nq;
  m.n_lists = n_lists;
  m.row_off = row_off;
  m.out_row = out_row;
  m.k_in = k_in;
  m.k = k;
  int pow2 = 32;
  while (pow2 < n_lists * k_in) pow2 <<= 1;
  if (pow2 > 8192) return fail(UV_EUNSUPPORTED, "merge of more than 8192 candidates per query");
  m.pow2 = pow2;
  const size_t per_warp = (size_t)pow2 * 12;  // id + key per entry
  m.warps = (int)std::max<size_t>(1, std::min<size_t>(8, (96 * 1024) / per_warp));
  m.in_key = in_key;
  m.in_score = in_score;
  m.in_id = in_id;
  m.out_id = out_id;
  m.out_score = out_score;
  const size_t smem = per_warp * m.warps;
  UV_CK(cudaFuncSetAttribute(uvb::merge_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem));
  const int grid = (int)((nq + m.warps - 1) / m.warps);
  void *args[] = {&m};
  ProfScope ps("merge_topk", st);
  UV_CK(cudaLaunchKernel((const void *)uvb::merge_topk_kernel, dim3(grid), dim3(32 * m.warps), args,
                         smem, st));
  return UV_OK;
}

int sm_count(int dev) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return sms;
}

// Normalize and rotate the queries (trellis.rs:2120-2183): q_r (rotated
// unit), qc (dots with the flat centroids), degenerate flags, and optionally
// the unrotated unit query u.  All buffers have rows of dim rounded up to 4.
int prep_launch(const uv_codec *c, const float *d_q, int64_t nq, const float *centroids,
                int n_centroids, float *q_r, float *qc, uint32_t *degen, float *u,
                cudaStream_t st) {
  const int d = c->cfg.dim;
  const int dim_pad = (d + 3) & ~3;
  uvb::PrepParams pp;
  std::memset(&pp, 0, sizeof(pp));
  pp.dim = d;
  pp.dim_pad = dim_pad;
  pp.nq = nq;
  pp.queries = d_q;
  pp.rot = c->rot;
  pp.centroids = centroids;
  pp.n_centroids = n_centroids;
  pp.q_r = q_r;
  pp.qc = qc;
  pp.degenerate = degen;
  pp.u = u;
  pp.teams = uvb::prep_teams(d);
  const size_t smem = (size_t)(dim_pad + 4) * 4 * pp.teams;
  UV_CK(cudaFuncSetAttribute(uvb::prep_queries_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem));
  const int grid = (int)std::max<int64_t>(
      1, std::min<int64_t>((nq + pp.teams - 1) / pp.teams, INT32_MAX));
  void *args[] = {&pp};
  ProfScope ps("prep_queries", st);
  UV_CK(cudaLaunchKernel((const void *)uvb::prep_queries_kernel, dim3(grid), dim3(256), args, smem,
                         st));
  return UV_OK;
}

}  // namespace uvcapi

namespace {

// The exact CUDA-core scan over prepared queries (flat_scan_kernel, or the
// K-chunked kernel for wide rows) with a per-split top-k, then the merge.
// The scan kernels' view of an index: rows of any width run as width d16
// (rounded up to 16) with the real width in dim_data (the decode-GEMM over
// the 16- and 8-wide blocks, then the reference's scalar tail).
void fill_scan_params(const uv_index *ix, const float *q_r, const float *qc,
                      const uint32_t *degen, int64_t nq, int k, int mode, int img_words,
                      bool table_smem, uvb::ScanParams *out) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int d16 = (d + 15) & ~15;
  uvb::ScanParams &sp = *out;
  std::memset(&sp, 0, sizeof(sp));
  sp.dim = d16;
  sp.dim_data = d16 != d ? d : 0;
  sp.mem = c->cfg.mem;
  sp.bits = c->cfg.bits;
  sp.nq = nq;
  sp.n = ix->n;
  sp.q_r = q_r;
  sp.q_stride = (d + 3) & ~3;
  sp.qc = qc;
  sp.n_centroids = ix->n_centroids;
  sp.degenerate = degen;
  sp.codes = ix->codes;
  sp.code_stride = c->code_stride;
  sp.start = ix->start;
  sp.rescale = ix->rescale;
  sp.rnorm = ix->rnorm;
  sp.norms = ix->norms;
  sp.cidx = ix->cidx;
  sp.code = c->d_table;
  sp.table_len = c->table_len;
  sp.table_in_smem = table_smem ? 1 : 0;
  sp.img_words = img_words;
  sp.mips = mode == UV_SEARCH_MIPS ? 1 : 0;
  sp.k = k;
  sp.ids = ix->ids;
  sp.id_base = 0;
}

int exact_scan(const uv_index *ix, const float *q_r, const float *qc, const uint32_t *degen,
               int64_t nq, int k, int mode, int64_t *d_ids, float *d_scores, cudaStream_t st,
               Scratch &sc) {
  const uv_codec *c = ix->codec;
  const int d = (c->cfg.dim + 15) & ~15;  // kernel width (fill_scan_params)
  const int dev = c->cfg.device;
  const int64_t n = ix->n;
  int64_t qtiles = (nq + uvb::kScanTQ - 1) / uvb::kScanTQ;
  const int rw = c->code_stride / 4;
  int img_words = 4 + rw + 3;
  if ((img_words & 1) == 0) img_words++;
  const bool table_smem = (size_t)c->table_len * 4 <= 16 * 1024;
  // rows up to 384 keep the whole query tile resident; wider rows stream it in
  // 128-coordinate chunks (chunked_scan_kernel)
  const bool chunked = uvb::scan_smem_bytes(d, img_words, c->table_len, table_smem) > 227 * 1024;
  const bool small_k = k <= 32;
  const size_t smem = chunked ? uvb::chunked_scan_smem_bytes(c->table_len, table_smem, small_k)
                              : uvb::scan_smem_bytes(d, img_words, c->table_len, table_smem);
  const void *scan_k = chunked ? uvb::chunked_scan_kernel_ptr(c->cfg.bits, table_smem, small_k)
                               : uvb::flat_scan_kernel_ptr(c->cfg.bits, table_smem);
  UV_CK(cudaFuncSetAttribute(scan_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  UV_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_k, 256, smem));
  per_sm = std::max(per_sm, 1);
  const int64_t slots = (int64_t)sm_count(dev) * per_sm;
  // Split each query tile's records so that the grid fills whole waves: the
  // smallest split count whose last wave is at least 90% full, else the best.
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
  const int64_t fixed_splits = g_scan_splits.load();
  if (fixed_splits > 0) splits = std::min<int64_t>(fixed_splits, std::max<int64_t>(1, n));
  uint32_t *part_key = nullptr;
  int64_t *part_id = nullptr;
  UV_TRY(sc.alloc(&part_key, (size_t)nq * splits * k));
  UV_TRY(sc.alloc(&part_id, (size_t)nq * splits * k));
  if (n == 0) {
    UV_CK(cudaMemsetAsync(part_key, 0, sizeof(uint32_t) * nq * splits * k, st));
    UV_CK(cudaMemsetAsync(part_id, 0xff, sizeof(int64_t) * nq * splits * k, st));
  } else {
    uvb::ScanParams sp;
    fill_scan_params(ix, q_r, qc, degen, nq, k, mode, img_words, table_smem, &sp);
    sp.part_key = part_key;
    sp.part_id = part_id;
    uvb::ScanWork work;
    std::memset(&work, 0, sizeof(work));
    void *args[] = {&sp, &work};
    ProfScope ps("flat_scan", st);
    UV_CK(cudaLaunchKernel(scan_k, dim3((unsigned)qtiles, (unsigned)splits), dim3(256), args,
                           smem, st));
  }
  // 3) merge the splits
  UV_TRY(merge_launch(nq, (int)splits, k, k, part_key, nullptr, part_id, d_ids, d_scores, st));
  return UV_OK;
}

// Sort `rows` segments of n (key, id) entries (buffers a, spare b) by (key
// desc, id asc), keeping the best klim of each (rank.cu); *result is the
// buffer that holds the sorted rows.
int rank_sort_rows(uint32_t *ka, int64_t *ia, uint32_t *kb, int64_t *ib, int64_t n, int64_t rows,
                   int64_t klim, cudaStream_t st, bool *in_b) {
  *in_b = false;
  if (n <= 0 || rows <= 0) return UV_OK;
  const int span = uvb::rank_merge_span();
  const unsigned tiles = (unsigned)((n + uvb::kRankTile - 1) / uvb::kRankTile);
  const unsigned g = (unsigned)((n + span - 1) / span);
  bool flip = false;
  for (int64_t r0 = 0; r0 < rows; r0 += 65535) {
    const unsigned m = (unsigned)std::min<int64_t>(65535, rows - r0);
    uint32_t *kin = ka + r0 * n, *kout = kb + r0 * n;
    int64_t *iin = ia + r0 * n, *iout = ib + r0 * n;
    {
      ProfScope ps("rank_sort", st);
      uvb::rank_tile_sort_kernel<<<dim3(tiles, m), 256, 0, st>>>(kin, iin, n);
      UV_CK(cudaGetLastError());
    }
    flip = false;
    for (int64_t w = uvb::kRankTile; w < n; w *= 2) {
      ProfScope ps("rank_merge", st);
      uvb::rank_merge_kernel<<<dim3(g, m), 256, 0, st>>>(kin, iin, kout, iout, n, w, klim);
      UV_CK(cudaGetLastError());
      std::swap(kin, kout);
      std::swap(iin, iout);
      flip = !flip;
    }
  }
  *in_b = flip;  // the same number of passes for every row chunk
  return UV_OK;
}

// Full ranking for k above the fused top-k capacity (src/trellis.rs:2120-2183
// with any limit; the MIPS harness asks for len(), src/bench.rs:1029-1045):
// per chunk of queries, every (query, record) score from the exact scan
// kernel (ScanParams::all_key), a sort of each query's n (key, id) pairs
// (rank.cu), then its first k.  Outputs go straight into device buffers, or
// through a chunk buffer into host ones.
}  // namespace

namespace uvcapi {

// Every (query, record) score of an exact scan kernel with all_key set
// (p0 describes all nq queries; chunks of queries re-base q_r, qc and
// degenerate), each query's n keys sorted (rank_sort_rows keeps the best k
// of every run), then the best k as ids and scores ranked (score desc, id
// asc); slots past n hold -1 / -inf.  Outputs: host or device memory.
int rank_all_scores(const uvb::ScanParams &p0, const void *scan_k, size_t smem, int64_t nq,
                    int64_t k, int64_t *ids_out, float *scores_out, int dev, cudaStream_t st,
                    Scratch &sc) {
  const int64_t n = p0.n;
  bool ids_dev = false, sc_dev = false;
  UV_TRY(classify(ids_out, dev, &ids_dev));
  UV_TRY(classify(scores_out, dev, &sc_dev));
  const bool direct = ids_dev && (scores_out == nullptr || sc_dev);
  // queries per chunk: two (key, id) buffers of n entries per query (24 B
  // each) and, for host outputs, the chunk's k results (12 B each), within
  // about 1 GiB; at least one query
  const double budget = 1024.0 * 1024.0 * 1024.0;
  const double per_q = 24.0 * (double)n + (direct ? 0.0 : 12.0 * (double)k);
  int64_t qb = (int64_t)std::max(1.0, std::floor(budget / std::max(per_q, 1.0)));
  qb = std::min<int64_t>(std::min<int64_t>(qb, nq), 65535);
  uint32_t *key0 = nullptr, *key1 = nullptr;
  int64_t *id0 = nullptr, *id1 = nullptr;
  int64_t *c_ids = nullptr;
  float *c_sc = nullptr;
  if (n > 0) {
    UV_TRY(sc.alloc(&key0, (size_t)qb * n));
    UV_TRY(sc.alloc(&key1, (size_t)qb * n));
    UV_TRY(sc.alloc(&id0, (size_t)qb * n));
    UV_TRY(sc.alloc(&id1, (size_t)qb * n));
  }
  if (!direct) {
    UV_TRY(sc.alloc(&c_ids, (size_t)qb * k));
    if (scores_out != nullptr) UV_TRY(sc.alloc(&c_sc, (size_t)qb * k));
  }
  UV_CK(cudaFuncSetAttribute(scan_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  UV_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_k, 256, smem));
  const int64_t slots = (int64_t)sm_count(dev) * std::max(per_sm, 1);
  const int qc_stride = std::max(1, p0.n_centroids);
  for (int64_t q0 = 0; q0 < nq; q0 += qb) {
    const int64_t m = std::min(qb, nq - q0);
    uint32_t *kin = key0;
    int64_t *iin = id0;
    if (n > 0) {
      // every score of the chunk
      const int64_t qtiles = (m + uvb::kScanTQ - 1) / uvb::kScanTQ;
      int64_t splits = std::max<int64_t>(1, (2 * slots + qtiles - 1) / qtiles);
      splits = std::min<int64_t>(std::min<int64_t>(splits, std::max<int64_t>(1, n / 256)), 65535);
      uvb::ScanParams sp = p0;
      sp.nq = m;
      sp.k = 1;
      sp.q_r = p0.q_r + q0 * (int64_t)p0.q_stride;
      sp.qc = p0.qc + q0 * (int64_t)qc_stride;
      sp.degenerate = p0.degenerate + q0;
      sp.all_key = key0;
      sp.all_id = id0;
      sp.part_key = nullptr;
      sp.part_id = nullptr;
      uvb::ScanWork work;
      std::memset(&work, 0, sizeof(work));
      void *args[] = {&sp, &work};
      {
        ProfScope ps("flat_scan", st);
        UV_CK(cudaLaunchKernel(scan_k, dim3((unsigned)qtiles, (unsigned)splits), dim3(256), args,
                               smem, st));
      }
      // sort each query's n entries: tiles, then merge passes keeping the best k
      bool in_b = false;
      UV_TRY(rank_sort_rows(key0, id0, key1, id1, n, m, k, st, &in_b));
      if (in_b) {
        kin = key1;
        iin = id1;
      }
    }
    int64_t *o_ids = direct ? ids_out + q0 * k : c_ids;
    float *o_sc = direct ? (scores_out ? scores_out + q0 * k : nullptr) : c_sc;
    {
      ProfScope ps("rank_emit", st);
      const int64_t total = m * k;
      const unsigned g = (unsigned)std::min<int64_t>((total + 255) / 256, slots * 8);
      uvb::rank_emit_kernel<<<std::max(g, 1u), 256, 0, st>>>(kin, iin, n, m, k,
                                                            p0.degenerate + q0, o_ids, o_sc);
      UV_CK(cudaGetLastError());
    }
    if (!direct) {
      UV_CK(cudaMemcpyAsync(ids_out + q0 * k, c_ids, sizeof(int64_t) * m * k,
                            ids_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
      if (scores_out != nullptr)
        UV_CK(cudaMemcpyAsync(scores_out + q0 * k, c_sc, sizeof(float) * m * k,
                              sc_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st));
      UV_CK(cudaStreamSynchronize(st));  // the chunk buffers are reused
    }
  }
  return UV_OK;
}

}  // namespace uvcapi

namespace {

int full_rank_search(const uv_index *ix, const float *q_r, const float *qc,
                     const uint32_t *degen, int64_t nq, int64_t k, int mode, int64_t *ids_out,
                     float *scores_out, cudaStream_t st, Scratch &sc) {
  const uv_codec *c = ix->codec;
  const int d = (c->cfg.dim + 15) & ~15;
  const int dev = c->cfg.device;
  const int rw = c->code_stride / 4;
  int img_words = 4 + rw + 3;
  if ((img_words & 1) == 0) img_words++;
  const bool table_smem = (size_t)c->table_len * 4 <= 16 * 1024;
  const bool chunked = uvb::scan_smem_bytes(d, img_words, c->table_len, table_smem) > 227 * 1024;
  const size_t smem = chunked ? uvb::chunked_scan_smem_bytes(c->table_len, table_smem, true)
                              : uvb::scan_smem_bytes(d, img_words, c->table_len, table_smem);
  const void *scan_k = chunked ? uvb::chunked_scan_kernel_ptr(c->cfg.bits, table_smem, true)
                               : uvb::flat_scan_kernel_ptr(c->cfg.bits, table_smem);
  if (scan_k == nullptr) return fail(UV_EUNSUPPORTED, "no scan kernel for these bits");
  uvb::ScanParams sp;
  fill_scan_params(ix, q_r, qc, degen, nq, 1, mode, img_words, table_smem, &sp);
  return rank_all_scores(sp, scan_k, smem, nq, k, ids_out, scores_out, dev, st, sc);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tiled_fn(EncodeTiledFn *out) {
  static std::mutex mu;
  static EncodeTiledFn fn = nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (fn == nullptr) {
    void *pfn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &pfn, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || pfn == nullptr) {
      cudaGetLastError();
      return fail(UV_ECUDA, "cuTensorMapEncodeTiled is not available");
    }
    fn = (EncodeTiledFn)pfn;
  }
  *out = fn;
  return UV_OK;
}

// Tensor-core prefilter + exact rescoring (tcscan.cu).  Sets *used = false
// when the configuration is outside what the kernels are built for.
// The k-th largest of each query's n_tiles values (one list: q * n_tiles + i;
// several lists gathered shard-major): one warp per query with the values
// in registers up to 2048 of them, else one CTA per query with a radix
// select.
int theta_launch(const float *vals, int64_t n_tiles, int64_t nq, int k, float *theta, int lists,
                 cudaStream_t st) {
  const void *wk = uvb::tc_theta_warp_kernel_ptr(n_tiles);
  if (wk != nullptr) {
    void *args[] = {&vals, &n_tiles, &nq, &k, &theta, &lists};
    UV_CK(cudaLaunchKernel(wk, dim3((unsigned)((nq + 7) / 8)), dim3(256), args, 0, st));
    return UV_OK;
  }
  const size_t tsm = n_tiles <= uvb::kThetaSmemKeys ? (size_t)n_tiles * 4 : 0;
  if (tsm > 48 * 1024)
    UV_CK(cudaFuncSetAttribute(uvb::tc_theta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)tsm));
  uvb::tc_theta_kernel<<<(unsigned)nq, 256, tsm, st>>>(vals, n_tiles, nq, k, theta, lists);
  UV_CK(cudaGetLastError());
  return UV_OK;
}

// The prefilter in two phases, so that shards of one base can exchange their
// first-pass bounds in between (uv_index_search_begin / uv_search_finish):
// tc_begin runs pass 1 and the local threshold, tc_finish pass 2, the exact
// rescoring and the fallback for overflowed queries.
struct TcState {
  bool used = false;
  bool wide = false;
  const void *k2 = nullptr;
  dim3 grid;
  size_t smem = 0;
  int threads = 0;
  int kchunks = 0;
  uvb::TcScanParams tp;
  alignas(64) CUtensorMap tmap_main;
  alignas(64) CUtensorMap tmap_ext;
  alignas(64) CUtensorMap tmap_a;
  alignas(64) CUtensorMap tmap_ax_hi;
  int cap = 0, regions = 0, region_cap = 0;
  int64_t cand_stride = 0, S = 1, n_groups1 = 0;
  float *tmax = nullptr, *theta = nullptr;
  uint32_t *cand = nullptr;
  int *flags = nullptr;
  int32_t *over_list = nullptr;
};

int tc_begin(const uv_index *ix, const float *q_r, const uint32_t *degen, int64_t nq, int k,
             int mode, int n_shards, cudaStream_t st, Scratch &sc, TcState *ts) {
  ts->used = false;
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int64_t n = ix->n;
  const int tc_mode = g_tc_mode.load();
  if (tc_mode == 1 || ix->n_centroids != 0) return UV_OK;
  // d = 128: tcscan.cu (the query tile resident for the CTA's life); any
  // other width up to 4096: tcwide.cu (queries and records streamed in K
  // chunks of 64)
  const bool wide = d != uvb::tc_dim();
  if (wide && (d % 16 != 0 || d > 4096)) return UV_OK;
  const int kpad = (d + 63) / 64 * 64;
  const int shape = g_tc_shape == 1 ? 1 : 3;  // CTA shape (tcscan.cu)
  const int TN = uvb::tc_tile_records(), TM = uvb::tc_tile_queries();
  const int64_t n_tiles = (n + TN - 1) / TN;
  // a useful threshold needs several bound groups per top-k slot (counted as
  // two per tile, the wide kernel's groups of half a tile), over all shards
  // whose bounds meet
  const int64_t shards = std::max(1, n_shards);
  if (2 * n_tiles * shards < (tc_mode == 2 ? (int64_t)k : 8 * (int64_t)k)) return UV_OK;
  // pass 1 bounds half tiles (both kernels); pass 2's candidate segments
  // follow the epilogue's column slices (2 per tile wide, 4 flat)
  const int gpt = wide ? 2 : uvb::tc_groups_per_tile();
  const int64_t n_groups = 2 * n_tiles;
  if (n_tiles * TN > INT32_MAX) return UV_OK;
  ts->used = true;
  ts->wide = wide;
  const int dev = c->cfg.device;
  const int dim_pad = (d + 3) & ~3;
  const int mips = mode == UV_SEARCH_MIPS ? 1 : 0;
  // fp16 operand rows with the bound constants folded in.  By default they
  // are made once per index version and score mode and kept (tuning key
  // "tc_cache").  A remake after a change of the records rewrites them in
  // place on this stream (adds do not overlap searches of the same index)
  // and records an event that later searches on any stream wait for; the
  // buffers are reallocated only when the index has outgrown them, after the
  // device has drained.
  const int64_t n_pad = n_tiles * TN;
  uint16_t *x16 = nullptr, *xext = nullptr;
  float *cmax = nullptr;
  auto make_rows = [&](uint16_t *rows16, uint16_t *rows_ext, float *rows_cmax) -> int {
    uint32_t *gmax = nullptr;
    UV_TRY(sc.alloc(&gmax, 1));
    UV_CK(cudaMemsetAsync(gmax, 0, sizeof(uint32_t), st));
    uvb::TcPrepareParams pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.mem = c->cfg.mem;
    pp.bits = c->cfg.bits;
    pp.code_stride = c->code_stride;
    pp.mips = mips;
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
    pp.rnorm = ix->rnorm;
    pp.norms = ix->norms;
    pp.gmax_bits = gmax;
    pp.x16 = rows16;
    pp.xext = rows_ext;
    void *args[] = {&pp};
    ProfScope ps("tc_prepare", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::tc_gmax_kernel, dim3((unsigned)((n + 255) / 256)),
                           dim3(256), args, 0, st));
    // widths 1, 2, 4 with a table of at most 64 KB: the shared-memory
    // table and 16-byte code reads (|x|^2 summed in f32; tuning key
    // tc_prepare 2: in f64); otherwise, or with tc_prepare 1, the generic
    // kernel
    const void *fk = uvb::tc_prepare_records_fast_ptr(c->cfg.bits, g_tc_prepare.load() != 2);
    const size_t tsm = (size_t)4 << (c->cfg.mem + c->cfg.bits);
    if (fk != nullptr && tsm <= 64 * 1024 && g_tc_prepare != 1) {
      UV_CK(cudaFuncSetAttribute(fk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsm));
      UV_CK(cudaLaunchKernel(fk, dim3((unsigned)((n_pad + 255) / 256)), dim3(256), args, tsm, st));
    } else {
      UV_CK(cudaLaunchKernel((const void *)uvb::tc_prepare_records_kernel,
                             dim3((unsigned)((n_pad + 127) / 128)), dim3(128), args, 0, st));
    }
    uvb::tc_chunk_cmax_kernel<<<(unsigned)((n_pad + 255) / 256), 256, 0, st>>>(rows_ext, n, n_pad,
                                                                               rows_cmax);
    UV_CK(cudaGetLastError());
    return UV_OK;
  };
  if (g_tc_cache.load() == 0) {
    UV_TRY(sc.alloc(&x16, (size_t)n_pad * kpad));
    UV_TRY(sc.alloc(&xext, (size_t)n_pad * 16));
    UV_TRY(sc.alloc(&cmax, (size_t)n_pad / 16));
    UV_TRY(make_rows(x16, xext, cmax));
  } else {
    std::lock_guard<std::mutex> rows_lock(ix->tc_mu);
    TcRows &rows = ix->tc_rows[mips];
    if (rows.version != ix->version || rows.n_pad != n_pad || rows.kpad != kpad) {
      rows.version = ~0ull;
      if (rows.cap < n_pad || rows.kpad != kpad) {
        if (rows.x16 != nullptr || rows.xext != nullptr || rows.cmax != nullptr) {
          UV_CK(cudaDeviceSynchronize());
          cudaFree(rows.x16);
          cudaFree(rows.xext);
          cudaFree(rows.cmax);
          rows.x16 = rows.xext = nullptr;
          rows.cmax = nullptr;
          rows.cap = 0;
        }
        UV_CK(cudaMalloc((void **)&rows.x16, sizeof(uint16_t) * (size_t)n_pad * kpad));
        UV_CK(cudaMalloc((void **)&rows.xext, sizeof(uint16_t) * (size_t)n_pad * 16));
        UV_CK(cudaMalloc((void **)&rows.cmax, sizeof(float) * (size_t)n_pad / 16));
        rows.cap = n_pad;
        rows.kpad = kpad;
      }
      UV_TRY(make_rows(rows.x16, rows.xext, rows.cmax));
      if (rows.ready == nullptr)
        UV_CK(cudaEventCreateWithFlags(&rows.ready, cudaEventDisableTiming));
      UV_CK(cudaEventRecord(rows.ready, st));
      rows.n_pad = n_pad;
      rows.version = ix->version;
    } else {
      UV_CK(cudaStreamWaitEvent(st, rows.ready, 0));
    }
    x16 = rows.x16;
    xext = rows.xext;
    cmax = rows.cmax;
  }
  TcRows *cache = g_tc_cache.load() == 0 ? nullptr : &ix->tc_rows[mips];
  // TMA maps: main rows of 128 fp16 (boxes of 64 x TN, 128-byte swizzle) and
  // the extra slice of 16 fp16 (boxes of 16 x TN, 32-byte swizzle)
  CUtensorMap &tmap_main = ts->tmap_main, &tmap_ext = ts->tmap_ext;
  {
    EncodeTiledFn enc = nullptr;
    UV_TRY(encode_tiled_fn(&enc));
    const cuuint32_t estride[2] = {1, 1};
    const cuuint64_t gdim[2] = {(cuuint64_t)kpad, (cuuint64_t)n_pad};
    const cuuint64_t gstride[1] = {(cuuint64_t)kpad * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)TN};
    CUresult r = enc(&tmap_main, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)x16, gdim, gstride,
                     box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(UV_ECUDA, "cuTensorMapEncodeTiled (main rows) failed");
    const cuuint64_t gdim_x[2] = {16, (cuuint64_t)n_pad};
    const cuuint64_t gstride_x[1] = {32};
    const cuuint32_t box_x[2] = {16, (cuuint32_t)TN};
    r = enc(&tmap_ext, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)xext, gdim_x, gstride_x, box_x,
            estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(UV_ECUDA, "cuTensorMapEncodeTiled (extra slice) failed");
  }
  // wide rows: the queries as fp16 rows too, with maps for both extra slices
  alignas(64) CUtensorMap tmap_ax_lo;
  CUtensorMap &tmap_a = ts->tmap_a, &tmap_ax_hi = ts->tmap_ax_hi;
  if (wide) {
    const int64_t nq_pad = (nq + 127) / 128 * 128;
    uint16_t *a16 = nullptr, *ax_lo = nullptr, *ax_hi = nullptr;
    UV_TRY(sc.alloc(&a16, (size_t)nq_pad * kpad));
    UV_TRY(sc.alloc(&ax_lo, (size_t)nq_pad * 16));
    UV_TRY(sc.alloc(&ax_hi, (size_t)nq_pad * 16));
    {
      ProfScope ps("tc_prepare", st);
      const int64_t chunks = nq_pad * (kpad / 8);
      uvb::tc_prepare_queries_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
          q_r, dim_pad, degen, nq, nq_pad, d, kpad, a16, ax_lo, ax_hi);
      UV_CK(cudaGetLastError());
    }
    EncodeTiledFn enc = nullptr;
    UV_TRY(encode_tiled_fn(&enc));
    const cuuint32_t estride[2] = {1, 1};
    const cuuint64_t gdim[2] = {(cuuint64_t)kpad, (cuuint64_t)nq_pad};
    const cuuint64_t gstride[1] = {(cuuint64_t)kpad * 2};
    const cuuint32_t box[2] = {64, 128};
    CUresult r = enc(&tmap_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *)a16, gdim, gstride, box,
                     estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(UV_ECUDA, "cuTensorMapEncodeTiled (query rows) failed");
    const cuuint64_t gdim_x[2] = {16, (cuuint64_t)nq_pad};
    const cuuint64_t gstride_x[1] = {32};
    const cuuint32_t box_x[2] = {16, 128};
    for (int h = 0; h < 2; h++) {
      r = enc(h == 0 ? &tmap_ax_lo : &tmap_ax_hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
              (void *)(h == 0 ? ax_lo : ax_hi), gdim_x, gstride_x, box_x, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) return fail(UV_ECUDA, "cuTensorMapEncodeTiled (query slice) failed");
    }
  }
  // units: query tiles x record splits, filling whole waves of one CTA per SM
  const size_t smem = wide ? uvb::tc_wide_smem_bytes() : uvb::tc_scan_smem_bytes(shape);
  const void *k1 = wide ? uvb::tc_wide_kernel_ptr(1) : uvb::tc_scan_kernel_ptr(1, shape);
  const void *k2 = wide ? uvb::tc_wide_kernel_ptr(2) : uvb::tc_scan_kernel_ptr(2, shape);
  UV_CK(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  UV_CK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t qtiles = (nq + TM - 1) / TM;
  const int64_t slots = sm_count(dev);
  const int64_t max_splits = std::max<int64_t>(1, std::min<int64_t>(n_tiles / 8, 64));
  int64_t splits = 1;
  double best_eff = 0.0;
  for (int64_t s2 = 1; s2 <= max_splits; s2++) {
    const int64_t ctas = qtiles * s2;
    const int64_t waves = (ctas + slots - 1) / slots;
    const double eff = (double)ctas / (double)(waves * slots) - 0.002 * (double)waves;
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      splits = s2;
    }
  }
  // Pass 1 bounds a sample of the tiles (every S-th): the k-th largest group
  // maximum of any subset of groups is still a score at least k records
  // reach, so theta stays valid, and pass 2 admits about k*S candidates
  // instead of k.  Pass 1 costs ~1/S, the candidates ~k*S: S = sqrt(1600/k)
  // balances them at the 1M x 10k bench shape (measured optimum 4 at
  // k = 100, 10 at k = 10), capped at 10 and so that k*S stays well inside
  // the candidate lists, and the sample keeps at least 8k groups.
  // The sample stride S: pass 1 costs about 1/S of pass 2; the candidates
  // grow with S.  Every S-th tile (tc_hot 1) admits about k*S candidates, so
  // S = round(sqrt(1600/k)), at most 10 and 900/k (measured optimum 4 at
  // k = 100, 10 at k = 10 on the 1M x 10k bench shape); the sample of
  // largest g keeps the candidates near k much longer (about 1.9k at S =
  // 12, k = 100), so S = round(sqrt(14400/k)), at most 24 and 2400/k
  // (measured: 12 at k = 100, 24 at k = 10).  The sample keeps at least 8k
  // groups.
  const int fixed_sample = g_tc_sample.load();
  const bool hot_default = g_tc_hot.load() != 1;
  const double s_num = hot_default ? 14400.0 : 1600.0;
  const int64_t s_cap = hot_default ? 24 : 10, s_kcap = hot_default ? 2400 : 900;
  int64_t S = fixed_sample > 0
                  ? fixed_sample
                  : std::max<int64_t>(1, std::min<int64_t>(
                                             s_cap, (int64_t)std::lround(std::sqrt(s_num / k))));
  if (fixed_sample <= 0) S = std::max<int64_t>(1, std::min<int64_t>(S, s_kcap / k));
  while (S > 1 && 2 * ((n_tiles + S - 1) / S) * shards < 8 * (int64_t)k) S--;
  // Pass 1's sample: by default the n/S records of largest g, copied into
  // their own rows (tc_hot_*_kernel); tuning key tc_hot 1: every S-th tile
  // of the full rows; N >= 2: the n/N records of largest g.
  const int hot_mode = g_tc_hot.load();
  const int64_t s_hot = hot_mode >= 2 ? hot_mode : S;
  int64_t hot_cap = ((n + s_hot - 1) / s_hot + TN - 1) / TN * TN;
  const bool hot = hot_mode != 1 && s_hot > 1 && n >= 8 * (int64_t)TN &&
                   2 * (hot_cap / TN) * shards >= 8 * (int64_t)k;
  uint16_t *x16_hot = nullptr, *xext_hot = nullptr;
  float *cmax_hot = nullptr;
  if (hot) {
    auto make_hot = [&](uint16_t *hx, uint16_t *he, float *hc) -> int {
      uvb::TcPrepareParams hp;
      std::memset(&hp, 0, sizeof(hp));
      hp.mips = mips;
      hp.kpad = kpad;
      hp.dim = d;
      hp.n = n;
      hp.rescale = ix->rescale;
      hp.rnorm = ix->rnorm;
      hp.norms = ix->norms;
      hp.x16 = x16;
      hp.xext = xext;
      // blocks of the ordered compaction: at most 4095 (their counts and the
      // total fit the one-CTA scan of 4096), spans of whole 256s
      const int64_t span = std::max<int64_t>(256, ((n + 4094) / 4095 + 255) / 256 * 256);
      const int cblocks = (int)((n + span - 1) / span);
      uint32_t *hist = nullptr, *sel = nullptr, *keys = nullptr, *offs = nullptr;
      UV_TRY(sc.alloc(&hist, 4096 + 8));
      UV_TRY(sc.alloc(&keys, (size_t)n));
      UV_TRY(sc.alloc(&offs, (size_t)cblocks + 1));
      sel = hist + 4096;
      ProfScope ps("tc_hot", st);
      const unsigned hg = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 1184));
      UV_CK(cudaMemsetAsync(hist, 0, sizeof(uint32_t) * (4096 + 8), st));
      uvb::tc_hot_keys_kernel<<<hg, 256, 0, st>>>(hp, keys, hist);
      uvb::tc_hot_pick_kernel<<<1, 256, 0, st>>>(hist, hot_cap, 0, sel);
      UV_CK(cudaMemsetAsync(hist, 0, sizeof(uint32_t) * 4096, st));
      uvb::tc_hot_hist_kernel<<<hg, 256, 0, st>>>(keys, n, sel, hist);
      uvb::tc_hot_pick_kernel<<<1, 256, 0, st>>>(hist, hot_cap, 1, sel);
      uvb::tc_hot_count_kernel<<<(unsigned)cblocks, 256, 0, st>>>(keys, n, span, sel, offs);
      // one more count slot past the last block: the scan turns it into the total
      UV_CK(cudaMemsetAsync(offs + cblocks, 0, sizeof(uint32_t), st));
      uvb::tc_hot_scan_kernel<<<1, 1024, 0, st>>>(offs, cblocks + 1);
      uvb::tc_hot_gather_kernel<<<(unsigned)cblocks, 256, 0, st>>>(hp, keys, span, sel, offs,
                                                                    hot_cap, hx, he);
      uvb::tc_hot_pad_kernel<<<(unsigned)std::min<int64_t>((hot_cap + 255) / 256, 1184), 256, 0,
                               st>>>(offs + cblocks, hot_cap, kpad, hx, he);
      uvb::tc_chunk_cmax_kernel<<<(unsigned)((hot_cap + 255) / 256), 256, 0, st>>>(
          he, hot_cap, hot_cap, hc);
      UV_CK(cudaGetLastError());
      return UV_OK;
    };
    if (cache == nullptr) {
      UV_TRY(sc.alloc(&x16_hot, (size_t)hot_cap * kpad));
      UV_TRY(sc.alloc(&xext_hot, (size_t)hot_cap * 16));
      UV_TRY(sc.alloc(&cmax_hot, (size_t)hot_cap / 16));
      UV_TRY(make_hot(x16_hot, xext_hot, cmax_hot));
    } else {
      std::lock_guard<std::mutex> rows_lock(ix->tc_mu);
      TcRows &rows = *cache;
      if (rows.hot_version != ix->version || rows.hot_cap != hot_cap) {
        rows.hot_version = ~0ull;
        if (rows.hot_alloc < hot_cap) {
          if (rows.x16_hot != nullptr) {
            UV_CK(cudaDeviceSynchronize());
            cudaFree(rows.x16_hot);
            cudaFree(rows.xext_hot);
            cudaFree(rows.cmax_hot);
            rows.x16_hot = rows.xext_hot = nullptr;
            rows.cmax_hot = nullptr;
            rows.hot_alloc = 0;
          }
          UV_CK(cudaMalloc((void **)&rows.x16_hot, sizeof(uint16_t) * (size_t)hot_cap * kpad));
          UV_CK(cudaMalloc((void **)&rows.xext_hot, sizeof(uint16_t) * (size_t)hot_cap * 16));
          UV_CK(cudaMalloc((void **)&rows.cmax_hot, sizeof(float) * (size_t)hot_cap / 16));
          rows.hot_alloc = hot_cap;
        }
        UV_TRY(make_hot(rows.x16_hot, rows.xext_hot, rows.cmax_hot));
        UV_CK(cudaEventRecord(rows.ready, st));
        rows.hot_cap = hot_cap;
        rows.hot_version = ix->version;
      } else {
        UV_CK(cudaStreamWaitEvent(st, rows.ready, 0));
      }
      x16_hot = rows.x16_hot;
      xext_hot = rows.xext_hot;
      cmax_hot = rows.cmax_hot;
    }
  }
  const int64_t n_tiles1 = hot ? hot_cap / TN : (n_tiles + S - 1) / S;
  g_tc_last_sample = S;
  const int64_t n_groups1 = 2 * n_tiles1;
  float *tmax = nullptr, *theta = nullptr;
  uint32_t *cand = nullptr;
  int *cand_cnt = nullptr, *flags = nullptr;
  int32_t *over_list = nullptr;
  // Pass 2's candidate list of a query is cut into one segment per (record
  // split, bound group of a tile), each appended by a single thread; the
  // rescoring gathers at most `cap` of them.
  const int cap = 2048;
  const int regions = (int)(gpt * splits);  // <= 256: splits <= 64
  // (the same footprint for both kernels: 2 x 256 or 4 x 128 slots per split)
  const int region_cap = std::max(512 / gpt, cap / regions);
  const int64_t cand_stride = (int64_t)regions * region_cap;
  UV_TRY(sc.alloc(&tmax, (size_t)nq * n_groups1));
  UV_TRY(sc.alloc(&theta, (size_t)nq));
  UV_TRY(sc.alloc(&cand, (size_t)nq * cand_stride));
  UV_TRY(sc.alloc(&cand_cnt, (size_t)nq * regions));
  UV_TRY(sc.alloc(&flags, 4));  // [0] timeout, [1] overflowed queries, [2..3] candidates
  UV_TRY(sc.alloc(&over_list, (size_t)nq));
  UV_CK(cudaMemsetAsync(cand_cnt, 0, sizeof(int) * nq * regions, st));
  UV_CK(cudaMemsetAsync(flags, 0, sizeof(int) * 4, st));
  uvb::TcScanParams tp;
  std::memset(&tp, 0, sizeof(tp));
  tp.q_stride = dim_pad;
  tp.cand_cap = (int)cand_stride;
  tp.regions = regions;
  tp.region_cap = region_cap;
  tp.nq = nq;
  tp.n = n;
  tp.n_tiles = n_tiles;
  tp.n_groups = n_groups;
  tp.tile_stride = 1;
  tp.q_r = q_r;
  tp.degenerate = degen;
  tp.tmax = tmax;
  tp.theta = theta;
  tp.cand = cand;
  tp.cand_cnt = cand_cnt;
  tp.cmax = cmax;
  tp.err = flags;
  const dim3 grid((unsigned)qtiles, (unsigned)splits);
  int kchunks = kpad / 64;
  {
    uvb::TcScanParams tp1 = tp;
    tp1.n_tiles = n_tiles1;
    tp1.n_groups = n_groups1;
    tp1.tile_stride = hot ? 1 : S;
    alignas(64) CUtensorMap hmap_main, hmap_ext;
    if (hot) {
      // the sample: every slot a distinct record or a padding row
      tp1.n = hot_cap;
      tp1.cmax = cmax_hot;
      UV_TRY(fp16_tensor_map(&hmap_main, x16_hot, hot_cap, kpad, 64, TN, true));
      UV_TRY(fp16_tensor_map(&hmap_ext, xext_hot, hot_cap, 16, 16, TN, false));
    }
    const dim3 grid1((unsigned)qtiles,
                     (unsigned)std::max<int64_t>(1, std::min<int64_t>(splits, n_tiles1 / 8)));
    CUtensorMap *m1 = hot ? &hmap_main : &tmap_main;
    CUtensorMap *e1 = hot ? &hmap_ext : &tmap_ext;
    void *args[] = {&tp1, m1};
    void *wargs[] = {&tp1, &kchunks, &tmap_a, &tmap_ax_lo, m1, e1};
    ProfScope ps("tc_pass1", st);
    UV_CK(cudaLaunchKernel(k1, grid1, dim3(wide ? uvb::tc_wide_threads() : uvb::tc_threads()),
                           wide ? wargs : args, smem, st));
  }
  {
    ProfScope ps("tc_theta", st);
    UV_TRY(theta_launch(tmax, n_groups1, nq, k, theta, 1, st));
  }
  ts->k2 = k2;
  ts->grid = grid;
  ts->smem = smem;
  ts->threads = wide ? uvb::tc_wide_threads() : uvb::tc_threads();
  ts->kchunks = kchunks;
  ts->tp = tp;
  ts->cap = cap;
  ts->regions = regions;
  ts->region_cap = region_cap;
  ts->cand_stride = cand_stride;
  ts->S = S;
  ts->n_groups1 = n_groups1;
  ts->tmax = tmax;
  ts->theta = theta;
  ts->cand = cand;
  ts->flags = flags;
  ts->over_list = over_list;
  return UV_OK;
}

int tc_check(const uv_index *ix, const float *q_r, const float *qc, const uint32_t *degen,
             int64_t nq, int k, int mode, int64_t *d_ids, float *d_scores, cudaStream_t st,
             Scratch &sc, TcState &ts, bool *overflowed);

// Pass 2 and the exact rescoring; then (unless defer) tc_check.  With defer
// the results are final only after tc_check has run on the same stream.
int tc_finish(const uv_index *ix, const float *q_r, const float *qc, const uint32_t *degen,
              int64_t nq, int k, int mode, int64_t *d_ids, float *d_scores, cudaStream_t st,
              Scratch &sc, TcState &ts, bool defer = false) {
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dim_pad = (d + 3) & ~3;
  const int mips = mode == UV_SEARCH_MIPS ? 1 : 0;
  const int cap = ts.cap, regions = ts.regions, region_cap = ts.region_cap;
  const int64_t cand_stride = ts.cand_stride, S = ts.S;
  uint32_t *cand = ts.cand;
  int *cand_cnt = ts.tp.cand_cnt;
  int *flags = ts.flags;
  int32_t *over_list = ts.over_list;
  {
    void *args[] = {&ts.tp, &ts.tmap_main};
    void *wargs[] = {&ts.tp, &ts.kchunks, &ts.tmap_a, &ts.tmap_ax_hi, &ts.tmap_main, &ts.tmap_ext};
    ProfScope ps("tc_pass2", st);
    UV_CK(cudaLaunchKernel(ts.k2, ts.grid, dim3(ts.threads), ts.wide ? wargs : args, ts.smem,
                           st));
  }
  {
    uvb::TcRescoreParams rp;
    std::memset(&rp, 0, sizeof(rp));
    rp.dim = d;
    rp.mem = c->cfg.mem;
    rp.bits = c->cfg.bits;
    rp.code_stride = c->code_stride;
    rp.q_stride = dim_pad;
    rp.cap = cap;
    rp.k = k;
    rp.mips = mips;
    rp.table_len = c->table_len;
    rp.table_in_smem = (size_t)c->table_len * 4 <= 64 * 1024 ? 1 : 0;
    rp.nq = nq;
    rp.q_r = q_r;
    rp.degenerate = degen;
    rp.codes = ix->codes;
    rp.start = ix->start;
    rp.code = c->d_table;
    rp.rescale = ix->rescale;
    rp.rnorm = ix->rnorm;
    rp.norms = ix->norms;
    rp.cand = cand;
    rp.cand_cnt = cand_cnt;
    rp.regions = regions;
    rp.region_cap = region_cap;
    rp.cand_stride = cand_stride;
    rp.ids = ix->ids;
    rp.out_id = d_ids;
    rp.out_score = d_scores;
    rp.over_list = over_list;
    rp.n_over = flags + 1;
    rp.n_cand = (unsigned long long *)(flags + 2);
    const bool per_thread = (int64_t)k * S >= 128;
    const size_t rsmem = (size_t)cap * 12 + (size_t)((regions + 4) & ~3) * 4 + (size_t)d * 4 +
                         (rp.table_in_smem ? (size_t)c->table_len * 4 : 0) +
                         (size_t)16 * (c->code_stride / 4 + 1) * 4;
    if (rsmem > 227 * 1024) return fail(UV_EUNSUPPORTED, "prefilter rescoring exceeds shared memory");
    // queries with short lists first, one warp each; the rest one CTA each
    const size_t wsmem = uvb::tc_rescore_warp_smem_bytes(c->table_len, regions);
    const void *wk = uvb::tc_rescore_warp_kernel_ptr(c->cfg.bits);
    if (g_rescore_warp.load() == 0 && wk != nullptr && d <= uvb::kRescoreWarpDim &&
        c->table_len <= 1024 && wsmem <= 227 * 1024) {
      UV_TRY(sc.alloc(&rp.big_list, (size_t)nq));
      UV_TRY(sc.alloc(&rp.n_big, 1));
      UV_CK(cudaMemsetAsync(rp.n_big, 0, sizeof(int), st));
      UV_CK(cudaFuncSetAttribute(wk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem));
      void *wargs[] = {&rp};
      ProfScope ps("tc_rescore", st);
      UV_CK(cudaLaunchKernel(wk, dim3((unsigned)((nq + uvb::kRescoreWarps - 1) / uvb::kRescoreWarps)),
                             dim3(32 * uvb::kRescoreWarps), wargs, wsmem, st));
    }
    // long candidate lists (about k*S per query) score one candidate per
    // thread; short ones half a warp per candidate
    const void *rk = uvb::tc_rescore_kernel_ptr(c->cfg.bits, per_thread);
    UV_CK(cudaFuncSetAttribute(rk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)rsmem));
    void *args[] = {&rp};
    ProfScope ps("tc_rescore", st);
    UV_CK(cudaLaunchKernel(rk, dim3((unsigned)nq), dim3(256), args,
                           rsmem, st));
  }
  if (defer) return UV_OK;
  bool over = false;
  return tc_check(ix, q_r, qc, degen, nq, k, mode, d_ids, d_scores, st, sc, ts, &over);
}

// The prefilter's outcome (waits for the stream): a pipeline wait that
// timed out is an error; queries whose candidate list overflowed are
// scanned exactly and their results replaced in d_ids / d_scores
// (*overflowed = true).
int tc_check(const uv_index *ix, const float *q_r, const float *qc, const uint32_t *degen,
             int64_t nq, int k, int mode, int64_t *d_ids, float *d_scores, cudaStream_t st,
             Scratch &sc, TcState &ts, bool *overflowed) {
  const int dim_pad = (ix->codec->cfg.dim + 3) & ~3;
  int *flags = ts.flags;
  int32_t *over_list = ts.over_list;
  *overflowed = false;
  int h_flags[4] = {0, 0, 0, 0};
  UV_CK(cudaMemcpyAsync(h_flags, flags, sizeof(h_flags), cudaMemcpyDeviceToHost, st));
  UV_CK(cudaStreamSynchronize(st));
  {
    unsigned long long nc = 0;
    std::memcpy(&nc, h_flags + 2, sizeof(nc));
    g_tc_last_candidates = (int64_t)nc;
  }
  if (h_flags[0]) return fail(UV_ETIMEDOUT, "tensor-core scan: a pipeline wait timed out");
  if (h_flags[1] > 0) {
    // queries whose candidate list overflowed: exact scan of those rows
    *overflowed = true;
    const int64_t m = h_flags[1];
    std::vector<int32_t> rows((size_t)m);
    UV_CK(cudaMemcpyAsync(rows.data(), over_list, sizeof(int32_t) * m, cudaMemcpyDeviceToHost, st));
    UV_CK(cudaStreamSynchronize(st));
    float *sub_q = nullptr;
    uint32_t *sub_deg = nullptr;
    int64_t *sub_ids = nullptr;
    float *sub_sc = nullptr;
    UV_TRY(sc.alloc(&sub_q, (size_t)m * dim_pad));
    UV_TRY(sc.alloc(&sub_deg, (size_t)m));
    UV_TRY(sc.alloc(&sub_ids, (size_t)m * k));
    UV_TRY(sc.alloc(&sub_sc, (size_t)m * k));
    for (int64_t i = 0; i < m; i++) {
      UV_CK(cudaMemcpyAsync(sub_q + i * dim_pad, q_r + (int64_t)rows[i] * dim_pad,
                            sizeof(float) * dim_pad, cudaMemcpyDeviceToDevice, st));
      UV_CK(cudaMemcpyAsync(sub_deg + i, degen + rows[i], sizeof(uint32_t),
                            cudaMemcpyDeviceToDevice, st));
    }
    UV_TRY(exact_scan(ix, sub_q, qc, sub_deg, m, k, mode, sub_ids, sub_sc, st, sc));
    for (int64_t i = 0; i < m; i++) {
      UV_CK(cudaMemcpyAsync(d_ids + (int64_t)rows[i] * k, sub_ids + i * k, sizeof(int64_t) * k,
                            cudaMemcpyDeviceToDevice, st));
      UV_CK(cudaMemcpyAsync(d_scores + (int64_t)rows[i] * k, sub_sc + i * k, sizeof(float) * k,
                            cudaMemcpyDeviceToDevice, st));
    }
    UV_CK(cudaStreamSynchronize(st));  // `rows` is host memory of this frame
  }
  return UV_OK;
}

// Tensor-core prefilter + exact rescoring (tcscan.cu / tcwide.cu) of one
// index.  Sets *used = false when the configuration is outside what the
// kernels are built for.
int tc_search(const uv_index *ix, const float *q_r, const float *qc, const uint32_t *degen,
              int64_t nq, int k, int mode, int64_t *d_ids, float *d_scores, cudaStream_t st,
              Scratch &sc, bool *used) {
  TcState ts;
  UV_TRY(tc_begin(ix, q_r, degen, nq, k, mode, 1, st, sc, &ts));
  *used = ts.used;
  if (!ts.used) return UV_OK;
  return tc_finish(ix, q_r, qc, degen, nq, k, mode, d_ids, d_scores, st, sc, ts);
}

}  // namespace

namespace uvcapi {

// A 2D fp16 tensor map over rows x cols elements (row stride cols * 2
// bytes), boxes of box_cols x box_rows, 128-byte or 32-byte swizzle.
int fp16_tensor_map(CUtensorMap *m, const void *base, int64_t rows, int cols, int box_cols,
                    int box_rows, bool sw128) {
  EncodeTiledFn enc = nullptr;
  UV_TRY(encode_tiled_fn(&enc));
  const cuuint32_t estride[2] = {1, 1};
  const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const CUresult r =
      enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), gdim, gstride, box,
          estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
          sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(UV_ECUDA, "cuTensorMapEncodeTiled failed");
  return UV_OK;
}

}  // namespace uvcapi

extern "C" {

int uv_index_search(const uv_index *ix, const float *queries, int64_t nq, int32_t k, int32_t mode,
                    int64_t *ids_out, float *scores_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1) return fail(UV_EINVAL, "k must be at least 1");
  if (mode != UV_SEARCH_COSINE && mode != UV_SEARCH_MIPS) return fail(UV_EINVAL, "bad mode");
  if (nq == 0) return UV_OK;
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const float *d_q = nullptr;
  UV_TRY(stage_in(queries, (size_t)nq * d, dev, sc, &d_q));
  if (k > uvb::kScanKCap) {
    // every record ranked.  A cosine search with the 1-bit shortlist keeps
    // the best max(c, k) entries by sign code (src/trellis.rs:854-948); that
    // selection is built for k <= 128 only.
    if (ix->sl_c > 0 && mode == UV_SEARCH_COSINE && std::max<int64_t>(ix->sl_c, k) < ix->n)
      return fail(UV_EUNSUPPORTED, "the shortlist search is built for k <= 128");
    const int dim_pad = (d + 3) & ~3;
    float *q_r = nullptr, *qc = nullptr;
    uint32_t *degen = nullptr;
    UV_TRY(sc.alloc(&q_r, (size_t)nq * dim_pad));
    UV_TRY(sc.alloc(&qc, (size_t)nq * std::max(1, ix->n_centroids)));
    UV_TRY(sc.alloc(&degen, (size_t)nq));
    UV_TRY(prep_launch(c, d_q, nq, ix->centroids, ix->n_centroids, q_r, qc, degen, nullptr, st));
    UV_TRY(full_rank_search(ix, q_r, qc, degen, nq, k, mode, ids_out, scores_out, st, sc));
    UV_CK(cudaStreamSynchronize(st));
    return UV_OK;
  }
  int64_t *d_ids = nullptr;
  float *d_scores = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, sc, &d_scores));
  } else {
    UV_TRY(sc.alloc(&d_scores, (size_t)nq * k));
  }
  // 1) prepare queries
  const int dim_pad = (d + 3) & ~3;
  float *q_r = nullptr, *qc = nullptr;
  uint32_t *degen = nullptr;
  UV_TRY(sc.alloc(&q_r, (size_t)nq * dim_pad));
  UV_TRY(sc.alloc(&qc, (size_t)nq * std::max(1, ix->n_centroids)));
  UV_TRY(sc.alloc(&degen, (size_t)nq));
  UV_TRY(prep_launch(c, d_q, nq, ix->centroids, ix->n_centroids, q_r, qc, degen, nullptr, st));
  // the 1-bit shortlist (src/trellis.rs:2121-2123) when it prunes anything;
  // the MIPS wrapper (src/bench.rs:1029-1045) asks for every record, where
  // the shortlist keeps all of them, so MIPS is the plain scan
  if (ix->sl_c > 0 && mode == UV_SEARCH_COSINE && std::max(ix->sl_c, k) < ix->n) {
    UV_TRY(shortlist_launch(c, ix->sl_c, ix->sl_asym, ix->sl_weight && ix->n_centroids > 0, k,
                            nq, 1, nullptr, nullptr, ix->n, ix->n, q_r, nullptr, nullptr, qc,
                            ix->n_centroids, degen, ix->codes, ix->signs, ix->start, ix->cidx,
                            ix->rescale, ix->rnorm, ix->ids, d_ids, d_scores, st));
    return outs.finish(st);
  }
  bool used = false;
  UV_TRY(tc_search(ix, q_r, qc, degen, nq, k, mode, d_ids, d_scores, st, sc, &used));
  if (!used) UV_TRY(exact_scan(ix, q_r, qc, degen, nq, k, mode, d_ids, d_scores, st, sc));
  return outs.finish(st);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Sharded search (uv_index_search_begin ... uv_search_finish): a search of
// one shard of a base split across GPUs, in two phases around the exchange
// of first-pass bounds.  Every buffer lives in the search's own stream-ordered
// scratch until uv_search_destroy.
// ---------------------------------------------------------------------------
struct uv_search {
  const uv_index *ix = nullptr;
  int dev = 0;
  cudaStream_t st = nullptr;
  Scratch sc;
  int64_t nq = 0;
  int k = 0, mode = 0;
  enum Path { kPrefilter, kExact, kShortlist, kFullRank } path = kExact;
  int m = 0;                  // bounds per query this shard contributes
  bool needs_bounds = false;  // several shards: the threshold comes from set_bounds
  bool bounds_set = false;
  bool finished = false;
  bool deferred = false;      // finished without its outcome check (uv_search_check)
  int64_t *out_ids = nullptr;  // the deferred search's outputs (device)
  float *out_scores = nullptr;
  const float *d_q = nullptr;
  float *q_r = nullptr, *qc = nullptr;
  uint32_t *degen = nullptr;
  TcState ts;
  explicit uv_search(cudaStream_t s) : st(s), sc(s) {}
};

extern "C" {

int uv_search_bounds_per_query(int32_t k, int32_t n_shards, int32_t *m) {
  if (m == nullptr) return fail(UV_EINVAL, "null argument");
  if (k < 1 || n_shards < 1) return fail(UV_EINVAL, "k and n_shards must be at least 1");
  // every shard's best 2 * ceil(k / n_shards) bounds: the union still holds k
  // values (its k-th largest stays a valid threshold, any subset's does), and
  // a shard holds more than that many of the union's best k only rarely
  *m = n_shards == 1 ? k : std::min<int32_t>(k, 2 * ((k + n_shards - 1) / n_shards));
  return UV_OK;
}

int uv_index_search_begin(const uv_index *ix, const float *queries, int64_t nq, int32_t k,
                          int32_t mode, int32_t n_shards, float *bounds_out, uv_search **out,
                          void *stream) {
  if (out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  if (ix == nullptr || bounds_out == nullptr || (nq > 0 && queries == nullptr))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1) return fail(UV_EINVAL, "k must be at least 1");
  if (n_shards < 1) return fail(UV_EINVAL, "n_shards must be at least 1");
  if (mode != UV_SEARCH_COSINE && mode != UV_SEARCH_MIPS) return fail(UV_EINVAL, "bad mode");
  const uv_codec *c = ix->codec;
  const int d = c->cfg.dim;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = (cudaStream_t)stream;
  uv_search *s = new (std::nothrow) uv_search(st);
  if (s == nullptr) return fail(UV_ENOMEM, "host allocation failed");
  auto run = [&]() -> int {
    s->ix = ix;
    s->dev = dev;
    s->nq = nq;
    s->k = k;
    s->mode = mode;
    UV_TRY(uv_search_bounds_per_query(k, n_shards, &s->m));
    const int m = s->m;
    s->needs_bounds = n_shards > 1;
    bool b_dev = false;
    UV_TRY(classify(bounds_out, dev, &b_dev));
    float *d_bounds = bounds_out;
    if (!b_dev) UV_TRY(s->sc.alloc(&d_bounds, (size_t)std::max<int64_t>(nq, 1) * m));
    if (nq == 0) return UV_OK;
    // a private copy of the queries: the caller's buffer may go away
    float *q_copy = nullptr;
    UV_TRY(s->sc.alloc(&q_copy, (size_t)nq * d));
    bool q_dev = false;
    UV_TRY(classify(queries, dev, &q_dev));
    UV_CK(cudaMemcpyAsync(q_copy, queries, sizeof(float) * nq * d,
                          q_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
    s->d_q = q_copy;
    const int dim_pad = (d + 3) & ~3;
    UV_TRY(s->sc.alloc(&s->q_r, (size_t)nq * dim_pad));
    UV_TRY(s->sc.alloc(&s->qc, (size_t)nq * std::max(1, ix->n_centroids)));
    UV_TRY(s->sc.alloc(&s->degen, (size_t)nq));
    UV_TRY(prep_launch(c, s->d_q, nq, ix->centroids, ix->n_centroids, s->q_r, s->qc, s->degen,
                       nullptr, st));
    const bool shortlist = ix->sl_c > 0 && mode == UV_SEARCH_COSINE &&
                           std::max<int64_t>(ix->sl_c, k) < ix->n;
    if (k > uvb::kScanKCap) {
      if (shortlist) return fail(UV_EUNSUPPORTED, "the shortlist search is built for k <= 128");
      s->path = uv_search::kFullRank;
    } else if (shortlist) {
      s->path = uv_search::kShortlist;
    } else {
      UV_TRY(tc_begin(ix, s->q_r, s->degen, nq, k, mode, n_shards, st, s->sc, &s->ts));
      s->path = s->ts.used ? uv_search::kPrefilter : uv_search::kExact;
    }
    if (s->path == uv_search::kPrefilter) {
      ProfScope ps("tc_bounds", st);
      // the m-th largest group bound of each query (the k-th is ts.theta),
      // then the best m bounds
      const float *th = s->ts.theta;
      if (m != k) {
        float *theta_m = nullptr;
        UV_TRY(s->sc.alloc(&theta_m, (size_t)nq));
        UV_TRY(theta_launch(s->ts.tmax, s->ts.n_groups1, nq, m, theta_m, 1, st));
        th = theta_m;
      }
      uvb::tc_bounds_kernel<<<(unsigned)nq, 256, 0, st>>>(s->ts.tmax, s->ts.n_groups1, nq, m, th,
                                                          d_bounds);
      UV_CK(cudaGetLastError());
    } else {
      // no first pass on this shard: it bounds nothing
      uvb::fill_value_kernel<<<(unsigned)std::min<int64_t>((nq * m + 255) / 256, 4096), 256, 0,
                               st>>>(d_bounds, nq * m, -INFINITY);
      UV_CK(cudaGetLastError());
    }
    if (!b_dev) {
      UV_CK(cudaMemcpyAsync(bounds_out, d_bounds, sizeof(float) * nq * m, cudaMemcpyDeviceToHost,
                            st));
      UV_CK(cudaStreamSynchronize(st));
    }
    return UV_OK;
  };
  const int rc = run();
  if (rc != UV_OK) {
    delete s;
    return rc;
  }
  *out = s;
  return UV_OK;
}

int uv_search_set_bounds(uv_search *s, const float *gathered, int32_t n_shards) {
  if (s == nullptr || (s->nq > 0 && gathered == nullptr)) return fail(UV_EINVAL, "null argument");
  if (n_shards < 1) return fail(UV_EINVAL, "n_shards must be at least 1");
  if (s->finished) return fail(UV_EINVAL, "the search has finished");
  s->bounds_set = true;
  if (s->nq == 0 || s->path != uv_search::kPrefilter) return UV_OK;
  const int dev = s->dev;
  DeviceGuard g(dev);
  const int64_t nq = s->nq;
  const int k = s->k;
  const size_t count = (size_t)n_shards * nq * s->m;
  const float *d_g = nullptr;
  UV_TRY(stage_in(gathered, count, dev, s->sc, &d_g));
  // the k-th largest of the union of every shard's best m bounds
  ProfScope ps("tc_bounds", s->st);
  const int64_t per = (int64_t)n_shards * s->m;
  UV_TRY(theta_launch(d_g, per, nq, k, s->ts.theta, n_shards, s->st));
  return UV_OK;
}

int uv_search_finish(uv_search *s, int64_t *ids_out, float *scores_out) {
  if (s == nullptr || (s->nq > 0 && ids_out == nullptr)) return fail(UV_EINVAL, "null argument");
  if (s->finished) return fail(UV_EINVAL, "the search has finished");
  if (s->needs_bounds && !s->bounds_set)
    return fail(UV_EINVAL, "a search of several shards needs uv_search_set_bounds before finish");
  s->finished = true;
  if (s->nq == 0) return UV_OK;
  const uv_index *ix = s->ix;
  const uv_codec *c = ix->codec;
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  cudaStream_t st = s->st;
  const int64_t nq = s->nq;
  const int k = s->k;
  if (s->path == uv_search::kFullRank) {
    UV_TRY(full_rank_search(ix, s->q_r, s->qc, s->degen, nq, k, s->mode, ids_out, scores_out, st,
                            s->sc));
    UV_CK(cudaStreamSynchronize(st));
    return UV_OK;
  }
  Outputs outs;
  int64_t *d_ids = nullptr;
  float *d_scores = nullptr;
  UV_TRY(outs.stage(ids_out, (size_t)nq * k, dev, s->sc, &d_ids));
  if (scores_out != nullptr) {
    UV_TRY(outs.stage(scores_out, (size_t)nq * k, dev, s->sc, &d_scores));
  } else {
    UV_TRY(s->sc.alloc(&d_scores, (size_t)nq * k));
  }
  switch (s->path) {
    case uv_search::kShortlist:
      UV_TRY(shortlist_launch(c, ix->sl_c, ix->sl_asym, ix->sl_weight && ix->n_centroids > 0, k,
                              nq, 1, nullptr, nullptr, ix->n, ix->n, s->q_r, nullptr, nullptr,
                              s->qc, ix->n_centroids, s->degen, ix->codes, ix->signs, ix->start,
                              ix->cidx, ix->rescale, ix->rnorm, ix->ids, d_ids, d_scores, st));
      break;
    case uv_search::kPrefilter:
      UV_TRY(tc_finish(ix, s->q_r, s->qc, s->degen, nq, k, s->mode, d_ids, d_scores, st, s->sc,
                       s->ts));
      break;
    default:
      UV_TRY(exact_scan(ix, s->q_r, s->qc, s->degen, nq, k, s->mode, d_ids, d_scores, st, s->sc));
      break;
  }
  return outs.finish(st);
}

int uv_search_finish_deferred(uv_search *s, int64_t *ids_out, float *scores_out) {
  if (s == nullptr || (s->nq > 0 && ids_out == nullptr)) return fail(UV_EINVAL, "null argument");
  if (s->path != uv_search::kPrefilter || s->nq == 0)
    return uv_search_finish(s, ids_out, scores_out);  // nothing to defer
  if (s->finished) return fail(UV_EINVAL, "the search has finished");
  if (s->needs_bounds && !s->bounds_set)
    return fail(UV_EINVAL, "a search of several shards needs uv_search_set_bounds before finish");
  const uv_index *ix = s->ix;
  const int dev = ix->codec->cfg.device;
  DeviceGuard g(dev);
  bool ids_dev = false, sc_dev = false;
  UV_TRY(classify(ids_out, dev, &ids_dev));
  if (scores_out != nullptr) UV_TRY(classify(scores_out, dev, &sc_dev));
  if (!ids_dev || (scores_out != nullptr && !sc_dev))
    return fail(UV_EINVAL, "uv_search_finish_deferred takes device buffers of the index's GPU");
  float *d_scores = scores_out;
  if (d_scores == nullptr) UV_TRY(s->sc.alloc(&d_scores, (size_t)s->nq * s->k));
  s->finished = true;
  UV_TRY(tc_finish(ix, s->q_r, s->qc, s->degen, s->nq, s->k, s->mode, ids_out, d_scores, s->st,
                   s->sc, s->ts, true));
  s->deferred = true;
  s->out_ids = ids_out;
  s->out_scores = d_scores;
  return UV_OK;
}

int uv_search_check(uv_search *s, int32_t *overflowed) {
  if (s == nullptr || overflowed == nullptr) return fail(UV_EINVAL, "null argument");
  *overflowed = 0;
  if (!s->finished) return fail(UV_EINVAL, "the search has not finished");
  DeviceGuard g(s->dev);
  if (!s->deferred) {
    UV_CK(cudaStreamSynchronize(s->st));
    return UV_OK;
  }
  s->deferred = false;
  bool over = false;
  UV_TRY(tc_check(s->ix, s->q_r, s->qc, s->degen, s->nq, s->k, s->mode, s->out_ids,
                  s->out_scores, s->st, s->sc, s->ts, &over));
  *overflowed = over ? 1 : 0;
  return UV_OK;
}

int uv_search_destroy(uv_search *s) {
  if (s == nullptr) return UV_OK;
  DeviceGuard g(s->dev);
  delete s;  // frees the scratch on the search's stream
  return UV_OK;
}

}  // extern "C"

namespace {

// The merge of per-shard (or per-split) top-k lists described by m (input
// pointers, strides, nq, n_lists, k_in, k) into d_ids / d_scores: the k-way
// merge kernel up to 8192 entries per row, the segmented sort above.
int merge_rows(uvb::MergeParams m, int64_t *d_ids, float *d_scores, cudaStream_t st, Scratch &sc) {
  const int64_t total = (int64_t)m.n_lists * m.k_in;
  m.out_id = d_ids;
  m.out_score = d_scores;
  if (total >= 512 && total <= 8192) {
    // one CTA per row: many entries per row
    int pow2 = 32;
    while (pow2 < total) pow2 <<= 1;
    m.pow2 = pow2;
    m.warps = 8;
    const size_t smem = (size_t)pow2 * 12;
    UV_CK(cudaFuncSetAttribute(uvb::merge_topk_block_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    void *args[] = {&m};
    ProfScope ps("merge_topk", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::merge_topk_block_kernel, dim3((unsigned)m.nq),
                           dim3(256), args, smem, st));
    return UV_OK;
  }
  if (total <= 8192) {
    int pow2 = 32;
    while (pow2 < total) pow2 <<= 1;
    m.pow2 = pow2;
    const size_t per_warp = (size_t)pow2 * 12;  // id + key per entry
    m.warps = (int)std::max<size_t>(1, std::min<size_t>(8, (96 * 1024) / per_warp));
    const size_t smem = per_warp * m.warps;
    UV_CK(cudaFuncSetAttribute(uvb::merge_topk_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const int grid = (int)((m.nq + m.warps - 1) / m.warps);
    void *args[] = {&m};
    ProfScope ps("merge_topk", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::merge_topk_kernel, dim3(grid), dim3(32 * m.warps),
                           args, smem, st));
    return UV_OK;
  }
  // rows in chunks whose two (key, id) buffers stay within about 1 GiB
  const int64_t rows = std::max<int64_t>(1, std::min<int64_t>(m.nq, (int64_t)(1 << 30) / (24 * total)));
  uint32_t *k0 = nullptr, *k1 = nullptr;
  int64_t *i0 = nullptr, *i1 = nullptr;
  UV_TRY(sc.alloc(&k0, (size_t)rows * total));
  UV_TRY(sc.alloc(&k1, (size_t)rows * total));
  UV_TRY(sc.alloc(&i0, (size_t)rows * total));
  UV_TRY(sc.alloc(&i1, (size_t)rows * total));
  const int64_t row_stride = m.row_stride > 0 ? m.row_stride : total;
  for (int64_t r0 = 0; r0 < m.nq; r0 += rows) {
    uvb::MergeParams part = m;
    part.nq = std::min(rows, m.nq - r0);
    if (part.in_packed) part.in_packed += 3 * r0 * row_stride;
    if (part.in_id) part.in_id += r0 * row_stride;
    if (part.in_key) part.in_key += r0 * row_stride;
    if (part.in_score) part.in_score += r0 * row_stride;
    part.row_stride = row_stride;
    {
      ProfScope ps("merge_topk", st);
      const int64_t all = part.nq * total;
      uvb::rank_gather_kernel<<<(unsigned)std::min<int64_t>((all + 255) / 256, 148 * 16), 256, 0,
                                st>>>(part, total, k0, i0);
      UV_CK(cudaGetLastError());
    }
    bool in_b = false;
    UV_TRY(rank_sort_rows(k0, i0, k1, i1, total, part.nq, m.k, st, &in_b));
    {
      ProfScope ps("merge_topk", st);
      const int64_t outs = part.nq * m.k;
      uvb::rank_emit_kernel<<<(unsigned)std::min<int64_t>((outs + 255) / 256, 148 * 16), 256, 0,
                              st>>>(in_b ? k1 : k0, in_b ? i1 : i0, total, part.nq, m.k, nullptr,
                                    d_ids + r0 * m.k, d_scores ? d_scores + r0 * m.k : nullptr);
      UV_CK(cudaGetLastError());
    }
  }
  return UV_OK;
}

}  // namespace

extern "C" {

int uv_topk_merge(int32_t device, const int64_t *in_ids, const float *in_scores, int64_t nq,
                  int32_t n_lists, int32_t k_in, int32_t k, int64_t *out_ids, float *out_scores,
                  void *stream) {
  if (nq < 0 || n_lists < 1 || k_in < 1 || k < 1 || k > n_lists * k_in)
    return fail(UV_EINVAL, "bad sizes");
  // no rows: nothing to read or write (an empty tensor's buffer may be null)
  if (nq == 0) return UV_OK;
  if (in_ids == nullptr || in_scores == nullptr || out_ids == nullptr)
    return fail(UV_EINVAL, "null argument");
  DeviceGuard g(device);
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  const size_t nin = (size_t)nq * n_lists * k_in;
  const int64_t *d_in_ids = nullptr;
  const float *d_in_scores = nullptr;
  UV_TRY(stage_in(in_ids, nin, device, sc, &d_in_ids));
  UV_TRY(stage_in(in_scores, nin, device, sc, &d_in_scores));
  int64_t *d_out_ids = nullptr;
  float *d_out_scores = nullptr;
  UV_TRY(outs.stage(out_ids, (size_t)nq * k, device, sc, &d_out_ids));
  if (out_scores != nullptr) {
    UV_TRY(outs.stage(out_scores, (size_t)nq * k, device, sc, &d_out_scores));
  } else {
    UV_TRY(sc.alloc(&d_out_scores, (size_t)nq * k));
  }
  uvb::MergeParams m;
  std::memset(&m, 0, sizeof(m));
  m.nq = nq;
  m.n_lists = n_lists;
  m.k_in = k_in;
  m.k = k;
  m.in_score = d_in_scores;
  m.in_id = d_in_ids;
  UV_TRY(merge_rows(m, d_out_ids, d_out_scores, st, sc));
  return outs.finish(st);
}

int uv_topk_pack(int32_t device, const int64_t *ids, const float *scores, int64_t n, void *packed,
                 void *stream) {
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  if (ids == nullptr || scores == nullptr || packed == nullptr)
    return fail(UV_EINVAL, "null argument");
  DeviceGuard g(device);
  for (const void *ptr : {(const void *)ids, (const void *)scores, (const void *)packed}) {
    bool on_dev = false;
    UV_TRY(classify(ptr, device, &on_dev));
    if (!on_dev) return fail(UV_EINVAL, "uv_topk_pack works on device buffers");
  }
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps("topk_pack", st);
  uvb::topk_pack_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(
      ids, scores, n, (int32_t *)packed);
  UV_CK(cudaGetLastError());
  return UV_OK;
}

int uv_topk_unpack(int32_t device, const void *packed, int64_t n, int64_t *ids, float *scores,
                   void *stream) {
  if (n < 0) return fail(UV_EINVAL, "negative size");
  if (n == 0) return UV_OK;
  if (packed == nullptr || ids == nullptr) return fail(UV_EINVAL, "null argument");
  DeviceGuard g(device);
  for (const void *ptr : {(const void *)packed, (const void *)ids, (const void *)scores}) {
    if (ptr == nullptr) continue;
    bool on_dev = false;
    UV_TRY(classify(ptr, device, &on_dev));
    if (!on_dev) return fail(UV_EINVAL, "uv_topk_unpack works on device buffers");
  }
  cudaStream_t st = (cudaStream_t)stream;
  ProfScope ps("topk_pack", st);
  uvb::topk_unpack_kernel<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(
      (const int32_t *)packed, n, ids, scores);
  UV_CK(cudaGetLastError());
  return UV_OK;
}

int uv_topk_merge_packed(int32_t device, const void *packed, int64_t nq, int32_t n_lists,
                         int32_t k_in, int64_t row_stride, int64_t list_stride, int32_t k,
                         int64_t *out_ids, float *out_scores, void *stream) {
  if (nq < 0 || n_lists < 1 || k_in < 1 || k < 1 || k > n_lists * k_in || row_stride < 0 ||
      list_stride < 0)
    return fail(UV_EINVAL, "bad sizes");
  // a rank whose query slice is empty (fewer queries than ranks) merges
  // nothing; its buffers are empty tensors, whose pointers may be null
  if (nq == 0) return UV_OK;
  if (packed == nullptr || out_ids == nullptr) return fail(UV_EINVAL, "null argument");
  DeviceGuard g(device);
  bool on_dev = false;
  UV_TRY(classify(packed, device, &on_dev));
  if (!on_dev) return fail(UV_EINVAL, "uv_topk_merge_packed reads device records");
  cudaStream_t st = (cudaStream_t)stream;
  Scratch sc(st);
  Outputs outs;
  int64_t *d_out_ids = nullptr;
  float *d_out_scores = nullptr;
  UV_TRY(outs.stage(out_ids, (size_t)nq * k, device, sc, &d_out_ids));
  if (out_scores != nullptr) {
    UV_TRY(outs.stage(out_scores, (size_t)nq * k, device, sc, &d_out_scores));
  } else {
    UV_TRY(sc.alloc(&d_out_scores, (size_t)nq * k));
  }
  uvb::MergeParams m;
  std::memset(&m, 0, sizeof(m));
  m.nq = nq;
  m.n_lists = n_lists;
  m.k_in = k_in;
  m.k = k;
  m.row_stride = row_stride;
  m.list_stride = list_stride;
  m.in_packed = (const int32_t *)packed;
  UV_TRY(merge_rows(m, d_out_ids, d_out_scores, st, sc));
  return outs.finish(st);
}

int uv_set_tuning(const char *key, int64_t value) {
  if (key == nullptr) return fail(UV_EINVAL, "null key");
  if (std::strcmp(key, "encode_back") == 0) {
    if (value < 0 || value > 2) return fail(UV_EINVAL, "encode_back must be 0, 1 or 2");
    uvb::g_encode_back_mode = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_scan") == 0) {
    if (value < 0 || value > 2) return fail(UV_EINVAL, "tc_scan must be 0, 1 or 2");
    g_tc_mode = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_shape") == 0) {
    if (value != 0 && value != 1 && value != 3) return fail(UV_EINVAL, "tc_shape must be 0, 1 or 3");
    g_tc_shape = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_cache") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "tc_cache must be 0 or 1");
    g_tc_cache = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "ivf_tc_probe") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "ivf_tc_probe must be 0 or 1");
    g_ivf_tc_probe = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "ivf_tc") == 0) {
    if (value < 0 || value > 2) return fail(UV_EINVAL, "ivf_tc must be 0, 1 or 2");
    g_ivf_tc = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_prepare") == 0) {
    if (value < 0 || value > 2) return fail(UV_EINVAL, "tc_prepare must be 0, 1 or 2");
    g_tc_prepare = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_sample") == 0) {
    if (value < 0 || value > 64) return fail(UV_EINVAL, "tc_sample must be 0..64");
    g_tc_sample = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "coset_nearest") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "coset_nearest must be 0 or 1");
    g_coset_nearest = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "cand_kernel") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "cand_kernel must be 0 or 1");
    g_cand_kernel = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "encode_staged") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "encode_staged must be 0 or 1");
    uvb::g_encode_staged = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "tc_hot") == 0) {
    if (value < 0 || value > 64) return fail(UV_EINVAL, "tc_hot must be 0..64");
    g_tc_hot = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "rescore_warp") == 0) {
    if (value < 0 || value > 1) return fail(UV_EINVAL, "rescore_warp must be 0 or 1");
    g_rescore_warp = (int)value;
    return UV_OK;
  }
  if (std::strcmp(key, "scan_splits") == 0) {
    if (value < 0 || value > 4096) return fail(UV_EINVAL, "scan_splits must be 0..4096");
    g_scan_splits = value;
    return UV_OK;
  }
  return fail(UV_EINVAL, std::string("unknown tuning key: ") + key);
}

int uv_profile_enable(int32_t on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto &r : g_prof) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  g_prof.clear();
  g_prof_on = on != 0;
  return UV_OK;
}

int uv_profile_read(const char *kernel, double *total_ms, int64_t *launches) {
  if (kernel == nullptr || total_ms == nullptr || launches == nullptr)
    return fail(UV_EINVAL, "null argument");
  if (std::strcmp(kernel, "tc_sample") == 0) {
    // statistic of the last tensor-core search: pass 1 bounded every S-th tile
    *total_ms = 0.0;
    *launches = g_tc_last_sample.load();
    return UV_OK;
  }
  if (std::strcmp(kernel, "ivf_tc_overflow") == 0) {
    // statistic of the last tensor-core IVF list scan: 1 when its kept-record
    // store was full (total_ms), and the queries with more candidates than
    // the per-query store holds (launches); either sends the search to the
    // CUDA-core scan
    const int64_t v = g_ivf_tc_overflow.load();
    *total_ms = (double)(v >> 32);
    *launches = v & 0xffffffffll;
    return UV_OK;
  }
  if (std::strcmp(kernel, "tc_candidates") == 0) {
    // statistic of the last tensor-core search: candidates scored exactly
    *total_ms = 0.0;
    *launches = g_tc_last_candidates.load();
    return UV_OK;
  }
  std::lock_guard<std::mutex> lk(g_prof_mu);
  double tot = 0.0;
  int64_t cnt = 0;
  const bool all = std::strcmp(kernel, "*") == 0;
  for (auto &r : g_prof) {
    if (!all && std::strcmp(r.name, kernel) != 0) continue;
    UV_CK(cudaEventSynchronize(r.b));
    float ms = 0.0f;
    UV_CK(cudaEventElapsedTime(&ms, r.a, r.b));
    tot += ms;
    cnt++;
  }
  *total_ms = tot;
  *launches = cnt;
  return UV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Search without device allocation (uv_index_search_noalloc).
//
// Some callers cannot allocate device memory at search time: a serving
// process that reserves its whole GPU budget at start-up, or a latency-bound
// thread that cannot accept the device-wide synchronization cudaMalloc and
// cudaFree may imply.  This entry point takes its per-call scratch from one
// fixed file-scope device array instead, carved into the same buffers
// uv_index_search allocates.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
constexpr int kNoAllocMaxDevices = 64;
void *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// The device address of g_noalloc_scratch on the current device, looked up
// once per device (the caller made that device current) and kept for the
// life of the process: after a cudaDeviceReset of that device the cached
// address is stale, so a process that resets a device must not call
// uv_index_search_noalloc on it again.
int noalloc_scratch(int dev, unsigned char **out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(UV_EINVAL, "device ordinal out of range");
  if (g_noalloc_ptr[dev] == nullptr) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(UV_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = (unsigned char *)g_noalloc_ptr[dev];
  return UV_OK;
}

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

extern "C" {

int uv_index_search_noalloc(const uv_index *ix, const float *queries, int64_t nq, int32_t k,
                            int32_t mode, int64_t *ids_out, float *scores_out, void *stream) {
  if (ix == nullptr || (nq > 0 && (queries == nullptr || ids_out == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (nq < 0) return fail(UV_EINVAL, "negative size");
  if (k < 1 || k > uvb::kScanKCap) return fail(UV_EINVAL, "k must be 1..128");
  if (mode != UV_SEARCH_COSINE && mode != UV_SEARCH_MIPS) return fail(UV_EINVAL, "bad mode");
  const uv_codec *c = ix->codec;
  const int d = (c->cfg.dim + 15) & ~15;  // kernel width (fill_scan_params)
  if (ix->sl_c > 0 && mode == UV_SEARCH_COSINE && std::max(ix->sl_c, k) < ix->n)
    return fail(UV_EUNSUPPORTED, "the shortlist search is not built without allocation");
  const int dev = c->cfg.device;
  DeviceGuard g(dev);
  // every buffer must already be on this GPU: staging would allocate
  for (const void *ptr : {(const void *)queries, (const void *)ids_out, (const void *)scores_out}) {
    if (ptr == nullptr) continue;
    bool on_dev = false;
    UV_TRY(classify(ptr, dev, &on_dev));
    if (!on_dev)
      return fail(UV_EINVAL, "uv_index_search_noalloc needs queries and outputs in device memory");
  }
  unsigned char *arena = nullptr;
  UV_TRY(noalloc_scratch(dev, &arena));
  if (nq == 0) return UV_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = ix->n;
  const int dim_pad = (c->cfg.dim + 3) & ~3;
  const int ncen = std::max(1, ix->n_centroids);
  // every query needs at least its rotated row: reject batches that cannot
  // fit before any size product below could wrap
  if (nq > (int64_t)(kNoAllocScratchBytes / (4 * (size_t)dim_pad)))
    return fail(UV_EINVAL, "this query batch cannot fit the no-allocation search's " +
                               std::to_string(kNoAllocScratchBytes) +
                               "-byte scratch; search fewer queries per call");
  const int rw = c->code_stride / 4;
  int img_words = 4 + rw + 3;
  if ((img_words & 1) == 0) img_words++;
  const bool table_smem = (size_t)c->table_len * 4 <= 16 * 1024;
  const size_t smem = uvb::scan_smem_bytes(d, img_words, c->table_len, table_smem);
  if (smem > 227 * 1024)
    return fail(UV_EUNSUPPORTED, "flat scan tile for this dim exceeds shared memory (dim <= 384)");
  const void *scan_k = uvb::flat_scan_kernel_ptr(c->cfg.bits, table_smem);
  UV_CK(cudaFuncSetAttribute(scan_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 1;
  UV_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_k, 256, smem));
  per_sm = std::max(per_sm, 1);
  const int64_t qtiles = (nq + uvb::kScanTQ - 1) / uvb::kScanTQ;
  const int64_t slots = (int64_t)sm_count(dev) * per_sm;
  const int64_t max_splits =
      std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(2048 / k, 32), n / 1024));
  int64_t splits = 1;
  double best_eff = 0.0;
  for (int64_t sp = 1; sp <= max_splits; sp++) {
    const int64_t ctas = qtiles * sp;
    const int64_t waves = (ctas + slots - 1) / slots;
    const double eff = (double)ctas / (double)(waves * slots);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      splits = sp;
    }
    if (eff >= 0.9) break;
  }
  // carve the arena; fewer splits when the batch would not fit
  auto layout = [&](int64_t sp) {
    size_t b = 0;
    b += align256(sizeof(float) * (size_t)nq * dim_pad);
    b += align256(sizeof(float) * (size_t)nq * ncen);
    b += align256(sizeof(uint32_t) * (size_t)nq);
    if (scores_out == nullptr) b += align256(sizeof(float) * (size_t)nq * k);
    b += align256(sizeof(uint32_t) * (size_t)nq * sp * k);
    b += align256(sizeof(int64_t) * (size_t)nq * sp * k);
    return b;
  };
  while (splits > 1 && layout(splits) > kNoAllocScratchBytes) splits--;
  if (layout(splits) > kNoAllocScratchBytes)
    return fail(UV_EINVAL, "this query batch needs " + std::to_string(layout(1)) +
                               " bytes of scratch but the no-allocation search has " +
                               std::to_string(kNoAllocScratchBytes) +
                               "; search fewer queries per call");
  size_t off = 0;
  auto take = [&](size_t bytes) {
    unsigned char *ptr = arena + off;
    off += align256(bytes);
    return ptr;
  };
  float *q_r = (float *)take(sizeof(float) * (size_t)nq * dim_pad);
  float *qc = (float *)take(sizeof(float) * (size_t)nq * ncen);
  uint32_t *degen = (uint32_t *)take(sizeof(uint32_t) * (size_t)nq);
  float *d_scores = scores_out;
  if (d_scores == nullptr) d_scores = (float *)take(sizeof(float) * (size_t)nq * k);
  uint32_t *part_key = (uint32_t *)take(sizeof(uint32_t) * (size_t)nq * splits * k);
  int64_t *part_id = (int64_t *)take(sizeof(int64_t) * (size_t)nq * splits * k);

  // 1) prepare queries
  {
    uvb::PrepParams pp;
    std::memset(&pp, 0, sizeof(pp));
    pp.dim = c->cfg.dim;
    pp.dim_pad = dim_pad;
    pp.nq = nq;
    pp.queries = queries;
    pp.rot = c->rot;
    pp.centroids = ix->centroids;
    pp.n_centroids = ix->n_centroids;
    pp.q_r = q_r;
    pp.qc = qc;
    pp.degenerate = degen;
    pp.teams = uvb::prep_teams(d);
    const size_t psmem = (size_t)(dim_pad + 4) * 4 * pp.teams;
    UV_CK(cudaFuncSetAttribute(uvb::prep_queries_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psmem));
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((nq + pp.teams - 1) / pp.teams, INT32_MAX));
    void *args[] = {&pp};
    ProfScope ps("prep_queries", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::prep_queries_kernel, dim3(grid), dim3(256), args,
                           psmem, st));
  }
  // 2) scan with a per-split top-k
  if (n == 0) {
    UV_CK(cudaMemsetAsync(part_key, 0, sizeof(uint32_t) * nq * splits * k, st));
    UV_CK(cudaMemsetAsync(part_id, 0xff, sizeof(int64_t) * nq * splits * k, st));
  } else {
    uvb::ScanParams sp;
    fill_scan_params(ix, q_r, qc, degen, nq, k, mode, img_words, table_smem, &sp);
    sp.part_key = part_key;
    sp.part_id = part_id;
    void *args[] = {&sp};
    ProfScope ps("flat_scan", st);
    UV_CK(cudaLaunchKernel(scan_k, dim3((unsigned)qtiles, (unsigned)splits), dim3(256), args,
                           smem, st));
  }
  // 3) merge the splits
  {
    uvb::MergeParams m;
    std::memset(&m, 0, sizeof(m));
    m.nq = nq;
    m.n_lists = (int)splits;
    m.k_in = k;
    m.k = k;
    int pow2 = 32;
    while (pow2 < (int)splits * k) pow2 <<= 1;
    m.pow2 = pow2;
    const size_t per_warp = (size_t)pow2 * 12;  // id + key per entry
    m.warps = (int)std::max<size_t>(1, std::min<size_t>(8, (96 * 1024) / per_warp));
    m.in_key = part_key;
    m.in_id = part_id;
    m.out_id = ids_out;
    m.out_score = d_scores;
    const size_t msmem = per_warp * m.warps;
    UV_CK(cudaFuncSetAttribute(uvb::merge_topk_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
    const int grid = (int)((nq + m.warps - 1) / m.warps);
    void *args[] = {&m};
    ProfScope ps("merge_topk", st);
    UV_CK(cudaLaunchKernel((const void *)uvb::merge_topk_kernel, dim3(grid), dim3(32 * m.warps),
                           args, msmem, st));
  }
  return UV_OK;
}

}  // extern "C"
