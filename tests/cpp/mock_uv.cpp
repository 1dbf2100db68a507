// A CPU stand-in for the C ABI of ultravec_b200.h, for testing the C++ host
// API (include/ultravec_b200.hpp) without a GPU: each entry point the header
// calls checks the argument contract the library states, records what it
// was given in `mock`, and returns made-up results that the test can
// predict.  Linked instead of libultravec_b200.so; test infrastructure only.
#include "mock_uv.h"

#include <algorithm>
#include <cstring>
#include <string>

MockState mock;

namespace {

int fail(int code, const char *msg) {
  mock.error = msg;
  return code;
}

// an injected failure for the named call
bool injected(const char *name, int *rc) {
  if (mock.fail_call == name) {
    mock.error = "injected failure of " + mock.fail_call;
    *rc = mock.fail_code;
    return true;
  }
  return false;
}

#define MOCK_ENTER(name)                    \
  do {                                      \
    mock.calls.push_back(name);             \
    int rc_ = 0;                            \
    if (injected(name, &rc_)) return rc_;   \
  } while (0)

}  // namespace

struct uv_codec {
  uv_config cfg;
  mutable int live;  // indexes and IVF indexes made on this codec, not yet destroyed
};
struct uv_index {
  const uv_codec *codec;
  int64_t n;
};
struct uv_ivf {
  const uv_codec *codec;
  int32_t nlist;
  int64_t n;
};
struct uv_prepared {
  int64_t nq;
};
struct uv_coset {
  int32_t dim, bits, mem;
  int64_t n;
};

extern "C" {

int uv_abi_version(void) { return UV_ABI_VERSION; }
const char *uv_last_error(void) { return mock.error.c_str(); }

void uv_config_default(uv_config *cfg, int32_t dim, int32_t bits, int32_t mem) {
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->dim = dim;
  cfg->bits = bits;
  cfg->mem = mem;
  cfg->rotation_rounds = 3;
  cfg->rotation_seed = 42;
  cfg->start_bits = mem;
}

int uv_codec_create(const uv_config *cfg, uv_codec **out) {
  MOCK_ENTER("uv_codec_create");
  if (cfg == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  if (cfg->dim < 1 || cfg->bits < 1 || cfg->bits > 4 || cfg->mem < 1)
    return fail(UV_EINVAL, "bad configuration");
  mock.cfg = *cfg;
  *out = new uv_codec{*cfg, 0};
  mock.live_codecs++;
  return UV_OK;
}

int uv_codec_destroy(uv_codec *codec) {
  if (codec == nullptr) return UV_OK;
  mock.calls.push_back("uv_codec_destroy");
  mock.live_codecs--;
  // an index or IVF still alive on this codec would read freed tables
  if (codec->live > 0) mock.order_errors++;
  delete codec;
  return UV_OK;
}

int uv_codec_code_table_bits(const uv_codec *c, uint32_t *out, int64_t capacity) {
  MOCK_ENTER("uv_codec_code_table_bits");
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  const int64_t len = (int64_t)1 << (c->cfg.mem + c->cfg.bits);
  if (capacity < len) return fail(UV_EINVAL, "capacity too small");
  for (int64_t i = 0; i < len; i++) out[i] = (uint32_t)i * 3u;
  return UV_OK;
}

int uv_codec_rotation_sign_rounds(const uv_codec *c, float *out, int64_t capacity) {
  MOCK_ENTER("uv_codec_rotation_sign_rounds");
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  const int64_t len = (int64_t)c->cfg.rotation_rounds * c->cfg.dim;
  if (capacity < len) return fail(UV_EINVAL, "capacity too small");
  for (int64_t i = 0; i < len; i++) out[i] = (i % 3 == 0) ? -1.0f : 1.0f;
  return UV_OK;
}

int uv_codec_memory_bits(const uv_codec *c, int32_t *mem) {
  MOCK_ENTER("uv_codec_memory_bits");
  if (c == nullptr || mem == nullptr) return fail(UV_EINVAL, "null argument");
  *mem = c->cfg.mem;
  return UV_OK;
}

int uv_codec_record_bytes(const uv_codec *c, int32_t *code_bytes, int32_t *start_bytes,
                          int32_t *rescale_bytes) {
  MOCK_ENTER("uv_codec_record_bytes");
  if (c == nullptr) return fail(UV_EINVAL, "null argument");
  if (code_bytes) *code_bytes = (c->cfg.dim * c->cfg.bits + 7) / 8;
  if (start_bytes) *start_bytes = (c->cfg.start_bits + 7) / 8;
  if (rescale_bytes) *rescale_bytes = 4;
  return UV_OK;
}

// record i of a batch: codes byte j = (row[0] + i + j), start = 7 + i
int uv_encode(const uv_codec *c, const float *rows, int64_t n, const float *centroids,
              int32_t n_centroids, uint8_t *codes, uint32_t *start, float *rescale, float *rnorm,
              uint32_t *cidx, void *stream) {
  MOCK_ENTER("uv_encode");
  (void)centroids, (void)n_centroids, (void)rnorm, (void)cidx, (void)stream;
  if (c == nullptr || (n > 0 && (rows == nullptr || rescale == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (n_centroids > 0 && centroids == nullptr) return fail(UV_EINVAL, "null centroids");
  mock.n_centroids = n_centroids;
  const int cb = (c->cfg.dim * c->cfg.bits + 7) / 8;
  for (int64_t i = 0; i < n; i++) {
    for (int j = 0; j < cb; j++) codes[i * cb + j] = (uint8_t)((int)rows[i * c->cfg.dim] + i + j);
    start[i] = 7u + (uint32_t)i;
    rescale[i] = 1.0f;
    if (rnorm) rnorm[i] = n_centroids > 0 ? 0.5f : 1.0f;
    if (cidx) cidx[i] = n_centroids > 0 ? (uint32_t)(n_centroids - 1) : 0u;
  }
  return UV_OK;
}

int uv_encode_rotated(const uv_codec *c, const float *u_r, int64_t n, uint8_t *codes,
                      uint32_t *start, void *stream) {
  MOCK_ENTER("uv_encode_rotated");
  (void)stream;
  if (c == nullptr || (n > 0 && u_r == nullptr)) return fail(UV_EINVAL, "null argument");
  const int cb = (c->cfg.dim * c->cfg.bits + 7) / 8;
  for (int64_t i = 0; i < n; i++) {
    for (int j = 0; j < cb; j++) codes[i * cb + j] = (uint8_t)(100 + j);
    start[i] = 9u;
  }
  return UV_OK;
}

int uv_rotate(const uv_codec *c, const float *rows, int64_t n, float *out, void *stream) {
  MOCK_ENTER("uv_rotate");
  (void)stream;
  if (c == nullptr || rows == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  for (int64_t i = 0; i < n * c->cfg.dim; i++) out[i] = 2.0f * rows[i];
  return UV_OK;
}

int uv_decode(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
              float *out, void *stream) {
  MOCK_ENTER("uv_decode");
  (void)stream;
  if (c == nullptr || codes == nullptr || start == nullptr || out == nullptr)
    return fail(UV_EINVAL, "null argument");
  for (int64_t i = 0; i < n * c->cfg.dim; i++) out[i] = (float)(start[i / c->cfg.dim]) + codes[0];
  return UV_OK;
}

int uv_windows(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
               uint32_t *out, void *stream) {
  MOCK_ENTER("uv_windows");
  (void)stream;
  if (c == nullptr || codes == nullptr || start == nullptr || out == nullptr)
    return fail(UV_EINVAL, "null argument");
  for (int64_t i = 0; i < n * c->cfg.dim; i++) out[i] = 1000u * start[0] + (uint32_t)i;
  return UV_OK;
}

int uv_digest(const uv_codec *c, const uint8_t *codes, const uint32_t *start, int64_t n,
              uint64_t *digest, void *stream) {
  MOCK_ENTER("uv_digest");
  (void)stream;
  if (c == nullptr || digest == nullptr || (n > 0 && (codes == nullptr || start == nullptr)))
    return fail(UV_EINVAL, "null argument");
  // each record's start and first code byte (records of code_bytes each)
  const int cb = (c->cfg.dim * c->cfg.bits + 7) / 8;
  uint64_t h = 0;
  for (int64_t i = 0; i < n; i++) h ^= ((uint64_t)start[i] << 8) ^ codes[i * cb];
  *digest = h;
  return UV_OK;
}

int uv_index_create(const uv_codec *c, uv_index **out) {
  MOCK_ENTER("uv_index_create");
  if (c == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = new uv_index{c, 0};
  c->live++;
  mock.live_indexes++;
  return UV_OK;
}

int uv_index_destroy(uv_index *x) {
  if (x == nullptr) return UV_OK;
  mock.calls.push_back("uv_index_destroy");
  x->codec->live--;
  mock.live_indexes--;
  delete x;
  return UV_OK;
}

int uv_index_set_centroids(uv_index *x, const float *centroids, int32_t n) {
  MOCK_ENTER("uv_index_set_centroids");
  if (x == nullptr || (n > 0 && centroids == nullptr)) return fail(UV_EINVAL, "null argument");
  if (x->n != 0) return fail(UV_EINVAL, "the index is not empty");
  mock.rows.assign(centroids, centroids + (size_t)n * x->codec->cfg.dim);
  mock.n_centroids = n;
  return UV_OK;
}

int uv_index_set_shortlist(uv_index *x, int32_t c, int32_t asym, int32_t rnorm) {
  MOCK_ENTER("uv_index_set_shortlist");
  if (x == nullptr) return fail(UV_EINVAL, "null argument");
  if (x->n != 0) return fail(UV_EINVAL, "the index is not empty");
  mock.sl_c = c;
  mock.sl_asym = asym;
  mock.sl_rnorm = rnorm;
  return UV_OK;
}

int uv_index_reserve(uv_index *x, int64_t additional) {
  MOCK_ENTER("uv_index_reserve");
  if (x == nullptr || additional < 0) return fail(UV_EINVAL, "bad argument");
  mock.reserved = additional;
  return UV_OK;
}

int uv_index_add(uv_index *x, const int64_t *ids, const float *rows, int64_t n, void *stream) {
  MOCK_ENTER("uv_index_add");
  (void)stream;
  if (x == nullptr || (n > 0 && (ids == nullptr || rows == nullptr)))
    return fail(UV_EINVAL, "null argument");
  mock.rows.assign(rows, rows + (size_t)n * x->codec->cfg.dim);
  mock.ids.assign(ids, ids + n);
  x->n += n;
  return UV_OK;
}

int uv_index_add_batch(uv_index *x, const float *rows, int64_t n, void *stream) {
  MOCK_ENTER("uv_index_add_batch");
  (void)stream;
  if (x == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  mock.rows.assign(rows, rows + (size_t)n * x->codec->cfg.dim);
  mock.ids.clear();
  x->n += n;
  return UV_OK;
}

int uv_index_len(const uv_index *x, int64_t *len) {
  MOCK_ENTER("uv_index_len");
  if (x == nullptr || len == nullptr) return fail(UV_EINVAL, "null argument");
  *len = x->n;
  return UV_OK;
}

int uv_index_mem_bytes(const uv_index *x, int64_t *bytes) {
  MOCK_ENTER("uv_index_mem_bytes");
  if (x == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = x->n * 41;
  return UV_OK;
}

// slot j of query q: id = j while j < min(len, k) - (q odd), then unfilled;
// score = 10 - j (MIPS: 100 - j)
int uv_index_search(const uv_index *x, const float *queries, int64_t nq, int32_t k, int32_t mode,
                    int64_t *ids, float *scores, void *stream) {
  MOCK_ENTER("uv_index_search");
  (void)stream;
  if (x == nullptr || (nq > 0 && (queries == nullptr || ids == nullptr)))
    return fail(UV_EINVAL, "null argument");
  if (k < 1) return fail(UV_EINVAL, "k must be at least 1");
  if (mode != UV_SEARCH_COSINE && mode != UV_SEARCH_MIPS) return fail(UV_EINVAL, "bad mode");
  mock.k = k;
  mock.mode = mode;
  mock.nq = nq;
  mock.rows.assign(queries, queries + (size_t)nq * x->codec->cfg.dim);
  for (int64_t q = 0; q < nq; q++)
    for (int32_t j = 0; j < k; j++) {
      const bool filled = j < (int32_t)std::min<int64_t>(x->n, k) - (int32_t)(q & 1);
      ids[q * k + j] = filled ? j : -1;
      if (scores)
        scores[q * k + j] = filled ? (mode == UV_SEARCH_MIPS ? 100.0f : 10.0f) - j : -1e30f;
    }
  return UV_OK;
}

int uv_index_scorer_model_bytes(const uv_index *x, int64_t *bytes) {
  MOCK_ENTER("uv_index_scorer_model_bytes");
  if (x == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = 4096;
  return UV_OK;
}

int uv_index_prepare(const uv_index *x, const float *queries, int64_t nq, uv_prepared **out,
                     void *stream) {
  MOCK_ENTER("uv_index_prepare");
  (void)stream;
  if (x == nullptr || queries == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = new uv_prepared{nq};
  mock.live_prepared++;
  return UV_OK;
}

int uv_prepared_destroy(uv_prepared *p) {
  if (p == nullptr) return UV_OK;
  mock.live_prepared--;
  delete p;
  return UV_OK;
}

// score of position p = 0.5 * p; a position at or past 1000 is outside the index
int uv_prepared_score(const uv_prepared *p, const int64_t *offsets, const int64_t *positions,
                      int64_t n, float *scores, void *stream) {
  MOCK_ENTER("uv_prepared_score");
  (void)stream;
  if (p == nullptr || positions == nullptr || scores == nullptr)
    return fail(UV_EINVAL, "null argument");
  if (offsets == nullptr && p->nq != 1) return fail(UV_EINVAL, "offsets needed");
  for (int64_t i = 0; i < n; i++) {
    if (positions[i] < 0 || positions[i] >= 1000) return fail(UV_EINVAL, "position outside the index");
    scores[i] = 0.5f * (float)positions[i];
  }
  return UV_OK;
}

int uv_index_save(const uv_index *x, const char *path) {
  MOCK_ENTER("uv_index_save");
  if (x == nullptr || path == nullptr) return fail(UV_EINVAL, "null argument");
  mock.path = path;
  return UV_OK;
}

int uv_index_load(const uv_codec *c, const char *path, uv_index **out) {
  MOCK_ENTER("uv_index_load");
  if (c == nullptr || path == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  mock.path = path;
  *out = new uv_index{c, 5};
  c->live++;
  mock.live_indexes++;
  return UV_OK;
}

int uv_kmeans(int32_t device, const float *rows, int64_t n, int32_t dim, int32_t nlist,
              uint64_t seed, int32_t iters, float *centroids_out, void *stream) {
  MOCK_ENTER("uv_kmeans");
  (void)device, (void)stream;
  if (rows == nullptr || centroids_out == nullptr || n < 1 || nlist < 1)
    return fail(UV_EINVAL, "bad argument");
  mock.seed = seed;
  mock.iters = iters;
  for (int64_t j = 0; j < (int64_t)nlist * dim; j++) centroids_out[j] = (float)j;
  return UV_OK;
}

int uv_ivf_assign(int32_t device, const float *rows, int64_t n, int32_t dim,
                  const float *centroids, int32_t nlist, uint32_t *assign_out, void *stream) {
  MOCK_ENTER("uv_ivf_assign");
  (void)device, (void)rows, (void)dim, (void)centroids, (void)stream;
  if (assign_out == nullptr || nlist < 1) return fail(UV_EINVAL, "bad argument");
  for (int64_t i = 0; i < n; i++) assign_out[i] = (uint32_t)(i % nlist);
  return UV_OK;
}

int uv_ivf_create(const uv_codec *c, const float *centroids, int32_t nlist, int32_t centered,
                  uv_ivf **out) {
  MOCK_ENTER("uv_ivf_create");
  if (c == nullptr || centroids == nullptr || out == nullptr || nlist < 1)
    return fail(UV_EINVAL, "bad argument");
  mock.centered = centered;
  mock.nlist = nlist;
  *out = new uv_ivf{c, nlist, 0};
  c->live++;
  mock.live_indexes++;
  return UV_OK;
}

int uv_ivf_destroy(uv_ivf *x) {
  if (x == nullptr) return UV_OK;
  mock.calls.push_back("uv_ivf_destroy");
  x->codec->live--;
  mock.live_indexes--;
  delete x;
  return UV_OK;
}

int uv_ivf_set_shortlist(uv_ivf *x, int32_t c, int32_t asym, int32_t rnorm) {
  MOCK_ENTER("uv_ivf_set_shortlist");
  if (x == nullptr) return fail(UV_EINVAL, "null argument");
  mock.sl_c = c;
  mock.sl_asym = asym;
  mock.sl_rnorm = rnorm;
  return UV_OK;
}

int uv_ivf_build(uv_ivf *x, const float *rows, int64_t n, const uint32_t *assign,
                 const int64_t *ids, void *stream) {
  MOCK_ENTER("uv_ivf_build");
  (void)ids, (void)stream;
  if (x == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  for (int64_t i = 0; i < n; i++)
    if (assign != nullptr && assign[i] >= (uint32_t)x->nlist) return fail(UV_EINVAL, "bad assignment");
  x->n = n;
  return UV_OK;
}

int uv_ivf_search(const uv_ivf *x, const float *queries, int64_t nq, int32_t k, int32_t nprobe,
                  int64_t *ids, float *scores, void *stream) {
  MOCK_ENTER("uv_ivf_search");
  (void)queries, (void)stream;
  if (x == nullptr || ids == nullptr || scores == nullptr) return fail(UV_EINVAL, "null argument");
  if (k < 1 || k > 128) return fail(UV_EINVAL, "k must be 1..128");
  mock.k = k;
  mock.nprobe = nprobe;
  for (int64_t i = 0; i < nq * k; i++) {
    ids[i] = (i % k) < 3 ? 40 + (i % k) : -1;
    scores[i] = 1.0f - 0.1f * (float)(i % k);
  }
  return UV_OK;
}

int uv_ivf_search_rerank(const uv_ivf *x, const float *queries, int64_t nq, int32_t k,
                         int32_t nprobe, int32_t rdepth, const float *db, int64_t n_db,
                         int64_t *ids, float *scores, void *stream) {
  MOCK_ENTER("uv_ivf_search_rerank");
  (void)queries, (void)stream;
  if (x == nullptr || db == nullptr || ids == nullptr || scores == nullptr)
    return fail(UV_EINVAL, "null argument");
  mock.k = k;
  mock.nprobe = nprobe;
  mock.rdepth = rdepth;
  mock.n_db = n_db;
  for (int64_t i = 0; i < nq * k; i++) {
    ids[i] = 70 + i;
    scores[i] = 0.9f;
  }
  return UV_OK;
}

int uv_ivf_len(const uv_ivf *x, int64_t *len) {
  MOCK_ENTER("uv_ivf_len");
  if (x == nullptr || len == nullptr) return fail(UV_EINVAL, "null argument");
  *len = x->n;
  return UV_OK;
}

int uv_ivf_nlist(const uv_ivf *x, int32_t *nlist) {
  MOCK_ENTER("uv_ivf_nlist");
  if (x == nullptr || nlist == nullptr) return fail(UV_EINVAL, "null argument");
  *nlist = x->nlist;
  return UV_OK;
}

int uv_ivf_mem_bytes(const uv_ivf *x, int64_t *bytes) {
  MOCK_ENTER("uv_ivf_mem_bytes");
  if (x == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = x->n * 45;
  return UV_OK;
}

int uv_coset_create(int32_t dim, int32_t bits, int32_t mem, uint64_t rotation_seed,
                    int32_t rotation_rounds, int32_t device, uv_coset **out) {
  MOCK_ENTER("uv_coset_create");
  (void)device;
  if (out == nullptr) return fail(UV_EINVAL, "null argument");
  if (dim % 8 != 0 || bits < 1 || bits > 3 || mem < 1 || mem > 20)
    return fail(UV_EINVAL, "bad coset configuration");
  mock.cfg.dim = dim;
  mock.cfg.bits = bits;
  mock.cfg.mem = mem;
  mock.cfg.rotation_seed = rotation_seed;
  mock.cfg.rotation_rounds = rotation_rounds;
  *out = new uv_coset{dim, bits, mem, 0};
  mock.live_indexes++;
  return UV_OK;
}

int uv_coset_destroy(uv_coset *c) {
  if (c == nullptr) return UV_OK;
  mock.live_indexes--;
  delete c;
  return UV_OK;
}

int uv_coset_set_centroids(uv_coset *c, const float *centroids, int32_t n) {
  MOCK_ENTER("uv_coset_set_centroids");
  if (c == nullptr || (n > 0 && centroids == nullptr)) return fail(UV_EINVAL, "null argument");
  if (c->n != 0) return fail(UV_EINVAL, "the index is not empty");
  mock.n_centroids = n;
  return UV_OK;
}

int uv_coset_add(uv_coset *c, const int64_t *ids, const float *rows, int64_t n, void *stream) {
  MOCK_ENTER("uv_coset_add");
  (void)stream;
  if (c == nullptr || (n > 0 && rows == nullptr)) return fail(UV_EINVAL, "null argument");
  mock.ids.assign(ids ? ids : nullptr, ids ? ids + n : nullptr);
  mock.rows.assign(rows, rows + (size_t)n * c->dim);
  c->n += n;
  return UV_OK;
}

int uv_coset_search(const uv_coset *c, const float *queries, int64_t nq, int32_t k,
                    int64_t *ids, float *scores, void *stream) {
  MOCK_ENTER("uv_coset_search");
  (void)queries, (void)stream;
  if (c == nullptr || ids == nullptr || scores == nullptr || k < 1)
    return fail(UV_EINVAL, "bad argument");
  mock.k = k;
  mock.nq = nq;
  for (int64_t i = 0; i < nq * k; i++) {
    ids[i] = (i % k) < c->n ? (i % k) : -1;
    scores[i] = 5.0f - (float)(i % k);
  }
  return UV_OK;
}

int uv_coset_len(const uv_coset *c, int64_t *n) {
  MOCK_ENTER("uv_coset_len");
  if (c == nullptr || n == nullptr) return fail(UV_EINVAL, "null argument");
  *n = c->n;
  return UV_OK;
}

int uv_coset_mem_bytes(const uv_coset *c, int64_t *bytes) {
  MOCK_ENTER("uv_coset_mem_bytes");
  if (c == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = c->n * 50;
  return UV_OK;
}

int uv_coset_model_bytes(const uv_coset *c, int64_t *bytes) {
  MOCK_ENTER("uv_coset_model_bytes");
  if (c == nullptr || bytes == nullptr) return fail(UV_EINVAL, "null argument");
  *bytes = 777;
  return UV_OK;
}

int uv_coset_reconstruct(const uv_coset *c, const float *rows, int64_t n, float *out,
                         void *stream) {
  MOCK_ENTER("uv_coset_reconstruct");
  (void)stream;
  if (c == nullptr || rows == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  for (int64_t i = 0; i < n * c->dim; i++) out[i] = -rows[i];
  return UV_OK;
}

}  // extern "C"
