/*
 * ultravec_b200.hpp -- C++17 host API of the B200 trellis codec, header only,
 * over the C ABI of ultravec_b200.h.
 *
 * It restates, under the reference crate's names and argument meanings, the
 * interfaces a caller of the trellis hot path uses:
 *   VectorBackend, CandidateScorer, PreparedQuery, MemoryBreakdown
 *                                      (src/lib.rs:55-155)
 *   TrellisConfig, TrellisQuantizer    (src/trellis.rs:352-458, 645-1000,
 *                                       2036-2247)
 *   IvfCodec, IvfIndex                 (src/ivf.rs:41-60, 98-290)
 *   kmeans, assign                     (src/bench.rs:298-349, src/ivf.rs:405-421)
 *   CosetTrellis                       (src/coset_trellis.rs:98-530)
 * so that code written against the reference's traits ports line for line.
 *
 * Error behaviour.  Where the reference panics (assert_eq! on a dimension
 * mismatch, a position outside the index) or where the device reports a
 * failure, these calls throw ultravec::Error with the library's status code
 * and message.  A query with |q| < f32::EPSILON gives an empty result, as in
 * the reference (src/trellis.rs:2124-2127).
 *
 * Threading.  search / prepare / score are const and may run concurrently
 * from several threads on one index; add, add_batch, reserve and the builder
 * methods must not overlap searches of the same index (the reference's
 * &self / &mut self split).
 *
 * Every call here is a single-row (or single-query) convenience, as the
 * reference's trait methods are; the *_batch forms pass whole batches to
 * the GPU in one call and are the ones to use for throughput.
 */
#ifndef ULTRAVEC_B200_HPP
#define ULTRAVEC_B200_HPP

#include "ultravec_b200.h"

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace ultravec {

using ItemId = int64_t;                              // src/lib.rs:45
using Hits = std::vector<std::pair<ItemId, float>>;  // search results, best first

/* A failed call: the library's status (UV_EINVAL, UV_ENOMEM, UV_ECUDA,
 * UV_ETIMEDOUT, UV_EUNSUPPORTED) and its message. */
class Error : public std::runtime_error {
 public:
  Error(int code, const std::string &msg)
      : std::runtime_error("ultravec_b200 error " + std::to_string(code) + ": " + msg),
        code_(code) {}
  int code() const noexcept { return code_; }

 private:
  int code_;
};

namespace detail {

inline void check(int rc) {
  if (rc != UV_OK) {
    const char *m = uv_last_error();
    throw Error(rc, m != nullptr ? m : "");
  }
}

inline void require(bool ok, const char *what) {
  if (!ok) throw Error(UV_EINVAL, what);
}

// rows of equal width dim, one after the other (the reference asserts each
// row's length, src/trellis.rs:2096, 2114)
inline std::vector<float> flatten(const std::vector<std::vector<float>> &rows, size_t dim) {
  std::vector<float> flat;
  flat.reserve(rows.size() * dim);
  for (const auto &r : rows) {
    require(r.size() == dim, "row length differs from the codec's dimension");
    flat.insert(flat.end(), r.begin(), r.end());
  }
  return flat;
}

// unfilled slots (id -1) are left out: the reference returns fewer hits
inline Hits collect(const int64_t *ids, const float *scores, size_t k) {
  Hits out;
  out.reserve(k);
  for (size_t i = 0; i < k; i++)
    if (ids[i] >= 0) out.emplace_back(ids[i], scores[i]);
  return out;
}

inline long env_long(const char *name, long fallback) {
  const char *v = std::getenv(name);
  if (v == nullptr || *v == '\0') return fallback;
  char *end = nullptr;
  const long x = std::strtol(v, &end, 10);
  return (end != nullptr && *end == '\0') ? x : fallback;
}

inline bool env_is(const char *name, const char *value) {
  const char *v = std::getenv(name);
  return v != nullptr && std::string(v) == value;
}

// l2_norm (src/lib.rs:215-217): the f32 sum of squares from -0.0, in
// order, then the square root.  Each product is rounded by itself (the
// volatile keeps a compiler from fusing it into the add, which rustc never
// does), so the result has the reference's bits under any build flags.
inline float l2_norm(const float *v, size_t n) {
  float s = -0.0f;
  for (size_t i = 0; i < n; i++) {
    volatile float p = v[i] * v[i];
    s = s + p;
  }
  return std::sqrt(s);
}

// the tail of reconstruct_from (src/trellis.rs:1640-1653): the decoded,
// inverse-rotated row normalized, then, for a centered record, recomposed
// as centroid + rnorm * direction and normalized again
inline std::vector<float> unit_direction(std::vector<float> recon, const float *centroid,
                                         float rnorm) {
  const size_t d = recon.size();
  const float n = std::fmax(l2_norm(recon.data(), d), FLT_EPSILON);
  for (auto &x : recon) x = x / n;
  if (centroid == nullptr) return recon;
  for (size_t i = 0; i < d; i++) {
    volatile float p = rnorm * recon[i];
    recon[i] = centroid[i] + p;
  }
  const float nf = std::fmax(l2_norm(recon.data(), d), FLT_EPSILON);
  for (auto &x : recon) x = x / nf;
  return recon;
}

struct CodecDel {
  void operator()(uv_codec *c) const { uv_codec_destroy(c); }
};
struct IndexDel {
  void operator()(uv_index *x) const { uv_index_destroy(x); }
};
struct IvfDel {
  void operator()(uv_ivf *x) const { uv_ivf_destroy(x); }
};
struct PreparedDel {
  void operator()(uv_prepared *x) const { uv_prepared_destroy(x); }
};
struct CosetDel {
  void operator()(uv_coset *x) const { uv_coset_destroy(x); }
};

}  // namespace detail

/* ---- the reference's traits (src/lib.rs:55-155) ------------------------- */

struct MemoryBreakdown {
  size_t code_bytes = 0;
  size_t model_bytes = 0;
  size_t index_bytes = 0;
  size_t cache_bytes = 0;
  size_t total_resident_bytes() const {
    return code_bytes + model_bytes + index_bytes + cache_bytes;
  }
};

class PreparedQuery {
 public:
  virtual ~PreparedQuery() = default;
  virtual float score_at(size_t index) = 0;
};

class CandidateScorer {
 public:
  virtual ~CandidateScorer() = default;
  virtual std::unique_ptr<PreparedQuery> prepare(const std::vector<float> &query) const = 0;
  virtual size_t scored_len() const = 0;
  virtual size_t scorer_model_bytes() const = 0;
};

class VectorBackend {
 public:
  virtual ~VectorBackend() = default;
  virtual size_t dimensions() const = 0;
  virtual size_t len() const = 0;
  bool is_empty() const { return len() == 0; }
  virtual void add(ItemId id, const std::vector<float> &embedding) = 0;
  // ids 0..n, order preserving (the default delegates to add)
  virtual void add_batch(const std::vector<std::vector<float>> &embeddings) {
    for (size_t i = 0; i < embeddings.size(); i++) add((ItemId)i, embeddings[i]);
  }
  virtual void reserve(size_t /*additional*/) {}
  virtual Hits search(const std::vector<float> &query, size_t limit) const = 0;
  virtual size_t mem_bytes() const = 0;
  virtual MemoryBreakdown memory_breakdown() const {
    MemoryBreakdown m;
    m.code_bytes = mem_bytes();
    return m;
  }
  virtual bool is_approximate() const { return false; }
  // the unit direction the codec stores for x, or nothing for a backend
  // that cannot reconstruct
  virtual std::optional<std::vector<float>> reconstruct_unit(const std::vector<float> &) const {
    return std::nullopt;
  }
};

/* ---- TrellisConfig (src/trellis.rs:352-391) ---------------------------- */

struct TrellisConfig {
  size_t dim = 0;
  uint8_t bits = 0;
  uint8_t mem = 0;
  uint64_t rotation_seed = 42;
  uint8_t rotation_rounds = 3;
  uint8_t start_bits = 0;
  uint8_t rescale_bits = 0;
  // The reference's recon-cache mode (false) and codes-only mode (true)
  // give the same scores (src/trellis.rs:1494-1502: "the products are
  // identical; only decode timing differs"); the device index is codes-only
  // either way, so the flag changes nothing here.
  bool codes_only = false;
  // Not in the reference's TrellisConfig: the anisotropic metric weight it
  // reads from ULTRAVEC_TRELLIS_ANISO, and the GPU the codec lives on.
  float branch_lambda = 0.0f;
  int device = 0;

  // TrellisConfig::new: seed 42, three rounds, full free start, exact rescale
  static TrellisConfig make(size_t dim, uint8_t bits, uint8_t mem) {
    TrellisConfig c;
    c.dim = dim;
    c.bits = bits;
    c.mem = mem;
    c.start_bits = mem;
    return c;
  }

  // the configuration TrellisQuantizer::new(dim, bits) builds from the
  // environment (src/trellis.rs:460-540): ULTRAVEC_TRELLIS_MEM (default 12),
  // _ANISO, _START_BITS (at most mem) and _RESCALE_BITS.  Knobs of research
  // arms that are not built (beam, residual sketch, tail biting, the 1MAD
  // code, vector trellis V > 1, fixed start) throw UV_EUNSUPPORTED when set
  // to anything but their default.
  static TrellisConfig from_env(size_t dim, uint8_t bits, int device = 0) {
    const long mem = detail::env_long("ULTRAVEC_TRELLIS_MEM", 12);
    if (detail::env_long("ULTRAVEC_TRELLIS_BEAM", 0) != 0 ||
        detail::env_long("ULTRAVEC_TRELLIS_RESID", 0) != 0 ||
        detail::env_is("ULTRAVEC_TRELLIS_TAILBITE", "1") ||
        detail::env_is("ULTRAVEC_TRELLIS_CODE", "1mad") ||
        detail::env_long("ULTRAVEC_TRELLIS_V", 1) > 1 ||
        detail::env_is("ULTRAVEC_TRELLIS_FIXEDSTART", "1"))
      throw Error(UV_EUNSUPPORTED, "this ULTRAVEC_TRELLIS_* research arm is not built");
    detail::require(mem >= 1 && mem <= 24, "ULTRAVEC_TRELLIS_MEM out of range");
    TrellisConfig cfg = make(dim, bits, (uint8_t)mem);
    const char *aniso = std::getenv("ULTRAVEC_TRELLIS_ANISO");
    if (aniso != nullptr && *aniso != '\0') cfg.branch_lambda = std::strtof(aniso, nullptr);
    cfg.start_bits = (uint8_t)std::min<long>(
        detail::env_long("ULTRAVEC_TRELLIS_START_BITS", mem), mem);
    cfg.rescale_bits = (uint8_t)detail::env_long("ULTRAVEC_TRELLIS_RESCALE_BITS", 0);
    cfg.device = device;
    return cfg;
  }

  uv_config raw() const {
    uv_config r;
    uv_config_default(&r, (int32_t)dim, (int32_t)bits, (int32_t)mem);
    r.rotation_seed = rotation_seed;
    r.rotation_rounds = rotation_rounds;
    r.start_bits = start_bits;
    r.rescale_bits = rescale_bits;
    r.branch_lambda = branch_lambda;
    r.device = device;
    return r;
  }
};

/* Search metric of the batched calls: cosine is the reference's search; MIPS
 * is its inner-product harness (src/bench.rs:1029-1045: the cosine score
 * times the row's exact norm, re-ranked), with the norms stored at add. */
enum class Metric : int32_t { Cosine = UV_SEARCH_COSINE, Mips = UV_SEARCH_MIPS };

/* Results of a batched search: nq x k, row-major, unfilled slots id -1 and
 * score -inf. */
struct SearchBatch {
  size_t nq = 0, k = 0;
  std::vector<ItemId> ids;
  std::vector<float> scores;
  Hits row(size_t q) const { return detail::collect(&ids[q * k], &scores[q * k], k); }
};

/* ---- TrellisQuantizer: the codec and its codes-only index -------------- */

class TrellisQuantizer : public VectorBackend, public CandidateScorer {
 public:
  // TrellisQuantizer::new(dim, bits).with_codes_only(true): the research
  // harness's constructor, which reads its knobs from the environment
  // (src/trellis.rs:418-420, 460-540; TrellisConfig::from_env) and the
  // shortlist knobs ULTRAVEC_TRELLIS_SHORTLIST, _ASYM and _RNORM.
  static TrellisQuantizer make(size_t dim, uint8_t bits, int device = 0) {
    TrellisConfig cfg = TrellisConfig::from_env(dim, bits, device);
    cfg.codes_only = true;
    TrellisQuantizer q = from_config(cfg);
    const long c = detail::env_long("ULTRAVEC_TRELLIS_SHORTLIST", 0);
    if (c > 0) {
      q.sl_c_ = (int32_t)c;
      q.sl_asym_ = detail::env_is("ULTRAVEC_TRELLIS_SHORTLIST_ASYM", "1");
      q.sl_rnorm_ = !detail::env_is("ULTRAVEC_TRELLIS_SHORTLIST_RNORM", "0");
      q.apply_shortlist();
    }
    return q;
  }

  // TrellisQuantizer::from_config: no environment read
  static TrellisQuantizer from_config(const TrellisConfig &cfg) {
    detail::require(cfg.mem >= 1, "trellis memory must be at least one bit");
    const uv_config raw = cfg.raw();
    uv_codec *c = nullptr;
    detail::check(uv_codec_create(&raw, &c));
    std::unique_ptr<uv_codec, detail::CodecDel> codec(c);
    uv_index *x = nullptr;
    detail::check(uv_index_create(codec.get(), &x));
    return TrellisQuantizer(std::move(codec), std::unique_ptr<uv_index, detail::IndexDel>(x),
                            cfg);
  }

  TrellisQuantizer(TrellisQuantizer &&) noexcept = default;
  // the old index goes before the old codec whose tables it reads
  TrellisQuantizer &operator=(TrellisQuantizer &&o) noexcept {
    if (this != &o) {
      index_ = std::move(o.index_);
      codec_ = std::move(o.codec_);
      cfg_ = o.cfg_;
      centroids_ = std::move(o.centroids_);
      sl_c_ = o.sl_c_;
      sl_asym_ = o.sl_asym_;
      sl_rnorm_ = o.sl_rnorm_;
    }
    return *this;
  }
  TrellisQuantizer(const TrellisQuantizer &) = delete;
  TrellisQuantizer &operator=(const TrellisQuantizer &) = delete;

  /* -- builders (the reference's consuming `with_*`) -- */

  // both modes score alike (see TrellisConfig::codes_only)
  TrellisQuantizer &with_codes_only(bool on) & {
    cfg_.codes_only = on;
    return *this;
  }
  TrellisQuantizer with_codes_only(bool on) && { return std::move(with_codes_only(on)); }

  // with_centroids (src/trellis.rs:952-956): centered records, on an empty index
  TrellisQuantizer &with_centroids(const std::vector<std::vector<float>> &centroids) & {
    std::vector<float> flat = detail::flatten(centroids, cfg_.dim);
    detail::check(uv_index_set_centroids(index_.get(), flat.data(), (int32_t)centroids.size()));
    centroids_ = std::move(flat);
    return *this;
  }
  TrellisQuantizer with_centroids(const std::vector<std::vector<float>> &centroids) && {
    return std::move(with_centroids(centroids));
  }
  // with_mean (src/trellis.rs:746-748): one centroid
  TrellisQuantizer &with_mean(const std::vector<float> &mean) & {
    return with_centroids(std::vector<std::vector<float>>{mean});
  }
  TrellisQuantizer with_mean(const std::vector<float> &mean) && {
    return std::move(with_mean(mean));
  }

  // with_shortlist / _asym / _rnorm (src/trellis.rs:805-851), on an empty index
  TrellisQuantizer &with_shortlist(size_t c) & {
    sl_c_ = (int32_t)c;
    apply_shortlist();
    return *this;
  }
  TrellisQuantizer with_shortlist(size_t c) && { return std::move(with_shortlist(c)); }
  TrellisQuantizer &with_shortlist_asym(bool on) & {
    sl_asym_ = on;
    apply_shortlist();
    return *this;
  }
  TrellisQuantizer with_shortlist_asym(bool on) && { return std::move(with_shortlist_asym(on)); }
  TrellisQuantizer &with_shortlist_rnorm(bool on) & {
    sl_rnorm_ = on;
    apply_shortlist();
    return *this;
  }
  TrellisQuantizer with_shortlist_rnorm(bool on) && {
    return std::move(with_shortlist_rnorm(on));
  }

  /* -- record API (src/trellis.rs:645-743, 970-990) -- */

  std::vector<uint32_t> code_table_bits() const {
    std::vector<uint32_t> out((size_t)1 << (cfg_.mem + cfg_.bits));
    detail::check(uv_codec_code_table_bits(codec_.get(), out.data(), (int64_t)out.size()));
    return out;
  }
  uint8_t memory_bits() const {
    int32_t m = 0;
    detail::check(uv_codec_memory_bits(codec_.get(), &m));
    return (uint8_t)m;
  }
  std::vector<std::vector<float>> rotation_sign_rounds() const {
    std::vector<float> flat((size_t)cfg_.rotation_rounds * cfg_.dim);
    detail::check(
        uv_codec_rotation_sign_rounds(codec_.get(), flat.data(), (int64_t)flat.size()));
    std::vector<std::vector<float>> out(cfg_.rotation_rounds);
    for (size_t r = 0; r < out.size(); r++)
      out[r].assign(flat.begin() + r * cfg_.dim, flat.begin() + (r + 1) * cfg_.dim);
    return out;
  }
  // encode_codes(row) -> (packed emissions, start state)
  std::pair<std::vector<uint8_t>, uint32_t> encode_codes(const std::vector<float> &row) const {
    detail::require(row.size() == cfg_.dim, "row length differs from the codec's dimension");
    std::vector<uint8_t> codes(code_bytes());
    uint32_t start = 0;
    float rescale = 0.0f;
    detail::check(uv_encode(codec_.get(), row.data(), 1, nullptr, 0, codes.data(), &start,
                            &rescale, nullptr, nullptr, nullptr));
    return {std::move(codes), start};
  }
  // rotate(unit): the forward rotation of a unit row
  std::vector<float> rotate(const std::vector<float> &unit) const {
    detail::require(unit.size() == cfg_.dim, "row length differs from the codec's dimension");
    std::vector<float> out(cfg_.dim);
    detail::check(uv_rotate(codec_.get(), unit.data(), 1, out.data(), nullptr));
    return out;
  }
  // encode_rotated(u_r): rows already rotated to unit u_r
  std::pair<std::vector<uint8_t>, uint32_t> encode_rotated(const std::vector<float> &u_r) const {
    detail::require(u_r.size() == cfg_.dim, "row length differs from the codec's dimension");
    std::vector<uint8_t> codes(code_bytes());
    uint32_t start = 0;
    detail::check(
        uv_encode_rotated(codec_.get(), u_r.data(), 1, codes.data(), &start, nullptr));
    return {std::move(codes), start};
  }
  // decode_codes: table values by window, inverse rotated, not normalized
  std::vector<float> decode_codes(const std::vector<uint8_t> &codes, uint32_t start) const {
    detail::require(codes.size() == code_bytes(), "record length differs from the codec's");
    std::vector<float> out(cfg_.dim);
    detail::check(uv_decode(codec_.get(), codes.data(), &start, 1, out.data(), nullptr));
    return out;
  }
  // window_at(codes, start, i)
  uint32_t window_at(const std::vector<uint8_t> &codes, uint32_t start, size_t i) const {
    detail::require(codes.size() == code_bytes(), "record length differs from the codec's");
    detail::require(i < cfg_.dim, "window index past the record");
    std::vector<uint32_t> w(cfg_.dim);
    detail::check(uv_windows(codec_.get(), codes.data(), &start, 1, w.data(), nullptr));
    return w[i];
  }
  // encode_digest(vectors): XOR-folded FNV-1a of every row's record
  uint64_t encode_digest(const std::vector<std::vector<float>> &vectors) const {
    const std::vector<float> flat = detail::flatten(vectors, cfg_.dim);
    const size_t n = vectors.size();
    std::vector<uint8_t> codes(n * code_bytes());
    std::vector<uint32_t> start(n);
    std::vector<float> rescale(n);
    detail::check(uv_encode(codec_.get(), n ? flat.data() : nullptr, (int64_t)n, nullptr, 0,
                            codes.data(), start.data(), rescale.data(), nullptr, nullptr,
                            nullptr));
    uint64_t h = 0;
    detail::check(uv_digest(codec_.get(), codes.data(), start.data(), (int64_t)n, &h, nullptr));
    return h;
  }

  /* -- VectorBackend (src/trellis.rs:2088-2247) -- */

  size_t dimensions() const override { return cfg_.dim; }
  size_t len() const override {
    int64_t n = 0;
    detail::check(uv_index_len(index_.get(), &n));
    return (size_t)n;
  }
  void add(ItemId id, const std::vector<float> &embedding) override {
    detail::require(embedding.size() == cfg_.dim,
                    "row length differs from the codec's dimension");
    detail::check(uv_index_add(index_.get(), &id, embedding.data(), 1, nullptr));
  }
  void add_batch(const std::vector<std::vector<float>> &embeddings) override {
    const std::vector<float> flat = detail::flatten(embeddings, cfg_.dim);
    detail::check(uv_index_add_batch(index_.get(), embeddings.empty() ? nullptr : flat.data(),
                                     (int64_t)embeddings.size(), nullptr));
  }
  void reserve(size_t additional) override {
    detail::check(uv_index_reserve(index_.get(), (int64_t)additional));
  }
  // any limit: above 128 every record is ranked, so search(q, len()) returns
  // the whole index in order (the MIPS harness's call, src/bench.rs:1033)
  Hits search(const std::vector<float> &query, size_t limit) const override {
    return search_metric(query, limit, Metric::Cosine);
  }
  size_t mem_bytes() const override {
    int64_t b = 0;
    detail::check(uv_index_mem_bytes(index_.get(), &b));
    return (size_t)b;
  }
  MemoryBreakdown memory_breakdown() const override {
    MemoryBreakdown m;
    m.code_bytes = mem_bytes();
    m.model_bytes = scorer_model_bytes();
    return m;
  }
  bool is_approximate() const override { return true; }
  // reconstruct_unit (src/trellis.rs:2241-2246): encode x, decode the
  // record, normalize (recomposed with its centroid when centered)
  std::optional<std::vector<float>> reconstruct_unit(const std::vector<float> &x) const override {
    detail::require(x.size() == cfg_.dim, "row length differs from the codec's dimension");
    const int32_t n_cen = (int32_t)(centroids_.size() / cfg_.dim);
    std::vector<uint8_t> codes(code_bytes());
    uint32_t start = 0, cidx = 0;
    float rescale = 0.0f, rnorm = 1.0f;
    detail::check(uv_encode(codec_.get(), x.data(), 1, n_cen ? centroids_.data() : nullptr, n_cen,
                            codes.data(), &start, &rescale, &rnorm, &cidx, nullptr));
    std::vector<float> recon(cfg_.dim);
    detail::check(uv_decode(codec_.get(), codes.data(), &start, 1, recon.data(), nullptr));
    return detail::unit_direction(std::move(recon),
                                  n_cen ? centroids_.data() + (size_t)cidx * cfg_.dim : nullptr,
                                  rnorm);
  }

  // the inner-product harness's ranking for one query (src/bench.rs:1029-1045)
  Hits search_mips(const std::vector<float> &query, size_t limit) const {
    return search_metric(query, limit, Metric::Mips);
  }

  /* -- batched forms: one GPU call per batch -- */

  // rows n x dim (host or device) under ids n, or under 0 .. n - 1 as
  // add_batch gives them when ids is null
  void add_rows(const float *rows, size_t n, const ItemId *ids = nullptr, void *stream = nullptr) {
    if (ids == nullptr)
      detail::check(uv_index_add_batch(index_.get(), rows, (int64_t)n, stream));
    else
      detail::check(uv_index_add(index_.get(), ids, rows, (int64_t)n, stream));
  }
  SearchBatch search_batch(const float *queries, size_t nq, size_t k,
                           Metric metric = Metric::Cosine, void *stream = nullptr) const {
    SearchBatch out;
    out.nq = nq;
    out.k = k;
    out.ids.assign(nq * k, -1);
    out.scores.assign(nq * k, 0.0f);
    if (nq == 0 || k == 0) return out;
    detail::require(k <= (size_t)INT32_MAX, "k too large");
    detail::check(uv_index_search(index_.get(), queries, (int64_t)nq, (int32_t)k,
                                  (int32_t)metric, out.ids.data(), out.scores.data(), stream));
    return out;
  }

  /* -- CandidateScorer (src/trellis.rs:2036-2086).  A PreparedQuery reads
   *    this index's arrays when it scores: it must not outlive the index (in
   *    the reference it borrows it). -- */

  std::unique_ptr<PreparedQuery> prepare(const std::vector<float> &query) const override {
    detail::require(query.size() == cfg_.dim, "query length differs from the codec's dimension");
    uv_prepared *p = nullptr;
    detail::check(uv_index_prepare(index_.get(), query.data(), 1, &p, nullptr));
    return std::unique_ptr<PreparedQuery>(new Prepared(p));
  }
  size_t scored_len() const override { return len(); }
  size_t scorer_model_bytes() const override {
    int64_t b = 0;
    detail::check(uv_index_scorer_model_bytes(index_.get(), &b));
    return (size_t)b;
  }

  /* -- the index file (build once, search many) -- */

  void save(const std::string &path) const {
    detail::check(uv_index_save(index_.get(), path.c_str()));
  }
  static TrellisQuantizer load(const TrellisConfig &cfg, const std::string &path) {
    const uv_config raw = cfg.raw();
    uv_codec *c = nullptr;
    detail::check(uv_codec_create(&raw, &c));
    std::unique_ptr<uv_codec, detail::CodecDel> codec(c);
    uv_index *x = nullptr;
    detail::check(uv_index_load(codec.get(), path.c_str(), &x));
    return TrellisQuantizer(std::move(codec), std::unique_ptr<uv_index, detail::IndexDel>(x),
                            cfg);
  }

  const TrellisConfig &config() const { return cfg_; }
  const uv_codec *codec_handle() const { return codec_.get(); }
  uv_index *index_handle() const { return index_.get(); }

  size_t code_bytes() const {
    int32_t cb = 0, sb = 0, rb = 0;
    detail::check(uv_codec_record_bytes(codec_.get(), &cb, &sb, &rb));
    return (size_t)cb;
  }

 private:
  class Prepared : public PreparedQuery {
   public:
    explicit Prepared(uv_prepared *p) : p_(p) {}
    float score_at(size_t index) override {
      const int64_t pos = (int64_t)index;
      float s = 0.0f;
      detail::check(uv_prepared_score(p_.get(), nullptr, &pos, 1, &s, nullptr));
      return s;
    }

   private:
    std::unique_ptr<uv_prepared, detail::PreparedDel> p_;
  };

  TrellisQuantizer(std::unique_ptr<uv_codec, detail::CodecDel> codec,
                   std::unique_ptr<uv_index, detail::IndexDel> index, const TrellisConfig &cfg)
      : codec_(std::move(codec)), index_(std::move(index)), cfg_(cfg) {}

  Hits search_metric(const std::vector<float> &query, size_t limit, Metric metric) const {
    detail::require(query.size() == cfg_.dim, "query length differs from the codec's dimension");
    const size_t k = std::min(limit, len());
    if (k == 0) return {};
    const SearchBatch b = search_batch(query.data(), 1, k, metric);
    return b.row(0);
  }

  void apply_shortlist() {
    detail::check(uv_index_set_shortlist(index_.get(), sl_c_, sl_asym_ ? 1 : 0,
                                         sl_rnorm_ ? 1 : 0));
  }

  // declared codec first, so that the index, which reads the codec's
  // tables, is destroyed before it
  std::unique_ptr<uv_codec, detail::CodecDel> codec_;
  std::unique_ptr<uv_index, detail::IndexDel> index_;
  TrellisConfig cfg_;
  std::vector<float> centroids_;  // with_centroids, flattened (reconstruct_unit)
  int32_t sl_c_ = 0;
  bool sl_asym_ = false, sl_rnorm_ = true;
};

/* ---- the coarse quantizer (src/bench.rs:298-349, src/ivf.rs:405-421) ---- */

// kmeans(dim, db, nlist, seed): splitmix64 initial picks, 5 Lloyd rounds
inline std::vector<std::vector<float>> kmeans(size_t dim, const std::vector<std::vector<float>> &db,
                                              size_t nlist, uint64_t seed, int device = 0) {
  const std::vector<float> flat = detail::flatten(db, dim);
  std::vector<float> cen(nlist * dim);
  detail::check(uv_kmeans(device, db.empty() ? nullptr : flat.data(), (int64_t)db.size(),
                          (int32_t)dim, (int32_t)nlist, seed, 5, cen.data(), nullptr));
  std::vector<std::vector<float>> out(nlist);
  for (size_t j = 0; j < nlist; j++) out[j].assign(cen.begin() + j * dim, cen.begin() + (j + 1) * dim);
  return out;
}

// the first strict maximum of <row / |row|, c_j> for every row
inline std::vector<uint32_t> assign(const std::vector<std::vector<float>> &db,
                                    const std::vector<std::vector<float>> &centroids,
                                    int device = 0) {
  detail::require(!centroids.empty(), "no centroids");
  const size_t dim = centroids[0].size();
  const std::vector<float> flat = detail::flatten(db, dim);
  const std::vector<float> cen = detail::flatten(centroids, dim);
  std::vector<uint32_t> out(db.size());
  detail::check(uv_ivf_assign(device, db.empty() ? nullptr : flat.data(), (int64_t)db.size(),
                              (int32_t)dim, cen.data(), (int32_t)centroids.size(), out.data(),
                              nullptr));
  return out;
}

/* ---- IvfCodec / IvfIndex (src/ivf.rs:41-60, 98-290) -------------------- */

// The posting-list codecs of the trellis path: TrellisCodes and
// TrellisShortlist{c, asym, rnorm}.  TrellisRecon scores exactly as
// TrellisCodes (see TrellisConfig::codes_only) and maps onto it; the
// comparator codecs (Baseline, Rabitq, Pvq) are not part of this library.
struct IvfCodec {
  enum class Kind { TrellisRecon, TrellisCodes, TrellisShortlist };
  Kind kind = Kind::TrellisCodes;
  size_t c = 0;
  bool asym = false, rnorm = true;

  static IvfCodec trellis_recon() { return IvfCodec{Kind::TrellisRecon, 0, false, true}; }
  static IvfCodec trellis_codes() { return IvfCodec{Kind::TrellisCodes, 0, false, true}; }
  static IvfCodec trellis_shortlist(size_t c, bool asym, bool rnorm) {
    return IvfCodec{Kind::TrellisShortlist, c, asym, rnorm};
  }
  std::string label() const {
    switch (kind) {
      case Kind::TrellisRecon: return "trellis_recon";
      case Kind::TrellisCodes: return "trellis_codes";
      case Kind::TrellisShortlist: return "trellis_shortlist_c" + std::to_string(c);
    }
    return "";
  }
};

class IvfIndex {
 public:
  // IvfIndex::build(dim, db, centroids, assign, codec, bits): each list's
  // codec is TrellisQuantizer::new(dim, bits) (its knobs from the
  // environment, TrellisConfig::from_env; the shortlist from `codec`, set
  // explicitly as the reference does), centered on its centroid when
  // ULTRAVEC_IVF_CENTER=1 (src/ivf.rs:98-150)
  static IvfIndex build(size_t dim, const std::vector<std::vector<float>> &db,
                        const std::vector<std::vector<float>> &centroids,
                        const std::vector<uint32_t> &assign, IvfCodec codec, uint8_t bits,
                        int device = 0) {
    const TrellisConfig cfg = TrellisConfig::from_env(dim, bits, device);
    return build_with(cfg, db, centroids, assign, codec,
                      detail::env_is("ULTRAVEC_IVF_CENTER", "1"));
  }

  // the same with an explicit configuration and centering, no environment read
  static IvfIndex build_with(const TrellisConfig &cfg, const std::vector<std::vector<float>> &db,
                             const std::vector<std::vector<float>> &centroids,
                             const std::vector<uint32_t> &assign, IvfCodec codec,
                             bool centered) {
    detail::require(assign.size() == db.size(), "one assignment per row");
    const uv_config raw = cfg.raw();
    uv_codec *c = nullptr;
    detail::check(uv_codec_create(&raw, &c));
    std::unique_ptr<uv_codec, detail::CodecDel> cd(c);
    const std::vector<float> cen = detail::flatten(centroids, cfg.dim);
    uv_ivf *x = nullptr;
    detail::check(uv_ivf_create(cd.get(), cen.data(), (int32_t)centroids.size(),
                                centered ? 1 : 0, &x));
    std::unique_ptr<uv_ivf, detail::IvfDel> ivf(x);
    if (codec.kind == IvfCodec::Kind::TrellisShortlist)
      detail::check(uv_ivf_set_shortlist(ivf.get(), (int32_t)codec.c, codec.asym ? 1 : 0,
                                         codec.rnorm ? 1 : 0));
    const std::vector<float> flat = detail::flatten(db, cfg.dim);
    detail::check(uv_ivf_build(ivf.get(), db.empty() ? nullptr : flat.data(),
                               (int64_t)db.size(), assign.data(), nullptr, nullptr));
    return IvfIndex(std::move(cd), std::move(ivf), cfg.dim, codec);
  }

  IvfIndex(IvfIndex &&) noexcept = default;
  // the old lists go before the old codec whose tables they read
  IvfIndex &operator=(IvfIndex &&o) noexcept {
    if (this != &o) {
      ivf_ = std::move(o.ivf_);
      codec_handle_ = std::move(o.codec_handle_);
      dim_ = o.dim_;
      codec_ = o.codec_;
    }
    return *this;
  }
  IvfIndex(const IvfIndex &) = delete;
  IvfIndex &operator=(const IvfIndex &) = delete;

  // search(query, k, nprobe): the best k over the nprobe nearest lists
  // (k <= 128)
  Hits search(const std::vector<float> &query, size_t k, size_t nprobe) const {
    detail::require(query.size() == dim_, "query length differs from the index's dimension");
    if (k == 0) return {};
    const SearchBatch b = search_batch(query.data(), 1, k, nprobe);
    return b.row(0);
  }

  // search_with_rerank(query, k, nprobe, rdepth, db): the codec's top
  // max(rdepth, k) re-scored by exact cosine against the fp32 rows
  Hits search_with_rerank(const std::vector<float> &query, size_t k, size_t nprobe,
                          size_t rdepth, const std::vector<std::vector<float>> &db) const {
    const std::vector<float> flat = detail::flatten(db, dim_);
    return search_with_rerank(query, k, nprobe, rdepth, flat.data(), db.size());
  }
  // the same over rows db (n_db x dim, host or device: device rows avoid
  // staging them per call)
  Hits search_with_rerank(const std::vector<float> &query, size_t k, size_t nprobe,
                          size_t rdepth, const float *db, size_t n_db) const {
    detail::require(query.size() == dim_, "query length differs from the index's dimension");
    if (k == 0) return {};
    std::vector<int64_t> ids(k, -1);
    std::vector<float> scores(k, 0.0f);
    detail::check(uv_ivf_search_rerank(ivf_.get(), query.data(), 1, (int32_t)k,
                                       (int32_t)nprobe, (int32_t)rdepth, db, (int64_t)n_db,
                                       ids.data(), scores.data(), nullptr));
    return detail::collect(ids.data(), scores.data(), k);
  }

  SearchBatch search_batch(const float *queries, size_t nq, size_t k, size_t nprobe,
                           void *stream = nullptr) const {
    SearchBatch out;
    out.nq = nq;
    out.k = k;
    out.ids.assign(nq * k, -1);
    out.scores.assign(nq * k, 0.0f);
    if (nq == 0 || k == 0) return out;
    detail::check(uv_ivf_search(ivf_.get(), queries, (int64_t)nq, (int32_t)k, (int32_t)nprobe,
                                out.ids.data(), out.scores.data(), stream));
    return out;
  }

  size_t len() const {
    int64_t n = 0;
    detail::check(uv_ivf_len(ivf_.get(), &n));
    return (size_t)n;
  }
  size_t nlist() const {
    int32_t n = 0;
    detail::check(uv_ivf_nlist(ivf_.get(), &n));
    return (size_t)n;
  }
  size_t mem_bytes() const {
    int64_t b = 0;
    detail::check(uv_ivf_mem_bytes(ivf_.get(), &b));
    return (size_t)b;
  }
  MemoryBreakdown memory_breakdown() const {
    MemoryBreakdown m;
    m.code_bytes = mem_bytes();
    m.model_bytes = nlist() * dim_ * sizeof(float);  // the centroids
    return m;
  }
  const IvfCodec &codec() const { return codec_; }
  uv_ivf *handle() const { return ivf_.get(); }

 private:
  IvfIndex(std::unique_ptr<uv_codec, detail::CodecDel> codec,
           std::unique_ptr<uv_ivf, detail::IvfDel> ivf, size_t dim, IvfCodec kind)
      : codec_handle_(std::move(codec)), ivf_(std::move(ivf)), dim_(dim), codec_(kind) {}

  // declared codec first, so that the lists are destroyed before it
  std::unique_ptr<uv_codec, detail::CodecDel> codec_handle_;
  std::unique_ptr<uv_ivf, detail::IvfDel> ivf_;
  size_t dim_;
  IvfCodec codec_;
};

/* ---- CosetTrellis (src/coset_trellis.rs) --------------------------------- */

// The reference's research arm behind ULTRAVEC_COSET_TRELLIS=1: trellis-coded
// quantization over the eight cosets of an E8 sublattice, one handle holding
// codec and entries.
class CosetTrellis : public VectorBackend {
 public:
  // CosetTrellis::new(dim, bits) (src/coset_trellis.rs:116-190): dim % 8 ==
  // 0, bits 1..3, memory from ULTRAVEC_TRELLIS_MEM (default 12, clamped to
  // 1..20), seed 42, three rotation rounds
  static CosetTrellis make(size_t dim, uint8_t bits, int device = 0) {
    const long mem = std::min(20L, std::max(1L, detail::env_long("ULTRAVEC_TRELLIS_MEM", 12)));
    return with_params(dim, bits, (uint8_t)mem, 42, 3, device);
  }
  static CosetTrellis with_params(size_t dim, uint8_t bits, uint8_t mem, uint64_t rotation_seed,
                                  uint8_t rotation_rounds, int device = 0) {
    uv_coset *c = nullptr;
    detail::check(uv_coset_create((int32_t)dim, bits, mem, rotation_seed, rotation_rounds,
                                  device, &c));
    return CosetTrellis(std::unique_ptr<uv_coset, detail::CosetDel>(c), dim);
  }

  CosetTrellis(CosetTrellis &&) noexcept = default;
  CosetTrellis &operator=(CosetTrellis &&) noexcept = default;
  CosetTrellis(const CosetTrellis &) = delete;
  CosetTrellis &operator=(const CosetTrellis &) = delete;

  // with_centroids (192-196), before the first add
  CosetTrellis &with_centroids(const std::vector<std::vector<float>> &centroids) & {
    const std::vector<float> flat = detail::flatten(centroids, dim_);
    detail::check(uv_coset_set_centroids(c_.get(), flat.data(), (int32_t)centroids.size()));
    return *this;
  }
  CosetTrellis with_centroids(const std::vector<std::vector<float>> &centroids) && {
    return std::move(with_centroids(centroids));
  }

  size_t dimensions() const override { return dim_; }
  size_t len() const override {
    int64_t n = 0;
    detail::check(uv_coset_len(c_.get(), &n));
    return (size_t)n;
  }
  void add(ItemId id, const std::vector<float> &embedding) override {
    detail::require(embedding.size() == dim_, "row length differs from the codec's dimension");
    detail::check(uv_coset_add(c_.get(), &id, embedding.data(), 1, nullptr));
  }
  // ids 0..n, as the reference's add_batch assigns them (454-469)
  void add_batch(const std::vector<std::vector<float>> &embeddings) override {
    const std::vector<float> flat = detail::flatten(embeddings, dim_);
    detail::check(uv_coset_add(c_.get(), nullptr, embeddings.empty() ? nullptr : flat.data(),
                               (int64_t)embeddings.size(), nullptr));
  }
  // any limit (the reference sorts every score and truncates)
  Hits search(const std::vector<float> &query, size_t limit) const override {
    detail::require(query.size() == dim_, "query length differs from the codec's dimension");
    const size_t k = std::min(limit, len());
    if (k == 0) return {};
    std::vector<int64_t> ids(k, -1);
    std::vector<float> scores(k, 0.0f);
    detail::require(k <= (size_t)INT32_MAX, "k too large");
    detail::check(uv_coset_search(c_.get(), query.data(), 1, (int32_t)k, ids.data(),
                                  scores.data(), nullptr));
    return detail::collect(ids.data(), scores.data(), k);
  }
  SearchBatch search_batch(const float *queries, size_t nq, size_t k,
                           void *stream = nullptr) const {
    SearchBatch out;
    out.nq = nq;
    out.k = k;
    out.ids.assign(nq * k, -1);
    out.scores.assign(nq * k, 0.0f);
    if (nq == 0 || k == 0) return out;
    detail::check(uv_coset_search(c_.get(), queries, (int64_t)nq, (int32_t)k, out.ids.data(),
                                  out.scores.data(), stream));
    return out;
  }
  size_t mem_bytes() const override {
    int64_t b = 0;
    detail::check(uv_coset_mem_bytes(c_.get(), &b));
    return (size_t)b;
  }
  MemoryBreakdown memory_breakdown() const override {
    MemoryBreakdown m;
    m.code_bytes = mem_bytes();
    int64_t b = 0;
    detail::check(uv_coset_model_bytes(c_.get(), &b));
    m.model_bytes = (size_t)b;
    return m;
  }
  bool is_approximate() const override { return true; }
  // reconstruct_unit (521-529)
  std::optional<std::vector<float>> reconstruct_unit(const std::vector<float> &x) const override {
    detail::require(x.size() == dim_, "row length differs from the codec's dimension");
    std::vector<float> out(dim_);
    detail::check(uv_coset_reconstruct(c_.get(), x.data(), 1, out.data(), nullptr));
    return out;
  }
  uv_coset *handle() const { return c_.get(); }

 private:
  CosetTrellis(std::unique_ptr<uv_coset, detail::CosetDel> c, size_t dim)
      : c_(std::move(c)), dim_(dim) {}

  std::unique_ptr<uv_coset, detail::CosetDel> c_;
  size_t dim_;
};

}  // namespace ultravec

#endif  // ULTRAVEC_B200_HPP
