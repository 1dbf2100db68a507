// The C++ host API (include/ultravec_b200.hpp) against a CPU stand-in of the
// C ABI (mock_uv.cpp): every call reaches the library with the arguments the
// reference's method means, results come back in the reference's shape,
// failures surface as ultravec::Error with the library's code and message,
// and handles are released index first, codec last.  Prints "ok <checks>"
// and exits 0, or prints the first failed check and exits 1.
#include "mock_uv.h"
#include "ultravec_b200.hpp"

#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

using namespace ultravec;

static int checks = 0;

#define CHECK(cond)                                                          \
  do {                                                                       \
    checks++;                                                                \
    if (!(cond)) {                                                           \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);          \
      std::exit(1);                                                          \
    }                                                                        \
  } while (0)

// runs f, which must throw ultravec::Error with this code
template <class F>
static std::string expect_error(int code, F f) {
  try {
    f();
  } catch (const Error &e) {
    CHECK(e.code() == code);
    return e.what();
  }
  CHECK(!"no ultravec::Error thrown");
  return "";
}

static std::vector<std::vector<float>> rows(size_t n, size_t dim, float base) {
  std::vector<std::vector<float>> r(n, std::vector<float>(dim));
  for (size_t i = 0; i < n; i++)
    for (size_t j = 0; j < dim; j++) r[i][j] = base + (float)(i * dim + j);
  return r;
}

static void config_and_errors() {
  mock.reset();
  TrellisConfig cfg = TrellisConfig::make(16, 2, 6);
  CHECK(cfg.rotation_seed == 42 && cfg.rotation_rounds == 3 && cfg.start_bits == 6 &&
        cfg.rescale_bits == 0 && !cfg.codes_only);
  cfg.rotation_seed = 7;
  cfg.rotation_rounds = 2;
  cfg.start_bits = 5;
  cfg.rescale_bits = 8;
  cfg.branch_lambda = 0.25f;
  {
    TrellisQuantizer q = TrellisQuantizer::from_config(cfg);
    CHECK(mock.cfg.dim == 16 && mock.cfg.bits == 2 && mock.cfg.mem == 6);
    CHECK(mock.cfg.rotation_seed == 7 && mock.cfg.rotation_rounds == 2);
    CHECK(mock.cfg.start_bits == 5 && mock.cfg.rescale_bits == 8);
    CHECK(mock.cfg.branch_lambda == 0.25f && mock.cfg.device == 0);
    CHECK(q.dimensions() == 16 && q.is_empty() && q.is_approximate());
  }
  CHECK(mock.live_codecs == 0 && mock.live_indexes == 0 && mock.order_errors == 0);

  // the reference asserts mem >= 1 before building anything
  mock.reset();
  expect_error(UV_EINVAL, [] { TrellisQuantizer::from_config(TrellisConfig::make(16, 2, 0)); });
  CHECK(!mock.called("uv_codec_create"));

  // a library failure keeps its code and message; nothing leaks
  mock.reset();
  mock.fail_call = "uv_index_create";
  const std::string msg = expect_error(
      UV_ECUDA, [] { TrellisQuantizer::from_config(TrellisConfig::make(16, 2, 6)); });
  CHECK(msg.find("injected failure of uv_index_create") != std::string::npos);
  CHECK(mock.live_codecs == 0);
}

static void environment_constructor() {
  mock.reset();
  setenv("ULTRAVEC_TRELLIS_MEM", "8", 1);
  setenv("ULTRAVEC_TRELLIS_START_BITS", "3", 1);
  setenv("ULTRAVEC_TRELLIS_SHORTLIST", "64", 1);
  setenv("ULTRAVEC_TRELLIS_SHORTLIST_ASYM", "1", 1);
  {
    TrellisQuantizer q = TrellisQuantizer::make(32, 2);
    CHECK(mock.cfg.mem == 8 && mock.cfg.start_bits == 3 && mock.cfg.bits == 2);
    CHECK(mock.sl_c == 64 && mock.sl_asym == 1 && mock.sl_rnorm == 1);
    CHECK(q.config().codes_only);
  }
  unsetenv("ULTRAVEC_TRELLIS_START_BITS");
  unsetenv("ULTRAVEC_TRELLIS_SHORTLIST");
  unsetenv("ULTRAVEC_TRELLIS_SHORTLIST_ASYM");
  unsetenv("ULTRAVEC_TRELLIS_MEM");
  mock.reset();
  {
    TrellisQuantizer q = TrellisQuantizer::make(32, 2);
    CHECK(mock.cfg.mem == 12 && mock.cfg.start_bits == 12);  // the reference's MEM
    CHECK(!mock.called("uv_index_set_shortlist"));
  }
  // research arms that are not built are refused, not silently ignored
  setenv("ULTRAVEC_TRELLIS_BEAM", "4", 1);
  expect_error(UV_EUNSUPPORTED, [] { TrellisQuantizer::make(32, 2); });
  unsetenv("ULTRAVEC_TRELLIS_BEAM");
}

static void backend() {
  mock.reset();
  TrellisQuantizer q = TrellisQuantizer::from_config(TrellisConfig::make(4, 2, 6));
  // dimension mismatches are refused before the library is called
  expect_error(UV_EINVAL, [&] { q.add(3, std::vector<float>(5)); });
  expect_error(UV_EINVAL, [&] { q.add_batch(rows(2, 3, 0.0f)); });
  CHECK(!mock.called("uv_index_add") && !mock.called("uv_index_add_batch"));
  // search of an empty index: no hits, no device call
  CHECK(q.search(std::vector<float>(4, 1.0f), 10).empty());
  CHECK(!mock.called("uv_index_search"));

  q.add(77, std::vector<float>{1, 2, 3, 4});
  CHECK(mock.ids.size() == 1 && mock.ids[0] == 77);
  CHECK(mock.rows == (std::vector<float>{1, 2, 3, 4}));
  q.add_batch(rows(4, 4, 10.0f));
  CHECK(mock.rows.size() == 16 && mock.rows[0] == 10.0f && mock.rows[15] == 25.0f);
  CHECK(q.len() == 5);
  q.reserve(100);
  CHECK(mock.reserved == 100);

  // search(q, limit): k = min(limit, len()), cosine, best first
  const Hits h = q.search(std::vector<float>{0.5f, 0, 0, 0}, 100);
  CHECK(mock.k == 5 && mock.mode == UV_SEARCH_COSINE && mock.nq == 1);
  CHECK(mock.rows == (std::vector<float>{0.5f, 0, 0, 0}));
  CHECK(h.size() == 5 && h[0].first == 0 && h[0].second == 10.0f && h[4].second == 6.0f);
  // the inner-product harness's ranking
  const Hits m = q.search_mips(std::vector<float>{0.5f, 0, 0, 0}, 3);
  CHECK(mock.k == 3 && mock.mode == UV_SEARCH_MIPS && m.size() == 3 && m[0].second == 100.0f);
  // a batch: unfilled slots (id -1) are dropped from a row
  std::vector<float> qs(8, 1.0f);
  const SearchBatch b = q.search_batch(qs.data(), 2, 4, Metric::Mips);
  CHECK(b.ids.size() == 8 && mock.nq == 2 && mock.k == 4);
  CHECK(b.row(0).size() == 4 && b.row(1).size() == 3);

  CHECK(q.mem_bytes() == 5 * 41);
  const MemoryBreakdown mb = q.memory_breakdown();
  CHECK(mb.code_bytes == 5 * 41 && mb.model_bytes == 4096 && mb.cache_bytes == 0);
  CHECK(mb.total_resident_bytes() == 5 * 41 + 4096);

  // centering and the shortlist need an empty index, as in the library
  expect_error(UV_EINVAL, [&] { q.with_centroids(rows(2, 4, 0.0f)); });
  expect_error(UV_EINVAL, [&] { q.with_shortlist(32); });

  // the index file
  q.save("/tmp/x.uvb");
  CHECK(mock.path == "/tmp/x.uvb");
  TrellisQuantizer r = TrellisQuantizer::load(TrellisConfig::make(4, 2, 6), "/tmp/y.uvb");
  CHECK(mock.path == "/tmp/y.uvb" && r.len() == 5);

  // CandidateScorer
  CHECK(q.scored_len() == 5 && q.scorer_model_bytes() == 4096);
  {
    std::unique_ptr<PreparedQuery> p = q.prepare(std::vector<float>{1, 0, 0, 0});
    CHECK(mock.live_prepared == 1);
    CHECK(p->score_at(4) == 2.0f);
    expect_error(UV_EINVAL, [&] { p->score_at(5000); });  // outside the index
  }
  CHECK(mock.live_prepared == 0);
}

static void builders_and_lifetimes() {
  mock.reset();
  {
    // consuming builders on a temporary, as the reference chains them
    TrellisQuantizer q = TrellisQuantizer::from_config(TrellisConfig::make(4, 2, 6))
                             .with_codes_only(true)
                             .with_mean(std::vector<float>{1, 2, 3, 4})
                             .with_shortlist(16)
                             .with_shortlist_rnorm(false);
    CHECK(q.config().codes_only);
    CHECK(mock.n_centroids == 1 && mock.rows == (std::vector<float>{1, 2, 3, 4}));
    CHECK(mock.sl_c == 16 && mock.sl_asym == 0 && mock.sl_rnorm == 0);
    // and on a named one
    TrellisQuantizer p = TrellisQuantizer::from_config(TrellisConfig::make(4, 2, 6));
    p.with_centroids(rows(3, 4, 0.0f)).with_shortlist_asym(true);
    CHECK(mock.n_centroids == 3 && mock.sl_asym == 1);
    // move assignment releases the old index before the old codec
    p = std::move(q);
    CHECK(mock.order_errors == 0 && mock.live_codecs == 1 && mock.live_indexes == 1);
    TrellisQuantizer t = std::move(p);
    CHECK(t.dimensions() == 4);
  }
  CHECK(mock.live_codecs == 0 && mock.live_indexes == 0 && mock.order_errors == 0);
}

static void record_api() {
  mock.reset();
  TrellisQuantizer q = TrellisQuantizer::from_config(TrellisConfig::make(8, 2, 5));
  const std::vector<uint32_t> t = q.code_table_bits();
  CHECK(t.size() == 128 && t[5] == 15u);
  CHECK(q.memory_bits() == 5);
  const std::vector<std::vector<float>> s = q.rotation_sign_rounds();
  CHECK(s.size() == 3 && s[0].size() == 8 && s[0][0] == -1.0f && s[2][7] == 1.0f);
  CHECK(q.code_bytes() == 2);
  const auto rec = q.encode_codes(std::vector<float>{5, 0, 0, 0, 0, 0, 0, 0});
  CHECK(rec.first == (std::vector<uint8_t>{5, 6}) && rec.second == 7u);
  const auto rot = q.rotate(std::vector<float>(8, 1.5f));
  CHECK(rot.size() == 8 && rot[3] == 3.0f);
  const auto rr = q.encode_rotated(std::vector<float>(8, 0.1f));
  CHECK(rr.first == (std::vector<uint8_t>{100, 101}) && rr.second == 9u);
  const auto dec = q.decode_codes(std::vector<uint8_t>{4, 0}, 3);
  CHECK(dec.size() == 8 && dec[0] == 7.0f);
  CHECK(q.window_at(std::vector<uint8_t>{0, 0}, 2, 6) == 2006u);
  expect_error(UV_EINVAL, [&] { q.window_at(std::vector<uint8_t>{0, 0}, 2, 8); });
  expect_error(UV_EINVAL, [&] { q.decode_codes(std::vector<uint8_t>{0}, 2); });
  // encode_digest over a batch: every row's record, one digest
  const uint64_t d = q.encode_digest(rows(2, 8, 1.0f));
  CHECK(d == ((((uint64_t)7 << 8) ^ 1u) ^ (((uint64_t)8 << 8) ^ 10u)));
}

static void coarse_and_ivf() {
  mock.reset();
  const auto db = rows(6, 4, 0.0f);
  const auto cen = kmeans(4, db, 3, 42);
  CHECK(cen.size() == 3 && cen[2][3] == 11.0f && mock.iters == 5 && mock.seed == 42);
  const auto asg = assign(db, cen);
  CHECK(asg.size() == 6 && asg[4] == 1u);

  TrellisConfig cfg = TrellisConfig::make(4, 2, 6);
  {
    IvfIndex ivf = IvfIndex::build_with(cfg, db, cen, asg,
                                        IvfCodec::trellis_shortlist(32, true, false), true);
    CHECK(mock.centered == 1 && mock.nlist == 3);
    CHECK(mock.sl_c == 32 && mock.sl_asym == 1 && mock.sl_rnorm == 0);
    CHECK(ivf.len() == 6 && ivf.nlist() == 3 && ivf.mem_bytes() == 6 * 45);
    CHECK(ivf.codec().label() == "trellis_shortlist_c32");
    const Hits h = ivf.search(std::vector<float>{1, 0, 0, 0}, 10, 4);
    CHECK(mock.k == 10 && mock.nprobe == 4 && h.size() == 3 && h[0].first == 40);
    // the library's k limit surfaces as an error
    expect_error(UV_EINVAL, [&] { ivf.search(std::vector<float>{1, 0, 0, 0}, 200, 4); });
    const Hits r = ivf.search_with_rerank(std::vector<float>{1, 0, 0, 0}, 2, 3, 50, db);
    CHECK(mock.rdepth == 50 && mock.nprobe == 3 && mock.n_db == 6 && r.size() == 2);
    CHECK(ivf.memory_breakdown().model_bytes == 3 * 4 * sizeof(float));
    expect_error(UV_EINVAL, [&] {
      IvfIndex::build_with(cfg, db, cen, std::vector<uint32_t>(2), IvfCodec::trellis_codes(),
                           false);
    });
  }
  CHECK(mock.live_codecs == 0 && mock.live_indexes == 0 && mock.order_errors == 0);
  // the reference's build: memory and centering from the environment
  mock.reset();
  setenv("ULTRAVEC_IVF_CENTER", "1", 1);
  setenv("ULTRAVEC_TRELLIS_MEM", "7", 1);
  setenv("ULTRAVEC_TRELLIS_START_BITS", "4", 1);
  setenv("ULTRAVEC_TRELLIS_SHORTLIST", "99", 1);  // ignored: the codec says no shortlist
  {
    IvfIndex ivf = IvfIndex::build(4, db, cen, asg, IvfCodec::trellis_codes(), 2);
    CHECK(mock.centered == 1 && mock.cfg.mem == 7 && mock.cfg.start_bits == 4);
    CHECK(!mock.called("uv_ivf_set_shortlist"));
    CHECK(ivf.codec().label() == "trellis_codes");
  }
  unsetenv("ULTRAVEC_IVF_CENTER");
  unsetenv("ULTRAVEC_TRELLIS_MEM");
  unsetenv("ULTRAVEC_TRELLIS_START_BITS");
  unsetenv("ULTRAVEC_TRELLIS_SHORTLIST");
}

static void reconstruct_and_coset() {
  mock.reset();
  {
    // reconstruct_unit: encode (with the centroids when set), decode, normalize
    TrellisQuantizer q = TrellisQuantizer::from_config(TrellisConfig::make(8, 2, 5));
    const auto u = q.reconstruct_unit(std::vector<float>(8, 1.0f));
    CHECK(u.has_value() && u->size() == 8 && mock.n_centroids == 0);
    float ss = 0.0f;
    for (float v : *u) ss += v * v;
    CHECK(ss > 0.999f && ss < 1.001f);
    TrellisQuantizer c = TrellisQuantizer::from_config(TrellisConfig::make(8, 2, 5))
                             .with_centroids(rows(2, 8, 0.0f));
    const auto uc = c.reconstruct_unit(std::vector<float>(8, 1.0f));
    CHECK(mock.n_centroids == 2 && uc.has_value() && uc->size() == 8);
    expect_error(UV_EINVAL, [&] { q.reconstruct_unit(std::vector<float>(7)); });
  }
  mock.reset();
  setenv("ULTRAVEC_TRELLIS_MEM", "30", 1);  // clamped to 20, as the reference does
  {
    CosetTrellis ct = CosetTrellis::make(16, 2);
    CHECK(mock.cfg.mem == 20 && mock.cfg.rotation_seed == 42 && mock.cfg.rotation_rounds == 3);
  }
  unsetenv("ULTRAVEC_TRELLIS_MEM");
  // the reference panics on dim % 8 != 0: an error here
  expect_error(UV_EINVAL, [] { CosetTrellis::make(12, 2); });
  {
    CosetTrellis ct = CosetTrellis::with_params(16, 2, 6, 42, 3).with_centroids(rows(2, 16, 0.0f));
    CHECK(mock.n_centroids == 2);
    ct.add_batch(rows(3, 16, 1.0f));
    CHECK(mock.ids.empty() && mock.rows.size() == 48 && ct.len() == 3);  // ids 0..n
    ct.add(9, std::vector<float>(16, 0.5f));
    CHECK(mock.ids.size() == 1 && mock.ids[0] == 9 && ct.len() == 4);
    const Hits h = ct.search(std::vector<float>(16, 1.0f), 1000);
    CHECK(mock.k == 4 && h.size() == 4 && h[0].second == 5.0f);
    CHECK(ct.mem_bytes() == 200 && ct.memory_breakdown().model_bytes == 777);
    const auto r = ct.reconstruct_unit(std::vector<float>(16, 2.0f));
    CHECK(r.has_value() && (*r)[3] == -2.0f);
    expect_error(UV_EINVAL, [&] { ct.search(std::vector<float>(8), 3); });
    VectorBackend &b = ct;  // usable through the reference's trait
    CHECK(b.dimensions() == 16 && b.is_approximate() && !b.is_empty());
  }
  CHECK(mock.live_indexes == 0);
}

int main() {
  reconstruct_and_coset();
  config_and_errors();
  environment_constructor();
  backend();
  builders_and_lifetimes();
  record_api();
  coarse_and_ivf();
  std::printf("ok %d\n", checks);
  return 0;
}
