// capi_store.cu -- the index file: one list-major SoA per index, so an index
// is built once and searched from many processes, and checkpointed.
//
// It replaces the reference's in-memory per-entry records (TVec,
// src/trellis.rs:158-198: 64 B per entry plus heap codes) with flat arrays
// that load straight into the device layout.  Little-endian:
//
//   magic "UVB200IX", u32 version (2; 1 is read too), u32 kind (1 flat, 2 IVF)
//   codec config: i32 dim, bits, mem, rotation_rounds; u64 rotation_seed;
//                 i32 start_bits, rescale_bits; f32 branch_lambda
//   i64 n; i32 code_bytes; i32 n_centroids (flat) or nlist (IVF);
//   i32 centered (IVF); i32 0
//   version 2: i32 shortlist c (0 off), asym, rnorm, sign bytes per record
//   arrays, each as u64 byte length + bytes:
//     flat: codes (n x code_bytes), start u32, rescale f32, rnorm f32,
//           norms f32, cidx u32, ids i64, centroids (n_centroids x dim f32)
//     IVF:  list_off i64 (nlist + 1), ids i64, codes, start u32, rescale f32,
//           rnorm f32, centroids (nlist x dim f32)
//     version 2, both kinds: the shortlist sign codes (n x sign bytes; empty
//           when the shortlist is off)
//   u64 FNV-1a of every preceding byte
//
// Loading checks the magic, version, kind, the codec configuration (a file
// only loads into a codec that decodes its records identically), every array
// length and the checksum; any mismatch returns UV_EINVAL.
#include "capi_internal.h"

#include <cstdio>

using namespace uvcapi;

namespace {

constexpr char kMagic[8] = {'U', 'V', 'B', '2', '0', '0', 'I', 'X'};
constexpr uint32_t kVersion = 2;

struct Header {
  char magic[8];
  uint32_t version, kind;
  int32_t dim, bits, mem, rotation_rounds;
  uint64_t rotation_seed;
  int32_t start_bits, rescale_bits;
  float branch_lambda;
  int64_t n;
  int32_t code_bytes, count, centered, zero;
};

struct Writer {
  FILE *f = nullptr;
  uint64_t h = 0xcbf29ce484222325ULL;
  bool ok = true;
  explicit Writer(const char *path) { f = std::fopen(path, "wb"); }
  ~Writer() {
    if (f) std::fclose(f);
  }
  void put(const void *p, size_t bytes) {
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < bytes; i++) {
      h ^= b[i];
      h *= 0x00000100000001b3ULL;
    }
    if (ok && bytes > 0 && std::fwrite(p, 1, bytes, f) != bytes) ok = false;
  }
  void array(const void *p, size_t bytes) {
    const uint64_t len = bytes;
    put(&len, sizeof(len));
    put(p, bytes);
  }
  int finish() {
    const uint64_t sum = h;
    if (ok && std::fwrite(&sum, 1, sizeof(sum), f) != sizeof(sum)) ok = false;
    if (ok && std::fflush(f) != 0) ok = false;
    return ok ? UV_OK : fail(UV_EINVAL, "index file: write failed");
  }
};

struct Reader {
  FILE *f = nullptr;
  uint64_t h = 0xcbf29ce484222325ULL;
  uint64_t left = 0;  // bytes not yet read
  bool ok = true;
  explicit Reader(const char *path) {
    f = std::fopen(path, "rb");
    if (f != nullptr && std::fseek(f, 0, SEEK_END) == 0) {
      const long end = std::ftell(f);
      left = end > 0 ? (uint64_t)end : 0;
      std::fseek(f, 0, SEEK_SET);
    }
  }
  ~Reader() {
    if (f) std::fclose(f);
  }
  bool get(void *p, size_t bytes) {
    if (!ok || bytes > left || (bytes > 0 && std::fread(p, 1, bytes, f) != bytes))
      return ok = false;
    left -= bytes;
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < bytes; i++) {
      h ^= b[i];
      h *= 0x00000100000001b3ULL;
    }
    return true;
  }
  // one length-prefixed array of exactly `bytes` bytes
  template <class T>
  bool array(std::vector<T> &v, size_t count) {
    uint64_t len = 0;
    // the length is checked against the bytes left before anything is allocated
    if (!get(&len, sizeof(len)) || len != count * sizeof(T) || len > left) return ok = false;
    v.resize(count);
    return get(v.data(), len);
  }
  bool checksum() {
    const uint64_t want = h;
    uint64_t got = 0;
    if (!ok || std::fread(&got, 1, sizeof(got), f) != sizeof(got)) return false;
    return got == want && std::fgetc(f) == EOF;
  }
};

Header make_header(const uv_codec *c, uint32_t kind, int64_t n, int32_t count, int32_t centered) {
  Header hd;
  std::memset(&hd, 0, sizeof(hd));
  std::memcpy(hd.magic, kMagic, 8);
  hd.version = kVersion;
  hd.kind = kind;
  hd.dim = c->cfg.dim;
  hd.bits = c->cfg.bits;
  hd.mem = c->cfg.mem;
  hd.rotation_rounds = c->cfg.rotation_rounds;
  hd.rotation_seed = c->cfg.rotation_seed;
  hd.start_bits = c->cfg.start_bits;
  hd.rescale_bits = c->cfg.rescale_bits;
  hd.branch_lambda = c->cfg.branch_lambda;
  hd.n = n;
  hd.code_bytes = c->code_bytes;
  hd.count = count;
  hd.centered = centered;
  return hd;
}

int check_header(const Header &hd, const uv_codec *c, uint32_t kind) {
  if (std::memcmp(hd.magic, kMagic, 8) != 0) return fail(UV_EINVAL, "index file: bad magic");
  if (hd.version != 1 && hd.version != kVersion)
    return fail(UV_EINVAL, "index file: unknown version");
  if (hd.kind != kind) return fail(UV_EINVAL, "index file: holds another kind of index");
  if (hd.dim != c->cfg.dim || hd.bits != c->cfg.bits || hd.mem != c->cfg.mem ||
      hd.rotation_rounds != c->cfg.rotation_rounds || hd.rotation_seed != c->cfg.rotation_seed ||
      hd.start_bits != c->cfg.start_bits || hd.rescale_bits != c->cfg.rescale_bits ||
      std::memcmp(&hd.branch_lambda, &c->cfg.branch_lambda, sizeof(float)) != 0 ||
      hd.code_bytes != c->code_bytes)
    return fail(UV_EINVAL, "index file: written by a codec with another configuration");
  if (hd.n < 0 || hd.count < 0) return fail(UV_EINVAL, "index file: bad sizes");
  return UV_OK;
}

// The shortlist block of a version-2 file (after the header).
struct ShortlistBlock {
  int32_t c, asym, rnorm, sign_bytes;
};

int check_shortlist(const ShortlistBlock &sl, const uv_codec *c) {
  if (sl.c < 0 || (sl.asym != 0 && sl.asym != 1) || (sl.rnorm != 0 && sl.rnorm != 1) ||
      sl.sign_bytes != c->sign_bytes)
    return fail(UV_EINVAL, "index file: bad shortlist block");
  return UV_OK;
}

// sign codes between the device (sign_stride rows) and the file (sign_bytes)
int download_signs(std::vector<uint8_t> &h, const uv_codec *c, const uint8_t *d, int64_t n) {
  h.resize((size_t)n * c->sign_bytes);
  if (n > 0 && d != nullptr)
    UV_CK(cudaMemcpy2D(h.data(), c->sign_bytes, d, c->sign_stride, c->sign_bytes, n,
                       cudaMemcpyDeviceToHost));
  return UV_OK;
}

int upload_signs(uint8_t *d, const uv_codec *c, const std::vector<uint8_t> &h, int64_t n) {
  if (n == 0) return UV_OK;
  UV_CK(cudaMemset(d, 0, (size_t)n * c->sign_stride));
  UV_CK(cudaMemcpy2D(d, c->sign_stride, h.data(), c->sign_bytes, c->sign_bytes, n,
                     cudaMemcpyHostToDevice));
  return UV_OK;
}

template <class T>
int download(std::vector<T> &h, const T *d, size_t count) {
  h.resize(count);
  if (count > 0) UV_CK(cudaMemcpy(h.data(), d, sizeof(T) * count, cudaMemcpyDeviceToHost));
  return UV_OK;
}

template <class T>
int upload_to(T *d, const std::vector<T> &h) {
  if (!h.empty()) UV_CK(cudaMemcpy(d, h.data(), sizeof(T) * h.size(), cudaMemcpyHostToDevice));
  return UV_OK;
}

}  // namespace

extern "C" {

int uv_index_save(const uv_index *ix, const char *path) {
  if (ix == nullptr || path == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  UV_CK(cudaDeviceSynchronize());
  const int64_t n = ix->n;
  const int d = c->cfg.dim;
  std::vector<uint8_t> codes((size_t)n * c->code_bytes);
  if (n > 0)
    UV_CK(cudaMemcpy2D(codes.data(), c->code_bytes, ix->codes, c->code_stride, c->code_bytes, n,
                       cudaMemcpyDeviceToHost));
  std::vector<uint32_t> start, cidx;
  std::vector<float> rescale, rnorm, norms, cen;
  std::vector<int64_t> ids;
  UV_TRY(download(start, ix->start, (size_t)n));
  UV_TRY(download(rescale, ix->rescale, (size_t)n));
  UV_TRY(download(rnorm, ix->rnorm, (size_t)n));
  UV_TRY(download(norms, ix->norms, (size_t)n));
  UV_TRY(download(cidx, ix->cidx, (size_t)n));
  UV_TRY(download(ids, ix->ids, (size_t)n));
  UV_TRY(download(cen, (const float *)ix->centroids, (size_t)ix->n_centroids * d));
  std::vector<uint8_t> signs;
  UV_TRY(download_signs(signs, c, ix->signs, ix->sl_c > 0 ? n : 0));
  Writer w(path);
  if (w.f == nullptr) return fail(UV_EINVAL, std::string("index file: cannot create ") + path);
  const Header hd = make_header(c, 1, n, ix->n_centroids, 0);
  w.put(&hd, sizeof(hd));
  const ShortlistBlock sl = {ix->sl_c, ix->sl_asym, ix->sl_weight, c->sign_bytes};
  w.put(&sl, sizeof(sl));
  w.array(codes.data(), codes.size());
  w.array(start.data(), 4 * start.size());
  w.array(rescale.data(), 4 * rescale.size());
  w.array(rnorm.data(), 4 * rnorm.size());
  w.array(norms.data(), 4 * norms.size());
  w.array(cidx.data(), 4 * cidx.size());
  w.array(ids.data(), 8 * ids.size());
  w.array(cen.data(), 4 * cen.size());
  w.array(signs.data(), signs.size());
  return w.finish();
}

int uv_index_load(const uv_codec *c, const char *path, uv_index **out) {
  if (c == nullptr || path == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  Reader r(path);
  if (r.f == nullptr) return fail(UV_EINVAL, std::string("index file: cannot open ") + path);
  Header hd;
  if (!r.get(&hd, sizeof(hd))) return fail(UV_EINVAL, "index file: truncated header");
  UV_TRY(check_header(hd, c, 1));
  ShortlistBlock sl = {0, 0, 1, c->sign_bytes};
  if (hd.version >= 2) {
    if (!r.get(&sl, sizeof(sl))) return fail(UV_EINVAL, "index file: truncated header");
    UV_TRY(check_shortlist(sl, c));
  }
  const size_t n = (size_t)hd.n;
  const int d = c->cfg.dim;
  std::vector<uint8_t> codes, signs;
  std::vector<uint32_t> start, cidx;
  std::vector<float> rescale, rnorm, norms, cen;
  std::vector<int64_t> ids;
  r.array(codes, n * c->code_bytes);
  r.array(start, n);
  r.array(rescale, n);
  r.array(rnorm, n);
  r.array(norms, n);
  r.array(cidx, n);
  r.array(ids, n);
  r.array(cen, (size_t)hd.count * d);
  if (hd.version >= 2) r.array(signs, sl.c > 0 ? n * c->sign_bytes : 0);
  if (!r.ok) return fail(UV_EINVAL, "index file: truncated or malformed arrays");
  if (!r.checksum()) return fail(UV_EINVAL, "index file: checksum mismatch");
  uv_index *ix = nullptr;
  UV_TRY(uv_index_create(c, &ix));
  int rc = uv_index_set_centroids(ix, hd.count > 0 ? cen.data() : nullptr, hd.count);
  if (rc == UV_OK) rc = uv_index_set_shortlist(ix, sl.c, sl.asym, sl.rnorm);
  if (rc == UV_OK) rc = uv_index_reserve(ix, (int64_t)n);
  if (rc == UV_OK && n > 0) {
    DeviceGuard g(c->cfg.device);
    cudaError_t e = cudaMemcpy2D(ix->codes, c->code_stride, codes.data(), c->code_bytes,
                                 c->code_bytes, n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && c->code_stride > c->code_bytes)
      e = cudaMemset2D(ix->codes + c->code_bytes, c->code_stride, 0,
                       c->code_stride - c->code_bytes, n);
    rc = e == cudaSuccess ? UV_OK : fail(UV_ECUDA, cudaGetErrorString(e));
    if (rc == UV_OK) rc = upload_to(ix->start, start);
    if (rc == UV_OK) rc = upload_to(ix->rescale, rescale);
    if (rc == UV_OK) rc = upload_to(ix->rnorm, rnorm);
    if (rc == UV_OK) rc = upload_to(ix->norms, norms);
    if (rc == UV_OK) rc = upload_to(ix->cidx, cidx);
    if (rc == UV_OK) rc = upload_to(ix->ids, ids);
    if (rc == UV_OK && sl.c > 0) rc = upload_signs(ix->signs, c, signs, (int64_t)n);
  }
  if (rc != UV_OK) {
    uv_index_destroy(ix);
    return rc;
  }
  ix->n = (int64_t)n;
  *out = ix;
  return UV_OK;
}

int uv_ivf_save(const uv_ivf *ix, const char *path) {
  if (ix == nullptr || path == nullptr) return fail(UV_EINVAL, "null argument");
  const uv_codec *c = ix->codec;
  DeviceGuard g(c->cfg.device);
  UV_CK(cudaDeviceSynchronize());
  const int64_t n = ix->n;
  const int d = c->cfg.dim;
  std::vector<uint8_t> codes((size_t)n * c->code_bytes);
  if (n > 0)
    UV_CK(cudaMemcpy2D(codes.data(), c->code_bytes, ix->codes, c->code_stride, c->code_bytes, n,
                       cudaMemcpyDeviceToHost));
  std::vector<uint32_t> start;
  std::vector<float> rescale, rnorm, cen;
  std::vector<int64_t> ids;
  UV_TRY(download(start, ix->start, (size_t)n));
  UV_TRY(download(rescale, ix->rescale, (size_t)n));
  UV_TRY(download(rnorm, ix->rnorm, (size_t)n));
  UV_TRY(download(ids, ix->ids, (size_t)n));
  UV_TRY(download(cen, (const float *)ix->centroids, (size_t)ix->nlist * d));
  std::vector<uint8_t> signs;
  UV_TRY(download_signs(signs, c, ix->signs, ix->sl_c > 0 ? n : 0));
  Writer w(path);
  if (w.f == nullptr) return fail(UV_EINVAL, std::string("index file: cannot create ") + path);
  const Header hd = make_header(c, 2, n, ix->nlist, ix->centered);
  w.put(&hd, sizeof(hd));
  const ShortlistBlock sl = {ix->sl_c, ix->sl_asym, ix->sl_weight, c->sign_bytes};
  w.put(&sl, sizeof(sl));
  w.array(ix->off.data(), 8 * ix->off.size());
  w.array(ids.data(), 8 * ids.size());
  w.array(codes.data(), codes.size());
  w.array(start.data(), 4 * start.size());
  w.array(rescale.data(), 4 * rescale.size());
  w.array(rnorm.data(), 4 * rnorm.size());
  w.array(cen.data(), 4 * cen.size());
  w.array(signs.data(), signs.size());
  return w.finish();
}

int uv_ivf_load(const uv_codec *c, const char *path, uv_ivf **out) {
  if (c == nullptr || path == nullptr || out == nullptr) return fail(UV_EINVAL, "null argument");
  *out = nullptr;
  Reader r(path);
  if (r.f == nullptr) return fail(UV_EINVAL, std::string("index file: cannot open ") + path);
  Header hd;
  if (!r.get(&hd, sizeof(hd))) return fail(UV_EINVAL, "index file: truncated header");
  UV_TRY(check_header(hd, c, 2));
  if (hd.count < 1) return fail(UV_EINVAL, "index file: no lists");
  ShortlistBlock sl = {0, 0, 1, c->sign_bytes};
  if (hd.version >= 2) {
    if (!r.get(&sl, sizeof(sl))) return fail(UV_EINVAL, "index file: truncated header");
    UV_TRY(check_shortlist(sl, c));
  }
  const size_t n = (size_t)hd.n;
  const int d = c->cfg.dim;
  std::vector<int64_t> off, ids;
  std::vector<uint8_t> codes, signs;
  std::vector<uint32_t> start;
  std::vector<float> rescale, rnorm, cen;
  r.array(off, (size_t)hd.count + 1);
  r.array(ids, n);
  r.array(codes, n * c->code_bytes);
  r.array(start, n);
  r.array(rescale, n);
  r.array(rnorm, n);
  r.array(cen, (size_t)hd.count * d);
  if (hd.version >= 2) r.array(signs, sl.c > 0 ? n * c->sign_bytes : 0);
  if (!r.ok) return fail(UV_EINVAL, "index file: truncated or malformed arrays");
  if (!r.checksum()) return fail(UV_EINVAL, "index file: checksum mismatch");
  if (off.front() != 0 || off.back() != (int64_t)n) return fail(UV_EINVAL, "index file: bad offsets");
  for (size_t j = 0; j + 1 < off.size(); j++)
    if (off[j + 1] < off[j]) return fail(UV_EINVAL, "index file: bad offsets");
  uv_ivf *ix = nullptr;
  UV_TRY(uv_ivf_create(c, cen.data(), hd.count, hd.centered, &ix));
  DeviceGuard g(c->cfg.device);
  const size_t cap = std::max<size_t>(n, 1);
  cudaError_t e = cudaMalloc(&ix->codes, cap * c->code_stride);
  if (e == cudaSuccess) e = cudaMalloc(&ix->start, sizeof(uint32_t) * cap);
  if (e == cudaSuccess) e = cudaMalloc(&ix->rescale, sizeof(float) * cap);
  if (e == cudaSuccess) e = cudaMalloc(&ix->rnorm, sizeof(float) * cap);
  if (e == cudaSuccess) e = cudaMalloc(&ix->ids, sizeof(int64_t) * cap);
  if (e == cudaSuccess) e = cudaMalloc(&ix->d_off, sizeof(int64_t) * off.size());
  if (e == cudaSuccess && n > 0)
    e = cudaMemcpy2D(ix->codes, c->code_stride, codes.data(), c->code_bytes, c->code_bytes, n,
                     cudaMemcpyHostToDevice);
  if (e == cudaSuccess && n > 0 && c->code_stride > c->code_bytes)
    e = cudaMemset2D(ix->codes + c->code_bytes, c->code_stride, 0, c->code_stride - c->code_bytes,
                     n);
  int rc = e == cudaSuccess ? UV_OK : fail(UV_ECUDA, cudaGetErrorString(e));
  if (rc == UV_OK) rc = upload_to(ix->start, start);
  if (rc == UV_OK) rc = upload_to(ix->rescale, rescale);
  if (rc == UV_OK) rc = upload_to(ix->rnorm, rnorm);
  if (rc == UV_OK) rc = upload_to(ix->ids, ids);
  if (rc == UV_OK) rc = upload_to(ix->d_off, off);
  if (rc == UV_OK) rc = uv_ivf_set_shortlist(ix, sl.c, sl.asym, sl.rnorm);
  if (rc == UV_OK && sl.c > 0) {
    e = cudaMalloc(&ix->signs, cap * c->sign_stride);
    rc = e == cudaSuccess ? upload_signs(ix->signs, c, signs, (int64_t)n)
                          : fail(UV_ECUDA, cudaGetErrorString(e));
  }
  if (rc != UV_OK) {
    uv_ivf_destroy(ix);
    return rc;
  }
  ix->off = off;
  ix->n = (int64_t)n;
  *out = ix;
  return UV_OK;
}

}  // extern "C"
