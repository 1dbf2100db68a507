// capi_internal.h -- helpers shared by the extern "C" translation units
// (capi.cu: codec and flat index; capi_ivf.cu: the IVF index).  Internal.
#pragma once

#include "ultravec_b200.h"

#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "codebook.h"
#include "uv_kernels.h"
#include "uv_util.h"

namespace uvcapi {

extern thread_local std::string g_err;

inline int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}

#define UV_CK(call)                                                                  \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess)                                                           \
      return fail(e_ == cudaErrorMemoryAllocation ? UV_ENOMEM : UV_ECUDA,            \
                  std::string(#call) + ": " + cudaGetErrorString(e_));               \
  } while (0)

#define UV_TRY(expr)        \
  do {                      \
    int rc_ = (expr);       \
    if (rc_ != UV_OK) return rc_; \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Where a caller pointer lives.  Returns UV_EINVAL for device memory of
// another GPU.
inline int classify(const void *p, int device, bool *on_device) {
  *on_device = false;
  if (p == nullptr) return UV_OK;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return UV_OK;  // unregistered host memory
  }
  if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
    if (a.type == cudaMemoryTypeDevice && a.device != device)
      return fail(UV_EINVAL, "device buffer belongs to another GPU");
    *on_device = true;
  }
  return UV_OK;
}

// The library's own stream-ordered memory pool on the current device.  It
// keeps freed blocks (release threshold = max) so that back-to-back calls
// reuse their scratch instead of mapping it again after every synchronize.
cudaMemPool_t scratch_pool();

// Stream-ordered scratch freed at scope exit (on the same stream).
struct Scratch {
  cudaStream_t st;
  std::vector<void *> ptrs;
  explicit Scratch(cudaStream_t s) : st(s) {}
  ~Scratch() {
    for (void *p : ptrs) cudaFreeAsync(p, st);
  }
  template <class T>
  int alloc(T **out, size_t count) {
    *out = nullptr;
    if (count == 0) count = 1;
    void *p = nullptr;
    cudaMemPool_t pool = scratch_pool();
    cudaError_t e = pool ? cudaMallocFromPoolAsync(&p, count * sizeof(T), pool, st)
                         : cudaMallocAsync(&p, count * sizeof(T), st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(UV_ENOMEM, std::string("cudaMallocAsync: ") + cudaGetErrorString(e));
    }
    ptrs.push_back(p);
    *out = (T *)p;
    return UV_OK;
  }
};

// A caller input viewed on the device: used in place when it is device
// memory, otherwise copied through scratch.
template <class T>
int stage_in(const T *src, size_t count, int device, Scratch &sc, const T **dev) {
  bool on_dev = false;
  UV_TRY(classify(src, device, &on_dev));
  if (src == nullptr || on_dev) {
    *dev = src;
    return UV_OK;
  }
  T *d = nullptr;
  UV_TRY(sc.alloc(&d, count));
  UV_CK(cudaMemcpyAsync(d, src, count * sizeof(T), cudaMemcpyHostToDevice, sc.st));
  *dev = d;
  return UV_OK;
}

// A caller output: written in place on the device, or produced in scratch
// and copied back (see Outputs::finish).
struct Outputs {
  struct Pending {
    void *host;
    const void *dev;
    size_t bytes;
  };
  std::vector<Pending> pend;
  template <class T>
  int stage(T *dst, size_t count, int device, Scratch &sc, T **dev) {
    bool on_dev = false;
    UV_TRY(classify(dst, device, &on_dev));
    if (dst == nullptr || on_dev) {
      *dev = dst;
      return UV_OK;
    }
    T *d = nullptr;
    UV_TRY(sc.alloc(&d, count));
    pend.push_back({(void *)dst, (const void *)d, count * sizeof(T)});
    *dev = d;
    return UV_OK;
  }
  int finish(cudaStream_t st) {
    for (auto &p : pend) UV_CK(cudaMemcpyAsync(p.host, p.dev, p.bytes, cudaMemcpyDeviceToHost, st));
    if (!pend.empty()) UV_CK(cudaStreamSynchronize(st));
    return UV_OK;
  }
};

// ---- kernel timing hook (uv_profile_enable / uv_profile_read) ----
struct ProfRec {
  const char *name;
  cudaEvent_t a, b;
};
extern std::mutex g_prof_mu;
extern std::atomic<int64_t> g_scan_splits;  // uv_set_tuning("scan_splits")
extern std::atomic<int> g_tc_mode;          // uv_set_tuning("tc_scan")
extern std::atomic<int> g_cand_kernel;      // uv_set_tuning("cand_kernel")
extern std::atomic<int> g_tc_shape;         // uv_set_tuning("tc_shape")
extern std::atomic<int> g_tc_cache;         // uv_set_tuning("tc_cache")
extern std::atomic<int> g_coset_nearest;    // uv_set_tuning("coset_nearest")
extern std::atomic<int> g_tc_sample;        // uv_set_tuning("tc_sample")
extern std::atomic<int> g_tc_prepare;       // uv_set_tuning("tc_prepare")
extern std::atomic<int> g_ivf_tc_probe;     // uv_set_tuning("ivf_tc_probe")
extern std::atomic<int> g_ivf_tc;           // uv_set_tuning("ivf_tc")
extern std::atomic<int64_t> g_tc_last_candidates;  // uv_profile_read("tc_candidates")
extern std::atomic<int64_t> g_ivf_tc_overflow;     // uv_profile_read("ivf_tc_overflow")
extern std::atomic<int> g_rescore_warp;     // uv_set_tuning("rescore_warp")
extern std::atomic<int> g_tc_hot;           // uv_set_tuning("tc_hot")
extern std::atomic<bool> g_prof_on;
extern std::vector<ProfRec> g_prof;

struct ProfScope {
  const char *name;
  cudaStream_t st;
  cudaEvent_t a = nullptr, b = nullptr;
  ProfScope(const char *n, cudaStream_t s) : name(n), st(s) {
    if (!g_prof_on) return;
    if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) {
      a = b = nullptr;
      return;
    }
    cudaEventRecord(a, st);
  }
  ~ProfScope() {
    if (a == nullptr) return;
    cudaEventRecord(b, st);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof.push_back({name, a, b});
  }
};

template <class T>
int grow(T **buf, int64_t old_n, int64_t new_cap, cudaStream_t st) {
  T *nb = nullptr;
  UV_CK(cudaMallocAsync((void **)&nb, (size_t)std::max<int64_t>(new_cap, 1) * sizeof(T), st));
  if (*buf != nullptr && old_n > 0)
    UV_CK(cudaMemcpyAsync(nb, *buf, (size_t)old_n * sizeof(T), cudaMemcpyDeviceToDevice, st));
  if (*buf != nullptr) cudaFreeAsync(*buf, st);
  *buf = nb;
  return UV_OK;
}

// Shared launchers (capi.cu).
int sm_count(int dev);

}  // namespace uvcapi

struct uv_codec {
  uv_config cfg;
  int code_bytes = 0, code_stride = 0, table_len = 0;
  int sign_bytes = 0, sign_stride = 0;  // shortlist sign code: ceil(dim/8), padded to 16
  float code_absmax = 0.0f;
  std::vector<float> h_table;
  uvb::RotationHost rot_host;
  float *d_table = nullptr;
  float *d_signs = nullptr;
  uvb::RotParams rot;
  uvb::EncodePlan plan;
  int plan_status = 0;
  std::string plan_why;
};

// The tensor-core prefilter's fp16 operand rows (tcscan.cu / tcwide.cu),
// kept between searches: one set per score mode (the MIPS rows carry the row
// norm), rebuilt when the index has changed since they were made.
struct TcRows {
  uint16_t *x16 = nullptr;      // cap x kpad
  uint16_t *xext = nullptr;     // cap x 16
  float *cmax = nullptr;        // cap / 32 chunk maxima of the bound constants
  int64_t cap = 0, n_pad = 0;   // rows allocated / rows made
  int kpad = 0;
  uint64_t version = ~0ull;     // index version the rows were made from
  cudaEvent_t ready = nullptr;  // recorded after the rows were made
  // pass 1's sample of the records of largest g (its own rows and constants)
  uint16_t *x16_hot = nullptr, *xext_hot = nullptr;
  float *cmax_hot = nullptr;
  int64_t hot_alloc = 0, hot_cap = 0;
  uint64_t hot_version = ~0ull;
};

// The IVF index (capi_ivf.cu): centroids and list-major posting lists.
struct uv_ivf {
  const uv_codec *codec = nullptr;
  int device = 0;              // destroy reads this, not the codec (which may be gone)
  int nlist = 0, centered = 0;
  float *centroids = nullptr;  // nlist x dim
  float *cnorm = nullptr;      // |c_j| (lib.rs:215-217)
  int64_t n = 0;
  std::vector<int64_t> off;    // nlist + 1
  int64_t *d_off = nullptr;
  uint8_t *codes = nullptr;
  uint32_t *start = nullptr;
  float *rescale = nullptr, *rnorm = nullptr;
  int64_t *ids = nullptr;
  int sl_c = 0, sl_asym = 0, sl_weight = 1;  // the 1-bit shortlist (0 = off)
  uint8_t *signs = nullptr;                  // n x sign_stride when the shortlist is on
  // the probe's tensor-core operand rows of the unit centroids (made on the
  // first probe that can use them; state -1 when a centroid norm is not finite)
  mutable std::mutex tc_mu;
  mutable int tc_state = 0;
  mutable uint16_t *c16 = nullptr;   // c_pad x kpad
  mutable uint16_t *cext = nullptr;  // c_pad x 16, zero
  mutable int64_t c_pad = 0;
  // the records' fp16 operand rows for the tensor-core list scan (made on
  // the first search that uses them, freed with the lists) and their scale
  mutable TcRows list_rows;
  mutable float *list_scale = nullptr;
};


struct uv_index {
  const uv_codec *codec = nullptr;
  int device = 0;              // destroy reads this, not the codec (which may be gone)
  uint64_t version = 0;        // bumped by every change of the records
  mutable std::mutex tc_mu;    // guards tc_rows
  mutable TcRows tc_rows[2];   // [mips]
  int64_t n = 0, cap = 0;
  uint8_t *codes = nullptr;
  uint32_t *start = nullptr;
  float *rescale = nullptr, *rnorm = nullptr, *norms = nullptr;
  uint32_t *cidx = nullptr;
  int64_t *ids = nullptr;
  float *centroids = nullptr;
  int n_centroids = 0;
  int sl_c = 0, sl_asym = 0, sl_weight = 1;  // the 1-bit shortlist (0 = off)
  uint8_t *signs = nullptr;                  // cap x sign_stride when the shortlist is on
};


namespace uvcapi {

// Every (query, record) score of an exact scan kernel (p0 with all_key
// filled by the routine; nq queries), sorted per query; the best k as ids
// and scores ranked (score desc, id asc), slots past n -1 / -inf.  Outputs:
// host or device memory.  For k above the scan's top-k capacity (capi.cu).
int rank_all_scores(const uvb::ScanParams &p0, const void *scan_k, size_t smem, int64_t nq,
                    int64_t k, int64_t *ids_out, float *scores_out, int dev, cudaStream_t st,
                    Scratch &sc);

int encode_device(const uv_codec *c, const float *rows, int64_t n, const float *centroids,
                  int n_centroids, bool rotated, uint8_t *codes, uint32_t *start, float *rescale,
                  float *rnorm, uint32_t *cidx, float *norms, cudaStream_t st, Scratch &sc,
                  const float *list_centroids = nullptr, const uint32_t *row_list = nullptr,
                  const int64_t *row_index = nullptr, uint8_t *signs = nullptr);
// The shortlist search (shortlist.cu): one pair per (query, list) with IVF
// lists (lists != null, per_query lists per query, max_len the longest
// list) or one pair per query over [0, n_flat).  Writes npairs x k results.
int shortlist_launch(const uv_codec *c, int cs, int asym, int weight, int k, int64_t npairs,
                     int per_query, const int32_t *lists, const int64_t *list_off,
                     int64_t max_len, int64_t n_flat, const float *q_r, const float *u,
                     const float *centroids, const float *qc, int n_centroids,
                     const uint32_t *degen, const uint8_t *codes, const uint8_t *signs,
                     const uint32_t *start, const uint32_t *cidx, const float *rescale,
                     const float *rnorm, const int64_t *ids, int64_t *out_id, float *out_score,
                     cudaStream_t st);
// Merge top-k lists: row q takes n_lists lists of k_in, or with row_off the
// ragged lists [row_off[q], row_off[q+1]) (n_lists is then their maximum) and
// writes output row out_row[q] when out_row is given.
int merge_launch(int64_t nq, int n_lists, int k_in, int k, const uint32_t *in_key,
                 const float *in_score, const int64_t *in_id, int64_t *out_id, float *out_score,
                 cudaStream_t st, const int64_t *row_off = nullptr,
                 const int32_t *out_row = nullptr);
// a 2D fp16 TMA tensor map (capi.cu)
int fp16_tensor_map(CUtensorMap *m, const void *base, int64_t rows, int cols, int box_cols,
                    int box_rows, bool sw128);
// normalize + rotate queries; u (unit, unrotated) optional
int prep_launch(const uv_codec *c, const float *d_q, int64_t nq, const float *centroids,
                int n_centroids, float *q_r, float *qc, uint32_t *degen, float *u,
                cudaStream_t st);

}  // namespace uvcapi
