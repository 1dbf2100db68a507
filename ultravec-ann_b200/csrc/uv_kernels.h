// uv_kernels.h -- launch interface between the C ABI (capi.cpp) and the
// CUDA kernels (encode.cu, scan.cu, ivf.cu).  Internal; not installed.
#pragma once

#include <cstdint>
#include <string>
#include <algorithm>
#include <atomic>
#include <cuda_runtime.h>

#include "uv_common.cuh"

namespace uvb {

struct EncodeParams {
  int dim, dim_pad, n_states, T, teams_per_cta, team_smem_words;
  int64_t n;
  const float *rows;        // n x dim
  const float *code;        // 2^(mem+bits) table
  RotParams rot;
  float lambda;
  float2 one2;              // (1.0f, 1.0f), passed at run time (see the forward loop)
  int start_bits, rescale_bits;
  const float *centroids;   // flat centering (assign among n_centroids)
  int n_centroids;
  const float *list_centroids;  // IVF centering: row i uses list_centroids[row_list[i]]
  const uint32_t *row_list;
  const int64_t *row_index;   // or null: position i encodes rows[row_index[i]]
  uint8_t *codes;           // n x code_stride
  int code_stride, code_bytes;
  uint32_t *start;
  float *rescale, *rnorm;
  uint32_t *cidx;
  float *norms;             // exact l2 norm of the raw row (MIPS sidecar)
  uint8_t *signs;           // or null: n x sign_stride sign codes of u_r (shortlist)
  int sign_stride;
  int rotated_input;        // rows are already rotated units (encode_rotated)
  uint32_t *back_global;    // per-team back-pointer slots (global mode)
  int64_t back_words_team;
};

struct EncodePlan {
  int B, WPT, T, n_states, dim_pad, teams_per_cta, threads, team_smem_words;
  int cluster = 0;           // > 0: one cluster of this many CTAs per row (encode_cluster.cu)
  int staged = 0;            // > 0: batches of rows one step per launch (encode_staged.cu);
                             // 2: the general pass for mem < bits
  bool back_smem;
  int64_t back_words_team;
  size_t smem_bytes;
  const void *kernel;
};

extern std::atomic<int> g_encode_back_mode;  // placement of back-pointers; never changes results
extern std::atomic<int> g_encode_staged;     // 1: the staged encoder for every window above 14 bits

// 0 ok, 1 invalid, 2 unsupported (message in *why)
int encode_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why);
cudaError_t encode_grid(const EncodePlan &plan, int64_t n, int *grid);
cudaError_t encode_launch(const EncodePlan &plan, EncodeParams p, int grid, cudaStream_t st);
// encode_cluster.cu: rows whose trellis needs more than one 512-thread CTA
int encode_cluster_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why);
cudaError_t encode_cluster_grid(const EncodePlan &plan, int64_t n, int *grid);
cudaError_t encode_cluster_launch(const EncodePlan &plan, EncodeParams p, int grid,
                                  cudaStream_t st);
// encode_staged.cu: every other shape (mem + bits >= 15 at 3 and 4 bits, mem
// + bits above 18, mem < bits), a batch of rows per call, one launch per step
int staged_plan(int dim, int bits, int mem, EncodePlan *plan, std::string *why);
int64_t staged_rows_per_batch(const EncodePlan &plan, int dim, int64_t n);
size_t staged_scratch_bytes(const EncodePlan &plan, int dim, int64_t R, size_t *offs);
cudaError_t encode_staged_launch(const EncodePlan &plan, EncodeParams p, int64_t row0, int64_t R,
                                 uint8_t *scratch, const size_t *offs, cudaStream_t st);

struct PrepParams {
  int dim, dim_pad;
  int64_t nq;
  const float *queries;  // nq x dim
  RotParams rot;
  const float *centroids;
  int n_centroids;
  float *q_r;            // nq x dim_pad
  float *qc;             // nq x n_centroids
  uint32_t *degenerate;  // nq
  float *u;              // or null: nq x dim_pad unit queries (before rotation)
  int clamp_norm;        // |q| clamped at EPS instead of a degenerate query
  int teams;             // queries per CTA of 256 threads: 8 (a warp each) or 1 (0: 8)
};
// prep_queries_kernel's teams per CTA for rows of width dim (prep_teams(dim)
// x (dim_pad + 4) floats of dynamic shared memory)
int prep_teams(int dim);

// The coset trellis's model (coset.cu, src/coset_trellis.rs): book points
// are 64-bit keys, norm << 40 | the eight raw doubled coordinates offset by
// 16, five bits each (first coordinate highest), sorted per coset.
struct CosetModel {
  int dim, mem, m_bits, per_coset, start_bytes, code_len, code_stride;
  const uint64_t *books;  // 8 x per_coset sorted keys
  uint64_t bound[8];      // last key of each coset's book
  float scale_mean, scale_std;
  double pi4;             // pi^4 as the reference's constant PI.powi(4)
  const float *xval;      // 32: (R/2 - mean) / std for raw R = -16..15
};

struct ScanParams {
  int dim, mem, bits;
  int64_t nq, n;
  const float *q_r;   // nq x q_stride
  int q_stride;
  const float *qc;    // nq x n_centroids
  int n_centroids;
  const uint32_t *degenerate;
  const uint8_t *codes;  // n x code_stride
  int code_stride;
  const uint32_t *start;
  const float *rescale, *rnorm, *norms;
  const uint32_t *cidx;
  const float *code;  // table
  int table_len, table_in_smem;
  int img_words;
  int mips, k;
  const int64_t *ids;  // record -> id (may be null: id_base + record)
  int64_t id_base;
  uint32_t *part_key;  // nq x splits x k
  int64_t *part_id;
  CosetModel coset;    // coset records (coset_scan_kernel)
  // Rows whose width is not a multiple of 16: `dim` is the width rounded up
  // to 16 and dim_data the real width (0: dim).  The 16- and 8-wide blocks
  // below dim_data & ~7 run through the decode-GEMM (zero query lanes above);
  // the last dim_data % 8 coordinates are added after the hsum tree, one
  // separately rounded product and sum at a time (src/simd.rs:240-243).
  int dim_data;
  // Full ranking (k above the top-k capacity): every (query, record) score
  // key (score_key32) and id is written to all_key / all_id [q * n + record]
  // instead of a per-split top-k; part_key / part_id are unused.
  uint32_t *all_key;
  int64_t *all_id;
};

// Work items of the chunked scan.  Flat (ivf == 0): the grid is query tiles x
// record splits, as for flat_scan_kernel.  IVF: item i scans the records of
// list item_list[i] for up to 32 (query, probe) pairs starting at
// item_pair[i]; each pair writes its top-k to output slot pair_slot[j].
// Long lists are split into record ranges of range_size; item i scans range
// item_range[i] of list item_list[i] for up to 32 pairs, and pair j of list l
// writes range r to slot list_rbase[l] + (j - list_pair_off[l]) * nr(l) + r.
struct ScanWork {
  int ivf;
  const int32_t *item_list;
  const int32_t *item_pair;
  const int32_t *item_npairs;
  const int32_t *item_range;
  const int64_t *list_off;       // nlist + 1
  const int32_t *list_pair_off;  // first pair of each list (bucketed order)
  const int64_t *list_rbase;     // first range slot of each list
  int64_t range_size;
  const int32_t *pair_query;     // query row of q_r
  const float *pair_qm;          // <u, c_list> (centered lists) or null
  const int32_t *n_items;        // IVF: CTAs at or past *n_items exit
};

// Sequential-dot tiles of the IVF coarse stage (ivf.cu).
struct SeqDotParams {
  int dim, lda, ldb;
  int64_t nA, nB;
  const float *A, *B;
  float2 one2;              // (1.0f, 1.0f), passed at run time
  uint64_t *out_key;        // mode 0: nA keys (zeroed before the launch)
  float *out;               // mode 1: nA x nB cosines
  const float *a_norm, *b_norm;
};

struct RerankParams {
  int64_t nq;
  int dim, r, k;
  const float *queries;     // nq x dim, raw
  const float *db;          // n_db x dim, raw
  int64_t n_db;
  int *err;                 // set to 1 when a candidate id is >= n_db
  const int64_t *cand;      // nq x r ids (-1 = empty)
  int64_t *out_id;
  float *out_score;
};

// Batched per-candidate scoring (candidates.cu).
struct CandParams {
  int dim, mem, bits, code_stride, q_stride, n_centroids, table_len, table_in_smem;
  int table_rep;               // lane kernel: copies of the table in shared memory (0: global)
  int64_t nq, n, n_records;
  const int64_t *offsets;      // nq + 1 (CSR over candidates), or null: all on query 0
  const int64_t *positions;    // n record positions
  const float *q_r;            // nq x q_stride rotated unit queries
  const float *qc;             // nq x n_centroids
  const uint32_t *degenerate;  // nq
  const uint8_t *codes;
  const uint32_t *start, *cidx;
  const float *code, *rescale, *rnorm;
  float *out;
  int *n_bad;                  // candidates with a position outside the index
};

// The 1-bit companion shortlist (shortlist.cu).  One CTA per pair: pair p
// is query p / per_query over the records of list lists[p] (IVF) or over
// [0, n_flat) (flat); it writes its top-k to row p of out_id / out_score.
struct ShortlistParams {
  int dim, mem, bits, code_stride, sign_stride, q_stride, u_stride;
  int cs, k, cp, weight, table_len, n_centroids, per_query;
  int64_t npairs, n_flat;
  const int32_t *lists;        // npairs (IVF) or null (flat)
  const int64_t *list_off;     // nlist + 1 (IVF)
  const float *q_r;            // rotated unit queries
  const float *u;              // unit queries (IVF centered: qm = <u, c_list>) or null
  const float *centroids;      // IVF list centroids (centered) or null
  const float *qc;             // flat centered: nq x n_centroids
  const uint32_t *degenerate;
  const uint8_t *codes, *signs;
  const uint32_t *start, *cidx;
  const float *code, *rescale, *rnorm;
  const int64_t *ids;          // output ids by record, or null: the record position
  int64_t *out_id;
  float *out_score;
};

// Tensor-core prefilter of the flat scan (tcscan.cu).
struct TcScanParams {
  int q_stride, cand_cap;
  int64_t nq, n, n_tiles, n_groups;
  int64_t tile_stride;         // tile t covers records of tile t * tile_stride (pass-1 sample)
  const float *q_r;            // nq x q_stride rotated unit queries
  const uint32_t *degenerate;  // nq
  float *tmax;                 // mode 1: nq x n_groups lower-bound maxima
  const float *theta;          // mode 2: per-query threshold
  uint32_t *cand;              // mode 2: nq x cand_cap record indices, in segments:
                               // region = split * 2 + column half, region_cap each
  int *cand_cnt;               // mode 2: nq x regions segment counts
  int regions, region_cap;
  const float *cmax;           // n_pad / 16: largest C' of each 16-record chunk (records
                               // below n; tc_scan_kernel applies it in the epilogue)
  int *err;
};

struct TcPrepareParams {
  int mem, bits, code_stride, mips;
  int dim, kpad;               // record dimension; row stride of x16 (dim rounded up to 64)
  int64_t n, n_pad;
  double eps;
  float code_absmax;           // max |code table value|
  const uint8_t *codes;
  const uint32_t *start;
  const float *code;           // f32 code table
  const float *rescale, *rnorm, *norms;
  uint32_t *gmax_bits;         // largest finite g (zeroed before tc_gmax_kernel)
  uint16_t *x16;               // n_pad x kpad fp16 main operand rows
  uint16_t *xext;              // n_pad x 16 fp16 extra slice (bound constant)
};

struct TcRescoreParams {
  int dim, mem, bits, code_stride, q_stride, cap, k, mips, table_len, table_in_smem;
  int64_t nq;
  const float *q_r;
  const uint32_t *degenerate;
  const uint8_t *codes;
  const uint32_t *start;
  const float *code, *rescale, *rnorm, *norms;
  const uint32_t *cand;        // nq x cand_stride: `regions` segments of region_cap
  const int *cand_cnt;         // nq x regions
  int regions, region_cap;
  int64_t cand_stride;
  const int64_t *ids;
  int64_t *out_id;
  float *out_score;
  int32_t *over_list;
  int *n_over;
  unsigned long long *n_cand;  // total candidates scored (statistics)
  int32_t *big_list;           // or null: tc_rescore_warp_kernel scored every query but
  int *n_big;                  // the *n_big listed here, left to tc_rescore_kernel
};

struct MergeParams {
  int64_t nq;                // rows to merge
  int n_lists, k_in, k, pow2, warps;
  // fixed rows: list l of row q starts at entry q * row_stride + l * list_stride
  // (0, 0: rows of n_lists * k_in contiguous entries)
  int64_t row_stride, list_stride;
  const int32_t *in_packed;  // or null: 3 x int32 per entry (id low, id high, score bits)
  const int64_t *row_off;    // or null: row q merges lists [row_off[q], row_off[q+1])
  const int32_t *out_row;    // or null: row q writes output row out_row[q]
  const uint32_t *in_key;  // or null
  const float *in_score;   // or null
  const int64_t *in_id;
  int64_t *out_id;
  float *out_score;
};

__global__ void prep_queries_kernel(const PrepParams p);
const void *flat_scan_kernel_ptr(int bits, bool table_in_smem);
// K-chunked scan for wide rows and IVF lists; small_k selects the 32-entry
// top-k (k <= 32) that keeps two CTAs per SM.
const void *chunked_scan_kernel_ptr(int bits, bool table_in_smem, bool small_k);
size_t chunked_scan_smem_bytes(int table_len, bool table_in_smem, bool small_k);
constexpr int kScanKChunk = 128;
__global__ void merge_topk_kernel(const MergeParams p);
__global__ void merge_topk_block_kernel(const MergeParams p);
__global__ void topk_pack_kernel(const int64_t *ids, const float *scores, int64_t n,
                                 int32_t *packed);
__global__ void topk_unpack_kernel(const int32_t *packed, int64_t n, int64_t *ids,
                                   float *scores);

// tcscan.cu
// shape 1: the queries (A) in shared memory; 3: A in TMEM (the default)
const void *tc_scan_kernel_ptr(int mode, int shape);
size_t tc_scan_smem_bytes(int shape);
int tc_threads();          // tc_scan_kernel's block
int tc_groups_per_tile();  // pass-2 candidate segments per tile column range and split
int tc_wide_threads();     // tc_wide_kernel's block
int tc_tile_records();
int tc_tile_queries();
int tc_dim();
__global__ void tc_gmax_kernel(const TcPrepareParams p);
__global__ void tc_prepare_records_kernel(const TcPrepareParams p);
// widths 1, 2, 4 with the table in shared memory (4 << (mem + bits) bytes,
// 256 threads); null for other widths.  f32sum: |x|^2 summed in f32 under a
// rigorous inflation and paired fp16 conversions; else the f64 sum of
// tc_prepare_records_kernel
const void *tc_prepare_records_fast_ptr(int bits, bool f32sum);
// cmax[c] = largest C' (element 0 of the extra slice) of records 16c ..
// 16c + 15 below n, 0 for a chunk of padding only; n_pad % 16 == 0, blocks
// of 256 threads
__global__ void tc_chunk_cmax_kernel(const uint16_t *xext, int64_t n, int64_t n_pad,
                                     float *cmax);
// pass 1's sample: the records of largest score scale g (tcscan.cu)
__global__ void tc_hot_keys_kernel(const TcPrepareParams p, uint32_t *keys, uint32_t *hist);
__global__ void tc_hot_hist_kernel(const uint32_t *keys, int64_t n, const uint32_t *sel,
                                   uint32_t *hist);
__global__ void tc_hot_pick_kernel(const uint32_t *hist, int64_t want, int level, uint32_t *sel);
__global__ void tc_hot_count_kernel(const uint32_t *keys, int64_t n, int64_t span,
                                    const uint32_t *sel, uint32_t *counts);
__global__ void tc_hot_scan_kernel(uint32_t *counts, int blocks);
__global__ void tc_hot_gather_kernel(const TcPrepareParams p, const uint32_t *keys, int64_t span,
                                     const uint32_t *sel, const uint32_t *offs, int64_t cap,
                                     uint16_t *x16_hot, uint16_t *xext_hot);
__global__ void tc_hot_pad_kernel(const uint32_t *offs_end, int64_t cap, int kpad,
                                  uint16_t *x16_hot, uint16_t *xext_hot);
// per-query k-th largest tile maximum; the n_tiles keys are staged in dynamic
// shared memory (4 bytes each) when n_tiles <= kThetaSmemKeys
constexpr int kThetaSmemKeys = 12288;
__global__ void tc_theta_kernel(const float *tmax, int64_t n_tiles, int64_t nq, int k,
                                float *theta, int lists);
__global__ void tc_bounds_kernel(const float *tmax, int64_t n_groups, int64_t nq, int k,
                                 const float *theta, float *bounds);
// the same selection, one warp per query (8 per CTA of 256) with the keys in
// registers, for up to 2048 values per query (null above)
const void *tc_theta_warp_kernel_ptr(int64_t n_tiles);
// bits 1..4; per_thread: one thread per candidate (long lists), else half a
// warp per candidate (short lists)
const void *tc_rescore_kernel_ptr(int bits, bool per_thread);
// One warp per query for short candidate lists: kRescoreWarps queries per CTA
// of 32 * kRescoreWarps threads, up to kRescoreWarpCap candidates each, rows
// up to kRescoreWarpDim wide, the code table (up to 1024 entries) in
// kRescoreCopies bank-interleaved copies.
constexpr int kRescoreWarps = 16;
constexpr int kRescoreWarpCap = 128;
constexpr int kRescoreWarpDim = 256;
constexpr int kRescoreCopies = 8;
const void *tc_rescore_warp_kernel_ptr(int bits);
size_t tc_rescore_warp_smem_bytes(int table_len, int regions);
// tcwide.cu: the prefilter for rows of any width (K streamed in chunks of 64)
const void *tc_wide_kernel_ptr(int mode);
size_t tc_wide_smem_bytes();
// queries -> fp16 operand rows (nq_pad x kpad) and the two extra slices
// (-1 for lower bounds, +1 for upper bounds)
__global__ void tc_prepare_queries_kernel(const float *q_r, int q_stride, const uint32_t *degen,
                                          int64_t nq, int64_t nq_pad, int dim, int kpad,
                                          uint16_t *a16, uint16_t *aext_lo, uint16_t *aext_hi);

// ivf.cu
template <int MODE>
__global__ void seqdot_kernel(const SeqDotParams p);
int seqdot_tile();
__global__ void argmax_index_kernel(const uint64_t *key, int64_t n, uint32_t *out);
__global__ void row_norms_kernel(const float *rows, int64_t n, int dim, float *norms);
__global__ void normalize_rows_kernel(const float *rows, const float *norms, int64_t n, int dim,
                                      float *units);
__global__ void gather_rows_kernel(const float *src, const int64_t *pick, int nrows, int dim,
                                   float *dst);
__global__ void list_means_kernel(const float *units, const int64_t *order, const int64_t *off,
                                  int nlist, int dim, float *cent);
// the IVF probe from tensor-core dots (ivf.cu)
struct ProbeRefineParams {
  int64_t m;             // queries
  int nlist, np, dim, pow2, ld_out;
  int cosine;            // 1: cosine over the norms; 0: the plain dot
  int64_t ld;            // leading dimension of approx
  float bound;           // |approx - exact cosine| <= bound
  const float *approx;   // m x ld fp16-operand dots of unit rows
  const float *queries;  // m x dim raw queries
  const float *qnorm;    // m
  const float *cent;     // nlist x dim
  const float *cnorm;    // nlist
  int32_t *out;          // m x ld_out lists
};
__global__ void probe_refine_kernel(const ProbeRefineParams p);
__global__ void unit_flags_kernel(const float *norms, int64_t n, uint32_t *flags);
__global__ void select_top_kernel(const float *scores, int64_t n, int nb, int pow2, int np,
                                  int ld_out, int32_t *out);
__global__ void fill_empty_kernel(int64_t *ids, float *scores, int64_t n);
__global__ void pair_count_kernel(const int32_t *lists, int64_t npairs, int32_t *cnt);
__global__ void drop_empty_lists_kernel(int32_t *lists, int64_t npairs, const int64_t *list_off,
                                        int nlist, int *bad);
// per_item: pairs of one list per scan item (kScanTQ for chunked_scan_kernel,
// kIvfTcRows for tc_ivf_kernel)
__global__ void pair_scan_kernel(const int32_t *cnt, const int64_t *list_off, int nlist,
                                 int64_t range_size, int per_item, int32_t *pair_off,
                                 int32_t *item_off, int64_t *list_rbase, int64_t *totals);
__global__ void pair_scatter_kernel(const int32_t *lists, int64_t nq, int np,
                                    const int32_t *pair_off, int32_t *fill, int32_t *pair_query,
                                    int32_t *pair_slot, int32_t *pair_list);
__global__ void item_fill_kernel(const int32_t *cnt, const int32_t *pair_off,
                                 const int32_t *item_off, const int64_t *list_off, int nlist,
                                 int64_t range_size, int per_item, int32_t *item_list,
                                 int32_t *item_pair, int32_t *item_npairs, int32_t *item_range);
__global__ void pair_rows_kernel(const int32_t *pair_list, const int32_t *pair_off,
                                 const int64_t *list_rbase, const int64_t *list_off,
                                 int64_t range_size, int npairs, int64_t *row_off);
constexpr int kPairQmWarps = 4;  // pair_qm_kernel: warps per block (32 pairs each)
__global__ void pair_qm_kernel(const float *u, int u_stride, const float *cent, int dim,
                               const int32_t *pair_query, const int32_t *pair_list, int npairs,
                               float *qm);
__global__ void rerank_kernel(const RerankParams p);

// ivftc.cu: the IVF list scan on the tensor cores.  Work items as for the
// chunked scan (ScanWork), with up to kIvfTcRows pairs per item and record
// ranges of at most kIvfTcRange records; (pair, range) slot s gets
// slot_cnt[s] kept records at cand_*[slot_base[s] ...] (-1: the store was
// full, *err |= 2), and each query's q_theta0 (zeroed before the launch) the
// largest of its slots' thresholds (the k-th largest lower bound of s *
// score over a range) as an order-preserving key.
constexpr int kIvfTcRows = 128;
constexpr int kIvfTcRange = 512;
struct TcIvfParams {
  int k, kchunks;              // kchunks: record row width / 64
  int64_t range_size;
  const int32_t *n_items;
  const int32_t *item_list, *item_pair, *item_npairs, *item_range;
  const int64_t *list_off;
  const int32_t *list_pair_off;
  const int64_t *list_rbase;
  const int32_t *pair_query;
  const float *pair_qm;        // or null
  const uint32_t *degenerate;
  const float *scale;          // s, a power of two (tc_scale_kernel)
  const uint16_t *xext;        // record extra slices: C' in element 0
  uint32_t *q_theta0;
  int32_t *slot_cnt;
  int64_t *slot_base;
  uint32_t *cand_rec;
  float *cand_lb, *cand_ub;
  unsigned long long *cand_used;  // entries handed out so far
  int64_t cand_cap;
  int *err;                    // 1: a wait timed out, 2: the store is full
};
// Per query: the threshold over all its slots, the candidates that reach
// it, their exact scores and the top k by (score desc, id asc).
struct IvfSelectParams {
  int dim, mem, bits, code_stride, q_stride, k, np, table_len;
  int64_t nq;
  const float *q_r;
  const uint32_t *degenerate;
  const int32_t *pair_of;      // nq x np: bucketed pair of probe j of query q
  const int64_t *row_off;      // pair -> its slots [row_off[p], row_off[p + 1])
  const float *pair_qm;        // or null
  const uint32_t *q_theta0;
  const int32_t *slot_cnt;
  const int64_t *slot_base;
  const uint32_t *cand_rec;
  const float *cand_lb, *cand_ub;
  const uint8_t *codes;
  const uint32_t *start;
  const float *code, *rescale, *rnorm;
  const int64_t *ids;
  int64_t *out_id;
  float *out_score;
  int *n_over;                 // queries with more candidates than kIvfSelCand
  unsigned long long *n_cand;  // candidates scored exactly (statistics)
};
constexpr int kIvfSelWarps = 8;
constexpr int kIvfSelLb = 512;     // lower bounds per query at the threshold step
constexpr int kIvfSelCand = 256;   // candidates per query
const void *tc_ivf_kernel_ptr(int k);  // k <= 32; null above
size_t tc_ivf_smem_bytes();
int tc_ivf_threads();
const void *ivf_select_kernel_ptr(int bits);
size_t ivf_select_smem_bytes(int table_len, int code_stride);
__global__ void ivf_pair_rows16_kernel(const uint16_t *a16, const int32_t *pair_query,
                                       int64_t npairs, int kpad, uint16_t *pa16);
__global__ void ivf_pair_of_kernel(const int32_t *pair_slot, int64_t npairs, int32_t *pair_of);
__global__ void ivf_neg_slice_kernel(uint16_t *ax);  // kIvfTcRows x 16, one thread per entry
__global__ void tc_scale_kernel(const uint32_t *gmax_bits, float code_absmax, float *scale);
__global__ void score_candidates_kernel(const CandParams p);
const void *score_candidates_lane_kernel_ptr(int bits);  // bits 1..4; else null
const void *shortlist_kernel_ptr(int bits, bool asym);
size_t shortlist_smem_bytes(int cp, int q_stride, int sign_stride, int table_len);

// ---------------------------------------------------------------------------
// Coset trellis (coset.cu): trellis-coded quantization over the eight cosets
// of an index-8 sublattice of E8 (src/coset_trellis.rs).  Book points are
// 64-bit keys, norm << 40 | the eight raw doubled coordinates offset by 16,
// five bits each (first coordinate highest), sorted per coset.
// ---------------------------------------------------------------------------

struct CosetEncParams {
  CosetModel m;
  int64_t n;                 // rows of this launch
  const float *rows;         // n x dim
  RotParams rot;
  const float *centroids;
  int n_centroids;
  float *u_r, *y;            // n x dim
  uint32_t *blk_idx;         // n x (dim/8) x 8
  float *blk_cost;           // n x (dim/8) x 8
  uint8_t *back;             // n x (dim/8) x 2^mem, unless in shared memory
  float *cost;               // n x 2 x 2^mem, unless in shared memory
  int back_smem, cost_smem;
  uint8_t *codes;            // n x code_stride
  float *rescale, *rnorm;
  uint32_t *cidx;
  float *recon;              // n x dim (reconstruction kernel)
};

__global__ void coset_prep_kernel(const CosetEncParams p);
__global__ void coset_nearest_kernel(const CosetEncParams p);
__global__ void coset_nearest_brute_kernel(const CosetEncParams p);
size_t coset_brute_smem_bytes(int per_coset);
constexpr int kCosetBruteY = 8;  // y-blocks per thread of coset_nearest_brute_kernel
__global__ void coset_viterbi_kernel(const CosetEncParams p);
__global__ void coset_reconstruct_kernel(const CosetEncParams p);
__global__ void iota_i64_kernel(int64_t *out, int64_t n, int64_t base);
size_t coset_viterbi_smem_bytes(int dim, int mem, bool back_smem, bool cost_smem);
const void *coset_scan_kernel_ptr();

// scan tiling constants shared with the host planner
constexpr int kScanTQ = 32;
constexpr int kScanTN = 32;
constexpr int kScanKCap = 128;

// Full ranking (rank.cu) for k above kScanKCap: sort every query's n score
// keys and ids.
constexpr int kRankTile = 2048;  // elements per block-sort tile (= rank_merge_span())
__global__ void rank_tile_sort_kernel(uint32_t *key, int64_t *id, int64_t n);
__global__ void rank_merge_kernel(const uint32_t *ik, const int64_t *ii, uint32_t *ok, int64_t *oi,
                                  int64_t n, int64_t w, int64_t klim);
__global__ void rank_emit_kernel(const uint32_t *key, const int64_t *id, int64_t n, int64_t nq,
                                 int64_t k, const uint32_t *degen, int64_t *out_id,
                                 float *out_score);
__global__ void rank_gather_kernel(const MergeParams p, int64_t total, uint32_t *keys,
                                   int64_t *ids);
__global__ void fill_value_kernel(float *out, int64_t n, float v);
int rank_merge_span();

size_t scan_smem_bytes(int dim, int img_words, int table_len, bool table_in_smem);

}  // namespace uvb
