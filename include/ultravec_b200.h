/*
 * ultravec_b200.h -- C ABI of the B200 trellis codec (encode) and codes-only
 * scan (flat + IVF).
 *
 * A drop-in for the two data-parallel hot paths of ultravec-ann:
 *   - the free-start Viterbi trellis encoder (src/trellis.rs), and
 *   - the codes-only MIPS / cosine scan with RaBitQ's rescaled estimator and a
 *     per-query top-k (src/trellis.rs search/score, src/ivf.rs, src/bench.rs).
 * Every entry point names the reference item it replaces (file:line).
 *
 * Conventions
 *   - Plain pointers and sizes only.  Array arguments may live in host memory
 *     or in device memory of the handle's GPU; the library detects which and
 *     stages host buffers through the call's stream.  Host results are valid
 *     when the call returns; device results are ordered on `stream`.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call returns UV_OK (0) or a UV_E* status; nothing throws across the
 *     ABI and nothing aborts.  uv_last_error() gives a message for the calling
 *     thread.
 *   - Handles are immutable during a search: concurrent uv_*_search calls on one
 *     index from several threads/streams are safe (per-call scratch).  Adds and
 *     builds must not overlap searches of the same index.
 *   - Rows are `dim` f32 values, already zero-padded to a power of two by the
 *     caller exactly as the reference loader does (src/datasets.rs:95-103).
 *   - Ranking everywhere is score descending, then id ascending; NaN scores
 *     rank last.  Unfilled top-k slots hold id -1 and score -inf.  A query with
 *     |q| < f32::EPSILON returns only unfilled slots (the reference returns an
 *     empty list, src/trellis.rs:2124-2127).
 */
#ifndef ULTRAVEC_B200_H
#define ULTRAVEC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UV_OK 0
#define UV_EINVAL 1        /* bad argument or configuration */
#define UV_ENOMEM 2        /* device or host allocation failed */
#define UV_ECUDA 3         /* a CUDA call failed; see uv_last_error() */
#define UV_ETIMEDOUT 4     /* a bounded device wait gave up */
#define UV_EUNSUPPORTED 5  /* valid for the reference, not built for sm_100a yet */

#define UV_ABI_VERSION 1

/* Mirrors TrellisConfig (src/trellis.rs:352-391). */
typedef struct uv_config {
    int32_t dim;             /* padded dimension */
    int32_t bits;            /* emitted bits per coordinate, 1..4 */
    int32_t mem;             /* trellis memory M (state bits) */
    int32_t rotation_rounds; /* rounds of seeded sign flip + FWHT (3) */
    uint64_t rotation_seed;  /* 42 */
    int32_t start_bits;      /* free-start width, <= mem (mem) */
    int32_t rescale_bits;    /* 0 = exact f32 rescale */
    float branch_lambda;     /* anisotropic metric weight; 0 = plain MSE */
    int32_t device;          /* CUDA device ordinal the handle lives on */
} uv_config;

typedef struct uv_codec uv_codec;
typedef struct uv_index uv_index;
typedef struct uv_ivf uv_ivf;

int uv_abi_version(void);
const char *uv_last_error(void);

/* TrellisConfig::new (src/trellis.rs:379-390): seed 42, 3 rounds, full free
 * start, exact rescale, device 0. */
void uv_config_default(uv_config *cfg, int32_t dim, int32_t bits, int32_t mem);

/* TrellisQuantizer::from_config (src/trellis.rs:430-458).  Builds the code
 * table (593-610) and rotation signs (src/lib.rs:428-463) on the host and
 * uploads them to cfg->device. */
int uv_codec_create(const uv_config *cfg, uv_codec **out);
int uv_codec_destroy(uv_codec *codec);

/* code_table_bits (src/trellis.rs:649-655): 2^(mem+bits) f32 bit patterns. */
int uv_codec_code_table_bits(const uv_codec *codec, uint32_t *out, int64_t capacity);
/* rotation_sign_rounds (src/trellis.rs:663-667): rounds x dim, +-1.0 */
int uv_codec_rotation_sign_rounds(const uv_codec *codec, float *out, int64_t capacity);
/* memory_bits (src/trellis.rs:658-660) */
int uv_codec_memory_bits(const uv_codec *codec, int32_t *mem);
/* record layout: ceil(dim*bits/8) code bytes, ceil(start_bits/8) start bytes,
 * 4 rescale bytes (scalar_bytes, src/trellis.rs:401-418) */
int uv_codec_record_bytes(const uv_codec *codec, int32_t *code_bytes, int32_t *start_bytes,
                          int32_t *rescale_bytes);

/* encode_codes over a batch (src/trellis.rs:672-675, 1164-1212; the per-row
 * work of add_batch 2103-2119).  rows: n x dim.  Outputs: codes n x
 * code_bytes (packed MSB-first), start n, rescale n (+inf when <= 1e-6),
 * rnorm n (1.0 uncentered; may be NULL).  centroids (n_centroids x dim) turns
 * on centering (with_centroids, 952-956): each row is assigned to its
 * first-maximum centroid, cidx n receives it (may be NULL). */
int uv_encode(const uv_codec *codec, const float *rows, int64_t n, const float *centroids,
              int32_t n_centroids, uint8_t *codes, uint32_t *start, float *rescale,
              float *rnorm, uint32_t *cidx, void *stream);

/* encode_rotated (src/trellis.rs:689-699): rows are already rotated units. */
int uv_encode_rotated(const uv_codec *codec, const float *u_r, int64_t n, uint8_t *codes,
                      uint32_t *start, void *stream);

/* rotate (src/trellis.rs:680-682 -> src/lib.rs:472-484), n rows. */
int uv_rotate(const uv_codec *codec, const float *rows, int64_t n, float *out, void *stream);

/* decode_codes (src/trellis.rs:705-720): table values by window, inverse
 * rotated, not normalized.  n records -> n x dim. */
int uv_decode(const uv_codec *codec, const uint8_t *codes, const uint32_t *start, int64_t n,
              float *out, void *stream);

/* window_at (src/trellis.rs:727-743) for all i: n records -> n x dim windows */
int uv_windows(const uv_codec *codec, const uint8_t *codes, const uint32_t *start, int64_t n,
               uint32_t *out, void *stream);

/* encode_digest (src/trellis.rs:970-990) of n records: XOR of per-record
 * FNV-1a over start (LE u32) then the code bytes. */
int uv_digest(const uv_codec *codec, const uint8_t *codes, const uint32_t *start, int64_t n,
              uint64_t *digest, void *stream);

/* ---- flat codes-only index: VectorBackend for TrellisQuantizer
 *      (src/lib.rs:104-155, src/trellis.rs:2088-2247) ---- */

/* TrellisQuantizer::new(..).with_codes_only(true): an empty device index. */
int uv_index_create(const uv_codec *codec, uv_index **out);
int uv_index_destroy(uv_index *index);
/* with_centroids / with_mean (src/trellis.rs:952-956, 746-748) */
int uv_index_set_centroids(uv_index *index, const float *centroids, int32_t n_centroids);
/* reserve (src/lib.rs:131, src/trellis.rs:2100-2102) */
int uv_index_reserve(uv_index *index, int64_t additional);
/* add (src/trellis.rs:2095-2099) for n rows with explicit ids; also stores
 * each row's exact l2 norm, the MIPS sidecar of src/bench.rs:1019. */
int uv_index_add(uv_index *index, const int64_t *ids, const float *rows, int64_t n,
                 void *stream);
/* add_batch (src/trellis.rs:2103-2119): ids 0..n-1, order preserving. */
int uv_index_add_batch(uv_index *index, const float *rows, int64_t n, void *stream);
/* len / dimensions / mem_bytes (src/trellis.rs:2089-2092, 2184-2201) */
int uv_index_len(const uv_index *index, int64_t *len);
int uv_index_dimensions(const uv_index *index, int32_t *dim);
int uv_index_mem_bytes(const uv_index *index, int64_t *bytes);

#define UV_SEARCH_COSINE 0 /* VectorBackend::search: the codec's score */
#define UV_SEARCH_MIPS 1   /* score x exact row norm (src/bench.rs:1029-1045) */

/* search (src/trellis.rs:2120-2183) for nq queries, the best k per query:
 * ids_out/scores_out are nq x k (scores_out may be NULL).  Any k >= 1: up to
 * 128 the scan keeps a fused per-query top-k; above 128 every record is
 * ranked (all scores, then a device sort of each query's list), so
 * k = len() returns the whole index in ranking order, as the reference's
 * MIPS harness asks for (src/bench.rs:1029-1045); slots past len() are
 * unfilled.  Rows of any width (the last dim % 8 coordinates are the
 * reference's scalar tail, src/simd.rs:240-243).  UV_EUNSUPPORTED for a
 * cosine search with k > 128 on an index whose 1-bit shortlist prunes. */
int uv_index_search(const uv_index *index, const float *queries, int64_t nq, int32_t k,
                    int32_t mode, int64_t *ids_out, float *scores_out, void *stream);

/* The records, for export or parity checks: any pointer may be NULL. */
int uv_index_export(const uv_index *index, uint8_t *codes, uint32_t *start, float *rescale,
                    float *rnorm, float *norms, int64_t *ids, void *stream);
/* encode_digest of the stored records. */
int uv_index_digest(const uv_index *index, uint64_t *digest, void *stream);

/* uv_index_search without any device allocation.  No counterpart in the
 * reference: it exists for callers that must not allocate device memory while
 * they serve queries -- a process that reserves its whole GPU memory budget at
 * start-up, or a latency-bound thread that cannot accept the device-wide
 * synchronization that cudaMalloc/cudaFree may bring.  Same arguments and
 * results (ids and score bits) as uv_index_search, with these limits:
 *   - queries, ids_out and scores_out (if given) must be device memory of the
 *     index's GPU; host buffers are rejected (copying them would allocate);
 *   - it always runs the exact CUDA-core scan (never the tensor-core
 *     prefilter, whose scratch is larger), so it is slower than
 *     uv_index_search on large batches;
 *   - 1 <= k <= 128;
 *   - UV_EUNSUPPORTED for dim > 384 (no room for the resident query tile of
 *     the exact scan) and for a cosine search of an index with the 1-bit
 *     shortlist on (the shortlist search is not built without allocation);
 *   - per-call scratch comes from one 16 MiB array that the library keeps on
 *     every GPU that loads it, until the process exits.  A batch needs, per
 *     query, 4*dim_pad + 4*max(1, n_centroids) + 4 bytes (dim_pad = dim
 *     rounded up to 4), plus 12*k bytes per record split (at least one),
 *     plus 4*k when scores_out is NULL, each of those arrays rounded up to
 *     256 bytes for the whole batch; a batch that does not fit even with one
 *     split is rejected with UV_EINVAL -- search fewer queries per call;
 *   - the first call on a device looks up that array's device address, so
 *     make it before any stream capture; the address is kept until exit and
 *     is stale after a cudaDeviceReset of that device;
 *   - all calls on a device share the array: calls whose GPU work overlaps
 *     (different streams or threads without ordering) race and corrupt each
 *     other's results; order them on one stream. */
int uv_index_search_noalloc(const uv_index *index, const float *queries, int64_t nq, int32_t k,
                            int32_t mode, int64_t *ids_out, float *scores_out, void *stream);

/* Drop every record but keep the device capacity: the state of a freshly
 * constructed codec after reserve(len) (src/trellis.rs:2100-2102). */
int uv_index_clear(uv_index *index);

/* Merge per-shard top-k lists (the multi-GPU combine after an all-gather):
 * in_ids/in_scores are nq x n_lists x k_in, each list sorted by the ranking
 * above; out is nq x k (k <= n_lists x k_in).  Device or host memory.  Up
 * to 8192 entries per row a k-way merge of the sorted lists, above that a
 * segmented sort.  nq = 0 returns UV_OK without reading any buffer. */
int uv_topk_merge(int32_t device, const int64_t *in_ids, const float *in_scores, int64_t nq,
                  int32_t n_lists, int32_t k_in, int32_t k, int64_t *out_ids, float *out_scores,
                  void *stream);

/* ---- a base split across GPUs (one index shard per GPU) ---------------- */

/* No counterpart in the reference (a single-process CPU crate): the
 * multi-GPU form of search (src/trellis.rs:2120-2183) over a base whose
 * records are split into disjoint shards, one uv_index per GPU, each added
 * with its rows' global ids.  Every shard answers a search in two phases
 * around one exchange, and the shards' lists then merge into the answer a
 * single index over the whole base gives (ids and score bits):
 *   1. uv_index_search_begin on every shard, with the number of shards:
 *      query preparation and the prefilter's first pass.  bounds_out
 *      receives nq x m lower bounds (uv_search_bounds_per_query; any order):
 *      scores that m distinct records of this shard reach (-inf where it
 *      has no such bound).
 *   2. The caller gathers every shard's bounds, shard-major (n_shards x nq x
 *      m floats: one all-gather), and hands them to uv_search_set_bounds on
 *      every shard.  The k-th largest of their union is a score that k
 *      records of the whole base reach, so no shard keeps a record below it;
 *      each shard then scores exactly only the records that can still be in
 *      the global top k, instead of its own top k's worth.  With one shard
 *      this step may be skipped (the shard's own top k, as uv_index_search);
 *      with several, uv_search_finish refuses to run before it.
 *   3. uv_search_finish: this shard's best (at most) k, ranked as
 *      uv_index_search, unfilled slots (id -1) where fewer records pass.
 *   4. uv_search_destroy (before the index is destroyed).
 * The lists of all shards then merge into the global top k: uv_topk_pack
 * the shard's lists, exchange query slices (all-to-all), and
 * uv_topk_merge_packed each slice over the shards.  All calls of one search
 * run on the stream given to begin; a search is used by one thread.  Any k
 * (above 128 every shard ranks all its records and step 2 changes
 * nothing); queries and outputs in host or device memory. */
typedef struct uv_search uv_search;
/* m, the bounds per query each of n_shards shards contributes for a top k:
 * k for one shard, else min(k, 2 * ceil(k / n_shards)).  bounds_out and
 * every shard's part of the gathered bounds are nq x m. */
int uv_search_bounds_per_query(int32_t k, int32_t n_shards, int32_t *m);
int uv_index_search_begin(const uv_index *index, const float *queries, int64_t nq, int32_t k,
                          int32_t mode, int32_t n_shards, float *bounds_out, uv_search **out,
                          void *stream);
int uv_search_set_bounds(uv_search *search, const float *gathered, int32_t n_shards);
int uv_search_finish(uv_search *search, int64_t *ids_out, float *scores_out);
/* Step 3 without waiting for the device: the same work as uv_search_finish
 * is queued on the search's stream and the call returns at once, so the
 * caller can queue the merge's collectives behind it.  Device buffers of the
 * index's GPU only.  The lists are final only after uv_search_check, which
 * waits for the stream: when a query's candidates overflowed the prefilter
 * (rare; *overflowed = 1) it scans that query exactly and rewrites its slots
 * in ids_out / scores_out, and a caller that already exchanged the lists
 * must merge them again.  A pipeline wait that timed out returns
 * UV_ETIMEDOUT there.  Searches that take the exact path finish at once
 * (uv_search_check then only waits). */
int uv_search_finish_deferred(uv_search *search, int64_t *ids_out, float *scores_out);
int uv_search_check(uv_search *search, int32_t *overflowed);
int uv_search_destroy(uv_search *search);

/* n (id, score) pairs as 12-byte records -- int32 id low, int32 id high,
 * f32 score bits -- so that a shard's lists travel in one collective.
 * Device buffers of `device`. */
int uv_topk_pack(int32_t device, const int64_t *ids, const float *scores, int64_t n, void *packed,
                 void *stream);
/* The inverse of uv_topk_pack (scores may be NULL).  Device buffers. */
int uv_topk_unpack(int32_t device, const void *packed, int64_t n, int64_t *ids, float *scores,
                   void *stream);
/* uv_topk_merge over packed records (device memory): list l of row q starts
 * at record q * row_stride + l * list_stride (0, 0: rows of n_lists x k_in
 * contiguous records).  After an all-to-all of query slices the lists of
 * slice row q from shard l sit at l * (rows * k_in) + q * k_in, i.e.
 * row_stride = k_in, list_stride = rows * k_in.  Any sizes (above 8192
 * entries per row a segmented sort replaces the k-way merge); nq = 0 (a
 * rank with an empty query slice) returns UV_OK without reading any
 * buffer, as uv_topk_merge does. */
int uv_topk_merge_packed(int32_t device, const void *packed, int64_t nq, int32_t n_lists,
                         int32_t k_in, int64_t row_stride, int64_t list_stride, int32_t k,
                         int64_t *out_ids, float *out_scores, void *stream);

/* Launch-shape tuning, no counterpart in the reference (results never depend
 * on it): "scan_splits" fixes the number of record ranges each query tile is
 * split into (0 = automatic); "encode_back" places the encoder's
 * back-pointers for codecs created afterwards (0 automatic, 1 global scratch,
 * 2 shared memory whenever one row's array fits); "encode_staged" 1 makes
 * codecs created afterwards encode every window wider than 14 bits with the
 * staged encoder (batches of rows, one launch per trellis step) instead of
 * one thread-block cluster per row (0 automatic: clusters up to 18 bits at
 * 1 and 2 bits per coordinate); "tc_scan" selects the flat
 * search's tensor-core prefilter (0 automatic, 1 never, 2 wherever it is
 * built); "tc_shape" where the prefilter keeps its queries (0 automatic =
 * 3: tensor memory; 1: shared memory); "tc_cache" keeps the prefilter's
 * fp16 record rows on the device between searches (1, the default: made on
 * the first search after a change of the records, per score mode, and held
 * until the next change or uv_index_destroy; (2 x dim rounded up to 64 + 32)
 * bytes per record and mode) or makes them in per-search scratch (0);
 * "ivf_tc_probe" 1 makes the IVF probe and the k-means / IVF assignment
 * compute every cosine or dot on the CUDA cores (0 automatic: tensor-core
 * dots, exact values for the centroids that can still be chosen, the same
 * lists and assignments); "ivf_tc" selects the IVF list scan (0 automatic:
 * the tensor-core bounds with exact rescoring for rows of 256 or more
 * coordinates and k <= 32; 1 the CUDA-core scan of every record; 2 the
 * tensor-core scan wherever it is built: k <= 32 and widths that are a
 * multiple of 16; its record rows, (2 x dim rounded up to 64 + 32) bytes per
 * record, are made on the first such search and kept with the lists);
 * "tc_sample" fixes the prefilter's first-pass sampling stride S (0
 * automatic: round(sqrt(14400/k)), at most 24 and 2400/k, with the sample
 * of largest g; round(sqrt(1600/k)), at most 10 and 900/k, with every S-th
 * tile); "tc_hot" chooses that
 * sample (0 automatic: the n/S records of largest score scale g, copied
 * into their own rows when the index changes; 1: every S-th record tile;
 * N >= 2: the n/N records of largest g); "tc_prepare" 1 makes the
 * prefilter's rows with the generic kernel, 2 with the shared-memory-table
 * kernel summing |x|^2 in f64 (0 automatic: that kernel for widths 1, 2, 4
 * summing in f32 under a rigorous inflation);
 * "coset_nearest" selects how the coset trellis finds each block's nearest
 * kept point (0 automatic: every book point scored for books of <= 8192
 * points, the reference's bisection + ball search where the minimum is tied
 * and for three bits; 1 the reference's search everywhere);
 * "rescore_warp" 1 makes the prefilter's exact rescoring use one CTA per
 * query throughout (0 automatic: one warp per query whose candidate list is
 * short, at widths up to 256 with tables of up to 1024 entries);
 * "cand_kernel" selects the
 * candidate scorer's kernel (0 automatic:
 * one thread per candidate at bits 1, 2, 4; 1 half a warp per candidate).
 * Process-wide; returns UV_EINVAL for an unknown key. */
int uv_set_tuning(const char *key, int64_t value);

/* Measurement aid, no counterpart in the reference: while enabled, every
 * kernel the library launches is bracketed by CUDA events on its launch
 * stream.  uv_profile_read waits for those events and returns the summed
 * device time and launch count of one kernel family ("encode",
 * "prep_queries", "flat_scan", "merge_topk", "tc_prepare" (the prefilter's
 * operand rows), "tc_hot" (its first pass's sample), "tc_pass1",
 * "tc_theta", "tc_pass2", "tc_rescore", "score_candidates", "shortlist", the IVF families
 * "ivf_*", or "*" for
 * all).  "tc_candidates" returns, as the count, the number of candidates the
 * last tensor-core search scored exactly.  Enabling clears previous records.
 * Not for concurrent use. */
int uv_profile_enable(int32_t on);
int uv_profile_read(const char *kernel, double *total_ms, int64_t *launches);

/* ---- the 1-bit companion shortlist ------------------------------------- */

/* with_shortlist(c) + with_shortlist_asym(asym) + with_shortlist_rnorm(rnorm)
 * (src/trellis.rs:803-839): records added afterwards also store the 1-bit
 * sign code of u_r (pack_indices(u_r > 0, 1), ceil(dim/8) bytes,
 * src/trellis.rs:1084-1094), and a cosine search becomes search_shortlist
 * (src/trellis.rs:854-948): stage 1 keeps the C = max(c, k) entries with the
 * best sign-code similarity -- dim - 2 * Hamming distance of the query's
 * sign code (asym 0) or the sequential sum of +-q_r[i] (asym 1), times rnorm
 * when rnorm is 1 and the index is centered -- and stage 2 scores those
 * with the codec's estimator.  Entries of equal stage-1 similarity are taken
 * lowest position first (the reference's select_nth_unstable leaves the
 * choice unspecified).  c = 0 switches it off.  Switching on or off needs an
 * empty index.  C is built up to 4096; MIPS searches ask for every record in
 * the reference (src/bench.rs:1029-1045), which no shortlist prunes, and use
 * the plain scan. */
int uv_index_set_shortlist(uv_index *index, int32_t c, int32_t asym, int32_t rnorm);
/* The sign codes, n x ceil(dim/8) (UV_EINVAL when the shortlist is off). */
int uv_index_export_signs(const uv_index *index, uint8_t *signs, void *stream);

/* ---- per-candidate scoring: CandidateScorer / PreparedQuery ----------- */

/* A codes-only graph walk (src/hnsw.rs:346-404) scores scattered records
 * through CandidateScorer::prepare(query) -> PreparedQuery::score_at(index)
 * (src/lib.rs:83-102, impl src/trellis.rs:2003-2086).  The batched form
 * prepares nq queries at once and scores CSR candidate lists: candidate i
 * belongs to query q where offsets[q] <= i < offsets[q+1] and names the
 * record at positions[i] (0 .. len-1, insertion order).  Each score is
 * score_at's: qm + rnorm * (dot / rescale), 0.0 for a query with
 * |q| < f32::EPSILON.  A position outside the index (the reference panics)
 * returns UV_EINVAL, with NaN in that slot.  The prepared batch reads the
 * index's arrays when it scores: keep the index alive while scoring
 * (uv_prepared_destroy may come after uv_index_destroy). */
typedef struct uv_prepared uv_prepared;
int uv_index_prepare(const uv_index *index, const float *queries, int64_t nq,
                     uv_prepared **out, void *stream);
int uv_prepared_destroy(uv_prepared *prepared);
int uv_prepared_len(const uv_prepared *prepared, int64_t *nq);
/* offsets: nq + 1 entries from 0 to n, or NULL when one query was prepared. */
int uv_prepared_score(const uv_prepared *prepared, const int64_t *offsets,
                      const int64_t *positions, int64_t n, float *scores_out, void *stream);
/* prepare + score for one query. */
int uv_index_score_candidates(const uv_index *index, const float *query,
                              const int64_t *positions, int64_t n, float *scores_out,
                              void *stream);
/* scored_len is uv_index_len.  scorer_model_bytes (src/trellis.rs:2084,
 * 2200-2218): code table + rotation signs + centroids. */
int uv_index_scorer_model_bytes(const uv_index *index, int64_t *bytes);

/* ---- IVF: coarse quantizer, posting lists of trellis records ----------- */

/* Every dot below is the reference's sequential f32 fold from -0.0 (product
 * and sum rounded separately), so centroids, assignments, probes and scores
 * are bit-identical to the reference's CPU results. */

/* bench.rs:298-349 kmeans: nlist centroids of the unit-normalized rows.
 * Initial centroids are units[splitmix64(seed) % n] (with replacement); each
 * of `iters` Lloyd rounds (the reference runs 5) assigns every unit to the
 * first strict maximum of <u, c_j>, then sets each non-empty list's centroid
 * to the sum of its units in row order from +0.0 divided by the count.
 * rows n x dim and centroids_out nlist x dim, host or device. */
int uv_kmeans(int32_t device, const float *rows, int64_t n, int32_t dim, int32_t nlist,
              uint64_t seed, int32_t iters, float *centroids_out, void *stream);

/* ivf.rs:405-421: assign[i] = the first strict maximum over j of
 * <rows[i] / max(|rows[i]|, EPS), c_j> (index 0 when every dot is NaN). */
int uv_ivf_assign(int32_t device, const float *rows, int64_t n, int32_t dim,
                  const float *centroids, int32_t nlist, uint32_t *assign_out, void *stream);

typedef struct uv_ivf uv_ivf;

/* IvfIndex (ivf.rs:155-170) over one codec: nlist centroids (copied) and one
 * posting list per centroid.  centered != 0 is ULTRAVEC_IVF_CENTER=1
 * (ivf.rs:98-150): each list's codec holds that list's centroid, so records
 * are residuals to it (rnorm kept) and scores add qm = <u, c_list>. */
int uv_ivf_create(const uv_codec *codec, const float *centroids, int32_t nlist, int32_t centered,
                  uv_ivf **out);
int uv_ivf_destroy(uv_ivf *ivf);

/* IvfIndex::build (ivf.rs:171-205): bucket the rows by assign (NULL computes
 * it as uv_ivf_assign does), rows in input order inside each list, encode
 * every list.  ids NULL gives id = row index.  Replaces earlier content. */
int uv_ivf_build(uv_ivf *ivf, const float *rows, int64_t n, const uint32_t *assign,
                 const int64_t *ids, void *stream);

int uv_ivf_len(const uv_ivf *ivf, int64_t *len);
int uv_ivf_nlist(const uv_ivf *ivf, int32_t *nlist);
/* Sum over the lists of the trellis mem_bytes (src/trellis.rs:2184-2201). */
int uv_ivf_mem_bytes(const uv_ivf *ivf, int64_t *bytes);

/* probe (ivf.rs:209-223): the min(nprobe, nlist) lists of best exact cosine
 * (lib.rs:240-248) to each raw query, ordered (cosine desc, list asc; the
 * reference leaves exact ties in any order).  lists_out is nq x nprobe;
 * columns past nlist hold -1. */
int uv_ivf_probe(const uv_ivf *ivf, const float *queries, int64_t nq, int32_t nprobe,
                 int32_t *lists_out, void *stream);

/* search (ivf.rs:229-239): each probed list scores its records with the list
 * codec (qm + rnorm * (dot / rescale)); the best k over the probed lists,
 * ranked as uv_index_search.  1 <= k <= 128. */
int uv_ivf_search(const uv_ivf *ivf, const float *queries, int64_t nq, int32_t k,
                  int32_t nprobe, int64_t *ids_out, float *scores_out, void *stream);

/* search over lists chosen beforehand: lists (host or device, nq x nprobe,
 * -1 = no list) as uv_ivf_probe returns them, possibly from another index
 * with the same centroids -- an IVF base split by posting list across GPUs
 * probes each query once, shares the lists, and every shard scans the
 * probed lists it holds (lists without records here are skipped).  The
 * results equal uv_ivf_search's for the same lists.  A list id >= nlist
 * returns UV_EINVAL.  1 <= k <= 128.  No counterpart in the reference (its
 * search probes and scans in one call, ivf.rs:229-239). */
int uv_ivf_search_lists(const uv_ivf *ivf, const float *queries, int64_t nq, int32_t k,
                        int32_t nprobe, const int32_t *lists, int64_t *ids_out, float *scores_out,
                        void *stream);

/* search_with_rerank (ivf.rs:248-274): the best r = max(rdepth, k) <= 128 by
 * the codec score, then exact fp32 cosine(query, db[id]) of those r, best k
 * by (cosine desc, id asc).  db is n_db x dim, host or device; an id >= n_db
 * returns UV_EINVAL. */
int uv_ivf_search_rerank(const uv_ivf *ivf, const float *queries, int64_t nq, int32_t k,
                         int32_t nprobe, int32_t rdepth, const float *db, int64_t n_db,
                         int64_t *ids_out, float *scores_out, void *stream);

/* The posting lists as one list-major SoA (the on-disk layout): list_off
 * (nlist + 1 entries), ids, codes (dense code_bytes per record), start,
 * rescale, rnorm.  NULL skips a field; host or device. */
int uv_ivf_export(const uv_ivf *ivf, int64_t *list_off, int64_t *ids, uint8_t *codes,
                  uint32_t *start, float *rescale, float *rnorm, void *stream);

/* IvfCodec::TrellisShortlist{c, asym, rnorm} (src/ivf.rs:52-60, 111-135):
 * every probed list runs search_shortlist(query, k, c) on its own entries
 * (see uv_index_set_shortlist; the rnorm weight applies to centered lists).
 * Set before uv_ivf_build; also used by uv_ivf_search_rerank's codec stage. */
int uv_ivf_set_shortlist(uv_ivf *ivf, int32_t c, int32_t asym, int32_t rnorm);
int uv_ivf_export_signs(const uv_ivf *ivf, uint8_t *signs, void *stream);

/* XOR-folded per-record FNV-1a digest of every posting (as uv_digest). */
int uv_ivf_digest(const uv_ivf *ivf, uint64_t *digest, void *stream);

/* ---- index files: one list-major SoA per index ------------------------- */

/* Build once, search many (and checkpoint): the records, sidecars, ids and
 * centroids of a flat index, or the lists of an IVF index, as one file of
 * flat little-endian arrays with a header carrying the codec configuration
 * and an FNV-1a checksum.  It replaces the reference's in-memory per-entry
 * records (TVec, src/trellis.rs:158-198).  Load returns UV_EINVAL for a
 * file that is not an index of this kind, was written by a codec of another
 * configuration, is truncated, or fails its checksum. */
int uv_index_save(const uv_index *index, const char *path);
int uv_index_load(const uv_codec *codec, const char *path, uv_index **out);
int uv_ivf_save(const uv_ivf *ivf, const char *path);
int uv_ivf_load(const uv_codec *codec, const char *path, uv_ivf **out);

/* ---- coset trellis (src/coset_trellis.rs) ------------------------------ */

/* The reference's research arm behind ULTRAVEC_COSET_TRELLIS=1: trellis-coded
 * quantization over the eight cosets of an index-8 sublattice of E8, one
 * 8-wide block per step, 2 branch bits + (8*bits - 3) book-index bits per
 * block, a free-start Viterbi over 2^mem states with 4 branches each.
 * One handle is the whole CosetTrellis backend (codec + entries). */
typedef struct uv_coset uv_coset;

/* CosetTrellis::new (coset_trellis.rs:121-190): dim % 8 == 0 and bits 1..3
 * (UV_EINVAL otherwise, where the reference panics), dim <= 4096
 * (UV_EUNSUPPORTED above); mem 1..20 (the
 * reference reads ULTRAVEC_TRELLIS_MEM, default 12); the rotation as
 * Rotor::new_oblivious (seed 42, 3 rounds by default).  The books of a bit
 * width are built once per process (three bits: 2^24 points, seconds). */
int uv_coset_create(int32_t dim, int32_t bits, int32_t mem, uint64_t rotation_seed,
                    int32_t rotation_rounds, int32_t device, uv_coset **out);
int uv_coset_destroy(uv_coset *coset);
/* with_centroids (192-196); before the first add. */
int uv_coset_set_centroids(uv_coset *coset, const float *centroids, int32_t n_centroids);
/* add (ids given) / add_batch (ids NULL: the batch's positions 0..n-1, as
 * the reference's add_batch assigns them, 454-469).  Rows n x dim f32. */
int uv_coset_add(uv_coset *coset, const int64_t *ids, const float *rows, int64_t n,
                 void *stream);
/* search (471-497), any k >= 1: score = <q,c> + rnorm * dot(q_r, x-bar) /
 * rescale, descending, ties by insertion position; slots past len() hold id
 * -1 and score -inf.  Above k = 128 every record's score is ranked (the
 * reference sorts them all and truncates).  Host or device buffers. */
int uv_coset_search(const uv_coset *coset, const float *queries, int64_t nq, int32_t k,
                    int64_t *ids_out, float *scores_out, void *stream);
int uv_coset_len(const uv_coset *coset, int64_t *n);
/* bytes per record as stored by the reference (start state + packed
 * symbols) and points per coset book */
int uv_coset_shape(const uv_coset *coset, int32_t *code_len, int32_t *per_coset);
/* the books (8 x per_coset keys: norm << 40 | raw doubled coordinates + 16,
 * five bits each, first coordinate highest) and {mean, std}; host memory */
int uv_coset_books(const uv_coset *coset, uint64_t *keys, float *scale);
/* mem_bytes (498-504) and memory_breakdown().model_bytes (505-517) */
int uv_coset_mem_bytes(const uv_coset *coset, int64_t *bytes);
int uv_coset_model_bytes(const uv_coset *coset, int64_t *bytes);
/* the records: n x code_len bytes, rescale, rnorm, cidx, ids (NULL skips) */
int uv_coset_export(const uv_coset *coset, uint8_t *codes, float *rescale, float *rnorm,
                    uint32_t *cidx, int64_t *ids, void *stream);
/* reconstruct_unit (521-529) of n rows, n x dim in and out */
int uv_coset_reconstruct(const uv_coset *coset, const float *rows, int64_t n, float *out,
                         void *stream);

#ifdef __cplusplus
}
#endif
#endif
