/*
 * uv_oracle.h -- CPU oracle for the UltraVec trellis hot paths.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a plain-C restatement of the
 * reference Rust arithmetic (ultravec-ann: src/trellis.rs, src/lib.rs,
 * src/simd.rs, src/dist.rs, src/bench.rs, src/ivf.rs).  It is the checker the
 * CUDA path is compared against and the timed CPU baseline; nothing in the
 * product links it.  Every function cites the reference lines it follows.
 *
 * Build: see oracle/Makefile (-O2 -ffp-contract=off -fno-fast-math -mfma).
 * No expression is contracted into an FMA except where the reference itself
 * issues one (_mm256_fmadd_ps in simd.rs), which is restated with fmaf().
 */
#ifndef UV_ORACLE_H
#define UV_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct uvo_codec uvo_codec;

/* --- primitives (lib.rs / dist.rs / trellis.rs) --- */
double uvo_inv_norm_cdf(double p);
float uvo_gaussian_code(uint32_t w);
uint64_t uvo_splitmix64(uint64_t *state);
double uvo_next_f64(uint64_t *state);
float uvo_l2_norm(const float *v, int n);
void uvo_l2_norms(const float *rows, int64_t n, int dim, float *out, int threads);
float uvo_std_about_mean(const float *v, int n);
void uvo_fwht(float *buf, int n);
int uvo_pack_indices(const uint16_t *idx, int n, int bits, uint8_t *out);
void uvo_unpack_indices(const uint8_t *data, int nbytes, int bits, uint16_t *out, int n);
float uvo_lut_dot_u32(const float *q, const uint32_t *idx, const float *book, int n);
float uvo_dense_dot(const float *a, const float *b, int n);
void uvo_acs_step(const float *cost, const float *total, int n_states, int n_emit,
                  float *next, uint8_t *back);

/* --- codec (trellis.rs TrellisQuantizer / TrellisConfig) --- */
uvo_codec *uvo_codec_new(int dim, int bits, int mem, uint64_t seed, int rounds,
                         int start_bits, int rescale_bits, float branch_lambda);
void uvo_codec_free(uvo_codec *c);
int uvo_codec_set_centroids(uvo_codec *c, const float *centroids, int n_centroids);
int uvo_codec_code_bytes(const uvo_codec *c);
int uvo_codec_table_len(const uvo_codec *c);
void uvo_codec_table(const uvo_codec *c, float *out);
void uvo_codec_signs(const uvo_codec *c, float *out); /* rounds*dim */
void uvo_rotate(const uvo_codec *c, const float *x, float *out);
void uvo_rotate_inverse(const uvo_codec *c, const float *y, float *out);

/* one row -> record.  Returns 0. */
int uvo_encode(const uvo_codec *c, const float *row, uint8_t *codes, uint32_t *start,
               float *rescale, float *rnorm, uint32_t *cidx);
/* the same record through the triple-loop scalar Viterbi (trellis.rs:2477-2528) */
int uvo_encode_scalar_ref(const uvo_codec *c, const float *row, uint8_t *codes,
                          uint32_t *start);
/* encode an already-rotated unit row (trellis.rs:689-699) */
int uvo_encode_rotated(const uvo_codec *c, const float *u_r, uint8_t *codes, uint32_t *start);
void uvo_encode_batch(const uvo_codec *c, const float *rows, int64_t n, uint8_t *codes,
                      uint32_t *start, float *rescale, float *rnorm, uint32_t *cidx,
                      int threads);
uint64_t uvo_record_digest(const uint8_t *codes, int code_bytes, uint32_t start);
uint64_t uvo_digest(const uint8_t *codes, const uint32_t *start, int64_t n, int code_bytes);

void uvo_windows(const uvo_codec *c, const uint8_t *codes, uint32_t start, uint32_t *out);
uint32_t uvo_window_at(const uvo_codec *c, const uint8_t *codes, uint32_t start, int i);
void uvo_decode_codes(const uvo_codec *c, const uint8_t *codes, uint32_t start, float *out);
void uvo_reconstruct_unit(const uvo_codec *c, const uint8_t *codes, uint32_t start,
                          float rnorm, uint32_t cidx, float *out);

/* query side (trellis.rs:2120-2183) */
int uvo_prepare_query(const uvo_codec *c, const float *q, float *q_r, float *qc);
float uvo_score(const uvo_codec *c, const float *q_r, float qm, const uint8_t *codes,
                uint32_t start, float rescale, float rnorm);

/* Flat scan over an SoA index: every record scored, top-k kept by
 * (score desc, id asc).  norms != NULL multiplies each score by norms[i]
 * (the MIPS sidecar, bench.rs:1029-1045).  ids of empty slots are -1. */
void uvo_search_topk(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                     const float *rescale, const float *rnorm, const uint32_t *cidx,
                     const float *norms, int64_t n, const float *queries, int64_t nq, int k,
                     int64_t *ids_out, float *scores_out, int threads);
/* encode_batch / ivf_encode plus the shortlist's 1-bit sign codes
 * (trellis.rs:1084-1094), n x ceil(dim/8) */
void uvo_encode_batch_signs(const uvo_codec *c, const float *rows, int64_t n, uint8_t *codes,
                            uint32_t *start, float *rescale, float *rnorm, uint32_t *cidx,
                            uint8_t *signs, int threads);
void uvo_ivf_encode_signs(const uvo_codec *c, const float *rows, int64_t n,
                          const float *centroids, const uint32_t *assign, uint8_t *codes,
                          uint32_t *start, float *rescale, float *rnorm, uint8_t *signs,
                          int threads);
/* search_shortlist (trellis.rs:854-948): flat and per IVF list */
void uvo_search_shortlist(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                          const float *rescale, const float *rnorm, const uint32_t *cidx,
                          const uint8_t *signs, int64_t n, const float *queries, int64_t nq,
                          int k, int cs, int asym, int weight, int64_t *ids_out,
                          float *scores_out, int threads);
void uvo_ivf_search_shortlist(const uvo_codec *c, const float *centroids, int nlist,
                              const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                              const uint32_t *start, const float *rescale, const float *rnorm,
                              const uint8_t *signs, int centered, const float *queries,
                              int64_t nq, int nprobe, int k, int cs, int asym, int weight,
                              int64_t *ids_out, float *scores_out, int threads);
/* batched CandidateScorer::prepare + score_at (trellis.rs:2016-2086) */
void uvo_score_candidates(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                          const float *rescale, const float *rnorm, const uint32_t *cidx,
                          const float *queries, int64_t nq, const int64_t *offsets,
                          const int64_t *positions, int64_t n, float *out, int threads);

/* exact ground truth, raw inner product (bench.rs:989-1001) or cosine
 * (bench.rs:126-146), ties by id */
void uvo_exact_topk(const float *db, int64_t n, int dim, const float *queries, int64_t nq,
                    int k, int cosine, int64_t *ids_out, int threads);

/* IVF (bench.rs:298-349, ivf.rs:171-239, 405-421) */
void uvo_kmeans(const float *db, int64_t n, int dim, int nlist, uint64_t seed, int iters,
                float *centroids_out, int threads);
void uvo_assign(const float *db, int64_t n, int dim, const float *centroids, int nlist,
                uint32_t *assign_out, int threads);
void uvo_ivf_probe(const float *centroids, int nlist, int dim, const float *query,
                   int nprobe, int32_t *lists_out);

void uvo_ivf_encode(const uvo_codec *c, const float *rows, int64_t n, const float *centroids,
                    const uint32_t *assign, uint8_t *codes, uint32_t *start, float *rescale,
                    float *rnorm, int threads);
void uvo_ivf_search_topk(const uvo_codec *c, const float *centroids, int nlist,
                         const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                         const uint32_t *start, const float *rescale, const float *rnorm,
                         int centered, const float *queries, int64_t nq, int nprobe, int k,
                         int64_t *ids_out, float *scores_out, int threads);

void uvo_ivf_search_rerank(const uvo_codec *c, const float *centroids, int nlist,
                           const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                           const uint32_t *start, const float *rescale, const float *rnorm,
                           int centered, const float *queries, int64_t nq, int nprobe, int k,
                           int rdepth, const float *db, int64_t *ids_out, float *scores_out,
                           int threads);

/* synthetic inputs used by the reference's own tests (trellis.rs:2387-2403) */
void uvo_rand_unit(int64_t n, int dim, uint64_t seed, float *out);

/* --- coset trellis (coset_trellis.rs, e8.rs): uv_oracle_coset.c --- */
typedef struct uvo_coset uvo_coset;
uint64_t uvo_e8_key(const int16_t *r);
void uvo_e8_unkey(uint64_t key, int16_t *r);
int uvo_coset_of(const int16_t *r);
void uvo_e8_nearest(const float *y, float *out);
int64_t uvo_e8_enumerate(float r2_max, uint64_t *keys, int64_t cap);
uvo_coset *uvo_coset_new(int dim, int bits, int mem, uint64_t seed, int rounds);
void uvo_coset_free(uvo_coset *c);
int uvo_coset_set_centroids(uvo_coset *c, const float *centroids, int n_centroids);
int uvo_coset_per_coset(const uvo_coset *c);
int uvo_coset_code_len(const uvo_coset *c);
void uvo_coset_books(const uvo_coset *c, uint64_t *out);
void uvo_coset_scale(const uvo_coset *c, float *out);
int64_t uvo_coset_index(const uvo_coset *c, int k, const int16_t *r);
void uvo_coset_nearest(const uvo_coset *c, int k, const float *y, int64_t *idx, float *dist);
void uvo_coset_nearest_exhaustive(const uvo_coset *c, int k, const float *y, int64_t *idx,
                                  float *dist);
void uvo_coset_encode_batch(const uvo_coset *c, const float *rows, int64_t n, uint8_t *codes,
                            float *rescale, float *rnorm, uint32_t *cidx);
void uvo_coset_decode(const uvo_coset *c, const uint8_t *rec, float *xbar);
void uvo_coset_reconstruct_unit(const uvo_coset *c, const float *row, float *out);
void uvo_coset_search(const uvo_coset *c, const uint8_t *codes, const float *rescale,
                      const float *rnorm, const uint32_t *cidx, const int64_t *ids, int64_t n,
                      const float *queries, int64_t nq, int k, int64_t *out_ids,
                      float *out_scores);
int64_t uvo_coset_mem_bytes(const uvo_coset *c, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
