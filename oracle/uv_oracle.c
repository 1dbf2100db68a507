/*
 * uv_oracle.c -- CPU oracle for the UltraVec trellis hot paths.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline.
 * A plain-C restatement of the reference Rust (ultravec-ann).  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Floating-point contract (matches rustc, which never contracts):
 *   - compiled with -ffp-contract=off -fno-fast-math, so a*b+c is two
 *     roundings everywhere;
 *   - fmaf() appears only where the reference issues _mm256_fmadd_ps
 *     (simd.rs:202-245), with the same per-lane association;
 *   - Rust's `.sum::<f32>()` is a sequential left fold from -0.0;
 *   - Rust's f32::max(a, b) returns the non-NaN operand, like fmaxf.
 */
#include "uv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define F32_EPS 1.1920928955078125e-7f /* f32::EPSILON */

struct uvo_codec {
    int dim, bits, mem, rounds, start_bits, rescale_bits;
    float lambda;
    uint64_t seed;
    int n_windows; /* 2^(mem+bits) */
    float *code;   /* normalized table, trellis.rs:588-610 */
    float *signs;  /* rounds x dim, lib.rs:428-463 */
    int n_blocks;
    int blk_off[32], blk_len[32]; /* greedy pow2 blocks, lib.rs:430-440 */
    int n_centroids;
    float *centroids; /* n_centroids x dim */
};

/* ------------------------------------------------------------------ */
/* dist.rs:158-201  inv_norm_cdf (Beasley-Springer-Moro), f64          */
/* ------------------------------------------------------------------ */
double uvo_inv_norm_cdf(double p) {
    static const double a[6] = {-3.969683028665376e1, 2.209460984245205e2,
                                -2.759285104469687e2, 1.383577518672690e2,
                                -3.066479806614716e1, 2.506628277459239e0};
    static const double b[5] = {-5.447609879822406e1, 1.615858368580409e2,
                                -1.556989798598866e2, 6.680131188771972e1,
                                -1.328068155288572e1};
    static const double c[6] = {-7.784894002430293e-3, -3.223964580411365e-1,
                                -2.400758277161838e0, -2.549732539343734e0,
                                4.374664141464968e0, 2.938163982698783e0};
    static const double d[4] = {7.784695709041462e-3, 3.224671290700398e-1,
                                2.445134137142996e0, 3.754408661907416e0};
    const double p_low = 0.02425;
    if (p < p_low) {
        double q = sqrt(-2.0 * log(p));
        return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
               ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
    } else if (p <= 1.0 - p_low) {
        double q = p - 0.5;
        double r = q * q;
        return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
               (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0);
    } else {
        double q = sqrt(-2.0 * log(1.0 - p));
        return -((((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
                 ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0));
    }
}

/* trellis.rs:136-145  lowbias32 hash -> uniform(0,1) -> inverse normal */
float uvo_gaussian_code(uint32_t w) {
    uint32_t h = w;
    h ^= h >> 16;
    h *= 0x7feb352dU;
    h ^= h >> 15;
    h *= 0x846ca68bU;
    h ^= h >> 16;
    double u = ((double)h + 0.5) / 4294967296.0;
    return (float)uvo_inv_norm_cdf(u);
}

/* lib.rs:259-265 */
uint64_t uvo_splitmix64(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* lib.rs:268-270 */
double uvo_next_f64(uint64_t *state) {
    return (double)(uvo_splitmix64(state) >> 11) / (double)(1ULL << 53);
}

/* Rust `.sum::<f32>()`: left fold starting from -0.0 */
static float seq_sum_sq(const float *v, int n) {
    float s = -0.0f;
    for (int i = 0; i < n; i++) s += v[i] * v[i];
    return s;
}

static float seq_dot(const float *a, const float *b, int n) {
    float s = -0.0f;
    for (int i = 0; i < n; i++) s += a[i] * b[i];
    return s;
}

/* lib.rs:215-217 */
float uvo_l2_norm(const float *v, int n) { return sqrtf(seq_sum_sq(v, n)); }

/* lib.rs:251-256 */
float uvo_std_about_mean(const float *x, int n) {
    float nf = (float)n;
    float s = -0.0f;
    for (int i = 0; i < n; i++) s += x[i];
    float mean = s / nf;
    float v = -0.0f;
    for (int i = 0; i < n; i++) v += (x[i] - mean) * (x[i] - mean);
    float var = v / nf;
    return sqrtf(var);
}

/* lib.rs:281-295 (+ the byte-identical AVX2 butterflies 300-364) */
void uvo_fwht(float *buf, int n) {
    for (int h = 1; h < n; h *= 2) {
        for (int i = 0; i < n; i += 2 * h) {
            for (int j = i; j < i + h; j++) {
                float u = buf[j], v = buf[j + h];
                buf[j] = u + v;
                buf[j + h] = u - v;
            }
        }
    }
    float inv = 1.0f / sqrtf((float)n);
    for (int i = 0; i < n; i++) buf[i] *= inv;
}

/* lib.rs:610-627  MSB-first packing; returns bytes written */
int uvo_pack_indices(const uint16_t *idx, int n, int bits, uint8_t *out) {
    uint32_t buf = 0, in_buf = 0;
    int o = 0;
    for (int i = 0; i < n; i++) {
        buf = (buf << bits) | (uint32_t)idx[i];
        in_buf += (uint32_t)bits;
        while (in_buf >= 8) {
            in_buf -= 8;
            out[o++] = (uint8_t)((buf >> in_buf) & 0xFF);
        }
    }
    if (in_buf > 0) out[o++] = (uint8_t)((buf << (8 - in_buf)) & 0xFF);
    return o;
}

/* lib.rs:630-652  stops at the end of the data, leaving later slots alone */
void uvo_unpack_indices(const uint8_t *data, int nbytes, int bits, uint16_t *out, int n) {
    uint32_t mask = (1u << bits) - 1, buf = 0, in_buf = 0;
    int byte = 0;
    for (int i = 0; i < n; i++) {
        while (in_buf < (uint32_t)bits && byte < nbytes) {
            buf = (buf << 8) | data[byte];
            in_buf += 8;
            byte++;
        }
        if (in_buf < (uint32_t)bits) return;
        in_buf -= (uint32_t)bits;
        out[i] = (uint16_t)((buf >> in_buf) & mask);
    }
}

/* simd.rs:202-262  two 8-lane FMA accumulators over 16-element blocks, one
 * optional 8-element block, hsum256 = ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)),
 * then a scalar mul+add tail. */
float uvo_lut_dot_u32(const float *q, const uint32_t *idx, const float *book, int n) {
    float acc0[8], acc1[8];
    for (int j = 0; j < 8; j++) acc0[j] = acc1[j] = 0.0f;
    int i = 0;
    while (i + 16 <= n) {
        for (int j = 0; j < 8; j++) {
            acc0[j] = fmaf(q[i + j], book[idx[i + j]], acc0[j]);
            acc1[j] = fmaf(q[i + 8 + j], book[idx[i + 8 + j]], acc1[j]);
        }
        i += 16;
    }
    if (i + 8 <= n) {
        for (int j = 0; j < 8; j++) acc0[j] = fmaf(q[i + j], book[idx[i + j]], acc0[j]);
        i += 8;
    }
    float v[8];
    for (int j = 0; j < 8; j++) v[j] = acc0[j] + acc1[j];
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    float total = (s0 + s1) + (s2 + s3);
    while (i < n) {
        total += q[i] * book[idx[i]];
        i++;
    }
    return total;
}

/* simd.rs:55-90  the dense twin of the above (recon-cache mode) */
float uvo_dense_dot(const float *a, const float *b, int n) {
    float acc0[8], acc1[8];
    for (int j = 0; j < 8; j++) acc0[j] = acc1[j] = 0.0f;
    int i = 0;
    while (i + 16 <= n) {
        for (int j = 0; j < 8; j++) {
            acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
            acc1[j] = fmaf(a[i + 8 + j], b[i + 8 + j], acc1[j]);
        }
        i += 16;
    }
    if (i + 8 <= n) {
        for (int j = 0; j < 8; j++) acc0[j] = fmaf(a[i + j], b[i + j], acc0[j]);
        i += 8;
    }
    float v[8];
    for (int j = 0; j < 8; j++) v[j] = acc0[j] + acc1[j];
    float s0 = v[0] + v[4], s1 = v[1] + v[5], s2 = v[2] + v[6], s3 = v[3] + v[7];
    float total = (s0 + s1) + (s2 + s3);
    while (i < n) {
        total += a[i] * b[i];
        i++;
    }
    return total;
}

/* trellis.rs:1734-1750 / 1878-1951  Phase B of one column: seed with k = 0,
 * refine with strict `<` over ascending k; back[ns] = winning k. */
void uvo_acs_step(const float *cost, const float *total, int n_states, int n_emit,
                  float *next, uint8_t *back) {
    int b_step = 0;
    while ((1 << b_step) < n_emit) b_step++;
    for (int ns = 0; ns < n_states; ns++) {
        float best = cost[ns >> b_step] + total[ns];
        uint8_t bestk = 0;
        for (int k = 1; k < n_emit; k++) {
            int w = ns + k * n_states;
            float c = cost[w >> b_step] + total[w];
            if (c < best) {
                best = c;
                bestk = (uint8_t)k;
            }
        }
        next[ns] = best;
        back[ns] = bestk;
    }
}

/* Rust f32::total_cmp key (core::f32::total_cmp) */
static inline int32_t total_key(float f) {
    int32_t x;
    memcpy(&x, &f, 4);
    x ^= (int32_t)(((uint32_t)(x >> 31)) >> 1);
    return x;
}

/* ------------------------------------------------------------------ */
/* codec construction: trellis.rs:430-458 (from_config), 563-643 (build)*/
/* ------------------------------------------------------------------ */
uvo_codec *uvo_codec_new(int dim, int bits, int mem, uint64_t seed, int rounds,
                         int start_bits, int rescale_bits, float branch_lambda) {
    if (dim <= 0 || bits < 1 || bits > 16 || mem < 1 || mem + bits > 24) return NULL;
    uvo_codec *c = (uvo_codec *)calloc(1, sizeof(uvo_codec));
    c->dim = dim;
    c->bits = bits;
    c->mem = mem;
    c->seed = seed;
    c->rounds = rounds < 1 ? 1 : rounds; /* lib.rs:449 n_rounds.max(1) */
    c->start_bits = start_bits < mem ? start_bits : mem;
    c->rescale_bits = rescale_bits;
    c->lambda = branch_lambda;
    c->n_windows = 1 << (mem + bits);
    /* table: gaussian_code per window, then normalize (trellis.rs:593-610) */
    int nw = c->n_windows;
    c->code = (float *)malloc(sizeof(float) * nw);
    for (int k = 0; k < nw; k++) c->code[k] = uvo_gaussian_code((uint32_t)k);
    float s = -0.0f;
    for (int k = 0; k < nw; k++) s += c->code[k];
    float mean = s / (float)nw;
    float v = -0.0f;
    for (int k = 0; k < nw; k++) v += (c->code[k] - mean) * (c->code[k] - mean);
    float var = v / (float)nw;
    float inv_std = 1.0f / fmaxf(sqrtf(var), 1e-9f);
    for (int k = 0; k < nw; k++) c->code[k] = (c->code[k] - mean) * inv_std;
    /* blocks (lib.rs:430-440) */
    int remaining = dim, offset = 0;
    c->n_blocks = 0;
    while (remaining > 0) {
        int bs = 1;
        while (bs * 2 <= remaining) bs *= 2;
        c->blk_off[c->n_blocks] = offset;
        c->blk_len[c->n_blocks] = bs;
        c->n_blocks++;
        offset += bs;
        remaining -= bs;
    }
    /* signs (lib.rs:449-462) */
    c->signs = (float *)malloc(sizeof(float) * (size_t)c->rounds * dim);
    uint64_t st = seed;
    for (int r = 0; r < c->rounds; r++)
        for (int i = 0; i < dim; i++)
            c->signs[(size_t)r * dim + i] = (uvo_splitmix64(&st) & 1) == 0 ? -1.0f : 1.0f;
    return c;
}

void uvo_codec_free(uvo_codec *c) {
    if (!c) return;
    free(c->code);
    free(c->signs);
    free(c->centroids);
    free(c);
}

/* trellis.rs:952-956 with_centroids */
int uvo_codec_set_centroids(uvo_codec *c, const float *centroids, int n_centroids) {
    free(c->centroids);
    c->centroids = NULL;
    c->n_centroids = 0;
    if (n_centroids > 0) {
        c->centroids = (float *)malloc(sizeof(float) * (size_t)n_centroids * c->dim);
        memcpy(c->centroids, centroids, sizeof(float) * (size_t)n_centroids * c->dim);
        c->n_centroids = n_centroids;
    }
    return 0;
}

int uvo_codec_code_bytes(const uvo_codec *c) { return (c->dim * c->bits + 7) / 8; }
int uvo_codec_table_len(const uvo_codec *c) { return c->n_windows; }
void uvo_codec_table(const uvo_codec *c, float *out) {
    memcpy(out, c->code, sizeof(float) * c->n_windows);
}
void uvo_codec_signs(const uvo_codec *c, float *out) {
    memcpy(out, c->signs, sizeof(float) * (size_t)c->rounds * c->dim);
}

/* lib.rs:472-484  R rounds of (sign flip, FWHT) per block */
void uvo_rotate(const uvo_codec *c, const float *x, float *out) {
    memmove(out, x, sizeof(float) * c->dim);
    for (int r = 0; r < c->rounds; r++) {
        const float *sg = c->signs + (size_t)r * c->dim;
        for (int b = 0; b < c->n_blocks; b++) {
            float *blk = out + c->blk_off[b];
            for (int i = 0; i < c->blk_len[b]; i++) blk[i] *= sg[c->blk_off[b] + i];
            uvo_fwht(blk, c->blk_len[b]);
        }
    }
}

/* lib.rs:487-499 */
void uvo_rotate_inverse(const uvo_codec *c, const float *y, float *out) {
    memmove(out, y, sizeof(float) * c->dim);
    for (int r = c->rounds - 1; r >= 0; r--) {
        const float *sg = c->signs + (size_t)r * c->dim;
        for (int b = 0; b < c->n_blocks; b++) {
            float *blk = out + c->blk_off[b];
            uvo_fwht(blk, c->blk_len[b]);
            for (int i = 0; i < c->blk_len[b]; i++) blk[i] *= sg[c->blk_off[b] + i];
        }
    }
}

/* trellis.rs:993-1004 assign: first strict maximum of the dot */
static int assign_centroid(const uvo_codec *c, const float *u) {
    int best = 0;
    float best_dot = -INFINITY;
    for (int j = 0; j < c->n_centroids; j++) {
        float d = seq_dot(u, c->centroids + (size_t)j * c->dim, c->dim);
        if (d > best_dot) {
            best_dot = d;
            best = j;
        }
    }
    return best;
}

/* trellis.rs:1144-1160 prep: unit vector, or the unit residual to its centroid.
 * `list_centroid` != NULL is the IVF case (ivf.rs:98-150): the posting list's
 * codec holds that single centroid, so the assignment is always index 0. */
static void prep_ex(const uvo_codec *c, const float *o, const float *list_centroid, float *r,
                    float *rnorm, uint32_t *cidx) {
    int d = c->dim;
    float norm = fmaxf(uvo_l2_norm(o, d), F32_EPS);
    for (int i = 0; i < d; i++) r[i] = o[i] / norm;
    if (c->n_centroids == 0 && list_centroid == NULL) {
        *rnorm = 1.0f;
        *cidx = 0;
        return;
    }
    int j = list_centroid ? 0 : assign_centroid(c, r);
    const float *cc = list_centroid ? list_centroid : c->centroids + (size_t)j * d;
    for (int i = 0; i < d; i++) r[i] = r[i] - cc[i];
    float rn = fmaxf(uvo_l2_norm(r, d), F32_EPS);
    for (int i = 0; i < d; i++) r[i] /= rn;
    *rnorm = rn;
    *cidx = (uint32_t)j;
}

static void prep(const uvo_codec *c, const float *o, float *r, float *rnorm, uint32_t *cidx) {
    prep_ex(c, o, NULL, r, rnorm, cidx);
}

/* trellis.rs:1349-1378: the general exact pass (taken when mem < bits): free
 * start limited to start_bits, infinite states skipped, strict `<` against a
 * column initialised to +inf, u32 back-pointers (zeroed), total_cmp argmin. */
static uint32_t viterbi_general(const uvo_codec *c, const float *u_rs, uint16_t *emissions,
                                int restrict_start) {
    int d = c->dim, n_states = 1 << c->mem, n_emit = 1 << c->bits, b = c->bits;
    uint32_t mask = (uint32_t)n_states - 1;
    float *cost = (float *)malloc(sizeof(float) * n_states);
    float *next = (float *)malloc(sizeof(float) * n_states);
    uint32_t *back = (uint32_t *)calloc((size_t)d * n_states, sizeof(uint32_t));
    for (int s = 0; s < n_states; s++) cost[s] = 0.0f;
    if (restrict_start && c->start_bits < c->mem)
        for (int s = 1 << c->start_bits; s < n_states; s++) cost[s] = INFINITY;
    for (int step = 0; step < d; step++) {
        for (int s = 0; s < n_states; s++) next[s] = INFINITY;
        for (int s = 0; s < n_states; s++) {
            float cs = cost[s];
            if (cs == INFINITY) continue;
            for (int e = 0; e < n_emit; e++) {
                uint32_t w = ((uint32_t)s << b) | (uint32_t)e;
                float xi = u_rs[step];
                float wi = 1.0f + c->lambda * xi * xi;
                float dd = xi - c->code[w];
                float d2 = 0.0f;
                d2 += wi * dd * dd;
                float cc = cs + d2;
                uint32_t nsx = w & mask;
                if (cc < next[nsx]) {
                    next[nsx] = cc;
                    back[(size_t)step * n_states + nsx] = ((uint32_t)s << b) | (uint32_t)e;
                }
            }
        }
        float *t = cost;
        cost = next;
        next = t;
    }
    int s = 0;
    int32_t bk = total_key(cost[0]);
    for (int i = 1; i < n_states; i++) {
        int32_t k = total_key(cost[i]);
        if (k < bk) {
            bk = k;
            s = i;
        }
    }
    uint32_t emit_mask = (1u << b) - 1;
    for (int step = d - 1; step >= 0; step--) {
        uint32_t packed = back[(size_t)step * n_states + s];
        emissions[step] = (uint16_t)(packed & emit_mask);
        s = (int)(packed >> b);
    }
    free(cost);
    free(next);
    free(back);
    return (uint32_t)s;
}

/* trellis.rs:1246-1347 (V=1 fast path, mem >= bits) + 1688-1751 + 1783-1802.
 * back is n_steps*n_states bytes of k; returns the start state. */
static uint32_t viterbi_fast(const uvo_codec *c, const float *u_rs, uint16_t *emissions,
                             float *cost, float *next, float *total, uint8_t *back) {
    int n_steps = c->dim, n_states = 1 << c->mem, n_emit = 1 << c->bits, b = c->bits;
    int n_win = n_emit * n_states;
    for (int s = 0; s < n_states; s++) cost[s] = 0.0f;
    if (c->start_bits < c->mem)
        for (int s = 1 << c->start_bits; s < n_states; s++) cost[s] = INFINITY;
    for (int step = 0; step < n_steps; step++) {
        float xi = u_rs[step];
        float wi = 1.0f + c->lambda * xi * xi;
        /* metric_scalar trellis.rs:1955-1961 */
        for (int w = 0; w < n_win; w++) {
            float d = xi - c->code[w];
            total[w] = (wi * d) * d;
        }
        uvo_acs_step(cost, total, n_states, n_emit, next, back + (size_t)step * n_states);
        float *t = cost;
        cost = next;
        next = t;
    }
    /* backtrack_packed 1783-1802: first minimum under total_cmp */
    int s = 0;
    int32_t bk = total_key(cost[0]);
    for (int i = 1; i < n_states; i++) {
        int32_t k = total_key(cost[i]);
        if (k < bk) {
            bk = k;
            s = i;
        }
    }
    uint32_t emit_mask = (1u << b) - 1;
    for (int step = n_steps - 1; step >= 0; step--) {
        int k = back[(size_t)step * n_states + s];
        uint32_t w = (uint32_t)(s + k * n_states);
        emissions[step] = (uint16_t)(w & emit_mask);
        s = (int)(w >> b);
    }
    return (uint32_t)s;
}

/* trellis.rs:1009-1133 finalize (codes-only: no recon, no residual sketch) */
static void finalize(const uvo_codec *c, const uint16_t *em, uint32_t start, const float *u_r,
                     uint8_t *codes, float *rescale_out) {
    uint32_t state = start, mask = (1u << c->mem) - 1;
    float rescale = 0.0f;
    for (int i = 0; i < c->dim; i++) {
        uint32_t w = (state << c->bits) | em[i];
        float cv = c->code[w];
        rescale += cv * u_r[i];
        state = w & mask;
    }
    if (c->rescale_bits > 0 && rescale > 1e-6f) {
        float levels = (float)((1u << c->rescale_bits) - 1);
        float sq = sqrtf((float)c->dim);
        float lo = 0.0f * sq, hi = 1.25f * sq;
        float t = (rescale - lo) / (hi - lo);
        t = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
        rescale = lo + roundf(t * levels) / levels * (hi - lo);
    }
    *rescale_out = rescale > 1e-6f ? rescale : INFINITY;
    uvo_pack_indices(em, c->dim, c->bits, codes);
}

typedef struct {
    float *r, *u_r, *u_rs, *cost, *next, *total;
    uint8_t *back;
    uint16_t *em;
} scratch_t;

static void scratch_init(const uvo_codec *c, scratch_t *s) {
    int d = c->dim, ns = 1 << c->mem;
    s->r = (float *)malloc(sizeof(float) * d);
    s->u_r = (float *)malloc(sizeof(float) * d);
    s->u_rs = (float *)malloc(sizeof(float) * d);
    s->cost = (float *)malloc(sizeof(float) * ns);
    s->next = (float *)malloc(sizeof(float) * ns);
    s->total = (float *)malloc(sizeof(float) * c->n_windows);
    s->back = (uint8_t *)malloc((size_t)d * ns);
    s->em = (uint16_t *)malloc(sizeof(uint16_t) * d);
}

static void scratch_free(scratch_t *s) {
    free(s->r);
    free(s->u_r);
    free(s->u_rs);
    free(s->cost);
    free(s->next);
    free(s->total);
    free(s->back);
    free(s->em);
}

/* trellis.rs:1164-1212 encode (exact free-start Viterbi, no tail-biting).
 * The V=1 fast path (mem >= bits) and the general pass pick the same path on
 * finite inputs; the choice mirrors trellis.rs:1284/1296. */
static uint32_t run_viterbi(const uvo_codec *c, const float *u_rs, scratch_t *s) {
    if (c->mem >= c->bits)
        return viterbi_fast(c, u_rs, s->em, s->cost, s->next, s->total, s->back);
    return viterbi_general(c, u_rs, s->em, 1);
}

/* trellis.rs:1084-1094: the 1-bit sign code of u_r, pack_indices(u_r > 0, 1)
 * (MSB-first, ceil(dim/8) bytes) */
static void sign_code(const float *u_r, int d, uint8_t *out) {
    for (int b = 0; b < (d + 7) / 8; b++) {
        uint8_t v = 0;
        for (int t = 0; t < 8; t++) {
            int i = 8 * b + t;
            if (i < d && u_r[i] > 0.0f) v |= (uint8_t)(0x80u >> t);
        }
        out[b] = v;
    }
}

static void encode_with(const uvo_codec *c, const float *row, const float *list_centroid,
                        uint8_t *codes, uint32_t *start, float *rescale, float *rnorm,
                        uint32_t *cidx, uint8_t *sign, scratch_t *s) {
    int d = c->dim;
    prep_ex(c, row, list_centroid, s->r, rnorm, cidx);
    uvo_rotate(c, s->r, s->u_r);
    if (sign) sign_code(s->u_r, d, sign);
    float scale = fmaxf(uvo_std_about_mean(s->u_r, d), F32_EPS);
    for (int i = 0; i < d; i++) s->u_rs[i] = s->u_r[i] / scale;
    uint32_t st = run_viterbi(c, s->u_rs, s);
    finalize(c, s->em, st, s->u_r, codes, rescale);
    *start = st;
}

int uvo_encode(const uvo_codec *c, const float *row, uint8_t *codes, uint32_t *start,
               float *rescale, float *rnorm, uint32_t *cidx) {
    scratch_t s;
    scratch_init(c, &s);
    encode_with(c, row, NULL, codes, start, rescale, rnorm, cidx, NULL, &s);
    scratch_free(&s);
    return 0;
}

/* trellis.rs:689-699 */
int uvo_encode_rotated(const uvo_codec *c, const float *u_r, uint8_t *codes, uint32_t *start) {
    scratch_t s;
    scratch_init(c, &s);
    int d = c->dim;
    float scale = fmaxf(uvo_std_about_mean(u_r, d), F32_EPS);
    for (int i = 0; i < d; i++) s.u_rs[i] = u_r[i] / scale;
    uint32_t st = run_viterbi(c, s.u_rs, &s);
    uvo_pack_indices(s.em, d, c->bits, codes);
    *start = st;
    scratch_free(&s);
    return 0;
}

/* trellis.rs:2477-2528  the ORIGINAL triple loop the fast path is pinned to
 * (every state a free start, infinite states skipped, strict `<`) */
int uvo_encode_scalar_ref(const uvo_codec *c, const float *row, uint8_t *codes,
                          uint32_t *start) {
    scratch_t s;
    scratch_init(c, &s);
    int d = c->dim;
    float rn;
    uint32_t ci;
    prep(c, row, s.r, &rn, &ci);
    uvo_rotate(c, s.r, s.u_r);
    float scale = fmaxf(uvo_std_about_mean(s.u_r, d), F32_EPS);
    for (int i = 0; i < d; i++) s.u_rs[i] = s.u_r[i] / scale;
    uint32_t st = viterbi_general(c, s.u_rs, s.em, 0);
    uvo_pack_indices(s.em, d, c->bits, codes);
    *start = st;
    scratch_free(&s);
    return 0;
}

static void encode_rows(const uvo_codec *c, const float *rows, int64_t n,
                        const float *centroids, const uint32_t *assign, uint8_t *codes,
                        uint32_t *start, float *rescale, float *rnorm, uint32_t *cidx,
                        uint8_t *signs, int threads) {
    int cb = uvo_codec_code_bytes(c), sb = (c->dim + 7) / 8;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        scratch_t s;
        scratch_init(c, &s);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
        for (int64_t i = 0; i < n; i++) {
            float rn, rs;
            uint32_t ci;
            const float *lc = centroids ? centroids + (size_t)assign[i] * c->dim : NULL;
            encode_with(c, rows + (size_t)i * c->dim, lc, codes + (size_t)i * cb, start + i, &rs,
                        &rn, &ci, signs ? signs + (size_t)i * sb : NULL, &s);
            rescale[i] = rs;
            if (rnorm) rnorm[i] = rn;
            if (cidx) cidx[i] = ci;
        }
        scratch_free(&s);
    }
}

void uvo_encode_batch(const uvo_codec *c, const float *rows, int64_t n, uint8_t *codes,
                      uint32_t *start, float *rescale, float *rnorm, uint32_t *cidx,
                      int threads) {
    encode_rows(c, rows, n, NULL, NULL, codes, start, rescale, rnorm, cidx, NULL, threads);
}

/* encode_batch with the shortlist's sign codes (n x ceil(dim/8)) */
void uvo_encode_batch_signs(const uvo_codec *c, const float *rows, int64_t n, uint8_t *codes,
                            uint32_t *start, float *rescale, float *rnorm, uint32_t *cidx,
                            uint8_t *signs, int threads) {
    encode_rows(c, rows, n, NULL, NULL, codes, start, rescale, rnorm, cidx, signs, threads);
}

/* ivf.rs:171-205 + 98-150 (ULTRAVEC_IVF_CENTER=1): row i is encoded by its
 * list's codec, centered on centroids[assign[i]]; pass centroids = NULL for
 * the uncentered lists.  Output rows stay in input order. */
void uvo_ivf_encode(const uvo_codec *c, const float *rows, int64_t n, const float *centroids,
                    const uint32_t *assign, uint8_t *codes, uint32_t *start, float *rescale,
                    float *rnorm, int threads) {
    encode_rows(c, rows, n, centroids, assign, codes, start, rescale, rnorm, NULL, NULL, threads);
}

void uvo_ivf_encode_signs(const uvo_codec *c, const float *rows, int64_t n,
                          const float *centroids, const uint32_t *assign, uint8_t *codes,
                          uint32_t *start, float *rescale, float *rnorm, uint8_t *signs,
                          int threads) {
    encode_rows(c, rows, n, centroids, assign, codes, start, rescale, rnorm, NULL, signs, threads);
}

/* trellis.rs:970-990  FNV-1a over start (LE) then codes, XOR-folded */
uint64_t uvo_record_digest(const uint8_t *codes, int code_bytes, uint32_t start) {
    uint64_t h = 0xcbf29ce484222325ULL;
    for (int i = 0; i < 4; i++) {
        h ^= (uint64_t)((start >> (8 * i)) & 0xFF);
        h *= 0x00000100000001b3ULL;
    }
    for (int i = 0; i < code_bytes; i++) {
        h ^= (uint64_t)codes[i];
        h *= 0x00000100000001b3ULL;
    }
    return h;
}

uint64_t uvo_digest(const uint8_t *codes, const uint32_t *start, int64_t n, int code_bytes) {
    uint64_t acc = 0;
    for (int64_t i = 0; i < n; i++)
        acc ^= uvo_record_digest(codes + (size_t)i * code_bytes, code_bytes, start[i]);
    return acc;
}

/* trellis.rs:1576-1600 windows_into: the (M+b)-bit field at offset i*b of
 * [start (M bits) || codes], MSB-first; a short stream zero-fills. */
void uvo_windows(const uvo_codec *c, const uint8_t *codes, uint32_t start, uint32_t *out) {
    uint32_t width = (uint32_t)(c->mem + c->bits);
    uint64_t wmask = (1ULL << width) - 1;
    uint64_t acc = start;
    uint32_t nbits = (uint32_t)c->mem;
    int byte = 0, len = uvo_codec_code_bytes(c);
    for (int i = 0; i < c->dim; i++) {
        while (nbits < width && byte < len) {
            acc = (acc << 8) | codes[byte];
            nbits += 8;
            byte++;
        }
        if (nbits < width) {
            acc <<= (width - nbits);
            nbits = width;
        }
        out[i] = (uint32_t)((acc >> (nbits - width)) & wmask);
        nbits -= (uint32_t)c->bits;
        acc &= (1ULL << nbits) - 1;
    }
}

/* trellis.rs:727-743 */
uint32_t uvo_window_at(const uvo_codec *c, const uint8_t *codes, uint32_t start, int i) {
    uint32_t width = (uint32_t)(c->mem + c->bits);
    uint64_t wmask = (1ULL << width) - 1;
    uint64_t acc = (uint64_t)start & ((1ULL << c->mem) - 1);
    uint32_t end_bit = (uint32_t)(i + 1) * (uint32_t)c->bits, consumed = 0;
    int byte = 0;
    while (consumed < end_bit) {
        acc = (acc << 8) | codes[byte];
        byte++;
        consumed += 8;
    }
    uint32_t extra = consumed - end_bit;
    return (uint32_t)((acc >> extra) & wmask);
}

/* trellis.rs:705-720 decode_codes: table values by window, inverse-rotated */
void uvo_decode_codes(const uvo_codec *c, const uint8_t *codes, uint32_t start, float *out) {
    uint32_t *w = (uint32_t *)malloc(sizeof(uint32_t) * c->dim);
    float *xbar = (float *)malloc(sizeof(float) * c->dim);
    uvo_windows(c, codes, start, w);
    for (int i = 0; i < c->dim; i++) xbar[i] = c->code[w[i]];
    uvo_rotate_inverse(c, xbar, out);
    free(w);
    free(xbar);
}

/* trellis.rs:1624-1654 reconstruct_from */
void uvo_reconstruct_unit(const uvo_codec *c, const uint8_t *codes, uint32_t start,
                          float rnorm, uint32_t cidx, float *out) {
    int d = c->dim;
    uvo_decode_codes(c, codes, start, out);
    float n = fmaxf(uvo_l2_norm(out, d), F32_EPS);
    for (int i = 0; i < d; i++) out[i] /= n;
    if (c->n_centroids == 0) return;
    const float *cc = c->centroids + (size_t)cidx * d;
    for (int i = 0; i < d; i++) out[i] = cc[i] + rnorm * out[i];
    float nf = fmaxf(uvo_l2_norm(out, d), F32_EPS);
    for (int i = 0; i < d; i++) out[i] /= nf;
}

/* trellis.rs:2120-2136  returns 1 (degenerate, empty result) when |q| < EPS */
int uvo_prepare_query(const uvo_codec *c, const float *q, float *q_r, float *qc) {
    int d = c->dim;
    float qn = uvo_l2_norm(q, d);
    if (qn < F32_EPS) return 1;
    float *u = (float *)malloc(sizeof(float) * d);
    for (int i = 0; i < d; i++) u[i] = q[i] / qn;
    for (int j = 0; j < c->n_centroids; j++)
        qc[j] = seq_dot(u, c->centroids + (size_t)j * d, d);
    uvo_rotate(c, u, q_r);
    free(u);
    return 0;
}

/* trellis.rs:1483-1536 (codes-only, no residual) + 1614-1618 */
float uvo_score(const uvo_codec *c, const float *q_r, float qm, const uint8_t *codes,
                uint32_t start, float rescale, float rnorm) {
    uint32_t w[4096];
    uint32_t *wp = c->dim <= 4096 ? w : (uint32_t *)malloc(sizeof(uint32_t) * c->dim);
    uvo_windows(c, codes, start, wp);
    float dot = uvo_lut_dot_u32(q_r, wp, c->code, c->dim);
    if (wp != w) free(wp);
    return qm + rnorm * (dot / rescale);
}

/* ranking used by every top-k here: score desc, then id asc; NaN ranks last */
static inline float rank_key(float s) { return isnan(s) ? -INFINITY : s; }
static inline int better(float a, int64_t ia, float b, int64_t ib) {
    float fa = rank_key(a), fb = rank_key(b);
    return fa > fb || (fa == fb && ia < ib);
}

typedef struct {
    float s;
    int64_t id;
} cand_t;

/* bounded max-k selection with a min-heap whose root is the worst kept item */
static void heap_sift_down(cand_t *h, int n, int i) {
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && better(h[m].s, h[m].id, h[l].s, h[l].id)) m = l;
        if (r < n && better(h[m].s, h[m].id, h[r].s, h[r].id)) m = r;
        if (m == i) return;
        cand_t t = h[i];
        h[i] = h[m];
        h[m] = t;
        i = m;
    }
}

static void heap_push_bounded(cand_t *h, int *n, int k, float s, int64_t id) {
    if (*n < k) {
        int i = (*n)++;
        h[i].s = s;
        h[i].id = id;
        while (i > 0) {
            int p = (i - 1) / 2;
            if (better(h[p].s, h[p].id, h[i].s, h[i].id)) {
                cand_t t = h[i];
                h[i] = h[p];
                h[p] = t;
                i = p;
            } else
                break;
        }
    } else if (better(s, id, h[0].s, h[0].id)) {
        h[0].s = s;
        h[0].id = id;
        heap_sift_down(h, *n, 0);
    }
}

static int cand_cmp(const void *a, const void *b) {
    const cand_t *x = (const cand_t *)a, *y = (const cand_t *)b;
    if (better(x->s, x->id, y->s, y->id)) return -1;
    if (better(y->s, y->id, x->s, x->id)) return 1;
    return 0;
}

static void emit_topk(cand_t *h, int n, int k, int64_t *ids, float *scores) {
    qsort(h, (size_t)n, sizeof(cand_t), cand_cmp);
    for (int i = 0; i < k; i++) {
        if (i < n) {
            ids[i] = h[i].id;
            if (scores) scores[i] = h[i].s;
        } else {
            ids[i] = -1;
            if (scores) scores[i] = -INFINITY;
        }
    }
}

void uvo_search_topk(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                     const float *rescale, const float *rnorm, const uint32_t *cidx,
                     const float *norms, int64_t n, const float *queries, int64_t nq, int k,
                     int64_t *ids_out, float *scores_out, int threads) {
    int d = c->dim, cb = uvo_codec_code_bytes(c);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *q_r = (float *)malloc(sizeof(float) * d);
        float *qc = (float *)malloc(sizeof(float) * (c->n_centroids + 1));
        uint32_t *w = (uint32_t *)malloc(sizeof(uint32_t) * d);
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (k > 0 ? k : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            int nh = 0;
            int degenerate = uvo_prepare_query(c, queries + (size_t)qi * d, q_r, qc);
            if (!degenerate) {
                for (int64_t i = 0; i < n; i++) {
                    uvo_windows(c, codes + (size_t)i * cb, start[i], w);
                    float dot = uvo_lut_dot_u32(q_r, w, c->code, d);
                    float qm = 0.0f, rn = 1.0f;
                    if (c->n_centroids > 0) {
                        uint32_t j = cidx ? cidx[i] : 0;
                        qm = qc[j];
                    }
                    if (rnorm) rn = rnorm[i];
                    float s = qm + rn * (dot / rescale[i]);
                    if (norms) s *= norms[i];
                    heap_push_bounded(h, &nh, k, s, i);
                }
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, scores_out ? scores_out + (size_t)qi * k : NULL);
        }
        free(q_r);
        free(qc);
        free(w);
        free(h);
    }
}

/* trellis.rs:2016-2086 CandidateScorer::prepare + PreparedQuery::score_at,
 * batched: candidate i of the CSR batch (offsets[q] <= i < offsets[q+1];
 * offsets NULL puts every candidate on query 0) is the record at
 * positions[i].  A degenerate query scores 0.0 (trellis.rs:2031-2033); qm is
 * qc[cidx] or 0.0 without centroids (trellis.rs:2035). */
void uvo_score_candidates(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                          const float *rescale, const float *rnorm, const uint32_t *cidx,
                          const float *queries, int64_t nq, const int64_t *offsets,
                          const int64_t *positions, int64_t n, float *out, int threads) {
    int d = c->dim, cb = uvo_codec_code_bytes(c);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *q_r = (float *)malloc(sizeof(float) * d);
        float *qc = (float *)malloc(sizeof(float) * (c->n_centroids + 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            int64_t i0 = offsets ? offsets[qi] : 0, i1 = offsets ? offsets[qi + 1] : n;
            int degenerate = uvo_prepare_query(c, queries + (size_t)qi * d, q_r, qc);
            for (int64_t i = i0; i < i1; i++) {
                int64_t r = positions[i];
                if (degenerate) {
                    out[i] = 0.0f;
                    continue;
                }
                float qm = 0.0f;
                if (c->n_centroids > 0) qm = qc[cidx ? cidx[r] : 0];
                out[i] = uvo_score(c, q_r, qm, codes + (size_t)r * cb, start[r], rescale[r],
                                   rnorm ? rnorm[r] : 1.0f);
            }
        }
        free(q_r);
        free(qc);
    }
}

/* bench.rs:989-1001 (raw IP) and bench.rs:126-146 (cosine), ties by id */
void uvo_exact_topk(const float *db, int64_t n, int dim, const float *queries, int64_t nq,
                    int k, int cosine, int64_t *ids_out, int threads) {
    float *dbn = NULL;
    if (cosine) {
        dbn = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
        for (int64_t i = 0; i < n; i++) dbn[i] = uvo_l2_norm(db + (size_t)i * dim, dim);
    }
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (k > 0 ? k : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            const float *q = queries + (size_t)qi * dim;
            int nh = 0;
            float qn = cosine ? uvo_l2_norm(q, dim) : 1.0f;
            if (!(cosine && qn < F32_EPS)) {
                for (int64_t i = 0; i < n; i++) {
                    float dot = seq_dot(q, db + (size_t)i * dim, dim);
                    float s = dot;
                    if (cosine) s = dbn[i] < F32_EPS ? 0.0f : dot / (qn * dbn[i]);
                    heap_push_bounded(h, &nh, k, s, i);
                }
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, NULL);
        }
        free(h);
    }
    free(dbn);
}

/* bench.rs:319-333: first strict maximum of <u, c_j> for rows already unit */
static void assign_units(const float *units, int64_t n, int dim, const float *cent, int nlist,
                         uint32_t *out, int threads) {
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int64_t i = 0; i < n; i++) {
        const float *u = units + (size_t)i * dim;
        uint32_t best = 0;
        float bd = -INFINITY;
        for (int j = 0; j < nlist; j++) {
            float dd = seq_dot(u, cent + (size_t)j * dim, dim);
            if (dd > bd) {
                bd = dd;
                best = (uint32_t)j;
            }
        }
        out[i] = best;
    }
}

/* ivf.rs:405-421: normalize the row (l2 .max(EPS)), then the first strict
 * maximum of the dot with each centroid */
void uvo_assign(const float *db, int64_t n, int dim, const float *cent, int nlist,
                uint32_t *out, int threads) {
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *u = (float *)malloc(sizeof(float) * dim);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t i = 0; i < n; i++) {
            const float *v = db + (size_t)i * dim;
            float nn = fmaxf(uvo_l2_norm(v, dim), F32_EPS);
            for (int j = 0; j < dim; j++) u[j] = v[j] / nn;
            uint32_t best = 0;
            float bd = -INFINITY;
            for (int j = 0; j < nlist; j++) {
                float dd = seq_dot(u, cent + (size_t)j * dim, dim);
                if (dd > bd) {
                    bd = dd;
                    best = (uint32_t)j;
                }
            }
            out[i] = best;
        }
        free(u);
    }
}

/* bench.rs:298-349 kmeans over the unit-normalized rows */
void uvo_kmeans(const float *db, int64_t n, int dim, int nlist, uint64_t seed, int iters,
                float *cent, int threads) {
    float *units = (float *)malloc(sizeof(float) * (size_t)n * dim);
    for (int64_t i = 0; i < n; i++) {
        const float *v = db + (size_t)i * dim;
        float nn = fmaxf(uvo_l2_norm(v, dim), F32_EPS);
        for (int j = 0; j < dim; j++) units[(size_t)i * dim + j] = v[j] / nn;
    }
    uint64_t st = seed;
    for (int j = 0; j < nlist; j++) {
        uint64_t pick = uvo_splitmix64(&st) % (uint64_t)n;
        memcpy(cent + (size_t)j * dim, units + (size_t)pick * dim, sizeof(float) * dim);
    }
    uint32_t *asg = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)n);
    float *sums = (float *)malloc(sizeof(float) * (size_t)nlist * dim);
    int64_t *counts = (int64_t *)malloc(sizeof(int64_t) * nlist);
    for (int it = 0; it < iters; it++) {
        assign_units(units, n, dim, cent, nlist, asg, threads);
        for (size_t t = 0; t < (size_t)nlist * dim; t++) sums[t] = 0.0f;
        for (int j = 0; j < nlist; j++) counts[j] = 0;
        for (int64_t i = 0; i < n; i++) {
            uint32_t b = asg[i];
            counts[b]++;
            float *s = sums + (size_t)b * dim;
            const float *u = units + (size_t)i * dim;
            for (int j = 0; j < dim; j++) s[j] += u[j];
        }
        for (int j = 0; j < nlist; j++)
            if (counts[j] > 0)
                for (int t = 0; t < dim; t++)
                    cent[(size_t)j * dim + t] = sums[(size_t)j * dim + t] / (float)counts[j];
    }
    free(units);
    free(asg);
    free(sums);
    free(counts);
}

/* ivf.rs:209-223 probe by exact cosine (lib.rs `cosine`); the nprobe best,
 * ordered by (cosine desc, list asc) */
void uvo_ivf_probe(const float *cent, int nlist, int dim, const float *query, int nprobe,
                   int32_t *lists_out) {
    cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (nprobe > 0 ? nprobe : 1));
    int nh = 0;
    float na = uvo_l2_norm(query, dim);
    for (int j = 0; j < nlist; j++) {
        const float *c = cent + (size_t)j * dim;
        float dot = seq_dot(query, c, dim);
        float nb = uvo_l2_norm(c, dim);
        float cs = (na < F32_EPS || nb < F32_EPS) ? 0.0f : dot / (na * nb);
        heap_push_bounded(h, &nh, nprobe, cs, j);
    }
    int64_t *ids = (int64_t *)malloc(sizeof(int64_t) * (nprobe > 0 ? nprobe : 1));
    emit_topk(h, nh, nprobe, ids, NULL);
    for (int i = 0; i < nprobe; i++) lists_out[i] = (int32_t)ids[i];
    free(ids);
    free(h);
}

/* trellis.rs:2387-2403 rand_unit: splitmix64 Box-Muller rows, normalized */
void uvo_rand_unit(int64_t n, int dim, uint64_t seed, float *out) {
    uint64_t st = seed;
    for (int64_t i = 0; i < n; i++) {
        float *v = out + (size_t)i * dim;
        for (int j = 0; j < dim; j++) {
            double u1 = uvo_next_f64(&st);
            if (u1 < 1e-12) u1 = 1e-12;
            double u2 = uvo_next_f64(&st);
            v[j] = (float)(sqrt(-2.0 * log(u1)) * cos(2.0 * 3.141592653589793 * u2));
        }
        float nn = fmaxf(uvo_l2_norm(v, dim), F32_EPS);
        for (int j = 0; j < dim; j++) v[j] /= nn;
    }
}

/* ivf.rs:229-239 IvfIndex::search over a list-major SoA index: probe the
 * nprobe lists by cosine, score each probed list's records exactly as that
 * list's codec does (qm = <u, c_list> when centered, else 0), keep the
 * global top-k by (score desc, id asc).  list_off has nlist+1 entries. */
void uvo_ivf_search_topk(const uvo_codec *c, const float *centroids, int nlist,
                         const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                         const uint32_t *start, const float *rescale, const float *rnorm,
                         int centered, const float *queries, int64_t nq, int nprobe, int k,
                         int64_t *ids_out, float *scores_out, int threads) {
    int d = c->dim, cb = uvo_codec_code_bytes(c);
    if (nprobe > nlist) nprobe = nlist;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *u = (float *)malloc(sizeof(float) * d);
        float *q_r = (float *)malloc(sizeof(float) * d);
        uint32_t *w = (uint32_t *)malloc(sizeof(uint32_t) * d);
        int32_t *lists = (int32_t *)malloc(sizeof(int32_t) * (nprobe > 0 ? nprobe : 1));
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (k > 0 ? k : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            const float *q = queries + (size_t)qi * d;
            int nh = 0;
            float qn = uvo_l2_norm(q, d);
            if (qn >= F32_EPS && nprobe > 0) {
                uvo_ivf_probe(centroids, nlist, d, q, nprobe, lists);
                for (int i = 0; i < d; i++) u[i] = q[i] / qn;
                uvo_rotate(c, u, q_r);
                for (int p = 0; p < nprobe; p++) {
                    int j = lists[p];
                    if (j < 0) continue;
                    float qm = centered ? seq_dot(u, centroids + (size_t)j * d, d) : 0.0f;
                    for (int64_t r = list_off[j]; r < list_off[j + 1]; r++) {
                        uvo_windows(c, codes + (size_t)r * cb, start[r], w);
                        float dot = uvo_lut_dot_u32(q_r, w, c->code, d);
                        float rn = rnorm ? rnorm[r] : 1.0f;
                        float s = qm + rn * (dot / rescale[r]);
                        heap_push_bounded(h, &nh, k, s, ids[r]);
                    }
                }
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, scores_out ? scores_out + (size_t)qi * k : NULL);
        }
        free(u);
        free(q_r);
        free(w);
        free(lists);
        free(h);
    }
}

/* ivf.rs:248-274 search_with_rerank: the global top-r (r = max(rdepth, k))
 * by the codec score (uvo_ivf_search_topk), then the exact fp32 cosine of
 * each candidate against db (lib.rs:240-248), best k by (cosine desc, id
 * asc; the reference leaves exact ties unordered). */
void uvo_ivf_search_rerank(const uvo_codec *c, const float *centroids, int nlist,
                           const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                           const uint32_t *start, const float *rescale, const float *rnorm,
                           int centered, const float *queries, int64_t nq, int nprobe, int k,
                           int rdepth, const float *db, int64_t *ids_out, float *scores_out,
                           int threads) {
    int d = c->dim;
    int r = rdepth > k ? rdepth : k;
    int64_t *cand = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nq > 0 ? nq : 1) * r);
    uvo_ivf_search_topk(c, centroids, nlist, list_off, ids, codes, start, rescale, rnorm, centered,
                        queries, nq, nprobe, r, cand, NULL, threads);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (size_t)r);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            const float *q = queries + (size_t)qi * d;
            int nh = 0;
            for (int j = 0; j < r; j++) {
                int64_t id = cand[(size_t)qi * r + j];
                if (id < 0) continue;
                const float *x = db + (size_t)id * d;
                float dot = seq_dot(q, x, d);
                float na = uvo_l2_norm(q, d), nb = uvo_l2_norm(x, d);
                float cs = (na < F32_EPS || nb < F32_EPS) ? 0.0f : dot / (na * nb);
                heap_push_bounded(h, &nh, r, cs, id);
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, scores_out ? scores_out + (size_t)qi * k : NULL);
        }
        free(h);
    }
    free(cand);
}

/* ---------------------------------------------------------------------- */
/* The 1-bit companion shortlist (trellis.rs:854-948, ivf.rs:52-60)        */
/* ---------------------------------------------------------------------- */

/* Stage-1 similarity of one entry (trellis.rs:887-899): the symmetric
 * dim - 2 * hamming(q_bits, sign) (2251-2266) or the asymmetric masked_sum
 * (2271-2279, a sequential fold of +-q_r[i]), times rnorm when weighted. */
static float shortlist_sim(int d, const float *q_r, const uint8_t *q_bits, const uint8_t *sign,
                           int asym, int weighted, float rnorm) {
    float sim;
    if (asym) {
        float s = 0.0f;
        for (int i = 0; i < d; i++) {
            int bit = (sign[i >> 3] >> (7 - (i & 7))) & 1;
            s += bit ? q_r[i] : -q_r[i];
        }
        sim = s;
    } else {
        uint32_t h = 0;
        for (int b = 0; b < (d + 7) / 8; b++) h += (uint32_t)__builtin_popcount(q_bits[b] ^ sign[b]);
        sim = (float)d - 2.0f * (float)h;
    }
    return weighted ? rnorm * sim : sim;
}

/* search_shortlist over the n entries [0, n) of one codec (a flat index or
 * one posting list): the c = min(max(c, limit), n) best by stage-1
 * similarity (ties: lower entry first -- select_nth_unstable leaves them
 * unspecified), then the estimator of score() on those, pushed into the
 * caller's top-limit heap under id ids[i] (or i).  qm is qc_all[cidx[i]]
 * (qc_all NULL: 0). */
static void shortlist_scan(const uvo_codec *c, int64_t n, const uint8_t *codes,
                           const uint32_t *start, const float *rescale, const float *rnorm,
                           const uint32_t *cidx, const uint8_t *signs, const int64_t *ids,
                           const float *q_r, const uint8_t *q_bits, const float *qc_all,
                           int limit, int cs, int asym, int weighted, cand_t *sel, cand_t *h,
                           int *nh) {
    int d = c->dim, cb = uvo_codec_code_bytes(c), sb = (d + 7) / 8;
    if (n <= 0) return;
    int64_t ce = cs > limit ? cs : limit;
    if (ce > n) ce = n;
    int ns = 0;
    for (int64_t i = 0; i < n; i++) {
        float rn = rnorm ? rnorm[i] : 1.0f;
        float sim = shortlist_sim(d, q_r, q_bits, signs + (size_t)i * sb, asym, weighted, rn);
        heap_push_bounded(sel, &ns, (int)ce, sim, i);
    }
    for (int t = 0; t < ns; t++) {
        int64_t i = sel[t].id;
        float qm = qc_all ? qc_all[cidx ? cidx[i] : 0] : 0.0f;
        float s = uvo_score(c, q_r, qm, codes + (size_t)i * cb, start[i], rescale[i],
                            rnorm ? rnorm[i] : 1.0f);
        heap_push_bounded(h, nh, limit, s, ids ? ids[i] : i);
    }
}

static void query_bits(const float *q_r, int d, uint8_t *out) { sign_code(q_r, d, out); }

/* trellis.rs:2120-2122 -> 854-948: a flat index whose codec has the shortlist
 * on (with_shortlist(c), with_shortlist_asym, with_shortlist_rnorm).  The
 * stage-1 weight applies when `weight` and the codec has centroids. */
void uvo_search_shortlist(const uvo_codec *c, const uint8_t *codes, const uint32_t *start,
                          const float *rescale, const float *rnorm, const uint32_t *cidx,
                          const uint8_t *signs, int64_t n, const float *queries, int64_t nq,
                          int k, int cs, int asym, int weight, int64_t *ids_out,
                          float *scores_out, int threads) {
    int d = c->dim;
    int64_t ce = cs > k ? cs : k;
    if (ce > n) ce = n;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *q_r = (float *)malloc(sizeof(float) * d);
        float *qc = (float *)malloc(sizeof(float) * (c->n_centroids + 1));
        uint8_t *qb = (uint8_t *)malloc((size_t)(d + 7) / 8);
        cand_t *sel = (cand_t *)malloc(sizeof(cand_t) * (size_t)(ce > 0 ? ce : 1));
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (k > 0 ? k : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            int nh = 0;
            if (!uvo_prepare_query(c, queries + (size_t)qi * d, q_r, qc)) {
                query_bits(q_r, d, qb);
                shortlist_scan(c, n, codes, start, rescale, rnorm, cidx, signs, NULL, q_r, qb,
                               c->n_centroids > 0 ? qc : NULL, k, cs, asym,
                               weight && c->n_centroids > 0, sel, h, &nh);
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, scores_out ? scores_out + (size_t)qi * k : NULL);
        }
        free(q_r);
        free(qc);
        free(qb);
        free(sel);
        free(h);
    }
}

/* ivf.rs:229-239 with IvfCodec::TrellisShortlist{c, asym, rnorm}: each probed
 * list runs search_shortlist(query, k, c) over its own entries (stage-1
 * weight only for centered lists), the per-list results merge to top-k. */
void uvo_ivf_search_shortlist(const uvo_codec *c, const float *centroids, int nlist,
                              const int64_t *list_off, const int64_t *ids, const uint8_t *codes,
                              const uint32_t *start, const float *rescale, const float *rnorm,
                              const uint8_t *signs, int centered, const float *queries,
                              int64_t nq, int nprobe, int k, int cs, int asym, int weight,
                              int64_t *ids_out, float *scores_out, int threads) {
    int d = c->dim, cb = uvo_codec_code_bytes(c), sb = (d + 7) / 8;
    if (nprobe > nlist) nprobe = nlist;
    int64_t maxlen = 0;
    for (int j = 0; j < nlist; j++)
        if (list_off[j + 1] - list_off[j] > maxlen) maxlen = list_off[j + 1] - list_off[j];
    int64_t ce = cs > k ? cs : k;
    if (ce > maxlen) ce = maxlen;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads)
#endif
    {
        float *u = (float *)malloc(sizeof(float) * d);
        float *q_r = (float *)malloc(sizeof(float) * d);
        uint8_t *qb = (uint8_t *)malloc((size_t)sb);
        int32_t *lists = (int32_t *)malloc(sizeof(int32_t) * (nprobe > 0 ? nprobe : 1));
        cand_t *sel = (cand_t *)malloc(sizeof(cand_t) * (size_t)(ce > 0 ? ce : 1));
        cand_t *h = (cand_t *)malloc(sizeof(cand_t) * (k > 0 ? k : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t qi = 0; qi < nq; qi++) {
            const float *q = queries + (size_t)qi * d;
            int nh = 0;
            float qn = uvo_l2_norm(q, d);
            if (qn >= F32_EPS && nprobe > 0) {
                uvo_ivf_probe(centroids, nlist, d, q, nprobe, lists);
                for (int i = 0; i < d; i++) u[i] = q[i] / qn;
                uvo_rotate(c, u, q_r);
                query_bits(q_r, d, qb);
                for (int p = 0; p < nprobe; p++) {
                    int j = lists[p];
                    if (j < 0) continue;
                    int64_t o = list_off[j];
                    float qm = centered ? seq_dot(u, centroids + (size_t)j * d, d) : 0.0f;
                    shortlist_scan(c, list_off[j + 1] - o, codes + (size_t)o * cb, start + o,
                                   rescale + o, rnorm ? rnorm + o : NULL, NULL,
                                   signs + (size_t)o * sb, ids + o, q_r, qb,
                                   centered ? &qm : NULL, k, cs, asym, weight && centered, sel, h,
                                   &nh);
                }
            }
            emit_topk(h, nh, k, ids_out + (size_t)qi * k, scores_out ? scores_out + (size_t)qi * k : NULL);
        }
        free(u);
        free(q_r);
        free(qb);
        free(lists);
        free(sel);
        free(h);
    }
}

/* bench.rs:1019 norms[i] = l2_norm(db[i]) over a batch */
void uvo_l2_norms(const float *rows, int64_t n, int dim, float *out, int threads) {
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int64_t i = 0; i < n; i++) out[i] = uvo_l2_norm(rows + (size_t)i * dim, dim);
}
