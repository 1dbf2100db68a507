/*
 * uv_oracle_coset.c -- CPU oracle for the coset trellis (trellis-coded
 * quantization over the eight cosets of an index-8 sublattice of E8).
 *
 * TEST INFRASTRUCTURE ONLY: a plain-C restatement of ultravec-ann's
 * src/coset_trellis.rs (and the E8 helpers of src/e8.rs it uses), the checker
 * the CUDA coset path is compared against.  Nothing in the product links it.
 *
 * Parity unpinned: the reference ships no golden vectors for this arm and
 * cannot be built here (Rust).  The restatement is checked against the
 * reference's own tests of it (coset_trellis.rs:522-616: the partition is
 * closed and balanced, the fast nearest-in-coset search equals the
 * exhaustive scan, a record decodes to a reconstruction that correlates with
 * its input), re-run on the oracle, and its Viterbi against an exhaustive
 * search over every path of small trellises.
 *
 * Every book point is kept as a 64-bit key that sorts exactly like the
 * reference's (norm, lexicographic) order: key = norm << 40 | the eight raw
 * doubled coordinates offset by 16, five bits each, first coordinate highest.
 * Raw coordinates stay within [-16, 15] for every book (|R| <= 13 at three
 * bits), so the key decodes back to the point.
 */
#include "uv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <omp.h>

#define F32_EPS 1.1920928955078125e-7f /* f32::EPSILON */

struct uvo_coset {
    int dim, bits, mem, m_bits, per_coset, start_bytes, code_len;
    uvo_codec *rot;      /* rotation only (lib.rs Rotation, Rotor::new_oblivious) */
    uint64_t *books;     /* 8 x per_coset sorted keys */
    float scale_mean, scale_std;
    int n_centroids;
    float *centroids;
};

/* ------------------------------------------------------------------ */
/* keys                                                                 */
/* ------------------------------------------------------------------ */
uint64_t uvo_e8_key(const int16_t *r) {
    int64_t n = 0;
    uint64_t lex = 0;
    for (int j = 0; j < 8; j++) {
        n += (int64_t)r[j] * r[j];
        lex = (lex << 5) | (uint64_t)((r[j] + 16) & 31);
    }
    return ((uint64_t)n << 40) | lex;
}

void uvo_e8_unkey(uint64_t key, int16_t *r) {
    for (int j = 0; j < 8; j++) r[j] = (int16_t)((int)((key >> (5 * (7 - j))) & 31) - 16);
}

/* coset_trellis.rs:73-79  three-bit label ((R0-R1)/2, (R2-R3)/2, (R4-R5)/2) mod 2 */
int uvo_coset_of(const int16_t *r) {
    int a = ((r[0] - r[1]) / 2) & 1;
    int b = ((r[2] - r[3]) / 2) & 1;
    int c = ((r[4] - r[5]) / 2) & 1;
    return (a << 2) | (b << 1) | c;
}

/* coset_trellis.rs:90-94  parity of the whole state selects the coset half */
static inline int coset_for(uint32_t state, int br) {
    return ((__builtin_popcount(state) & 1) << 2) | br;
}

/* ------------------------------------------------------------------ */
/* e8.rs:37-80  nearest E8 point (Conway & Sloane)                      */
/* ------------------------------------------------------------------ */
static void nearest_d8(const float *y, float offset, float *pt) {
    int64_t isum = 0;
    int worst = 0;
    float worst_err = -1.0f, worst_dir = 1.0f;
    for (int i = 0; i < 8; i++) {
        float s = y[i] - offset;
        float r = roundf(s); /* f32::round: half away from zero */
        pt[i] = r + offset;
        isum += (int64_t)r;
        float resid = s - r;
        float err = fabsf(resid);
        if (err > worst_err) {
            worst_err = err;
            worst = i;
            worst_dir = resid >= 0.0f ? 1.0f : -1.0f;
        }
    }
    if (((isum % 2) + 2) % 2 != 0) pt[worst] += worst_dir;
}

void uvo_e8_nearest(const float *y, float *out) {
    float a[8], b[8];
    nearest_d8(y, 0.0f, a);
    nearest_d8(y, 0.5f, b);
    float da = -0.0f, db = -0.0f;
    for (int i = 0; i < 8; i++) da += (y[i] - a[i]) * (y[i] - a[i]);
    for (int i = 0; i < 8; i++) db += (y[i] - b[i]) * (y[i] - b[i]);
    memcpy(out, da <= db ? a : b, sizeof(float) * 8);
}

/* ------------------------------------------------------------------ */
/* e8.rs:82-141  every E8 point with |x|^2 <= r2 (raw doubled coords)   */
/* ------------------------------------------------------------------ */
typedef void (*point_fn)(const int16_t *r, void *ctx);

static void enum_rec(int pos, int64_t left, int64_t sum, int64_t parity, int16_t *cur,
                     point_fn fn, void *ctx) {
    if (pos == 8) {
        if (((sum % 4) + 4) % 4 == 0) fn(cur, ctx);
        return;
    }
    int64_t bound = (int64_t)floor(sqrt((double)left));
    int64_t r = -bound;
    while (((r % 2) + 2) % 2 != parity) r++;
    for (; r <= bound; r += 2) {
        int64_t r2 = r * r;
        if (r2 <= left) {
            cur[pos] = (int16_t)r;
            enum_rec(pos + 1, left - r2, sum + r, parity, cur, fn, ctx);
        }
    }
}

static void enumerate_raw(float r2_max, point_fn fn, void *ctx) {
    int64_t budget = (int64_t)floorf(4.0f * r2_max);
    for (int64_t parity = 0; parity < 2; parity++) {
        int16_t cur[8] = {0};
        enum_rec(0, budget, 0, parity, cur, fn, ctx);
    }
}

typedef struct {
    int64_t n, cap;
    uint64_t *keys;
    int64_t counts[8];
} collect_t;

static void count_fn(const int16_t *r, void *ctx) {
    collect_t *c = (collect_t *)ctx;
    c->counts[uvo_coset_of(r)]++;
    c->n++;
}

static void collect_fn(const int16_t *r, void *ctx) {
    collect_t *c = (collect_t *)ctx;
    if (c->n < c->cap) c->keys[c->n] = uvo_e8_key(r);
    c->n++;
}

/* every E8 point with |x|^2 <= r2 as keys (unsorted); returns the count even
 * when it exceeds cap */
int64_t uvo_e8_enumerate(float r2_max, uint64_t *keys, int64_t cap) {
    collect_t c;
    memset(&c, 0, sizeof(c));
    c.cap = keys ? cap : 0;
    c.keys = keys;
    enumerate_raw(r2_max, collect_fn, &c);
    return c.n;
}

static int cmp_u64(const void *a, const void *b) {
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* ------------------------------------------------------------------ */
/* coset_trellis.rs:121-190  construction                               */
/* ------------------------------------------------------------------ */
uvo_coset *uvo_coset_new(int dim, int bits, int mem, uint64_t seed, int rounds) {
    if (dim <= 0 || dim % 8 != 0 || bits < 1 || bits > 3 || mem < 1 || mem > 20) return NULL;
    uvo_coset *c = (uvo_coset *)calloc(1, sizeof(uvo_coset));
    c->dim = dim;
    c->bits = bits;
    c->mem = mem;
    c->m_bits = 8 * bits - 3;
    c->per_coset = 1 << c->m_bits;
    c->start_bytes = (mem + 7) / 8;
    c->code_len = c->start_bytes + ((dim / 8) * (2 + c->m_bits) + 7) / 8;
    c->rot = uvo_codec_new(dim, 1, 1, seed, rounds, 1, 0, 0.0f);
    /* grow the radius until every coset holds per_coset points (141-153) */
    float r2 = 2.0f;
    for (;;) {
        collect_t cnt;
        memset(&cnt, 0, sizeof(cnt));
        enumerate_raw(r2, count_fn, &cnt);
        int ok = 1;
        for (int k = 0; k < 8; k++) ok &= cnt.counts[k] >= c->per_coset;
        if (ok) break;
        r2 += 2.0f;
    }
    int64_t total = uvo_e8_enumerate(r2, NULL, 0);
    uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)total);
    uvo_e8_enumerate(r2, keys, total);
    /* sort by (norm, lex), deal the first per_coset of each coset (154-167) */
    qsort(keys, (size_t)total, sizeof(uint64_t), cmp_u64);
    c->books = (uint64_t *)malloc(sizeof(uint64_t) * 8 * (size_t)c->per_coset);
    int64_t fill[8] = {0};
    for (int64_t i = 0; i < total; i++) {
        int16_t r[8];
        uvo_e8_unkey(keys[i], r);
        int k = uvo_coset_of(r);
        if (fill[k] < c->per_coset) c->books[(size_t)k * c->per_coset + fill[k]++] = keys[i];
    }
    free(keys);
    /* unit-variance scaling over the union of kept points, f64 (172-186) */
    double sum = 0.0, sumsq = 0.0, cnt = 0.0;
    for (size_t i = 0; i < 8 * (size_t)c->per_coset; i++) {
        int16_t r[8];
        uvo_e8_unkey(c->books[i], r);
        for (int j = 0; j < 8; j++) {
            double x = (double)r[j] / 2.0;
            sum += x;
            sumsq += x * x;
            cnt += 1.0;
        }
    }
    double mean = sum / cnt;
    double var = sumsq / cnt - mean * mean;
    double sd = sqrt(var > 1e-12 ? var : 1e-12);
    c->scale_mean = (float)mean;
    c->scale_std = (float)sd;
    return c;
}

void uvo_coset_free(uvo_coset *c) {
    if (!c) return;
    uvo_codec_free(c->rot);
    free(c->books);
    free(c->centroids);
    free(c);
}

/* coset_trellis.rs:192-196 */
int uvo_coset_set_centroids(uvo_coset *c, const float *centroids, int n_centroids) {
    free(c->centroids);
    c->centroids = NULL;
    c->n_centroids = n_centroids;
    if (n_centroids > 0) {
        c->centroids = (float *)malloc(sizeof(float) * (size_t)n_centroids * c->dim);
        memcpy(c->centroids, centroids, sizeof(float) * (size_t)n_centroids * c->dim);
    }
    return 0;
}

int uvo_coset_per_coset(const uvo_coset *c) { return c->per_coset; }
int uvo_coset_code_len(const uvo_coset *c) { return c->code_len; }
void uvo_coset_books(const uvo_coset *c, uint64_t *out) {
    memcpy(out, c->books, sizeof(uint64_t) * 8 * (size_t)c->per_coset);
}
void uvo_coset_scale(const uvo_coset *c, float *out) {
    out[0] = c->scale_mean;
    out[1] = c->scale_std;
}

/* ------------------------------------------------------------------ */
/* coset_trellis.rs:199-296  nearest kept point of one coset            */
/* ------------------------------------------------------------------ */
static inline const uint64_t *book_of(const uvo_coset *c, int k) {
    return c->books + (size_t)k * c->per_coset;
}

/* coset_trellis.rs:199-205  position of a point in its coset's book, or -1 */
int64_t uvo_coset_index(const uvo_coset *c, int k, const int16_t *r) {
    for (int j = 0; j < 8; j++)
        if (r[j] < -16 || r[j] > 15) return -1; /* outside every book */
    uint64_t key = uvo_e8_key(r);
    const uint64_t *b = book_of(c, k);
    int64_t lo = 0, hi = c->per_coset;
    while (lo < hi) {
        int64_t mid = (lo + hi) / 2;
        if (b[mid] < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return (lo < c->per_coset && b[lo] == key) ? lo : -1;
}

static inline float dist2(const float *y, const int16_t *p) {
    float d = 0.0f;
    for (int j = 0; j < 8; j++) {
        float e = y[j] - (float)p[j] / 2.0f;
        d += e * e;
    }
    return d;
}

/* coset_trellis.rs:281-296 */
void uvo_coset_nearest_exhaustive(const uvo_coset *c, int k, const float *y, int64_t *idx,
                                  float *dist) {
    int64_t best = 0;
    float best_d = INFINITY;
    const uint64_t *b = book_of(c, k);
    for (int64_t i = 0; i < c->per_coset; i++) {
        int16_t p[8];
        uvo_e8_unkey(b[i], p);
        float d = dist2(y, p);
        if (d < best_d) {
            best_d = d;
            best = i;
        }
    }
    *idx = best;
    *dist = best_d;
}

typedef struct {
    const uvo_coset *c;
    int k;
    const float *y;
    int64_t best;
    float best_d;
} ball_t;

/* e8.rs:143-203  E8 points within sqrt(budget) of centre (raw doubled
 * coordinates), each handed to the nearest-in-coset filter in the order the
 * reference's Vec holds them */
static void ball_visit(ball_t *b, const int16_t *p) {
    if (uvo_coset_of(p) != b->k) return;
    int64_t i = uvo_coset_index(b->c, b->k, p);
    if (i < 0) return;
    float d = dist2(b->y, p);
    if (d < b->best_d) {
        b->best_d = d;
        b->best = i;
    }
}

static void ball_rec(int pos, double left, int64_t sum, int64_t parity, const float *centre,
                     int16_t *cur, ball_t *b) {
    if (pos == 8) {
        if (((sum % 4) + 4) % 4 == 0) ball_visit(b, cur);
        return;
    }
    double cc = (double)centre[pos];
    double span = sqrt(left > 0.0 ? left : 0.0);
    int64_t lo = (int64_t)floor(cc - span);
    int64_t hi = (int64_t)ceil(cc + span);
    int64_t r = lo;
    while (((r % 2) + 2) % 2 != parity) r++;
    for (; r <= hi; r += 2) {
        double d = (double)r - cc;
        double d2 = d * d;
        if (d2 <= left) {
            cur[pos] = (int16_t)r;
            ball_rec(pos + 1, left - d2, sum + r, parity, centre, cur, b);
        }
    }
}

/* coset_trellis.rs:214-278  bisection seed, then every E8 point within the
 * seed's distance */
void uvo_coset_nearest(const uvo_coset *c, int k, const float *y, int64_t *idx, float *dist) {
    const uint64_t *bk = book_of(c, k);
    int16_t t[8];
    uvo_e8_unkey(bk[0], t);
    int64_t best = 0;
    float best_d = dist2(y, t);
    float lo = 0.0f, hi = 1.0f;
    for (int it = 0; it < 12; it++) {
        float a = 0.5f * (lo + hi);
        float z[8], pt[8];
        for (int j = 0; j < 8; j++) z[j] = a * y[j] - (float)t[j] / 2.0f;
        uvo_e8_nearest(z, pt);
        int16_t r[8];
        for (int j = 0; j < 8; j++) r[j] = (int16_t)((int16_t)roundf(pt[j] * 2.0f) + t[j]);
        int64_t hit = uvo_coset_of(r) == k ? uvo_coset_index(c, k, r) : -1;
        if (hit >= 0) {
            float d = dist2(y, r);
            if (d < best_d) {
                best_d = d;
                best = hit;
            }
            lo = a;
        } else {
            hi = a;
        }
    }
    /* PI.powi(4) folds to pow(pi, 4); (best_d as f64).powi(4) is (x^2)^2 */
    double bd = (double)best_d, bd2 = bd * bd;
    double est = pow(3.14159265358979323846, 4.0) * (bd2 * bd2) / 24.0;
    if (!isfinite(est) || est > (double)c->per_coset) {
        uvo_coset_nearest_exhaustive(c, k, y, idx, dist);
        return;
    }
    float centre[8];
    for (int j = 0; j < 8; j++) centre[j] = y[j] * 2.0f;
    double budget = 4.0 * (double)best_d * (1.0 + 1e-6) + 1e-6;
    ball_t b = {c, k, y, best, best_d};
    for (int64_t parity = 0; parity < 2; parity++) {
        int16_t cur[8] = {0};
        ball_rec(0, budget, 0, parity, centre, cur, &b);
    }
    *idx = b.best;
    *dist = b.best_d;
}

/* ------------------------------------------------------------------ */
/* coset_trellis.rs:298-318  prep: unit vector, or the unit residual to  */
/* its nearest centroid (first strict minimum of the squared distance)   */
/* ------------------------------------------------------------------ */
static void coset_prep(const uvo_coset *c, const float *o, float *r, float *rnorm,
                       uint32_t *cidx) {
    int d = c->dim;
    float n = fmaxf(uvo_l2_norm(o, d), F32_EPS);
    for (int i = 0; i < d; i++) r[i] = o[i] / n;
    *rnorm = 1.0f;
    *cidx = 0;
    if (c->n_centroids == 0) return;
    int best = 0;
    float best_d = INFINITY;
    for (int j = 0; j < c->n_centroids; j++) {
        const float *cc = c->centroids + (size_t)j * d;
        float s = -0.0f;
        for (int i = 0; i < d; i++) s += (r[i] - cc[i]) * (r[i] - cc[i]);
        if (s < best_d) {
            best_d = s;
            best = j;
        }
    }
    const float *cc = c->centroids + (size_t)best * d;
    for (int i = 0; i < d; i++) r[i] = r[i] - cc[i];
    float rn = fmaxf(uvo_l2_norm(r, d), F32_EPS);
    for (int i = 0; i < d; i++) r[i] /= rn;
    *rnorm = rn;
    *cidx = (uint32_t)best;
}

/* lib.rs:662-683  MSB-first packing of `bits`-wide symbols */
static int pack_wide(const uint32_t *sym, int n, int bits, uint8_t *out) {
    uint64_t buf = 0;
    int in_buf = 0, o = 0;
    for (int i = 0; i < n; i++) {
        buf = (buf << bits) | sym[i];
        in_buf += bits;
        while (in_buf >= 8) {
            in_buf -= 8;
            out[o++] = (uint8_t)((buf >> in_buf) & 0xFF);
        }
    }
    if (in_buf > 0) out[o++] = (uint8_t)((buf << (8 - in_buf)) & 0xFF);
    return o;
}

/* lib.rs:685-707 */
static void unpack_wide(const uint8_t *data, int nbytes, int bits, uint32_t *out, int n) {
    uint32_t mask = bits >= 32 ? 0xFFFFFFFFu : ((1u << bits) - 1);
    uint64_t buf = 0;
    int in_buf = 0, byte = 0;
    for (int i = 0; i < n; i++) out[i] = 0;
    for (int i = 0; i < n; i++) {
        while (in_buf < bits && byte < nbytes) {
            buf = (buf << 8) | data[byte++];
            in_buf += 8;
        }
        if (in_buf < bits) return;
        in_buf -= bits;
        out[i] = (uint32_t)(buf >> in_buf) & mask;
    }
}

static inline uint32_t total_key_u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* ------------------------------------------------------------------ */
/* coset_trellis.rs:320-412  encode: per-block nearest-in-coset costs,   */
/* free-start Viterbi (4 branches per state), traceback, emission        */
/* ------------------------------------------------------------------ */
static void coset_encode_one(const uvo_coset *c, const float *row, uint8_t *rec,
                             float *rescale_out, float *rnorm, uint32_t *cidx) {
    const int d = c->dim, nb = d / 8, S = 1 << c->mem;
    const uint32_t mask = (uint32_t)S - 1;
    float *r = (float *)malloc(sizeof(float) * d);
    float *u_r = (float *)malloc(sizeof(float) * d);
    coset_prep(c, row, r, rnorm, cidx);
    uvo_rotate(c->rot, r, u_r);
    float scale = fmaxf(uvo_std_about_mean(u_r, d), F32_EPS);
    int64_t *bidx = (int64_t *)malloc(sizeof(int64_t) * nb * 8);
    float *bcost = (float *)malloc(sizeof(float) * nb * 8);
    for (int b = 0; b < nb; b++) {
        float y[8];
        for (int j = 0; j < 8; j++) y[j] = (u_r[b * 8 + j] / scale) * c->scale_std + c->scale_mean;
        for (int k = 0; k < 8; k++) uvo_coset_nearest(c, k, y, &bidx[b * 8 + k], &bcost[b * 8 + k]);
    }
    float *cost = (float *)calloc((size_t)S, sizeof(float));
    float *next = (float *)malloc(sizeof(float) * (size_t)S);
    uint32_t *back = (uint32_t *)calloc((size_t)nb * S, sizeof(uint32_t));
    for (int b = 0; b < nb; b++) {
        for (int s = 0; s < S; s++) next[s] = INFINITY;
        for (int s = 0; s < S; s++) {
            float cs = cost[s];
            if (cs == INFINITY) continue;
            for (int br = 0; br < 4; br++) {
                int k = coset_for((uint32_t)s, br);
                uint32_t w = ((uint32_t)s << 2) | (uint32_t)br;
                uint32_t ns = w & mask;
                float total = cs + bcost[b * 8 + k];
                if (total < next[ns]) {
                    next[ns] = total;
                    back[(size_t)b * S + ns] = w;
                }
            }
        }
        float *t = cost;
        cost = next;
        next = t;
    }
    /* first minimum under f32::total_cmp */
    uint32_t s = 0;
    for (int i = 1; i < S; i++)
        if (total_key_u(cost[i]) < total_key_u(cost[s])) s = (uint32_t)i;
    uint8_t *branches = (uint8_t *)malloc((size_t)nb);
    for (int b = nb - 1; b >= 0; b--) {
        uint32_t w = back[(size_t)b * S + s];
        branches[b] = (uint8_t)(w & 3);
        s = w >> 2;
    }
    const uint32_t start = s;
    uint32_t *syms = (uint32_t *)malloc(sizeof(uint32_t) * nb);
    float rescale = 0.0f;
    uint32_t st = start;
    for (int b = 0; b < nb; b++) {
        int br = branches[b];
        int k = coset_for(st, br);
        int64_t idx = bidx[b * 8 + k];
        syms[b] = ((uint32_t)br << c->m_bits) | (uint32_t)idx;
        int16_t p[8];
        uvo_e8_unkey(book_of(c, k)[idx], p);
        for (int j = 0; j < 8; j++) {
            float v = ((float)p[j] / 2.0f - c->scale_mean) / c->scale_std;
            rescale += v * u_r[b * 8 + j];
        }
        st = ((st << 2) | (uint32_t)br) & mask;
    }
    for (int i = 0; i < c->start_bytes; i++) rec[i] = (uint8_t)((start >> (8 * i)) & 0xFF);
    pack_wide(syms, nb, 2 + c->m_bits, rec + c->start_bytes);
    *rescale_out = fmaxf(rescale, F32_EPS);
    free(r);
    free(u_r);
    free(bidx);
    free(bcost);
    free(cost);
    free(next);
    free(back);
    free(branches);
    free(syms);
}

/* VectorBackend::add_batch (coset_trellis.rs:454-470): rows in parallel */
void uvo_coset_encode_batch(const uvo_coset *c, const float *rows, int64_t n, uint8_t *codes,
                            float *rescale, float *rnorm, uint32_t *cidx) {
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t i = 0; i < n; i++)
        coset_encode_one(c, rows + i * c->dim, codes + i * c->code_len, rescale + i, rnorm + i,
                         cidx + i);
}

/* coset_trellis.rs:414-434 */
void uvo_coset_decode(const uvo_coset *c, const uint8_t *rec, float *xbar) {
    const int nb = c->dim / 8;
    uint32_t st = 0;
    for (int i = 0; i < c->start_bytes; i++) st |= (uint32_t)rec[i] << (8 * i);
    const uint32_t mask = (1u << c->mem) - 1, imask = (1u << c->m_bits) - 1;
    uint32_t *syms = (uint32_t *)malloc(sizeof(uint32_t) * nb);
    unpack_wide(rec + c->start_bytes, c->code_len - c->start_bytes, 2 + c->m_bits, syms, nb);
    for (int b = 0; b < nb; b++) {
        int br = (int)(syms[b] >> c->m_bits);
        int k = coset_for(st, br);
        int16_t p[8];
        uvo_e8_unkey(book_of(c, k)[syms[b] & imask], p);
        for (int j = 0; j < 8; j++)
            xbar[b * 8 + j] = ((float)p[j] / 2.0f - c->scale_mean) / c->scale_std;
        st = ((st << 2) | (uint32_t)br) & mask;
    }
    free(syms);
}

/* coset_trellis.rs:521-529 reconstruct_unit: encode, decode, inverse
 * rotation, normalize */
void uvo_coset_reconstruct_unit(const uvo_coset *c, const float *row, float *out) {
    const int d = c->dim;
    uint8_t *rec = (uint8_t *)malloc((size_t)c->code_len);
    float rs, rn;
    uint32_t ci;
    coset_encode_one(c, row, rec, &rs, &rn, &ci);
    float *xbar = (float *)malloc(sizeof(float) * d);
    uvo_coset_decode(c, rec, xbar);
    uvo_rotate_inverse(c->rot, xbar, out);
    float n = fmaxf(uvo_l2_norm(out, d), F32_EPS);
    for (int i = 0; i < d; i++) out[i] /= n;
    free(rec);
    free(xbar);
}

/* coset_trellis.rs:471-497  search: q/|q| (|q| clamped at EPS), rotate,
 * score = qm + rnorm * (dot(q_r, xbar) / rescale), stable sort by score
 * descending under f32::total_cmp (ties keep insertion order) */
void uvo_coset_search(const uvo_coset *c, const uint8_t *codes, const float *rescale,
                      const float *rnorm, const uint32_t *cidx, const int64_t *ids, int64_t n,
                      const float *queries, int64_t nq, int k, int64_t *out_ids,
                      float *out_scores) {
    const int d = c->dim;
#pragma omp parallel
    {
        float *q = (float *)malloc(sizeof(float) * d);
        float *q_r = (float *)malloc(sizeof(float) * d);
        float *xbar = (float *)malloc(sizeof(float) * d);
        uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(n > 0 ? n : 1));
        float *sc = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
#pragma omp for schedule(dynamic, 1)
        for (int64_t qi = 0; qi < nq; qi++) {
            const float *src = queries + qi * d;
            float qn = fmaxf(uvo_l2_norm(src, d), F32_EPS);
            for (int i = 0; i < d; i++) q[i] = src[i] / qn;
            uvo_rotate(c->rot, q, q_r);
            for (int64_t r = 0; r < n; r++) {
                float qm = 0.0f;
                if (c->n_centroids > 0) {
                    const float *cc = c->centroids + (size_t)cidx[r] * d;
                    qm = -0.0f;
                    for (int i = 0; i < d; i++) qm += q[i] * cc[i];
                }
                uvo_coset_decode(c, codes + r * c->code_len, xbar);
                float dot = uvo_dense_dot(q_r, xbar, d);
                float s = qm + rnorm[r] * (dot / rescale[r]);
                sc[r] = s;
                /* descending score, then ascending position */
                keys[r] = ((uint64_t)(~total_key_u(s)) << 32) | (uint64_t)(uint32_t)r;
            }
            qsort(keys, (size_t)n, sizeof(uint64_t), cmp_u64);
            for (int i = 0; i < k; i++) {
                if (i < n) {
                    uint32_t r = (uint32_t)(keys[i] & 0xFFFFFFFFu);
                    out_ids[qi * k + i] = ids ? ids[r] : (int64_t)r;
                    out_scores[qi * k + i] = sc[r];
                } else {
                    out_ids[qi * k + i] = -1;
                    out_scores[qi * k + i] = -INFINITY;
                }
            }
        }
        free(q);
        free(q_r);
        free(xbar);
        free(keys);
        free(sc);
    }
}

/* coset_trellis.rs:498-504 + lib.rs:229-237 */
int64_t uvo_coset_mem_bytes(const uvo_coset *c, int64_t n) {
    int64_t center = 0;
    if (c->n_centroids == 1) {
        center = 4;
    } else if (c->n_centroids > 1) {
        int bitsn = 0;
        uint64_t v = (uint64_t)(c->n_centroids - 1);
        while (v) {
            bitsn++;
            v >>= 1;
        }
        center = 4 + (bitsn + 7) / 8;
    }
    return n * ((int64_t)c->code_len + 4 + center);
}
