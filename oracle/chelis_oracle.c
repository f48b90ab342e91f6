/*
 * chelis_oracle.c -- CPU restatement of the Chelis C backend's numeric
 * semantics for the tensor-DAG hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker).  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load this file's
 * library; the CUDA product never links it.
 *
 * Build flags follow the reference C lane (crates/chelis-backend-c/src/
 * toolchain.rs:235-246): -O2 -ffp-contract=off -fno-fast-math -fopenmp.
 * Every float operation below is one rounded IEEE operation at the stated
 * width; no FMA contraction happens.
 *
 * Reduction order.  Every Sum is the canonical adjacent-pair tree of
 * spec/05-risc-primitives.md:452-466,515-531: pass by pass, pair (2j, 2j+1),
 * carry an odd tail.  The C lane streams that tree through a "carry tree"
 * (crates/chelis-backend-c/src/emit.rs:8113-8220): leaf i merges once per
 * trailing one bit of i with the completed subtree at that depth, and the
 * waiting subtrees fold lowest level first at the end.  The same streaming
 * form is used here so no leaf buffer is needed.
 */
#include "chelis_oracle.h"

#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Correctly rounded kernels from the reference's vendored CORE-MATH
 * (crates/chelis-crmath/csrc/crmath_ffi.c:15-45), linked from oracle/_ref. */
float chelis_crmath_ffi_expf(float);
float chelis_crmath_ffi_logf(float);
float chelis_crmath_ffi_erfcf(float);
double chelis_crmath_ffi_exp(double);

float orc_expf(float x) { return chelis_crmath_ffi_expf(x); }
float orc_logf(float x) { return chelis_crmath_ffi_logf(x); }
float orc_erfcf(float x) { return chelis_crmath_ffi_erfcf(x); }
double orc_exp(double x) { return chelis_crmath_ffi_exp(x); }
double orc_sqrt(double x) { return sqrt(x); }

/* [04-NUM-2] canonical quiet NaN (crates/chelis-backend-c/src/fp_env.rs:45-53). */
static inline float canon_f32(float v) {
    if (isnan(v)) {
        uint32_t bits = 0x7fc00000u;
        memcpy(&v, &bits, 4);
    }
    return v;
}
static inline double canon_f64(double v) {
    if (isnan(v)) {
        uint64_t bits = 0x7ff8000000000000ull;
        memcpy(&v, &bits, 8);
    }
    return v;
}

/* ------------------------------------------------------------------------ */
/* keyed randomness: dtype_semantics.rs:4508-4540                           */
/* ------------------------------------------------------------------------ */

/* [05-RNG-1] splitmix64 (dtype_semantics.rs:4508-4513). */
uint64_t orc_splitmix64(uint64_t v) {
    v += 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}
static inline uint64_t rotl64(uint64_t v, unsigned r) { return (v << r) | (v >> (64 - r)); }

/* [05-RNG-2] derive(k, j) (dtype_semantics.rs:4518-4520). */
uint64_t orc_derive(uint64_t key, uint64_t j) {
    return orc_splitmix64(key ^ rotl64(orc_splitmix64(j), 29));
}
/* [05-RNG-2] word(key, index) (dtype_semantics.rs:4529-4531). */
uint64_t orc_word(uint64_t key, uint64_t index) {
    return orc_splitmix64(key ^ rotl64(orc_splitmix64(index), 41));
}
/* [05-RNG-1] unit = high 53 bits / 2^53 (dtype_semantics.rs:4536-4538). */
double orc_unit(uint64_t key, uint64_t index) {
    return (double)(orc_word(key, index) >> 11) / 9007199254740992.0;
}

/* ------------------------------------------------------------------------ */
/* canonical adjacent-pair tree                                             */
/* ------------------------------------------------------------------------ */

#define DEFINE_TREE(T, SUFFIX, CANON)                                                   \
    T orc_tree_sum_##SUFFIX(const T *x, int64_t n, int64_t stride) {                    \
        T level[64];                                                                    \
        int64_t count = 0;                                                              \
        for (int64_t i = 0; i < n; ++i) {                                               \
            T carry = x[i * stride];                                                    \
            int depth = 0;                                                              \
            for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)       \
                carry = level[depth] + carry;                                           \
            level[depth] = carry;                                                       \
        }                                                                               \
        T total = (T)0;                                                                 \
        int found = 0, depth = 0;                                                       \
        for (int64_t remaining = count; remaining; remaining >>= 1, ++depth) {          \
            if (remaining & 1) {                                                        \
                total = found ? level[depth] + total : level[depth];                    \
                found = 1;                                                              \
            }                                                                           \
        }                                                                               \
        return CANON(total);                                                            \
    }
DEFINE_TREE(float, f32, canon_f32)
DEFINE_TREE(double, f64, canon_f64)

/* A laned carry tree: LANES independent trees that share one leaf schedule
 * (the C lane's 8-column lane blocks, emit.rs:8113-8176, generalised). */
#define LANES 64
#define DEFINE_LANED(T, SUFFIX)                                                          \
    typedef struct {                                                                     \
        T level[64][LANES];                                                              \
        int64_t count;                                                                   \
    } laned_##SUFFIX;                                                                    \
    static inline void laned_push_##SUFFIX(laned_##SUFFIX *t, T *leaf, int lanes) {      \
        int depth = 0;                                                                   \
        for (int64_t pending = t->count++; pending & 1; pending >>= 1, ++depth)          \
            for (int l = 0; l < lanes; ++l) leaf[l] = t->level[depth][l] + leaf[l];      \
        for (int l = 0; l < lanes; ++l) t->level[depth][l] = leaf[l];                    \
    }                                                                                    \
    static inline void laned_total_##SUFFIX(const laned_##SUFFIX *t, T *out, int lanes) { \
        int found = 0, depth = 0;                                                        \
        for (int l = 0; l < lanes; ++l) out[l] = (T)0;                                   \
        for (int64_t remaining = t->count; remaining; remaining >>= 1, ++depth) {        \
            if (remaining & 1) {                                                         \
                for (int l = 0; l < lanes; ++l)                                          \
                    out[l] = found ? t->level[depth][l] + out[l] : t->level[depth][l];   \
                found = 1;                                                               \
            }                                                                            \
        }                                                                                \
    }
DEFINE_LANED(float, f32)
DEFINE_LANED(double, f64)

void orc_row_sum_f32(const float *x, int64_t rows, int64_t cols, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) out[r] = orc_tree_sum_f32(x + r * cols, cols, 1);
}

/* Column sums over rows (axis 0): one tree per column, leaves in row order. */
void orc_col_sum_f32(const float *x, int64_t rows, int64_t cols, float *out) {
    int64_t blocks = (cols + LANES - 1) / LANES;
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < blocks; ++b) {
        laned_f32 t;
        t.count = 0;
        float leaf[LANES];
        int64_t j0 = b * LANES;
        int lanes = (int)((cols - j0) < LANES ? (cols - j0) : LANES);
        for (int64_t r = 0; r < rows; ++r) {
            for (int l = 0; l < lanes; ++l) leaf[l] = x[r * cols + j0 + l];
            laned_push_f32(&t, leaf, lanes);
        }
        laned_total_f32(&t, leaf, lanes);
        for (int l = 0; l < lanes; ++l) out[j0 + l] = canon_f32(leaf[l]);
    }
}

/* [05-OP-12] max_reduce: the first NaN wins with its payload; otherwise the
 * maximum, first representation among equals (spec/05-risc-primitives.md:421-438). */
static float max_row_f32(const float *x, int64_t n) {
    float best = x[0];
    if (isnan(best)) return best;
    for (int64_t i = 1; i < n; ++i) {
        float v = x[i];
        if (isnan(v)) return v;
        if (v > best) best = v;
    }
    return best;
}
void orc_row_max_f32(const float *x, int64_t rows, int64_t cols, float *out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) out[r] = max_row_f32(x + r * cols, cols);
}

/* [05-OP-29] count: exact i64 tree of 0/1 leaves; integer addition is
 * associative so the tree value equals the plain count. */
int64_t orc_count_bool(const uint8_t *x, int64_t n) {
    int64_t c = 0;
    for (int64_t i = 0; i < n; ++i) c += x[i] ? 1 : 0;
    return c;
}

/* ------------------------------------------------------------------------ */
/* matmul: inlined product sum, emit.rs:8431-8640                           */
/* ------------------------------------------------------------------------ */


static void sgemm_rows(const float *a, int64_t sa0, int64_t sa1, const float *b, int64_t sb0,
                       int64_t sb1, float *c, int64_t ldc, int64_t n, int64_t k,
                       int64_t row_begin, int64_t row_end) {
    int64_t blocks = (n + LANES - 1) / LANES;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t i = row_begin; i < row_end; ++i) {
        for (int64_t bj = 0; bj < blocks; ++bj) {
            laned_f32 t;
            t.count = 0;
            float leaf[LANES];
            int64_t j0 = bj * LANES;
            int lanes = (int)((n - j0) < LANES ? (n - j0) : LANES);
            for (int64_t kk = 0; kk < k; ++kk) {
                float av = a[i * sa0 + kk * sa1];
                const float *brow = b + kk * sb0 + j0 * sb1;
                if (sb1 == 1) {
                    for (int l = 0; l < lanes; ++l) leaf[l] = av * brow[l];
                } else {
                    for (int l = 0; l < lanes; ++l) leaf[l] = av * brow[l * sb1];
                }
                laned_push_f32(&t, leaf, lanes);
            }
            laned_total_f32(&t, leaf, lanes);
            for (int l = 0; l < lanes; ++l) c[i * ldc + j0 + l] = canon_f32(leaf[l]);
        }
    }
}

static void dgemm_rows(const double *a, int64_t sa0, int64_t sa1, const double *b, int64_t sb0,
                       int64_t sb1, double *c, int64_t ldc, int64_t n, int64_t k,
                       int64_t row_begin, int64_t row_end) {
    int64_t blocks = (n + LANES - 1) / LANES;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t i = row_begin; i < row_end; ++i) {
        for (int64_t bj = 0; bj < blocks; ++bj) {
            laned_f64 t;
            t.count = 0;
            double leaf[LANES];
            int64_t j0 = bj * LANES;
            int lanes = (int)((n - j0) < LANES ? (n - j0) : LANES);
            for (int64_t kk = 0; kk < k; ++kk) {
                double av = a[i * sa0 + kk * sa1];
                const double *brow = b + kk * sb0 + j0 * sb1;
                if (sb1 == 1) {
                    for (int l = 0; l < lanes; ++l) leaf[l] = av * brow[l];
                } else {
                    for (int l = 0; l < lanes; ++l) leaf[l] = av * brow[l * sb1];
                }
                laned_push_f64(&t, leaf, lanes);
            }
            laned_total_f64(&t, leaf, lanes);
            for (int l = 0; l < lanes; ++l) c[i * ldc + j0 + l] = canon_f64(leaf[l]);
        }
    }
}

/* Row-major C[m,n] = A[m,k] . B[k,n]; only rows [row_begin, row_end) are
 * written (a bounded sample of a large product). */
void orc_sgemm(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
               int64_t row_begin, int64_t row_end) {
    (void)m;
    sgemm_rows(a, k, 1, b, n, 1, c, n, n, k, row_begin, row_end);
}
void orc_dgemm(const double *a, const double *b, double *c, int64_t m, int64_t n, int64_t k,
               int64_t row_begin, int64_t row_end) {
    (void)m;
    dgemm_rows(a, k, 1, b, n, 1, c, n, n, k, row_begin, row_end);
}
void orc_sgemm_strided(const float *a, int64_t sa0, int64_t sa1, const float *b, int64_t sb0,
                       int64_t sb1, float *c, int64_t m, int64_t n, int64_t k) {
    sgemm_rows(a, sa0, sa1, b, sb0, sb1, c, n, n, k, 0, m);
}
void orc_dgemm_strided(const double *a, int64_t sa0, int64_t sa1, const double *b, int64_t sb0,
                       int64_t sb1, double *c, int64_t m, int64_t n, int64_t k) {
    dgemm_rows(a, sa0, sa1, b, sb0, sb1, c, n, n, k, 0, m);
}

/* ------------------------------------------------------------------------ */
/* dropout: PreparedDropout::apply (dtype_semantics.rs:4256-4280)           */
/* ------------------------------------------------------------------------ */

/* An f32 draw compares its unit rounded to f32 (then widened exactly) with
 * the rate widened to f64; a draw below the rate drops to +0. */
static inline int dropout_keep(uint64_t key, uint64_t index, float rate) {
    double unit = orc_unit(key, index);
    float unit32 = (float)unit;
    return !((double)unit32 < (double)rate);
}
/* DropoutParameters::denominator: 1 - rate finalized at f32 (dtype_semantics.rs:4005-4010). */
static inline float dropout_denominator(float rate) {
    volatile float one = 1.0f;
    return one - rate;
}

void orc_dropout_mask(uint8_t *keep, int64_t n, uint64_t key, float rate, int64_t index_base) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) keep[i] = (uint8_t)dropout_keep(key, (uint64_t)(index_base + i), rate);
}

void orc_dropout_f32(const float *x, float *y, int64_t n, uint64_t key, float rate,
                     int64_t index_base) {
    float den = dropout_denominator(rate);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i)
        y[i] = dropout_keep(key, (uint64_t)(index_base + i), rate) ? canon_f32(x[i] / den) : 0.0f;
}

/* ------------------------------------------------------------------------ */
/* layer norm, softmax (tier2.rs:1079-1375; spec 05 sections 4.2, 4.4)      */
/* ------------------------------------------------------------------------ */

/* Per-row forward values of layer_norm, kept for the adjoint. */
typedef struct {
    float m, v, d;
} ln_row;

/* spec/05-risc-primitives.md:5065-5093: m = mean(x); c = x - m;
 * var = mean(c*c); normed = c / sqrt(var + eps); y = normed*gamma + beta.
 * mean = tree sum / extent (tier2.rs:1183-1245); the sqrt is elementwise on
 * the expanded var, so every column sees the same d. */
static ln_row ln_row_fwd(const float *x, const float *gamma, const float *beta, float eps,
                         int64_t h, float *c, float *n, float *y) {
    ln_row r;
    float hf = (float)h;
    r.m = orc_tree_sum_f32(x, h, 1) / hf;
    for (int64_t j = 0; j < h; ++j) c[j] = x[j] - r.m;
    for (int64_t j = 0; j < h; ++j) n[j] = c[j] * c[j];
    r.v = orc_tree_sum_f32(n, h, 1) / hf;
    float t = r.v + eps;
    r.d = sqrtf(t);
    for (int64_t j = 0; j < h; ++j) {
        n[j] = c[j] / r.d;
        float g = n[j] * gamma[j];
        y[j] = canon_f32(g + beta[j]);
    }
    return r;
}

void orc_layer_norm_f32(const float *x, const float *gamma, const float *beta, float eps,
                        float *y, int64_t rows, int64_t hidden) {
#pragma omp parallel
    {
        float *c = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *n = (float *)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r)
            ln_row_fwd(x + r * hidden, gamma, beta, eps, hidden, c, n, y + r * hidden);
        free(c);
        free(n);
    }
}

/* spec/05-risc-primitives.md:5021-5042: m = max; e = exp(x - m); s = sum(e); y = e / s. */
static void softmax_row(const float *x, float *y, int64_t n) {
    float m = max_row_f32(x, n);
    for (int64_t j = 0; j < n; ++j) y[j] = orc_expf(x[j] - m);
    float s = orc_tree_sum_f32(y, n, 1);
    for (int64_t j = 0; j < n; ++j) y[j] = canon_f32(y[j] / s);
}

void orc_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) softmax_row(x + r * cols, y + r * cols, cols);
}

/* Softmax adjoint (crates/chelis-dag-core/src/grad.rs:2248-2280):
 * dx = y * (g - sum(g * y)). `tmp` holds g*y. */
static void softmax_row_bwd(const float *y, const float *g, float *dx, float *tmp, int64_t n) {
    for (int64_t j = 0; j < n; ++j) tmp[j] = g[j] * y[j];
    float q = orc_tree_sum_f32(tmp, n, 1);
    for (int64_t j = 0; j < n; ++j) {
        float diff = g[j] - q;
        dx[j] = canon_f32(y[j] * diff);
    }
}

void orc_softmax_rows_bwd_f32(const float *y, const float *g, float *dx, int64_t rows,
                              int64_t cols) {
#pragma omp parallel
    {
        float *tmp = (float *)malloc(sizeof(float) * (size_t)cols);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r)
            softmax_row_bwd(y + r * cols, g + r * cols, dx + r * cols, tmp, cols);
        free(tmp);
    }
}

/* ------------------------------------------------------------------------ */
/* fused chain: layer_norm -> softmax -> dropout -> row sum                 */
/* ------------------------------------------------------------------------ */

void orc_chain_fwd(const float *x, const float *gamma, const float *beta, float eps,
                   uint64_t key, float rate, int64_t rows, int64_t hidden, int64_t index_base,
                   float *rowsum) {
    float den = dropout_denominator(rate);
#pragma omp parallel
    {
        float *c = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *n = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *y = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *s = (float *)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            ln_row_fwd(x + r * hidden, gamma, beta, eps, hidden, c, n, y);
            softmax_row(y, s, hidden);
            int64_t base = index_base + r * hidden;
            for (int64_t j = 0; j < hidden; ++j)
                s[j] = dropout_keep(key, (uint64_t)(base + j), rate) ? canon_f32(s[j] / den) : 0.0f;
            rowsum[r] = orc_tree_sum_f32(s, hidden, 1);
        }
        free(c);
        free(n);
        free(y);
        free(s);
    }
}

/*
 * Reverse mode for loss = sum(rowsum), following the adjoint graphs of
 * crates/chelis-dag-core/src/grad.rs: Sum -> Expand (:2586), Dropout ->
 * DropoutReplay on the cotangent (:2515-2525), Softmax (:2248-2280), Add,
 * Mul (:1934-1942), Div (:1943-1961), Sqrt (:2342-2355), Sub, Expand -> Sum.
 * Fan-in is summed by balanced_adjoint_sum (:1713-1745) in increasing
 * consumer order: c feeds mul(c, c) (slots 0, 1) before div(c, d), so
 * dc = (dcc*c + dcc*c) + dn/d; x feeds sum(x) before sub(x, m), so
 * dx = dS1 + dc.  dgamma and dbeta reduce over rows with one tree per
 * column, leaves in row order (the Expand adjoint of gamma_exp / beta_exp).
 */
void orc_chain_bwd(const float *x, const float *gamma, const float *beta, float eps,
                   uint64_t key, float rate, int64_t rows, int64_t hidden, int64_t index_base,
                   float *dx, float *dgamma, float *dbeta) {
    float den = dropout_denominator(rate);
    float hf = (float)hidden;
    float *dyn_rows = (float *)malloc(sizeof(float) * (size_t)(rows * hidden));
    float *dy_rows = (float *)malloc(sizeof(float) * (size_t)(rows * hidden));
#pragma omp parallel
    {
        float *c = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *n = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *y = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *s = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *ds = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *tmp = (float *)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const float *xr = x + r * hidden;
            ln_row lr = ln_row_fwd(xr, gamma, beta, eps, hidden, c, n, y);
            softmax_row(y, s, hidden);
            int64_t base = index_base + r * hidden;
            /* d(rowsum)/dp = 1, replayed through the dropout mask. */
            for (int64_t j = 0; j < hidden; ++j)
                ds[j] = dropout_keep(key, (uint64_t)(base + j), rate) ? 1.0f / den : 0.0f;
            /* softmax adjoint -> dy */
            float *dy = dy_rows + r * hidden;
            softmax_row_bwd(s, ds, dy, tmp, hidden);
            float *dyn = dyn_rows + r * hidden;
            for (int64_t j = 0; j < hidden; ++j) dyn[j] = dy[j] * n[j];
            /* dn = dy * gamma; div adjoint: dc1 = dn / d, dd = -(dn * n) / d;
             * sqrt adjoint: dt = dd / (2 * d); dvar = sum(dt). */
            for (int64_t j = 0; j < hidden; ++j) {
                float dn = dy[j] * gamma[j];
                float q = (dn * n[j]) / lr.d;
                float dd = -q;
                float two_d = 2.0f * lr.d;
                tmp[j] = dd / two_d;
                ds[j] = dn / lr.d; /* dc1 */
            }
            float dvar = orc_tree_sum_f32(tmp, hidden, 1);
            float dS2 = dvar / hf;
            /* dc = (dS2*c + dS2*c) + dc1 */
            for (int64_t j = 0; j < hidden; ++j) {
                float p = dS2 * c[j];
                float pair = p + p;
                ds[j] = pair + ds[j];
                tmp[j] = -ds[j];
            }
            float dm = orc_tree_sum_f32(tmp, hidden, 1);
            float dS1 = dm / hf;
            float *dxr = dx + r * hidden;
            for (int64_t j = 0; j < hidden; ++j) dxr[j] = canon_f32(dS1 + ds[j]);
        }
        free(c);
        free(n);
        free(y);
        free(s);
        free(ds);
        free(tmp);
    }
    orc_col_sum_f32(dyn_rows, rows, hidden, dgamma);
    orc_col_sum_f32(dy_rows, rows, hidden, dbeta);
    free(dyn_rows);
    free(dy_rows);
}

/* ------------------------------------------------------------------------ */
/* cumsum: spec/05-risc-primitives.md:4310-4325                             */
/* ------------------------------------------------------------------------ */

/* The first input is the first prefix (no base value); each later input is
 * added to the previous prefix.  `reverse` is the decreasing-axis scan. */
void orc_cumsum_f64(const double *x, double *y, int64_t lanes, int64_t len, int reverse) {
#pragma omp parallel for schedule(static)
    for (int64_t l = 0; l < lanes; ++l) {
        const double *xl = x + l * len;
        double *yl = y + l * len;
        if (len == 0) continue;
        if (!reverse) {
            double acc = xl[0];
            yl[0] = canon_f64(acc);
            for (int64_t t = 1; t < len; ++t) {
                acc = acc + xl[t];
                yl[t] = canon_f64(acc);
            }
        } else {
            double acc = xl[len - 1];
            yl[len - 1] = canon_f64(acc);
            for (int64_t t = len - 2; t >= 0; --t) {
                acc = acc + xl[t];
                yl[t] = canon_f64(acc);
            }
        }
    }
}
void orc_cumsum_f32(const float *x, float *y, int64_t lanes, int64_t len, int reverse) {
#pragma omp parallel for schedule(static)
    for (int64_t l = 0; l < lanes; ++l) {
        const float *xl = x + l * len;
        float *yl = y + l * len;
        if (len == 0) continue;
        if (!reverse) {
            float acc = xl[0];
            yl[0] = canon_f32(acc);
            for (int64_t t = 1; t < len; ++t) {
                acc = acc + xl[t];
                yl[t] = canon_f32(acc);
            }
        } else {
            float acc = xl[len - 1];
            yl[len - 1] = canon_f32(acc);
            for (int64_t t = len - 2; t >= 0; --t) {
                acc = acc + xl[t];
                yl[t] = canon_f32(acc);
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* vmap'd covariance / risk (f64).  The batch axis is vectorize_axis0's      */
/* leading axis (crates/chelis-ir-core/src/vmap.rs:9-56); per portfolio:    */
/*   mean_a = sum_t R[t,a] / T;  C = R - mean;                              */
/*   Sigma = matmul(transpose(C), C) / (T - 1);                             */
/*   risk = sqrt(matmul(w, matmul(Sigma, w)));  cum = cumsum_t(matmul(R, w)) */
/* ------------------------------------------------------------------------ */
void orc_portfolio(const double *r, const double *w, int64_t count, int64_t t, int64_t a,
                   double *sigma, double *risk, double *cum) {
    double tf = (double)t, tm1 = (double)(t - 1);
#pragma omp parallel
    {
        double *cen = (double *)malloc(sizeof(double) * (size_t)(t * a));
        double *mean = (double *)malloc(sizeof(double) * (size_t)a);
        double *u = (double *)malloc(sizeof(double) * (size_t)a);
        double *leaf = (double *)malloc(sizeof(double) * (size_t)(t > a ? t : a));
#pragma omp for schedule(static)
        for (int64_t p = 0; p < count; ++p) {
            const double *rp = r + p * t * a;
            const double *wp = w + p * a;
            double *sp = sigma + p * a * a;
            for (int64_t j = 0; j < a; ++j) mean[j] = orc_tree_sum_f64(rp + j, t, a) / tf;
            for (int64_t i = 0; i < t; ++i)
                for (int64_t j = 0; j < a; ++j) cen[i * a + j] = rp[i * a + j] - mean[j];
            for (int64_t i = 0; i < a; ++i) {
                for (int64_t j = 0; j < a; ++j) {
                    for (int64_t s = 0; s < t; ++s) leaf[s] = cen[s * a + i] * cen[s * a + j];
                    sp[i * a + j] = canon_f64(orc_tree_sum_f64(leaf, t, 1) / tm1);
                }
            }
            for (int64_t i = 0; i < a; ++i) {
                for (int64_t j = 0; j < a; ++j) leaf[j] = sp[i * a + j] * wp[j];
                u[i] = orc_tree_sum_f64(leaf, a, 1);
            }
            for (int64_t i = 0; i < a; ++i) leaf[i] = wp[i] * u[i];
            risk[p] = canon_f64(sqrt(orc_tree_sum_f64(leaf, a, 1)));
            double *cp = cum + p * t;
            for (int64_t s = 0; s < t; ++s) {
                for (int64_t j = 0; j < a; ++j) leaf[j] = rp[s * a + j] * wp[j];
                cp[s] = orc_tree_sum_f64(leaf, a, 1);
            }
            double acc = cp[0];
            for (int64_t s = 1; s < t; ++s) {
                acc = acc + cp[s];
                cp[s] = canon_f64(acc);
            }
        }
        free(cen);
        free(mean);
        free(u);
        free(leaf);
    }
}

/* ------------------------------------------------------------------------ */
/* 2-layer MLP: logits = relu(x W1 + b1) W2 + b2; loss = mean(CE(logits))   */
/* CE per spec/05-risc-primitives.md:5044-5063 (log(softmax), gather,       */
/* diagonal, neg); mean = tree sum / batch.  Adjoints from grad.rs.         */
/* ------------------------------------------------------------------------ */
void orc_mlp_step(const float *x, const int64_t *labels, const float *w1, const float *b1,
                  const float *w2, const float *b2, int64_t batch, int64_t din, int64_t dh,
                  int64_t dout, float *loss, float *dw1, float *db1, float *dw2, float *db2) {
    size_t bh = (size_t)(batch * dh), bo = (size_t)(batch * dout);
    float *pre = (float *)malloc(sizeof(float) * bh);
    float *h = (float *)malloc(sizeof(float) * bh);
    float *z = (float *)malloc(sizeof(float) * bo);
    float *s = (float *)malloc(sizeof(float) * bo);
    float *dz = (float *)malloc(sizeof(float) * bo);
    float *dhid = (float *)malloc(sizeof(float) * bh);
    float *nl = (float *)malloc(sizeof(float) * (size_t)batch);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)(dout > 1 ? dout : 1));
    float *g = (float *)malloc(sizeof(float) * (size_t)(dout > 1 ? dout : 1));

    /* forward */
    orc_sgemm(x, w1, pre, batch, dh, din, 0, batch);
    for (int64_t i = 0; i < batch; ++i)
        for (int64_t j = 0; j < dh; ++j) {
            float v = pre[i * dh + j] + b1[j];
            pre[i * dh + j] = v;
            /* relu = max_elem(x, 0) (spec 05 section 3.3, [05-OP-43]) */
            h[i * dh + j] = (v < 0.0f) ? 0.0f : v;
        }
    orc_sgemm(h, w2, z, batch, dout, dh, 0, batch);
    for (int64_t i = 0; i < batch; ++i)
        for (int64_t j = 0; j < dout; ++j) z[i * dout + j] = z[i * dout + j] + b2[j];
    orc_softmax_rows_f32(z, s, batch, dout);
    for (int64_t i = 0; i < batch; ++i) {
        float lp = orc_logf(s[i * dout + labels[i]]);
        nl[i] = -lp;
    }
    float bf = (float)batch;
    *loss = canon_f32(orc_tree_sum_f32(nl, batch, 1) / bf);

    /* adjoint: mean -> div by batch; neg; gather+diagonal scatter; log
     * (g / x); softmax (grad.rs:2248-2280). */
    float dnl = 1.0f / bf;
    float dsel = -dnl;
    for (int64_t i = 0; i < batch; ++i) {
        const float *si = s + i * dout;
        for (int64_t j = 0; j < dout; ++j) {
            float dlp = (j == labels[i]) ? dsel : 0.0f;
            g[j] = dlp / si[j];
        }
        softmax_row_bwd(si, g, dz + i * dout, tmp, dout);
    }
    orc_col_sum_f32(dz, batch, dout, db2);
    /* dW2 = h^T dz, tree over the batch axis */
    orc_sgemm_strided(h, 1, dh, dz, dout, 1, dw2, dh, dout, batch);
    /* dh = dz W2^T, tree over the output axis */
    orc_sgemm_strided(dz, dout, 1, w2, 1, dout, dhid, batch, dh, dout);
    /* relu adjoint: g where 0 < x, else +0 ([05-OP-43]) */
    for (size_t q = 0; q < bh; ++q) dhid[q] = (0.0f < pre[q]) ? dhid[q] : 0.0f;
    orc_col_sum_f32(dhid, batch, dh, db1);
    orc_sgemm_strided(x, 1, din, dhid, dh, 1, dw1, din, dh, batch);

    free(pre);
    free(h);
    free(z);
    free(s);
    free(dz);
    free(dhid);
    free(nl);
    free(tmp);
    free(g);
}

/* ------------------------------------------------------------------------ */
/* single finalized f32 operations ([04-NUM-2]), for pinning against the    */
/* reference's profile obligations (crates/chelis-crmath/tests/fixtures/    */
/* profile_obligations.txt)                                                 */
/* ------------------------------------------------------------------------ */
float orc_add_f32(float a, float b) { return canon_f32(a + b); }
float orc_mul_f32(float a, float b) { return canon_f32(a * b); }
float orc_div_f32(float a, float b) { return canon_f32(a / b); }
float orc_sqrt_f32(float a) { return canon_f32(sqrtf(a)); }

/* ------------------------------------------------------------------------ */
/* FusedElem groups: the chain of FusedStepOps (crates/chelis-dag-core/src/ */
/* dag.rs:494-526) evaluated per element as the C lane emits it             */
/* (crates/chelis-backend-c/src/emit.rs scalar_step_raw_expr :6744-6905,    */
/* each step finalized by fp_env.rs fused_step_nan_finalization :213-241:   */
/* canonical NaN after every op but MaxElem / MinElem), and reduced along   */
/* one axis as emit_fused_reduce does (emit.rs:9580-9860: Sum by the carry  */
/* tree, finalized once; Max folding chelis_fmax_propnan_f32 from -inf,     */
/* crates/chelis-runtime/include/chelis_simd.h:66-69).  Transcendentals     */
/* are the reference's CORE-MATH (chelis_cr_* -> crmath_ffi.c).             */
/* ------------------------------------------------------------------------ */
float chelis_crmath_ffi_sinf(float);
float chelis_crmath_ffi_cosf(float);
float chelis_crmath_ffi_tanf(float);
float chelis_crmath_ffi_atanf(float);
float chelis_crmath_ffi_tanhf(float);
float chelis_crmath_ffi_erff(float);
float chelis_crmath_ffi_powf(float, float);
double chelis_crmath_ffi_log(double);
double chelis_crmath_ffi_sin(double);
double chelis_crmath_ffi_cos(double);
double chelis_crmath_ffi_tan(double);
double chelis_crmath_ffi_atan(double);
double chelis_crmath_ffi_tanh(double);
double chelis_crmath_ffi_erf(double);
double chelis_crmath_ffi_erfc(double);
double chelis_crmath_ffi_pow(double, double);

enum {
    F_ADD, F_SUB, F_MUL, F_DIV, F_POW, F_FLOOR_DIV, F_TRUNC_DIV, F_MAX, F_MIN, F_NEG, F_RECIP,
    F_EXP, F_LOG, F_SIN, F_SQRT, F_COS, F_TAN, F_ATAN, F_TANH, F_ERF, F_ERFC, F_ABS, F_FLOOR,
    F_CEIL, F_ROUND
};

#define DEFINE_FUSED(T, SUFFIX, CANON, CR, FLOOR, CEIL, RINT, FABS, SQRT)                      \
    static T fused_step_##SUFFIX(int op, T x, T y) {                                           \
        switch (op) {                                                                          \
            case F_ADD: return CANON(x + y);                                                   \
            case F_SUB: return CANON((x) - (y));                                               \
            case F_MUL: return CANON(x * y);                                                   \
            case F_DIV: return CANON(x / y);                                                   \
            case F_POW: return CANON(CR(pow)(x, y));                                           \
            case F_FLOOR_DIV: return CANON(FLOOR(x / y));                                      \
            case F_MAX: return (isnan(x) || (!isnan(y) && x >= y)) ? x : y;                    \
            case F_MIN: return (isnan(x) || (!isnan(y) && x <= y)) ? x : y;                    \
            case F_NEG: return CANON(-x);                                                      \
            case F_RECIP: return CANON((T)1 / x);                                              \
            case F_EXP: return CANON(CR(exp)(x));                                              \
            case F_LOG: return CANON(CR(log)(x));                                              \
            case F_SIN: return CANON(CR(sin)(x));                                              \
            case F_SQRT: return CANON(SQRT(x));                                                \
            case F_COS: return CANON(CR(cos)(x));                                              \
            case F_TAN: return CANON(CR(tan)(x));                                              \
            case F_ATAN: return CANON(CR(atan)(x));                                            \
            case F_TANH: return CANON(CR(tanh)(x));                                            \
            case F_ERF: return CANON(CR(erf)(x));                                              \
            case F_ERFC: return CANON(CR(erfc)(x));                                            \
            case F_ABS: return CANON(FABS(x));                                                 \
            case F_FLOOR: return CANON(FLOOR(x));                                              \
            case F_CEIL: return CANON(CEIL(x));                                                \
            case F_ROUND: return CANON(RINT(x));                                               \
            default: abort();                                                                  \
        }                                                                                      \
    }                                                                                          \
    /* value of the chain at the element with coordinates `coord` */                          \
    static T fused_eval_##SUFFIX(const int32_t *steps, int n_steps, const T *const *in,         \
                                 const int64_t *strides, int n_in, const int64_t *coord,       \
                                 int rank, T *v) {                                             \
        T ext[8];                                                                              \
        for (int k = 0; k < n_in; ++k) {                                                       \
            int64_t off = 0;                                                                   \
            for (int d = 0; d < rank; ++d) off += coord[d] * strides[k * rank + d];            \
            ext[k] = in[k][off];                                                               \
        }                                                                                      \
        for (int s = 0; s < n_steps; ++s) {                                                    \
            int op = steps[3 * s], a = steps[3 * s + 1], b = steps[3 * s + 2];                 \
            T x = a >= 0 ? ext[a] : v[-1 - a];                                                 \
            T y = x;                                                                           \
            if (op <= F_MIN) y = b >= 0 ? ext[b] : v[-1 - b];                                  \
            v[s] = fused_step_##SUFFIX(op, x, y);                                              \
        }                                                                                      \
        return v[n_steps - 1];                                                                 \
    }                                                                                          \
    void orc_fused_elementwise_##SUFFIX(const int32_t *steps, int32_t n_steps,                 \
                                        const T *const *in, const int64_t *strides,            \
                                        int32_t n_in, const int64_t *shape, int32_t rank,      \
                                        T *out) {                                              \
        int64_t total = 1;                                                                     \
        for (int d = 0; d < rank; ++d) total *= shape[d];                                      \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int64_t i = 0; i < total; ++i) {                                                  \
            int64_t coord[8], rem = i;                                                         \
            T v[32];                                                                           \
            for (int d = rank - 1; d >= 0; --d) {                                              \
                coord[d] = rem % shape[d];                                                     \
                rem /= shape[d];                                                               \
            }                                                                                  \
            out[i] = fused_eval_##SUFFIX(steps, n_steps, in, strides, n_in, coord, rank, v);   \
        }                                                                                      \
    }                                                                                          \
    /* kind 0 = Sum, 1 = Max; out is dense over shape without `axis` */                       \
    void orc_fused_reduce_##SUFFIX(const int32_t *steps, int32_t n_steps, const T *const *in,  \
                                   const int64_t *strides, int32_t n_in, const int64_t *shape, \
                                   int32_t rank, int32_t axis, int32_t kind, T *out) {         \
        int64_t outputs = 1, len = shape[axis];                                                \
        for (int d = 0; d < rank; ++d)                                                         \
            if (d != axis) outputs *= shape[d];                                                \
        _Pragma("omp parallel for schedule(static)")                                           \
        for (int64_t o = 0; o < outputs; ++o) {                                                \
            int64_t coord[8], rem = o;                                                         \
            T v[32];                                                                           \
            for (int d = rank - 1; d >= 0; --d) {                                              \
                if (d == axis) continue;                                                       \
                coord[d] = rem % shape[d];                                                     \
                rem /= shape[d];                                                               \
            }                                                                                  \
            if (kind == 0) {                                                                   \
                T level[64];                                                                   \
                int64_t count = 0;                                                             \
                for (int64_t j = 0; j < len; ++j) {                                            \
                    coord[axis] = j;                                                           \
                    T carry = fused_eval_##SUFFIX(steps, n_steps, in, strides, n_in, coord,    \
                                                  rank, v);                                    \
                    int depth = 0;                                                             \
                    for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)       \
                        carry = level[depth] + carry;                                          \
                    level[depth] = carry;                                                      \
                }                                                                              \
                T total = (T)0;                                                                \
                int found = 0, depth = 0;                                                      \
                for (int64_t remaining = count; remaining; remaining >>= 1, ++depth)           \
                    if (remaining & 1) {                                                       \
                        total = found ? level[depth] + total : level[depth];                   \
                        found = 1;                                                             \
                    }                                                                          \
                out[o] = CANON(total);                                                         \
            } else {                                                                           \
                T acc = -INFINITY;                                                             \
                for (int64_t j = 0; j < len; ++j) {                                            \
                    coord[axis] = j;                                                           \
                    T x = fused_eval_##SUFFIX(steps, n_steps, in, strides, n_in, coord, rank,  \
                                              v);                                              \
                    /* chelis_fmax_propnan_f32(acc, x) */                                      \
                    acc = (acc != acc || x != x) ? CANON((T)NAN) : (acc > x ? acc : x);        \
                }                                                                              \
                out[o] = acc;                                                                  \
            }                                                                                  \
        }                                                                                      \
    }

#define CR_F32(name) chelis_crmath_ffi_##name##f
#define CR_F64(name) chelis_crmath_ffi_##name
static inline float cr_sqrtf(float x) { return sqrtf(x); }
DEFINE_FUSED(float, f32, canon_f32, CR_F32, floorf, ceilf, rintf, fabsf, cr_sqrtf)
DEFINE_FUSED(double, f64, canon_f64, CR_F64, floor, ceil, rint, fabs, sqrt)

/* ------------------------------------------------------------------------ */
/* activations, layer_norm adjoint, cross-entropy                           */
/* ------------------------------------------------------------------------ */
/* [05-OP-43] relu = max_elem(x, +0) (spec/05-risc-primitives.md:1439-1452):
 * a NaN keeps its bits, -0 stays -0 (first operand on ties). */
void orc_relu_f32(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = (isnan(x[i]) || x[i] >= 0.0f) ? x[i] : 0.0f;
}
void orc_relu_f64(const double *x, double *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = (isnan(x[i]) || x[i] >= 0.0) ? x[i] : 0.0;
}
/* ReluAdjoint: g where cmplt(0, x), exact +0 otherwise (grad.rs:2281-2294). */
void orc_relu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dx[i] = (0.0f < x[i]) ? g[i] : 0.0f;
}
void orc_relu_adjoint_f64(const double *x, const double *g, double *dx, int64_t n) {
    for (int64_t i = 0; i < n; ++i) dx[i] = (0.0 < x[i]) ? g[i] : 0.0;
}

/* gelu(x) = mul(m(x), Phi(x)) with the compensated Phi graph of
 * spec/05-risc-primitives.md:1353-1400 at f32 (tier2.rs lower_gelu); every
 * step one finalized f32 operation, erfc and exp CORE-MATH. */
static float phi_graph_f32(float x) {
    const float c = 0x1.6a09e6p-1f, cl = 0x1.9fcef4p-27f, k = 0x1.20dd76p+0f, s = 4097.0f;
    float e = canon_f32(chelis_crmath_ffi_erfcf(canon_f32(canon_f32(-x) * c)));
    float z = (fabsf(x) < 64.0f) ? x : 0.0f;
    float a = canon_f32(-z);
    float th = canon_f32(a * c);
    float ta = canon_f32(s * a);
    float ah = canon_f32(ta - canon_f32(ta - a));
    float al = canon_f32(a - ah);
    float tc = canon_f32(s * c);
    float ch = canon_f32(tc - canon_f32(tc - c));
    float cr = canon_f32(c - ch);
    float tl = canon_f32(canon_f32(ah * ch) - th);
    tl = canon_f32(tl + canon_f32(ah * cr));
    tl = canon_f32(tl + canon_f32(al * ch));
    tl = canon_f32(tl + canon_f32(al * cr));
    tl = canon_f32(tl + canon_f32(a * cl));
    float ex = canon_f32(chelis_crmath_ffi_expf(canon_f32(-canon_f32(th * th))));
    float corr = canon_f32(canon_f32(k * ex) * tl);
    return canon_f32(0.5f * canon_f32(e - corr));
}
void orc_gelu_f32(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float m = (x[i] < -0x1.fffffep+127f) ? -0.0f : x[i]; /* the multiplicand guard m(x) */
        y[i] = canon_f32(m * phi_graph_f32(x[i]));
    }
}

/* Adjoint of layer_norm over the last axis given dy: the LN part of
 * orc_chain_bwd on its own (the AD of tier2.rs:1248-1375; dgamma, dbeta by
 * the canonical tree over rows). */
void orc_layer_norm_bwd_f32(const float *x, const float *gamma, float eps, const float *dy_all,
                            int64_t rows, int64_t hidden, float *dx, float *dgamma, float *dbeta) {
    float hf = (float)hidden;
    float *dyn_rows = (float *)malloc(sizeof(float) * (size_t)(rows * hidden));
#pragma omp parallel
    {
        float *c = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *n = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *y = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *ds = (float *)malloc(sizeof(float) * (size_t)hidden);
        float *tmp = (float *)malloc(sizeof(float) * (size_t)hidden);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const float *xr = x + r * hidden;
            const float *dy = dy_all + r * hidden;
            ln_row lr = ln_row_fwd(xr, gamma, gamma, eps, hidden, c, n, y);
            float *dyn = dyn_rows + r * hidden;
            for (int64_t j = 0; j < hidden; ++j) dyn[j] = dy[j] * n[j];
            for (int64_t j = 0; j < hidden; ++j) {
                float dn = dy[j] * gamma[j];
                float q = (dn * n[j]) / lr.d;
                float dd = -q;
                float two_d = 2.0f * lr.d;
                tmp[j] = dd / two_d;
                ds[j] = dn / lr.d;
            }
            float dS2 = orc_tree_sum_f32(tmp, hidden, 1) / hf;
            for (int64_t j = 0; j < hidden; ++j) {
                float p = dS2 * c[j];
                ds[j] = (p + p) + ds[j];
                tmp[j] = -ds[j];
            }
            float dS1 = orc_tree_sum_f32(tmp, hidden, 1) / hf;
            float *dxr = dx + r * hidden;
            for (int64_t j = 0; j < hidden; ++j) dxr[j] = canon_f32(dS1 + ds[j]);
        }
        free(c);
        free(n);
        free(y);
        free(ds);
        free(tmp);
    }
    orc_col_sum_f32(dyn_rows, rows, hidden, dgamma);
    orc_col_sum_f32(dy_all, rows, hidden, dbeta);
    free(dyn_rows);
}

/* Cross-entropy (spec/05-risc-primitives.md:5044-5063): loss =
 * mean_r(-log softmax(z_r)[label_r]) and, when dz is non-NULL, its adjoint
 * through mean, neg, gather, log and softmax -- the loss head of
 * orc_mlp_step on its own.  Returns 1 on an out-of-range label. */
int orc_cross_entropy_f32(const float *z, const int64_t *labels, int64_t rows, int64_t classes,
                          float *loss, float *dz) {
    for (int64_t i = 0; i < rows; ++i)
        if (labels[i] < 0 || labels[i] >= classes) return 1;
    float *s = (float *)malloc(sizeof(float) * (size_t)(rows * classes));
    float *nl = (float *)malloc(sizeof(float) * (size_t)rows);
    float *g = (float *)malloc(sizeof(float) * (size_t)classes);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)classes);
    orc_softmax_rows_f32(z, s, rows, classes);
    for (int64_t i = 0; i < rows; ++i) nl[i] = -orc_logf(s[i * classes + labels[i]]);
    float bf = (float)rows;
    *loss = canon_f32(orc_tree_sum_f32(nl, rows, 1) / bf);
    if (dz) {
        float dsel = -(1.0f / bf);
        for (int64_t i = 0; i < rows; ++i) {
            const float *si = s + i * classes;
            for (int64_t j = 0; j < classes; ++j) g[j] = ((j == labels[i]) ? dsel : 0.0f) / si[j];
            softmax_row_bwd(si, g, dz + i * classes, tmp, classes);
        }
    }
    free(s);
    free(nl);
    free(g);
    free(tmp);
    return 0;
}
