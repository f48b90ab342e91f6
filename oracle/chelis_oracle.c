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

/* Compare n results of a binary32 exp (op 0) / log (op 1) at the consecutive
 * bit patterns start, start + 1, ... (wrapping at 2^32) with CORE-MATH: bit
 * for bit, any NaN matching any NaN.  Returns the mismatch count and the
 * offset of the first mismatch (-1 if none). */
int64_t orc_crmath_check_f32(int32_t op, uint32_t start, int64_t n, const float *got,
                             int64_t *first_bad) {
    int64_t bad = 0, first = -1;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (int64_t i = 0; i < n; ++i) {
        uint32_t xb = start + (uint32_t)i;
        float x;
        memcpy(&x, &xb, 4);
        const float want = op == 0 ? chelis_crmath_ffi_expf(x) : chelis_crmath_ffi_logf(x);
        uint32_t wb, gb;
        memcpy(&wb, &want, 4);
        memcpy(&gb, &got[i], 4);
        const int ok = (isnan(want) && isnan(got[i])) || wb == gb;
        if (!ok) {
            bad += 1;
#pragma omp critical
            if (first < 0 || i < first) first = i;
        }
    }
    if (first_bad) *first_bad = first;
    return bad;
}

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


/*
 * The C lane streams every output's tree over k through a carry tree, in
 * lane blocks of output columns that share one leaf schedule (emit.rs:
 * 8113-8176).  The restatement does the same with blocks of 64 columns
 * and one more step that leaves every value unchanged: an aligned run of 8
 * leaves is a complete subtree of the canonical tree, so the first
 * k - k % 8 leaves enter in groups, each group's subtree
 * ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)) formed in registers and pushed at
 * depth 3; the carry tree then sees exactly the sums it would have built
 * leaf by leaf.  The last k % 8 leaves enter one at a time.  Lanes are
 * independent IEEE operations (GCC vector extensions; no reassociation, no
 * contraction), so the values equal the scalar tree's bit for bit
 * (tests/test_oracle.py checks this against orc_tree_sum_f32).
 */
#define VL 8 /* vector lanes per vector */
#define NV (LANES / VL)
typedef float v8f __attribute__((vector_size(VL * sizeof(float))));
typedef double v8d __attribute__((vector_size(VL * sizeof(double))));

#define DEFINE_GEMM_ROWS(T, V, SUFFIX, CANON)                                                  \
    __attribute__((target_clones("avx2", "default"))) static void gemm_block_##SUFFIX(          \
        const T *arow, int64_t sa1, const T *b, int64_t ldb, T *crow, int64_t k) {             \
        V lv[64][NV];                                                                          \
        V leaf[NV];                                                                            \
        int64_t count = 0;                                                                     \
        const int64_t kb_end = k & ~(int64_t)7;                                                \
        for (int64_t kk = 0; kk < kb_end; kk += 8) {                                           \
            const T a0 = arow[(kk + 0) * sa1], a1 = arow[(kk + 1) * sa1];                      \
            const T a2 = arow[(kk + 2) * sa1], a3 = arow[(kk + 3) * sa1];                      \
            const T a4 = arow[(kk + 4) * sa1], a5 = arow[(kk + 5) * sa1];                      \
            const T a6 = arow[(kk + 6) * sa1], a7 = arow[(kk + 7) * sa1];                      \
            const T *bp = b + kk * ldb;                                                        \
            for (int v = 0; v < NV; ++v) {                                                     \
                V b0, b1, b2, b3, b4, b5, b6, b7;                                              \
                memcpy(&b0, bp + 0 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b1, bp + 1 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b2, bp + 2 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b3, bp + 3 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b4, bp + 4 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b5, bp + 5 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b6, bp + 6 * ldb + v * VL, sizeof(V));                                 \
                memcpy(&b7, bp + 7 * ldb + v * VL, sizeof(V));                                 \
                V p01 = (a0 * b0) + (a1 * b1), p23 = (a2 * b2) + (a3 * b3);                    \
                V p45 = (a4 * b4) + (a5 * b5), p67 = (a6 * b6) + (a7 * b7);                    \
                leaf[v] = (p01 + p23) + (p45 + p67);                                           \
            }                                                                                  \
            int depth = 3;                                                                     \
            for (int64_t pending = count >> 3; pending & 1; pending >>= 1, ++depth)            \
                for (int v = 0; v < NV; ++v) leaf[v] = lv[depth][v] + leaf[v];                 \
            for (int v = 0; v < NV; ++v) lv[depth][v] = leaf[v];                               \
            count += 8;                                                                        \
        }                                                                                      \
        for (int64_t kk = kb_end; kk < k; ++kk) {                                              \
            const T av = arow[kk * sa1];                                                       \
            for (int v = 0; v < NV; ++v) {                                                     \
                V bv;                                                                          \
                memcpy(&bv, b + kk * ldb + v * VL, sizeof(V));                                 \
                leaf[v] = av * bv;                                                             \
            }                                                                                  \
            int depth = 0;                                                                     \
            for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)               \
                for (int v = 0; v < NV; ++v) leaf[v] = lv[depth][v] + leaf[v];                 \
            for (int v = 0; v < NV; ++v) lv[depth][v] = leaf[v];                               \
        }                                                                                      \
        int found = 0, depth = 0;                                                              \
        for (int v = 0; v < NV; ++v) leaf[v] = (V){0};                                         \
        for (int64_t remaining = count; remaining; remaining >>= 1, ++depth) {                 \
            if (remaining & 1) {                                                               \
                for (int v = 0; v < NV; ++v) leaf[v] = found ? lv[depth][v] + leaf[v] : lv[depth][v]; \
                found = 1;                                                                     \
            }                                                                                  \
        }                                                                                      \
        for (int v = 0; v < NV; ++v)                                                           \
            for (int l = 0; l < VL; ++l) crow[v * VL + l] = CANON(leaf[v][l]);                 \
    }                                                                                          \
    static void gemm_rows_##SUFFIX(const T *a, int64_t sa0, int64_t sa1, const T *b0,          \
                                   int64_t sb0, int64_t sb1, T *c, int64_t ldc, int64_t n,     \
                                   int64_t k, int64_t row_begin, int64_t row_end) {            \
        /* a B that is not row-contiguous is first copied to row-major [k, n] */               \
        T *bt = NULL;                                                                          \
        const T *b = b0;                                                                       \
        int64_t ldb = sb0;                                                                     \
        if (sb1 != 1 && k > 0 && n > 0) {                                                      \
            bt = (T *)malloc(sizeof(T) * (size_t)(k * n));                                     \
            _Pragma("omp parallel for schedule(static)")                                       \
            for (int64_t kk = 0; kk < k; ++kk)                                                 \
                for (int64_t j = 0; j < n; ++j) bt[kk * n + j] = b0[kk * sb0 + j * sb1];       \
            b = bt;                                                                            \
            ldb = n;                                                                           \
        }                                                                                      \
        int64_t blocks = (n + LANES - 1) / LANES;                                              \
        _Pragma("omp parallel for schedule(dynamic, 1) collapse(2)")                           \
        for (int64_t i = row_begin; i < row_end; ++i) {                                        \
            for (int64_t bj = 0; bj < blocks; ++bj) {                                          \
                int64_t j0 = bj * LANES;                                                       \
                int lanes = (int)((n - j0) < LANES ? (n - j0) : LANES);                        \
                if (lanes == LANES) {                                                          \
                    gemm_block_##SUFFIX(a + i * sa0, sa1, b + j0, ldb, c + i * ldc + j0, k);   \
                    continue;                                                                  \
                }                                                                              \
                laned_##SUFFIX t;                                                              \
                t.count = 0;                                                                   \
                T leafs[LANES];                                                                \
                for (int64_t kk = 0; kk < k; ++kk) {                                           \
                    T av = a[i * sa0 + kk * sa1];                                              \
                    const T *brow = b + kk * ldb + j0;                                         \
                    for (int l = 0; l < lanes; ++l) leafs[l] = av * brow[l];                   \
                    laned_push_##SUFFIX(&t, leafs, lanes);                                     \
                }                                                                              \
                laned_total_##SUFFIX(&t, leafs, lanes);                                        \
                for (int l = 0; l < lanes; ++l) c[i * ldc + j0 + l] = CANON(leafs[l]);         \
            }                                                                                  \
        }                                                                                      \
        free(bt);                                                                              \
    }
DEFINE_GEMM_ROWS(float, v8f, f32, canon_f32)
DEFINE_GEMM_ROWS(double, v8d, f64, canon_f64)

static void sgemm_rows(const float *a, int64_t sa0, int64_t sa1, const float *b, int64_t sb0,
                       int64_t sb1, float *c, int64_t ldc, int64_t n, int64_t k,
                       int64_t row_begin, int64_t row_end) {
    gemm_rows_f32(a, sa0, sa1, b, sb0, sb1, c, ldc, n, k, row_begin, row_end);
}
static void dgemm_rows(const double *a, int64_t sa0, int64_t sa1, const double *b, int64_t sb0,
                       int64_t sb1, double *c, int64_t ldc, int64_t n, int64_t k,
                       int64_t row_begin, int64_t row_end) {
    gemm_rows_f64(a, sa0, sa1, b, sb0, sb1, c, ldc, n, k, row_begin, row_end);
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
#pragma omp parallel for schedule(static)
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

/* ------------------------------------------------------------------------ */
/* GELU adjoint: reverse mode through the Phi graph above                   */
/* ------------------------------------------------------------------------ */
/*
 * The adjoint graph of gelu = mul(m(x), Phi(x)) node by node, with the
 * rules of crates/chelis-dag-core/src/grad.rs: mul gives (g*b, g*a), sub
 * gives (g, neg(g)), neg gives neg(g), exp gives g*exp(x), erfc gives
 * neg(g*(k*exp(neg(x*x)))) with k = 2/sqrt(pi) rounded once to f32
 * ([05-OP-46], grad.rs:2408-2425), where gives g on the chosen side and
 * +0 on the other.  A node with several consumers sums their cotangents
 * with the adjacent-pair tree in consumer order (balanced_adjoint_sum,
 * grad.rs:1713-1745).  The constants ch, cr (the split of c) carry no
 * cotangent.
 */
static float gelu_adjoint_one(float x, float g) {
    const float c = 0x1.6a09e6p-1f, cl = 0x1.9fcef4p-27f, k = 0x1.20dd76p+0f, s = 4097.0f;
    const float k2 = (float)1.12837916709551257390; /* 2/sqrt(pi) rounded to f32 */
    /* forward values */
    float n1 = canon_f32(-x);
    float n2 = canon_f32(n1 * c);
    float e = canon_f32(chelis_crmath_ffi_erfcf(n2));
    int zc = fabsf(x) < 64.0f;
    float z = zc ? x : 0.0f;
    float a = canon_f32(-z);
    float th = canon_f32(a * c);
    float ta = canon_f32(s * a);
    float t1 = canon_f32(ta - a);
    float ah = canon_f32(ta - t1);
    float al = canon_f32(a - ah);
    float tc = canon_f32(s * c);
    float ch = canon_f32(tc - canon_f32(tc - c));
    float cr = canon_f32(c - ch);
    float tl0 = canon_f32(canon_f32(ah * ch) - th);
    float tl1 = canon_f32(tl0 + canon_f32(ah * cr));
    float tl2 = canon_f32(tl1 + canon_f32(al * ch));
    float tl3 = canon_f32(tl2 + canon_f32(al * cr));
    float tl = canon_f32(tl3 + canon_f32(a * cl));
    float sq = canon_f32(th * th);
    float ex = canon_f32(chelis_crmath_ffi_expf(canon_f32(-sq)));
    float kx = canon_f32(k * ex);
    float corr = canon_f32(kx * tl);
    float phi = canon_f32(0.5f * canon_f32(e - corr));
    int mc = x < -0x1.fffffep+127f;
    float m = mc ? -0.0f : x;
    (void)tl2;
    (void)tl3;
    (void)tl1;
    /* reverse sweep */
    float g_m = canon_f32(g * phi);
    float g_phi = canon_f32(g * m);
    float g_df = canon_f32(g_phi * 0.5f);
    float g_e = g_df;
    float g_corr = canon_f32(-g_df);
    float g_kx = canon_f32(g_corr * tl);
    float g_tl = canon_f32(g_corr * kx);
    float g_ex = canon_f32(g_kx * k);
    float g_nsq = canon_f32(g_ex * ex);
    float g_sq = canon_f32(-g_nsq);
    /* tl = ((((ah*ch - th) + ah*cr) + al*ch) + al*cr) + a*cl */
    float g_p1 = g_tl, g_p2 = g_tl, g_p3 = g_tl, g_p4 = g_tl, g_p5 = g_tl;
    float g_th_tl = canon_f32(-g_tl);
    /* th feeds tl0 (slot 1), then sq (slots 0 and 1) */
    float g_th = canon_f32(canon_f32(g_th_tl + canon_f32(g_sq * th)) + canon_f32(g_sq * th));
    /* al feeds p3 (al*ch), then p4 (al*cr) */
    float g_al = canon_f32(canon_f32(g_p3 * ch) + canon_f32(g_p4 * cr));
    /* ah feeds al = a - ah (slot 1), then p1, then p2 */
    float g_ah = canon_f32(canon_f32(canon_f32(-g_al) + canon_f32(g_p1 * ch)) + canon_f32(g_p2 * cr));
    /* t1 = ta - a feeds ah = ta - t1 (slot 1) */
    float g_t1 = canon_f32(-g_ah);
    /* ta feeds t1 (slot 0), then ah (slot 0) */
    float g_ta = canon_f32(g_t1 + g_ah);
    /* a feeds th, ta, t1 (slot 1), al (slot 0), p5: five cotangents */
    float ga0 = canon_f32(g_th * c), ga1 = canon_f32(g_ta * s), ga2 = canon_f32(-g_t1);
    float ga3 = g_al, ga4 = canon_f32(g_p5 * cl);
    float g_a = canon_f32(canon_f32(canon_f32(ga0 + ga1) + canon_f32(ga2 + ga3)) + ga4);
    float g_z = canon_f32(-g_a);
    /* erfc adjoint, then n2 = n1 * c, n1 = neg(x) */
    float dens = canon_f32(chelis_crmath_ffi_expf(canon_f32(-canon_f32(n2 * n2))));
    float g_n2 = canon_f32(-canon_f32(g_e * canon_f32(k2 * dens)));
    float g_n1 = canon_f32(g_n2 * c);
    float gx0 = canon_f32(-g_n1);
    float gx1 = zc ? g_z : 0.0f;
    float gx2 = mc ? 0.0f : g_m;
    return canon_f32(canon_f32(gx0 + gx1) + gx2);
}

void orc_gelu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) dx[i] = gelu_adjoint_one(x[i], g[i]);
}

/* ------------------------------------------------------------------------ */
/* transformer block: pre-LN, causal multi-head attention, GELU MLP         */
/* ------------------------------------------------------------------------ */
/*
 * Per sample (the batch is the vmap axis, crates/chelis-ir-core/src/
 * vmap.rs:9-56):
 *   h1 = layer_norm(x; g1, b1)                      tier2.rs:1248-1375
 *   [q k v] = h1 . Wqkv                             [S, 3D], row-major
 *   per head h (columns h*Dh .. h*Dh+Dh of q, k, v), spec/05-risc-
 *   primitives.md:5146-5181:
 *     raw = q_h . k_h^T; scores = raw * scale; masked = where(j <= i,
 *     scores, -inf); p = softmax(masked, last axis); o_h = p . v_h
 *   x2 = x + o . Wo
 *   h2 = layer_norm(x2; g2, b2)
 *   u = h2 . W1;  y = x2 + gelu(u) . W2
 * with scale = 1/sqrtf(Dh) at f32.  Every matmul is the tree over its
 * contracted axis in increasing order (emit.rs:8431-8640), the masked
 * entries included (their probabilities are +0).
 *
 * Reverse mode for an upstream cotangent dy (grad.rs adjoint graphs): the
 * matmul adjoint is a matmul with a transposed operand ([05-OP-51]); the
 * softmax adjoint p*(g - sum(g*p)) (grad.rs:2248-2280); where passes the
 * cotangent on the chosen side, +0 on the other; mul by the scale gives
 * g*scale; layer_norm's adjoint is orc_layer_norm_bwd_f32's graph; a node
 * with several consumers sums their cotangents in consumer order (x2: its
 * layer_norm, then the residual add; x: likewise).  A weight is broadcast
 * along the batch axis, so its gradient is the per-sample gradient (tree
 * over the sequence) summed over samples by the canonical tree (the Expand
 * adjoint, grad.rs Sum over the broadcast axis).
 */

/* Streaming canonical tree over equally sized arrays (one leaf per sample). */
typedef struct {
    float *level[64];
    int64_t count, n;
} array_tree;

static void array_tree_push(array_tree *t, float *leaf) {
    /* leaf is consumed: it becomes a level array or is freed */
    int depth = 0;
    for (int64_t pending = t->count++; pending & 1; pending >>= 1, ++depth) {
        float *lv = t->level[depth];
        for (int64_t i = 0; i < t->n; ++i) leaf[i] = lv[i] + leaf[i];
        free(lv);
        t->level[depth] = NULL;
    }
    t->level[depth] = leaf;
}

static void array_tree_total(array_tree *t, float *out) {
    int found = 0, depth = 0;
    for (int64_t remaining = t->count; remaining; remaining >>= 1, ++depth) {
        if (remaining & 1) {
            float *lv = t->level[depth];
            if (found)
                for (int64_t i = 0; i < t->n; ++i) out[i] = lv[i] + out[i];
            else
                memcpy(out, lv, sizeof(float) * (size_t)t->n);
            found = 1;
            free(lv);
            t->level[depth] = NULL;
        }
    }
    if (!found) memset(out, 0, sizeof(float) * (size_t)t->n);
    for (int64_t i = 0; i < t->n; ++i) out[i] = canon_f32(out[i]);
}

static float *falloc(int64_t n) { return (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1)); }

/* Causal attention of one head, forward: p [S,S] and o_h (ldo stride). */
static void attn_head_fwd(const float *q, const float *k, const float *v, int64_t ld, int64_t S,
                          int64_t Dh, float scale, float *p, float *o, int64_t ldo) {
    /* raw = q . k^T: A = q (rows of ld), B[kk][j] = k[j][kk] */
    sgemm_rows(q, ld, 1, k, 1, ld, p, S, S, Dh, 0, S);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < S; ++i) {
        float *pr = p + i * S;
        for (int64_t j = 0; j < S; ++j) pr[j] = (j <= i) ? canon_f32(pr[j] * scale) : -INFINITY;
        softmax_row(pr, pr, S);
    }
    /* o_h = p . v_h */
    sgemm_rows(p, S, 1, v, ld, 1, o, ldo, Dh, S, 0, S);
}

/* Reverse of one head: dq, dk, dv into dqkv columns (ld), given p and do_h. */
static void attn_head_bwd(const float *q, const float *k, const float *v, int64_t ld,
                          const float *p, const float *dout, int64_t lddo, int64_t S, int64_t Dh,
                          float scale, float *dp, float *dq, float *dk, float *dv) {
    /* dv = p^T . do_h */
    sgemm_rows(p, 1, S, dout, lddo, 1, dv, ld, Dh, S, 0, S);
    /* dp = do_h . v_h^T */
    sgemm_rows(dout, lddo, 1, v, 1, ld, dp, S, S, Dh, 0, S);
#pragma omp parallel
    {
        float *tmp = falloc(S);
#pragma omp for schedule(static)
        for (int64_t i = 0; i < S; ++i) {
            const float *pr = p + i * S;
            float *dr = dp + i * S;
            softmax_row_bwd(pr, dr, dr, tmp, S);
            for (int64_t j = 0; j < S; ++j) dr[j] = (j <= i) ? canon_f32(dr[j] * scale) : 0.0f;
        }
        free(tmp);
    }
    /* dq = ds . k_h; dk = ds^T . q_h */
    sgemm_rows(dp, S, 1, k, ld, 1, dq, ld, Dh, S, 0, S);
    sgemm_rows(dp, 1, S, q, ld, 1, dk, ld, Dh, S, 0, S);
}

int orc_block_step(const float *x, const float *dy, int64_t batch, int64_t S, int64_t D,
                   int64_t H, int64_t F, float eps, const float *w_qkv, const float *w_o,
                   const float *w_1, const float *w_2, const float *g1, const float *b1,
                   const float *g2, const float *b2, float *y, float *dx, float *dw_qkv,
                   float *dw_o, float *dw_1, float *dw_2, float *dg1, float *db1, float *dg2,
                   float *db2) {
    if (batch < 0 || S <= 0 || D <= 0 || H <= 0 || F <= 0 || D % H) return 1;
    const int64_t Dh = D / H, D3 = 3 * D, SD = S * D;
    const float scale = 1.0f / sqrtf((float)Dh);
    float *h1 = falloc(SD), *qkv = falloc(S * D3), *o = falloc(SD), *x2 = falloc(SD);
    float *h2 = falloc(SD), *u = falloc(S * F), *act = falloc(S * F), *ps = falloc(H * S * S);
    float *c = falloc(D), *nn = falloc(D);
    /* reverse scratch */
    float *da = falloc(S * F), *du = falloc(S * F), *dh2 = falloc(SD), *dx2 = falloc(SD);
    float *dln = falloc(SD), *dout = falloc(SD), *dqkv = falloc(S * D3), *dh1 = falloc(SD);
    float *dp = falloc(S * S);
    array_tree tw[8];
    const int64_t wn[8] = {D * D3, D * D, D * F, F * D, D, D, D, D};
    for (int t = 0; t < 8; ++t) {
        memset(&tw[t], 0, sizeof(tw[t]));
        tw[t].n = wn[t];
    }
    for (int64_t b = 0; b < batch; ++b) {
        const float *xb = x + b * SD;
        float *yb = y + b * SD;
        /* ---- forward ---- */
        orc_layer_norm_f32(xb, g1, b1, eps, h1, S, D);
        sgemm_rows(h1, D, 1, w_qkv, D3, 1, qkv, D3, D3, D, 0, S);
        for (int64_t h = 0; h < H; ++h)
            attn_head_fwd(qkv + h * Dh, qkv + D + h * Dh, qkv + 2 * D + h * Dh, D3, S, Dh, scale,
                          ps + h * S * S, o + h * Dh, D);
        sgemm_rows(o, D, 1, w_o, D, 1, x2, D, D, D, 0, S);
        for (int64_t i = 0; i < SD; ++i) x2[i] = canon_f32(xb[i] + x2[i]);
        orc_layer_norm_f32(x2, g2, b2, eps, h2, S, D);
        sgemm_rows(h2, D, 1, w_1, F, 1, u, F, F, D, 0, S);
        orc_gelu_f32(u, act, S * F);
        sgemm_rows(act, F, 1, w_2, D, 1, yb, D, D, F, 0, S);
        for (int64_t i = 0; i < SD; ++i) yb[i] = canon_f32(x2[i] + yb[i]);
        if (!dy) continue;
        /* ---- reverse ---- */
        const float *dyb = dy + b * SD;
        float *dw2b = falloc(F * D), *dw1b = falloc(D * F), *dwob = falloc(D * D);
        float *dwqkvb = falloc(D * D3);
        float *dg2b = falloc(D), *db2b = falloc(D), *dg1b = falloc(D), *db1b = falloc(D);
        /* y = x2 + act . W2 */
        sgemm_rows(act, 1, F, dyb, D, 1, dw2b, D, D, S, 0, F);   /* dW2 = act^T dy */
        sgemm_rows(dyb, D, 1, w_2, 1, D, da, F, F, D, 0, S);     /* da = dy W2^T */
        orc_gelu_adjoint_f32(u, da, du, S * F);
        sgemm_rows(h2, 1, D, du, F, 1, dw1b, F, F, S, 0, D);     /* dW1 = h2^T du */
        sgemm_rows(du, F, 1, w_1, 1, F, dh2, D, D, F, 0, S);     /* dh2 = du W1^T */
        orc_layer_norm_bwd_f32(x2, g2, eps, dh2, S, D, dln, dg2b, db2b);
        for (int64_t i = 0; i < SD; ++i) dx2[i] = canon_f32(dln[i] + dyb[i]);
        /* x2 = x + o . Wo */
        sgemm_rows(o, 1, D, dx2, D, 1, dwob, D, D, S, 0, D);     /* dWo = o^T dx2 */
        sgemm_rows(dx2, D, 1, w_o, 1, D, dout, D, D, D, 0, S);   /* do = dx2 Wo^T */
        for (int64_t h = 0; h < H; ++h)
            attn_head_bwd(qkv + h * Dh, qkv + D + h * Dh, qkv + 2 * D + h * Dh, D3,
                          ps + h * S * S, dout + h * Dh, D, S, Dh, scale, dp, dqkv + h * Dh,
                          dqkv + D + h * Dh, dqkv + 2 * D + h * Dh);
        sgemm_rows(h1, 1, D, dqkv, D3, 1, dwqkvb, D3, D3, S, 0, D); /* dWqkv = h1^T dqkv */
        sgemm_rows(dqkv, D3, 1, w_qkv, 1, D3, dh1, D, D, D3, 0, S); /* dh1 = dqkv Wqkv^T */
        orc_layer_norm_bwd_f32(xb, g1, eps, dh1, S, D, dln, dg1b, db1b);
        float *dxb = dx + b * SD;
        for (int64_t i = 0; i < SD; ++i) dxb[i] = canon_f32(dln[i] + dx2[i]);
        array_tree_push(&tw[0], dwqkvb);
        array_tree_push(&tw[1], dwob);
        array_tree_push(&tw[2], dw1b);
        array_tree_push(&tw[3], dw2b);
        array_tree_push(&tw[4], dg1b);
        array_tree_push(&tw[5], db1b);
        array_tree_push(&tw[6], dg2b);
        array_tree_push(&tw[7], db2b);
    }
    if (dy) {
        float *outs[8] = {dw_qkv, dw_o, dw_1, dw_2, dg1, db1, dg2, db2};
        for (int t = 0; t < 8; ++t) array_tree_total(&tw[t], outs[t]);
    }
    (void)c;
    (void)nn;
    free(h1); free(qkv); free(o); free(x2); free(h2); free(u); free(act); free(ps);
    free(c); free(nn); free(da); free(du); free(dh2); free(dx2); free(dln); free(dout);
    free(dqkv); free(dh1); free(dp);
    return 0;
}

/* The causal attention of one [S, Dh] head set on its own (q, k, v of shape
 * [bh, S, Dh]), forward and, with dout, reverse: the head loop of
 * orc_block_step. */
void orc_attention_causal(const float *q, const float *k, const float *v, const float *dout,
                          int64_t bh, int64_t S, int64_t Dh, float scale, float *o, float *dq,
                          float *dk, float *dv) {
    float *p = falloc(S * S), *dp = falloc(S * S);
    for (int64_t h = 0; h < bh; ++h) {
        const int64_t off = h * S * Dh;
        attn_head_fwd(q + off, k + off, v + off, Dh, S, Dh, scale, p, o + off, Dh);
        if (!dout) continue;
        /* dq, dk, dv share one leading dimension (Dh) in this layout */
        sgemm_rows(p, 1, S, dout + off, Dh, 1, dv + off, Dh, Dh, S, 0, S);
        sgemm_rows(dout + off, Dh, 1, v + off, 1, Dh, dp, S, S, Dh, 0, S);
#pragma omp parallel
        {
            float *tmp = falloc(S);
#pragma omp for schedule(static)
            for (int64_t i = 0; i < S; ++i) {
                const float *pr = p + i * S;
                float *dr = dp + i * S;
                softmax_row_bwd(pr, dr, dr, tmp, S);
                for (int64_t j = 0; j < S; ++j) dr[j] = (j <= i) ? canon_f32(dr[j] * scale) : 0.0f;
            }
            free(tmp);
        }
        sgemm_rows(dp, S, 1, k + off, Dh, 1, dq + off, Dh, Dh, S, 0, S);
        sgemm_rows(dp, 1, S, q + off, Dh, 1, dk + off, Dh, Dh, S, 0, S);
    }
    free(p);
    free(dp);
}
