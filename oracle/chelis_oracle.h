/*
 * chelis_oracle.h -- CPU restatement of the Chelis C backend's numeric
 * semantics for the tensor-DAG hot path (matmul, sum/max reductions, layer
 * norm, softmax, keyed dropout, cumsum, cross-entropy and their adjoints).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * backend.  Only the test suite, __graft_entry__.smoke() and the cpu_baseline
 * leg of bench.py may load it.  The product library (libchelis_cuda.so)
 * never links or calls it.
 *
 * Every function cites the reference file:line whose behaviour it restates.
 * Floating point follows the C lane's build: -O2 -ffp-contract=off
 * -fno-fast-math (crates/chelis-backend-c/src/toolchain.rs:235-246), so
 * every addition and multiplication is a separately rounded IEEE operation.
 * Transcendentals come from the reference's vendored CORE-MATH
 * (crates/chelis-crmath/csrc/crmath_ffi.c:15-45), built by oracle/Makefile
 * into oracle/_ref/.
 */
#ifndef CHELIS_ORACLE_H
#define CHELIS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- keyed randomness: crates/chelis-numeric-core/src/dtype_semantics.rs:4508-4540 ---- */
uint64_t orc_splitmix64(uint64_t v);
uint64_t orc_word(uint64_t key, uint64_t index);
uint64_t orc_derive(uint64_t key, uint64_t j);
double orc_unit(uint64_t key, uint64_t index);

/* ---- canonical adjacent-pair tree: spec/05-risc-primitives.md:515-531 ---- */
float orc_tree_sum_f32(const float *x, int64_t n, int64_t stride);
double orc_tree_sum_f64(const double *x, int64_t n, int64_t stride);
/* sum over axis 1 of a [rows, cols] row-major tensor -> out[rows] */
void orc_row_sum_f32(const float *x, int64_t rows, int64_t cols, float *out);
/* sum over axis 0 of a [rows, cols] row-major tensor -> out[cols] */
void orc_col_sum_f32(const float *x, int64_t rows, int64_t cols, float *out);
void orc_row_max_f32(const float *x, int64_t rows, int64_t cols, float *out);
int64_t orc_count_bool(const uint8_t *x, int64_t n);

/* ---- matmul = Sum(Mul(Expand A, Expand B)) over k, tree in increasing k:
 *      crates/chelis-backend-c/src/emit.rs:8431-8640 ---- */
void orc_sgemm(const float *a, const float *b, float *c, int64_t m, int64_t n, int64_t k,
               int64_t row_begin, int64_t row_end);
void orc_dgemm(const double *a, const double *b, double *c, int64_t m, int64_t n, int64_t k,
               int64_t row_begin, int64_t row_end);
/* general strides: C[i,j] = tree_k A[i*sa0 + k*sa1] * B[k*sb0 + j*sb1] */
void orc_sgemm_strided(const float *a, int64_t sa0, int64_t sa1, const float *b, int64_t sb0,
                       int64_t sb1, float *c, int64_t m, int64_t n, int64_t k);
void orc_dgemm_strided(const double *a, int64_t sa0, int64_t sa1, const double *b, int64_t sb0,
                       int64_t sb1, double *c, int64_t m, int64_t n, int64_t k);

/* ---- dropout: PreparedDropout::apply, dtype_semantics.rs:4256-4280 ---- */
void orc_dropout_f32(const float *x, float *y, int64_t n, uint64_t key, float rate,
                     int64_t index_base);
void orc_dropout_mask(uint8_t *keep, int64_t n, uint64_t key, float rate, int64_t index_base);

/* ---- row ops (tier2.rs:1079-1375, spec/05-risc-primitives.md:5021-5093) ---- */
void orc_layer_norm_f32(const float *x, const float *gamma, const float *beta, float eps,
                        float *y, int64_t rows, int64_t hidden);
void orc_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t cols);
void orc_softmax_rows_bwd_f32(const float *y, const float *g, float *dx, int64_t rows,
                              int64_t cols);

/* ---- the fused chain: layer_norm -> softmax -> dropout -> row sum (forward),
 *      and its reverse-mode adjoint for loss = sum of the row sums ---- */
void orc_chain_fwd(const float *x, const float *gamma, const float *beta, float eps,
                   uint64_t key, float rate, int64_t rows, int64_t hidden, int64_t index_base,
                   float *rowsum);
void orc_chain_bwd(const float *x, const float *gamma, const float *beta, float eps,
                   uint64_t key, float rate, int64_t rows, int64_t hidden, int64_t index_base,
                   float *dx, float *dgamma_rows, float *dbeta_rows);

/* ---- cumsum: spec/05-risc-primitives.md:4310-4325 ---- */
void orc_cumsum_f64(const double *x, double *y, int64_t lanes, int64_t len, int reverse);
void orc_cumsum_f32(const float *x, float *y, int64_t lanes, int64_t len, int reverse);

/* ---- vmap'd covariance / risk (f64) ---- */
void orc_portfolio(const double *r, const double *w, int64_t count, int64_t t, int64_t a,
                   double *sigma, double *risk, double *cum);

/* ---- 2-layer MLP forward + adjoint ---- */
void orc_mlp_step(const float *x, const int64_t *labels, const float *w1, const float *b1,
                  const float *w2, const float *b2, int64_t batch, int64_t din, int64_t dh,
                  int64_t dout, float *loss, float *dw1, float *db1, float *dw2, float *db2);

/* ---- single finalized f32 operations ([04-NUM-2]) ---- */
float orc_add_f32(float a, float b);
float orc_mul_f32(float a, float b);
float orc_div_f32(float a, float b);
float orc_sqrt_f32(float a);

/* ---- CORE-MATH passthroughs for pinning against the reference fixtures ---- */
float orc_expf(float x);
float orc_logf(float x);
int64_t orc_crmath_check_f32(int32_t op, uint32_t start, int64_t n, const float *got,
                             int64_t *first_bad);
float orc_erfcf(float x);
double orc_exp(double x);
double orc_sqrt(double x);


/* ---- FusedElem groups (emit.rs:6744-6905, 9580-9860) ----
 * steps: n_steps triplets (op, a, b), op the FusedStepOp index
 * (dag.rs:494-526), operand >= 0 an input, < 0 step -1 - operand.
 * Input k is read at sum(coord[d] * strides[k * rank + d]).  Reduce kind
 * 0 = Sum, 1 = Max; its output is dense over shape without `axis`. */
void orc_fused_elementwise_f32(const int32_t *steps, int32_t n_steps, const float *const *in,
                               const int64_t *strides, int32_t n_in, const int64_t *shape,
                               int32_t rank, float *out);
void orc_fused_elementwise_f64(const int32_t *steps, int32_t n_steps, const double *const *in,
                               const int64_t *strides, int32_t n_in, const int64_t *shape,
                               int32_t rank, double *out);
void orc_fused_reduce_f32(const int32_t *steps, int32_t n_steps, const float *const *in,
                          const int64_t *strides, int32_t n_in, const int64_t *shape, int32_t rank,
                          int32_t axis, int32_t kind, float *out);
void orc_fused_reduce_f64(const int32_t *steps, int32_t n_steps, const double *const *in,
                          const int64_t *strides, int32_t n_in, const int64_t *shape, int32_t rank,
                          int32_t axis, int32_t kind, double *out);


/* ---- activations, layer_norm adjoint, cross-entropy ---- */
void orc_relu_f32(const float *x, float *y, int64_t n);
void orc_relu_f64(const double *x, double *y, int64_t n);
void orc_relu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n);
void orc_relu_adjoint_f64(const double *x, const double *g, double *dx, int64_t n);
void orc_gelu_f32(const float *x, float *y, int64_t n);
void orc_layer_norm_bwd_f32(const float *x, const float *gamma, float eps, const float *dy,
                            int64_t rows, int64_t hidden, float *dx, float *dgamma, float *dbeta);
int orc_cross_entropy_f32(const float *z, const int64_t *labels, int64_t rows, int64_t classes,
                          float *loss, float *dz);

/* ---- GELU adjoint: reverse mode through the Phi graph (grad.rs rules) ---- */
void orc_gelu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n);

/* ---- transformer block (config 4): pre-LN, causal attention (spec/05-risc-
 * primitives.md:5146-5181), GELU MLP; forward and, when dy is non-NULL, the
 * vector-Jacobian product.  x, dy, y, dx are [batch, S, D]; w_qkv [D, 3D],
 * w_o [D, D], w_1 [D, F], w_2 [F, D]; returns 1 on a shape it does not admit. */
int orc_block_step(const float *x, const float *dy, int64_t batch, int64_t S, int64_t D,
                   int64_t H, int64_t F, float eps, const float *w_qkv, const float *w_o,
                   const float *w_1, const float *w_2, const float *g1, const float *b1,
                   const float *g2, const float *b2, float *y, float *dx, float *dw_qkv,
                   float *dw_o, float *dw_1, float *dw_2, float *dg1, float *db1, float *dg2,
                   float *db2);
/* causal attention per head, q/k/v/o [bh, S, Dh]; reverse when dout != NULL */
void orc_attention_causal(const float *q, const float *k, const float *v, const float *dout,
                          int64_t bh, int64_t S, int64_t Dh, float scale, float *o, float *dq,
                          float *dk, float *dv);

#ifdef __cplusplus
}
#endif
#endif
