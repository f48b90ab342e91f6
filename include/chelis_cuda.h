/*
 * chelis_cuda.h -- C ABI of the B200-native (sm_100a) CUDA backend for Chelis.
 *
 * This library fills the slot of the reference's GPU lane
 * (crates/chelis-backend-hip).  Its entry points are the ones generated Chelis
 * code and a future `chelis-backend-cuda` crate bind through `extern "C"`:
 * plain pointers, sizes and the `chelis_gpu_tensor` descriptor, no C++ or
 * torch types.  Each declaration names the reference interface it replaces
 * (file:line within the reference project).
 *
 * Conventions
 *  - Every function returning `int` returns CHELIS_CUDA_OK (0) on success or
 *    a CHELIS_CUDA_ERR_* code; `chelis_cuda_last_error()` then holds a
 *    message for the calling thread.  The reference aborts instead
 *    (crates/chelis-backend-hip/runtime/chelis_hip_runtime.h:20-44); the
 *    messages keep the reference's "numeric trap: <kind> in <op> at <dtype>"
 *    wording where one applies.
 *  - Work is enqueued on the calling thread's stream (chelis_cuda_set_stream;
 *    default: the legacy default stream) of the current device.  Pointers
 *    are device pointers unless a parameter name says `host`.
 *  - Row-major layouts throughout, as in the reference's GEMM helpers.
 */
#ifndef CHELIS_CUDA_H
#define CHELIS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtype ids: crates/chelis-runtime/include/chelis_runtime_dtype.h:6-18 ---- */
#ifndef CHELIS_RUNTIME_DTYPE_H
typedef uint8_t chelis_dtype;
enum {
    CHELIS_DTYPE_F32 = 0,
    CHELIS_DTYPE_F64 = 1,
    CHELIS_DTYPE_I32 = 2,
    CHELIS_DTYPE_BOOL = 3,
    CHELIS_DTYPE_I64 = 4,
    CHELIS_DTYPE_BF16 = 5,
    CHELIS_DTYPE_F16 = 6,
    CHELIS_DTYPE_I8 = 7,
    CHELIS_DTYPE_I16 = 8,
    CHELIS_DTYPE_KEY = 9
};
#endif

/* ---- device descriptor: crates/chelis-backend-hip/runtime/chelis_device_descriptor.h:8-18 ---- */
#ifndef CHELIS_DEVICE_DESCRIPTOR_H
typedef int64_t chelis_device_metadata;
typedef int32_t chelis_device_rank;
typedef struct {
    void *data;
    const int64_t *shape;
    const int64_t *strides; /* in elements */
    int64_t count;
    int64_t byte_capacity;
    int32_t rank;
    chelis_dtype dtype;
    uint8_t ownership; /* 0 = borrowed, 1 = owned */
    uint8_t reserved[2];
} chelis_gpu_tensor;
#endif

/* ---- status codes ---- */
enum {
    CHELIS_CUDA_OK = 0,
    CHELIS_CUDA_ERR_DOMAIN = 1,      /* "numeric trap: domain ..." */
    CHELIS_CUDA_ERR_OVERFLOW = 2,    /* "numeric trap: overflow ..." */
    CHELIS_CUDA_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
    CHELIS_CUDA_ERR_UNSUPPORTED = 4, /* shape/dtype/layout this build does not admit */
    CHELIS_CUDA_ERR_TIMEOUT = 5,     /* a bounded device wait gave up */
    CHELIS_CUDA_ERR_NO_DEVICE = 6,
    CHELIS_CUDA_ERR_FAIL = 7         /* a program's own abort fired (GuardedFail): its message */
};

/* GEMM arithmetic for f32 (matmul lowering, spec/05-risc-primitives.md:4962-5000). */
enum {
    CHELIS_CUDA_GEMM_3XTF32 = 0,   /* tcgen05 tensor cores, split-accumulate (default) */
    CHELIS_CUDA_GEMM_EXACT_TREE = 1 /* CUDA cores, canonical tree over k: bit-identical to the C lane */
};
/* Fused row kernels: EXACT follows the C lane op for op (IEEE div/sqrt, no
 * contraction, canonical trees); FAST rewrites divisions as reciprocal
 * multiplies (tolerance parity only). */
enum { CHELIS_CUDA_ROWS_EXACT = 0, CHELIS_CUDA_ROWS_FAST = 1 };
/* f64 GEMM kernel when the GEMM mode is not EXACT_TREE: the FP64 tensor
 * path (DMMA) or the CUDA cores' FP64 FMA pipe (FFMA, half DMMA's peak on
 * B200).  AUTO (default) picks per product: DMMA when its 128 x 128 tiles
 * number at least the SM count, FFMA (64 x 64 tiles, four times the CTAs)
 * for smaller products. */
enum { CHELIS_CUDA_DGEMM_AUTO = 0, CHELIS_CUDA_DGEMM_DMMA = 1, CHELIS_CUDA_DGEMM_FFMA = 2 };

/* =========================================================================
 * Runtime
 * replaces the per-call hiprtc compile + launch helpers
 * (crates/chelis-backend-hip/runtime/chelis_hip_runtime.h:409-485): kernels
 * are compiled ahead of time for sm_100a, except the per-chain FusedElem
 * kernels, which NVRTC compiles once per chain and device and caches.
 * ========================================================================= */
int chelis_cuda_version(void);
const char *chelis_cuda_last_error(void);
/* Select and initialise a device (the reference always uses hipGetDevice's
 * current device: chelis_device_owner.cpp current_device()). */
int chelis_cuda_init(int32_t device);
/* Per-thread stream used by every later call on this thread (NULL = legacy default). */
int chelis_cuda_set_stream(void *cuda_stream);
void *chelis_cuda_get_stream(void);
int chelis_cuda_synchronize(void);
/* Read-and-clear the device error word: CHELIS_CUDA_ERR_TIMEOUT if a bounded
 * device wait gave up; CHELIS_CUDA_ERR_FAIL with the message of a DAG's
 * GuardedFail that fired; CHELIS_CUDA_ERR_DOMAIN / _OVERFLOW for a numeric
 * trap raised on the device (an index operand out of range ([05-OP-52]), a
 * dropout rate outside [0, 1), integer overflow or division by zero, a
 * checked cast), with the reference's "numeric trap: <kind> in <op> at
 * <dtype>" message; since the last call.
 * Synchronises the stream.  Replaces the debug failure flag readback of
 * chelis_hip_runtime.h:487-524. */
int chelis_cuda_device_status(void);
/* Number of kernels this library launched since process start (all threads). */
uint64_t chelis_cuda_launch_count(void);
/* Probes every bounded device wait makes before it gives up and reports
 * CHELIS_CUDA_ERR_TIMEOUT (about 1 us each; 0 restores the default of
 * 2^22, a few seconds).  Device-wide for this process; for tests of the
 * timeout path.  No counterpart in the reference (its waits are unbounded). */
int chelis_cuda_set_wait_limit(uint32_t tries);
uint32_t chelis_cuda_get_wait_limit(void);
/* Self-test of the bounded wait: one CTA whose consumer thread waits on an
 * mbarrier for a producer thread's arrival; skip_arrival != 0 tells the
 * producer not to arrive, so the wait runs out after the wait limit and the
 * next chelis_cuda_device_status returns CHELIS_CUDA_ERR_TIMEOUT.  The
 * kernel always returns. */
int chelis_cuda_selftest_bounded_wait(int skip_arrival);
/* Process-wide default modes (a thread's own setting, below, wins). */
int chelis_cuda_set_gemm_mode(int mode);
int chelis_cuda_get_gemm_mode(void);
int chelis_cuda_set_rows_mode(int mode);
int chelis_cuda_get_rows_mode(void);
int chelis_cuda_set_dgemm_kernel(int kernel); /* CHELIS_CUDA_DGEMM_* */
int chelis_cuda_get_dgemm_kernel(void);
/* The calling thread's modes (GEMM, rows, f64 kernel; -1 = follow the
 * process default), so that threads choose exact or fast arithmetic
 * independently; every entry point on this thread uses them.  _get reports
 * the modes in force on this thread. */
int chelis_cuda_set_thread_modes(int gemm_mode, int rows_mode, int dgemm_kernel);
int chelis_cuda_get_thread_modes(int *gemm_mode, int *rows_mode, int *dgemm_kernel);
/* The f64 kernel AUTO picks for a product of this shape
 * (CHELIS_CUDA_DGEMM_DMMA or _FFMA). */
int chelis_cuda_dgemm_kernel_for(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                                 int64_t batch);
/* Release what the library created by itself: the scratch memory pools,
 * the compiled FusedElem kernels, the host-GEMM copy streams, event pools
 * and the data-parallel communicator (as chelis_cuda_dp_finalize(0)).  The
 * next call re-creates what it needs.  No other call may run concurrently.
 * The static scratch array of chelis_cuda_chain_bwd_noalloc belongs to the
 * loaded library and stays until exit.  Returns the first failure. */
int chelis_cuda_shutdown(void);

/* =========================================================================
 * Device tensor owner
 * crates/chelis-backend-hip/runtime/chelis_device_owner.h:16-24
 * ========================================================================= */
typedef struct chelis_device_tensor_owner chelis_device_tensor_owner;
/* chelis_device_tensor_alloc(plan) (owner.h:16): the metadata plan is a Rust
 * runtime object; this entry takes its dtype/rank/shape directly.  Owned,
 * zero-filled, canonical row-major strides. */
chelis_device_tensor_owner *chelis_device_tensor_alloc_shape(chelis_dtype dtype, int32_t rank,
                                                             const int64_t *shape);
/* chelis_device_tensor_borrow(plan, data, capacity) (owner.h:17). */
chelis_device_tensor_owner *chelis_device_tensor_borrow_shape(chelis_dtype dtype, int32_t rank,
                                                              const int64_t *shape, void *data,
                                                              int64_t byte_capacity);
/* owner.h:18 -- borrow a foreign packet (ownership must be 0). */
chelis_device_tensor_owner *chelis_device_tensor_import(const chelis_gpu_tensor *packet);
/* owner.h:19 */
const chelis_gpu_tensor *chelis_device_tensor_view(const chelis_device_tensor_owner *owner);
/* owner.h:20 */
int32_t chelis_device_tensor_device(const chelis_device_tensor_owner *owner);
/* owner.h:21 -- canonical-stride copy; strided sources gather in one kernel
 * (the reference issues one hipMemcpy per element: owner.cpp:224-237). */
chelis_device_tensor_owner *chelis_device_tensor_clone(const chelis_device_tensor_owner *source);
/* owner.h:22 */
void chelis_device_tensor_release(chelis_device_tensor_owner *owner);
/* owner.h:23-24 (chelis_tensor is a Rust host object; these take bytes). */
int chelis_device_tensor_copy_from_host_bytes(chelis_device_tensor_owner *destination,
                                              const void *host, int64_t bytes);
int chelis_device_tensor_copy_to_host_bytes(void *host, int64_t bytes,
                                            const chelis_device_tensor_owner *source);

/* =========================================================================
 * GEMM helper ABI
 * crates/chelis-backend-hip/runtime/chelis_hip_runtime.h:48-404
 * (chelis_hipblas_*_row_major), dispatched from emit.rs:4718-4842.
 * C = A.B, row-major, contiguous matrix slices (the reference's
 * chelis_gpu_matrix_slices_contiguous precondition, :80-87); count == 0 is a
 * no-op (emit.rs:4806).
 * ========================================================================= */
/* chelis_hipblas_sgemm_row_major (:48-78) */
int chelis_cuda_sgemm_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k);
/* chelis_hipblas_dgemm_row_major (:271-300) */
int chelis_cuda_dgemm_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k);
/* chelis_hipblas_sgemm_batched_row_major (:167-220): leading axes are the batch */
int chelis_cuda_sgemm_batched_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                        const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                        int64_t k, int64_t batch_count);
/* chelis_hipblas_sgemm_strided_batched_row_major (:222-267) */
int chelis_cuda_sgemm_strided_batched_row_major(const chelis_gpu_tensor *a,
                                                const chelis_gpu_tensor *b,
                                                const chelis_gpu_tensor *out, int64_t m,
                                                int64_t n, int64_t k, int64_t batch_count,
                                                int64_t a_batch_stride, int64_t b_batch_stride,
                                                int64_t out_batch_stride);
/* chelis_hipblas_dgemm_batched_row_major (:302-355) */
int chelis_cuda_dgemm_batched_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                        const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                        int64_t k, int64_t batch_count);
/* chelis_hipblas_dgemm_strided_batched_row_major (:357-404) */
int chelis_cuda_dgemm_strided_batched_row_major(const chelis_gpu_tensor *a,
                                                const chelis_gpu_tensor *b,
                                                const chelis_gpu_tensor *out, int64_t m,
                                                int64_t n, int64_t k, int64_t batch_count,
                                                int64_t a_batch_stride, int64_t b_batch_stride,
                                                int64_t out_batch_stride);

/* chelis_hipblas_bf16_gemm_f32_acc_row_major / _f16_ (chelis_hip_runtime.h:92-165):
 * A, B and out in bf16 (f16), products and sums in f32, out rounded to the
 * storage type once (nearest-even).  Same contiguity precondition and
 * count == 0 no-op as the f32 helpers. */
int chelis_cuda_bf16_gemm_f32_acc_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                            const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                            int64_t k);
int chelis_cuda_f16_gemm_f32_acc_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                           const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                           int64_t k);
/* Raw-pointer form for 16-bit storage (dtype CHELIS_DTYPE_BF16 or _F16):
 * the same arguments as chelis_cuda_sgemm. */
int chelis_cuda_gemm16(int32_t dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                       const void *a, int64_t lda, int64_t stride_a, const void *b, int64_t ldb,
                       int64_t stride_b, void *c, int64_t ldc, int64_t stride_c, int64_t batch);

/* Raw-pointer GEMM used by the helpers above and by the AD programs:
 * C[b] = op(A[b]) . op(B[b]) for b < batch, op = transpose when trans_* != 0.
 * Leading dimensions are row strides in elements.  The matmul adjoint of
 * [05-OP-51] (spec/05-risc-primitives.md:4247-4250) is this call with a
 * transposed operand.  Mode CHELIS_CUDA_GEMM_3XTF32 keeps split operand
 * copies in stream-ordered scratch for the duration of the call. */
int chelis_cuda_sgemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const float *a,
                      int64_t lda, int64_t stride_a, const float *b, int64_t ldb,
                      int64_t stride_b, float *c, int64_t ldc, int64_t stride_c, int64_t batch);
int chelis_cuda_dgemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const double *a,
                      int64_t lda, int64_t stride_a, const double *b, int64_t ldb,
                      int64_t stride_b, double *c, int64_t ldc, int64_t stride_c, int64_t batch);
/* The same products with the arithmetic chosen for this call only
 * (CHELIS_CUDA_GEMM_* and, for f64, CHELIS_CUDA_DGEMM_*); the thread's and
 * the process's settings are left as they were. */
int chelis_cuda_sgemm_ex(int gemm_mode, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                         const float *a, int64_t lda, int64_t stride_a, const float *b,
                         int64_t ldb, int64_t stride_b, float *c, int64_t ldc, int64_t stride_c,
                         int64_t batch);
int chelis_cuda_dgemm_ex(int gemm_mode, int dgemm_kernel, int trans_a, int trans_b, int64_t m,
                         int64_t n, int64_t k, const double *a, int64_t lda, int64_t stride_a,
                         const double *b, int64_t ldb, int64_t stride_b, double *c, int64_t ldc,
                         int64_t stride_c, int64_t batch);
/* Tile shape of the 3xTF32 main kernel: 1 (default) = 256 x 256 tiles on
 * CTA pairs (tcgen05 cta_group::2) for products with more than 128 rows,
 * 0 = 128 x 256 tiles on single CTAs.  Results are identical in both modes
 * up to the f32 accumulation order inside the tensor core.  Process-wide. */
int chelis_cuda_set_gemm_pairs(int enable);
int chelis_cuda_get_gemm_pairs(void);
/* [05-OP-30] matmul on HOST buffers (row-major, same argument meaning as
 * chelis_cuda_sgemm / chelis_cuda_dgemm, all pointers host pointers).  The
 * reference uploads both operands, runs hipBLAS and downloads C in sequence
 * (chelis_hip_runtime.h:48-78 plus its buffer copies); here the uploads of A
 * panels, the GEMM of earlier panels and the read-back of finished panels
 * overlap on three streams.  Stream-ordered on the thread's stream: C is
 * complete once that stream is synchronised.  Page-locked host memory lets
 * the copies run asynchronously. */
int chelis_cuda_sgemm_host(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                           const float *a, int64_t lda, int64_t stride_a, const float *b,
                           int64_t ldb, int64_t stride_b, float *c, int64_t ldc,
                           int64_t stride_c, int64_t batch);
int chelis_cuda_dgemm_host(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                           const double *a, int64_t lda, int64_t stride_a, const double *b,
                           int64_t ldb, int64_t stride_b, double *c, int64_t ldc,
                           int64_t stride_c, int64_t batch);
/* 3xTF32 in two halves, for operands reused across many products (weights).
 * chelis_cuda_tf32x3_split splits op(X) (rows x k, op = transpose when
 * trans != 0, element (r, kk) at src[r*ld + kk], or src[kk*ld + r] when
 * transposed) into hi/lo copies in one of two layouts:
 *   layout 0 (K-major):  [batch][rows][kp], kp = k rounded up to 32;
 *   layout 1 (MN-major): [batch][k][rp],    rp = rows rounded up to 4
 *                        (needs trans != 0: the source is already [k][rows]).
 * Padding is zero.  chelis_cuda_sgemm_tf32x3_presplit then computes
 * C[b] = A[b] . B[b]^T for pre-split A (m x k) and B (n x k) in the layouts
 * named by a_layout / b_layout; a row-major right operand B (k x n) is split
 * with trans = 1, layout = 1.  No reference counterpart: hipBLAS has no split
 * form (chelis_hip_runtime.h:48-78 is the single-call slot). */
int chelis_cuda_tf32x3_split(int trans, int layout, int64_t rows, int64_t k, const float *src,
                             int64_t ld, int64_t stride, int64_t batch, float *hi, float *lo);
int chelis_cuda_sgemm_tf32x3_presplit(int64_t m, int64_t n, int64_t k, int64_t batch,
                                      int a_layout, const float *a_hi, const float *a_lo,
                                      int b_layout, const float *b_hi, const float *b_lo,
                                      float *c, int64_t ldc, int64_t stride_c);

/* [05-OP-30..33] causal softmax attention per head, the block's attention
 * step (spec 05 section 4.7): o = softmax(where(causal, (q.k^T)*scale,
 * -inf)) . v for bh independent heads, q, k, v, o f32 [bh][seq][dh]
 * contiguous, lse [bh][seq] (optional, may be NULL) = max + log(sum) of each
 * row's scaled scores.  The reference materialises the [seq, seq] scores
 * (tier2.rs attention lowering); this keeps them in tensor memory.  Head dims
 * 32 and 64 (else CHELIS_CUDA_ERR_UNSUPPORTED). */
int chelis_cuda_attention_causal_fwd(int64_t bh, int64_t seq, int64_t dh, float scale,
                                     const float *q, const float *k, const float *v, float *o,
                                     float *lse);
/* Reverse mode of the same: given o and lse from the forward and the
 * cotangent dout ([bh][seq][dh]), dq, dk, dv ([bh][seq][dh]).  The reference
 * differentiates the materialised graph (grad.rs softmax / matmul adjoints);
 * this recomputes the scores blockwise from lse (no [seq, seq] tensor). */
int chelis_cuda_attention_causal_bwd(int64_t bh, int64_t seq, int64_t dh, float scale,
                                     const float *q, const float *k, const float *v,
                                     const float *o, const float *lse, const float *dout,
                                     float *dq, float *dk, float *dv);

/* =========================================================================
 * Fused elementwise / reduction groups and their adjoints.
 * The reference JIT-compiles per-DAG kernel strings (kernels.rs:2175-2468,
 * fused_elementwise / reduce_fused; row reductions :1703-2014) and rejects
 * Softmax, sqrt and Dropout on HIP (emit.rs:1572-1583, 2763-2775).
 * ========================================================================= */
/* A FusedElem group (dag.rs:1323-1325): a chain of steps, each one
 * FusedStepOp (dag.rs:494-526, same order and numbering) over operands that
 * are FusedInputs (dag.rs:673-678): a >= 0 is External(a), an input; a < 0
 * is PreviousStep(-1 - a), an earlier step.  Unary steps ignore b.  The
 * group's value is its last step. */
typedef enum {
    CHELIS_FUSED_ADD = 0,
    CHELIS_FUSED_SUB = 1,
    CHELIS_FUSED_MUL = 2,
    CHELIS_FUSED_DIV = 3,
    CHELIS_FUSED_POW = 4,
    CHELIS_FUSED_FLOOR_DIV = 5,
    CHELIS_FUSED_TRUNC_DIV = 6, /* integer-only: rejected on a float chain */
    CHELIS_FUSED_MAX_ELEM = 7,
    CHELIS_FUSED_MIN_ELEM = 8,
    CHELIS_FUSED_NEG = 9,
    CHELIS_FUSED_RECIP = 10,
    CHELIS_FUSED_EXP = 11,
    CHELIS_FUSED_LOG = 12,
    CHELIS_FUSED_SIN = 13,
    CHELIS_FUSED_SQRT = 14,
    CHELIS_FUSED_COS = 15,
    CHELIS_FUSED_TAN = 16,
    CHELIS_FUSED_ATAN = 17,
    CHELIS_FUSED_TANH = 18,
    CHELIS_FUSED_ERF = 19,
    CHELIS_FUSED_ERFC = 20,
    CHELIS_FUSED_ABS = 21,
    CHELIS_FUSED_FLOOR = 22,
    CHELIS_FUSED_CEIL = 23,
    CHELIS_FUSED_ROUND = 24
} chelis_fused_op;
typedef struct {
    int32_t op; /* chelis_fused_op */
    int32_t a, b;
} chelis_fused_step;
typedef enum { CHELIS_FUSED_REDUCE_SUM = 0, CHELIS_FUSED_REDUCE_MAX = 1 } chelis_fused_reduce_kind;
/* Evaluate the group over `shape` (rank <= 6) into the dense `out`.  Input k
 * is read at sum(coord[d] * strides[k * rank + d]) elements: stride 0 on a
 * dimension broadcasts it (the HIP lane's per-input strides, kernels.rs
 * fused_elementwise :2391-2468; the C lane's full-or-scalar inputs,
 * emit.rs:6984-7100, are the strides 1..., and 0...).  dtype F32 or F64;
 * <= 32 steps, <= 8 inputs.  Step results follow the C lane
 * (emit.rs:6744-6905 with fp_env.rs:213-241): canonical NaN after every step
 * but MaxElem / MinElem; transcendentals within a few ulp of its correctly
 * rounded CORE-MATH calls. */
int chelis_cuda_fused_elementwise(int32_t dtype, const chelis_fused_step *steps, int32_t n_steps,
                                  const void *const *inputs, const int64_t *strides,
                                  int32_t n_inputs, const int64_t *shape, int32_t rank, void *out);
/* Compiled chains for chelis_cuda_fused_elementwise: 1 (default) = a group
 * whose innermost extent is a whole number of 16-byte vectors, and whose
 * inputs are unit-stride (16-byte aligned) or broadcast along that axis, runs
 * as one kernel generated for its chain.  That kernel is compiled at run time
 * with NVRTC for sm_100a and cached per device and chain, the counterpart of
 * the HIP lane's per-chain kernel strings compiled with hiprtc
 * (kernels.rs:2391, chelis_hip_runtime.h:409-453).  Other groups, and every
 * group when NVRTC is absent, use the ahead-of-time interpreter.  0 = always
 * the interpreter.  Both give the same bits.  Process-wide.
 * chelis_cuda_fused_jit_launches counts the compiled-chain launches so far. */
int chelis_cuda_set_fused_jit(int enable);
int chelis_cuda_get_fused_jit(void);
int64_t chelis_cuda_fused_jit_launches(void);
/* The group reduced along `axis` of `shape` (emit_fused_reduce,
 * emit.rs:9580-9860; reduce_fused kernels.rs:2175-2390): Sum by the
 * canonical pair tree, Max folding chelis_fmax_propnan_f32 from -inf.  `out`
 * is dense over shape without `axis`.  An empty Max axis is the Domain trap
 * "max_reduce"; an empty Sum axis writes zeros. */
int chelis_cuda_fused_reduce(int32_t dtype, const chelis_fused_step *steps, int32_t n_steps,
                             const void *const *inputs, const int64_t *strides, int32_t n_inputs,
                             const int64_t *shape, int32_t rank, int32_t axis, int32_t kind,
                             void *out);
/* Correctly rounded binary32 exp / log (round to nearest even), the results
 * of the C lane's CORE-MATH calls (crates/chelis-crmath, crmath_ffi.c:15-45)
 * bit for bit; NaN inputs give a quiet NaN.  The EXACT rows mode and the
 * fused groups use them.  _sweep evaluates op at the n consecutive bit
 * patterns start, start + 1, ... (wrapping at 2^32), for exhaustive checks. */
enum { CHELIS_CRMATH_EXP = 0, CHELIS_CRMATH_LOG = 1 };
int chelis_cuda_crmath_f32(int32_t op, const float *x, float *y, int64_t n);
int chelis_cuda_crmath_sweep_f32(int32_t op, uint32_t start, int64_t n, float *y);
/* [05-OP-30] sum over the last axis / first axis of a [rows, cols] f32 tensor,
 * canonical adjacent-pair tree (kernels.rs:1703-1755 left-folds instead). */
int chelis_cuda_row_sum_f32(const float *x, int64_t rows, int64_t cols, float *out);
int chelis_cuda_col_sum_f32(const float *x, int64_t rows, int64_t cols, float *out);
/* [05-OP-12] max_reduce over the last axis (first NaN wins). kernels.rs:1802 */
int chelis_cuda_row_max_f32(const float *x, int64_t rows, int64_t cols, float *out);
/* [05-OP-29] exact i64 count of a bool tensor (kernels.rs:375-520). */
int chelis_cuda_count_bool(const uint8_t *x, int64_t n, int64_t *out_device);
/* [05-OP-37] keyed dropout / DropoutReplay on a flat f32 tensor whose first
 * element has flat index `index_base` (dtype_semantics.rs:4256-4280). */
int chelis_cuda_dropout_f32(const float *x, float *y, int64_t n, uint64_t key, float rate,
                            int64_t index_base);
/* Keep mask (1 = kept) of the same draw; bit-exact with the C lane. */
int chelis_cuda_dropout_mask(uint8_t *keep, int64_t n, uint64_t key, float rate,
                             int64_t index_base);
/* layer_norm over the last axis (tier2.rs:1248-1375). */
int chelis_cuda_layer_norm_f32(const float *x, const float *gamma, const float *beta, float eps,
                               float *y, int64_t rows, int64_t hidden);
/* softmax over the last axis (tier2.rs:1079-1180) and its adjoint
 * y * (g - sum(g * y)) (grad.rs:2248-2280). */
int chelis_cuda_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t cols);
int chelis_cuda_softmax_rows_bwd_f32(const float *y, const float *g, float *dx, int64_t rows,
                                     int64_t cols);
/* [05-OP-43] relu = max_elem(x, +0) (a NaN keeps its bits, -0 stays -0) and
 * ReluAdjoint: g's bits where 0 < x, exact +0 elsewhere (dag.rs:957,965,
 * grad.rs:2281-2294).  f32 or f64, n elements, bit-exact. */
int chelis_cuda_relu(int32_t dtype, const void *x, void *y, int64_t n);
int chelis_cuda_relu_adjoint(int32_t dtype, const void *x, const void *g, void *dx, int64_t n);
/* gelu = m(x) * Phi(x), Phi the compensated standard normal CDF graph of
 * spec 05 section 3.3 (tier2.rs lower_gelu), and its adjoint
 * dx = g * (Phi(x) + x * phi(x)).  f32; CUDA erfc / exp stand in for
 * CORE-MATH's. */
int chelis_cuda_gelu_f32(const float *x, float *y, int64_t n);
int chelis_cuda_gelu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n);
/* Adjoint of y = layer_norm(x, gamma, beta, eps) over the last axis
 * (tier2.rs:1248-1375 through grad.rs): dx [rows, hidden] and the complete
 * dgamma, dbeta [hidden] from dy.  hidden <= 8192. */
int chelis_cuda_layer_norm_bwd_f32(const float *x, const float *gamma, float eps, const float *dy,
                                   int64_t rows, int64_t hidden, float *dx, float *dgamma,
                                   float *dbeta);
/* Cross-entropy of spec 05 section 4.3: loss = mean_r(-log softmax(z_r)[label_r])
 * written to the device scalar *loss; with dlogits non-NULL also d loss / d z
 * (the AD graph through mean, neg, gather, log and softmax).  labels int64 in
 * [0, classes): another value is the gather's Domain trap, reported by
 * chelis_cuda_device_status. */
int chelis_cuda_cross_entropy_f32(const float *logits, const int64_t *labels, int64_t rows,
                                  int64_t classes, float *loss, float *dlogits);
/* The fused chain layer_norm -> softmax -> dropout -> row sum over a
 * [rows, hidden] f32 tensor.  `row_stats` (optional, 4 floats per row:
 * mean, sqrt(var+eps), softmax max, softmax denominator) is written for the
 * adjoint to reuse. */
int chelis_cuda_chain_fwd(const float *x, const float *gamma, const float *beta, float eps,
                          uint64_t key, float rate, int64_t rows, int64_t hidden,
                          int64_t index_base, float *rowsum, float *row_stats);
/* Adjoint of loss = sum(rowsum) w.r.t. x, gamma and beta.  With row_stats
 * NULL the forward statistics are recomputed.  dgamma/dbeta are complete
 * (reduced over all rows) on return. */
int chelis_cuda_chain_bwd(const float *x, const float *gamma, const float *beta, float eps,
                          uint64_t key, float rate, int64_t rows, int64_t hidden,
                          int64_t index_base, const float *row_stats, float *dx, float *dgamma,
                          float *dbeta);
/* The chain forward that also saves what its adjoint needs: per-row
 * statistics and the keyed-dropout keep bits (one bit per element), in a
 * 16-byte aligned device buffer of chelis_cuda_chain_saved_bytes(rows,
 * hidden) bytes.  chelis_cuda_chain_bwd_saved then runs the adjoint without
 * recomputing the RNG or any forward reduction.  PyTorch-style saved state;
 * the reference materialises forward intermediates instead (the C lane
 * keeps every DAG node's tensor). */
int64_t chelis_cuda_chain_saved_bytes(int64_t rows, int64_t hidden);
int chelis_cuda_chain_fwd_save(const float *x, const float *gamma, const float *beta, float eps,
                               uint64_t key, float rate, int64_t rows, int64_t hidden,
                               int64_t index_base, float *rowsum, void *saved);
int chelis_cuda_chain_bwd_saved(const float *x, const float *gamma, const float *beta, float eps,
                                float rate, int64_t rows, int64_t hidden, const void *saved,
                                float *dx, float *dgamma, float *dbeta);
/* chelis_cuda_chain_bwd for callers that cannot let the library allocate
 * device memory (a host that budgets its whole device arena up front and
 * hands out every buffer itself, or one that bans driver allocation while it
 * runs).  No counterpart in the reference.  Same arguments and results as
 * chelis_cuda_chain_bwd; its scratch is one 10 MiB device array per GPU,
 * held until the process exits.  Limits: hidden <= 4096 (larger rows return
 * CHELIS_CUDA_ERR_UNSUPPORTED).  Calls that overlap on the GPU share that
 * array and race; order them.  The first call on a device resolves the
 * array's address with that device current: make it before any stream
 * capture; a device reset invalidates that address (do not call it on a
 * device after resetting it).  The grid is two CTAs per SM, at most 296 (the
 * array's capacity): dx is bit for bit chelis_cuda_chain_bwd's on any GPU,
 * and on a 148-SM B200 so are dgamma / dbeta; on a GPU with more SMs they
 * group rows differently and agree within f32 rounding. */
int chelis_cuda_chain_bwd_noalloc(const float *x, const float *gamma, const float *beta,
                                  float eps, uint64_t key, float rate, int64_t rows,
                                  int64_t hidden, int64_t index_base, const float *row_stats,
                                  float *dx, float *dgamma, float *dbeta);
/* Cumsum ([05-OP-53], spec/05-risc-primitives.md:4310-4325) along the last
 * axis of [lanes, len]; reverse != 0 is the decreasing scan (the adjoint).
 * kernels.rs:2793-2895 */
int chelis_cuda_cumsum_f64(const double *x, double *y, int64_t lanes, int64_t len, int reverse);
int chelis_cuda_cumsum_f32(const float *x, float *y, int64_t lanes, int64_t len, int reverse);

/* =========================================================================
 * vmap'd programs (vectorize_axis0, crates/chelis-ir-core/src/vmap.rs:9-56)
 * ========================================================================= */
/* Covariance / risk per portfolio, f64: r [count, t, a], w [count, a] ->
 * sigma [count, a, a] = (R-mean)^T (R-mean) / (t-1), risk [count] =
 * sqrt(w^T sigma w), cum [count, t] = cumsum_t(R.w). */
int chelis_cuda_portfolio_f64(const double *r, const double *w, int64_t count, int64_t t,
                              int64_t a, double *sigma, double *risk, double *cum);

/* 2-layer MLP forward + adjoint (matmul, add, relu, softmax cross-entropy,
 * mean; grads w.r.t. w1, b1, w2, b2).  labels are i64 class ids.  The call
 * does not synchronise: a label outside [0, dout) is recorded on the device
 * and reported as CHELIS_CUDA_ERR_DOMAIN ("numeric trap: domain in gather")
 * by the next chelis_cuda_device_status(). */
int chelis_cuda_mlp_step(const float *x, const int64_t *labels, const float *w1,
                         const float *b1, const float *w2, const float *b2, int64_t batch,
                         int64_t din, int64_t dh, int64_t dout, float *loss, float *dw1,
                         float *db1, float *dw2, float *db2);

/* A pre-LN transformer block (the post-LN ReLU block of
 * examples/transformer_block.ch rearranged): causal multi-head softmax
 * attention (spec/05-risc-primitives.md:5146-5181), layer_norm
 * (:5065-5093) and a GELU MLP (gelu = m(x)*Phi(x), :1353-1400), forward and,
 * when dy != NULL, the vector-Jacobian product for upstream cotangent dy.
 * Row-major f32; w_qkv is [d_model, 3*d_model] with the q, k and v column
 * blocks in that order and heads contiguous inside each (head h owns
 * columns h*head_dim .. (h+1)*head_dim - 1 of a block); no biases.  The
 * attention scale is 1/sqrt(head_dim). */
typedef struct {
    int64_t batch, seq, d_model, heads, d_ff;
    float eps;
    const float *x, *dy;                 /* [batch, seq, d_model]; dy may be NULL */
    const float *w_qkv, *w_o, *w_1, *w_2;
    const float *ln1_gamma, *ln1_beta, *ln2_gamma, *ln2_beta;
    float *y, *dx;
    float *dw_qkv, *dw_o, *dw_1, *dw_2;
    float *dln1_gamma, *dln1_beta, *dln2_gamma, *dln2_beta;
} chelis_block_params;
/* Bytes of device workspace chelis_cuda_block_step needs (-1: shape not admitted). */
int64_t chelis_cuda_block_workspace_bytes(const chelis_block_params *p);
/* workspace: device memory of chelis_cuda_block_workspace_bytes bytes, or
 * NULL to take it from the library's stream-ordered pool for the call. */
int chelis_cuda_block_step(const chelis_block_params *p, void *workspace);
/* chelis_cuda_block_step for one rank of a data-parallel step: with a
 * communicator open (chelis_cuda_dp_init, more than one rank), each of the
 * eight parameter gradients is summed across the ranks as soon as the
 * reverse pass has written it, on the library's communication stream, while
 * the reverse pass goes on (dln*_gamma / dln*_beta in one reduction when
 * beta follows gamma in memory).  The call's stream waits for all of them
 * before later work, so on return (stream order) every d<weight> holds the
 * all-rank sum; x, y and dx stay this rank's.  With one rank, or dy == NULL,
 * it is chelis_cuda_block_step.  No counterpart in the reference (it has no
 * multi-GPU lane).  One host thread per device at a time. */
int chelis_cuda_block_step_dp(const chelis_block_params *p, void *workspace);
/* Phase timing of chelis_cuda_block_step (a diagnostic; no counterpart in the
 * reference).  enable != 0 creates CUDA events on the current device; every
 * later block step records them on its stream at its 16 phase boundaries
 * (layer norms, each matmul pair, attention forward and reverse, GELU).
 * chelis_cuda_block_phase_ms waits for the last step and writes each phase's
 * milliseconds (0 for phases that step did not run) into ms[0..15] (n >= 16).
 * Process-wide: use from one host thread at a time. */
int chelis_cuda_block_timing(int enable);
int chelis_cuda_block_phase_ms(float *ms, int32_t n);
const char *chelis_cuda_block_phase_name(int32_t i);

/* =========================================================================
 * Data parallel across the GPUs of one node (new: the reference has no
 * multi-GPU lane).  One process per GPU; NCCL is opened at run time
 * (libnccl.so.2), without it these return CHELIS_CUDA_ERR_UNSUPPORTED.
 * ========================================================================= */
/* Contiguous [start, stop) of n batch items for `rank`: shard sizes differ by
 * at most one and tile [0, n) in rank order (the vmap axis,
 * crates/chelis-ir-core/src/vmap.rs:9-56). */
int chelis_cuda_dp_shard(int64_t n, int32_t nranks, int32_t rank, int64_t *start, int64_t *stop);
/* 128 bytes identifying a new communicator; rank 0 makes it, every rank
 * passes the same bytes to chelis_cuda_dp_init. */
int chelis_cuda_dp_unique_id(uint8_t *id);
/* Join the communicator on the current device (every rank calls it). */
int chelis_cuda_dp_init(int32_t nranks, int32_t rank, const uint8_t *id);
/* In-place sum over ranks of count elements (f32, f64, i32, i64), enqueued
 * on the calling thread's stream: the gradient all-reduce of a data-parallel
 * step.  Every rank calls it in the same order. */
int chelis_cuda_dp_allreduce_sum(int32_t dtype, void *buf, int64_t count);
/* nranks / rank of the open communicator (1 / 0 without one). */
int chelis_cuda_dp_world(int32_t *nranks, int32_t *rank);
/* Close the communicator; abort != 0 abandons collectives in flight (a rank
 * that learned of a failed peer on the host). */
int chelis_cuda_dp_finalize(int32_t abort);

/* =========================================================================
 * Generated-entry device ABI (emit.rs:838-958, `f_device`): inputs borrowed,
 * outputs newly allocated owners the caller releases.  One entry per program
 * this backend ships whole.
 * ========================================================================= */
/* inputs: x[rows,hidden], gamma[hidden], beta[hidden]; outputs: rowsum[rows].
 * eps = 1e-5, key = 42, rate = 0.1 are the program's constants. */
int chelis_chain_fwd_device(const chelis_device_tensor_owner *const *inputs,
                            chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                            chelis_device_rank n_out);
/* inputs: x, gamma, beta; outputs: dx, dgamma, dbeta */
int chelis_chain_grad_device(const chelis_device_tensor_owner *const *inputs,
                             chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                             chelis_device_rank n_out);
/* inputs: r[count,t,a], w[count,a]; outputs: sigma, risk, cum */
int chelis_portfolio_device(const chelis_device_tensor_owner *const *inputs,
                            chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                            chelis_device_rank n_out);
/* inputs: a[m,k], b[k,n] (f32 or f64, batched when rank 3); outputs: c */
int chelis_matmul_device(const chelis_device_tensor_owner *const *inputs,
                         chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                         chelis_device_rank n_out);

#ifdef __cplusplus
}
#endif
#endif
