// abi.cu -- the descriptor-level entry points generated Chelis code calls:
// the row-major GEMM helpers (chelis_hip_runtime.h:48-404, dispatched from
// emit.rs:4718-4842) and whole-program `*_device` entries with the
// generated-entry device ABI (emit.rs:838-958).
#include <cuda_runtime.h>

#include "common.cuh"

using namespace chelis;

namespace {

// chelis_gpu_matrix_slices_contiguous (chelis_hip_runtime.h:80-87): the two
// trailing axes are a dense row-major matrix with `cols` columns.
bool slices_contiguous(const chelis_gpu_tensor *t, int64_t cols) {
    if (!t || t->rank < 2) return false;
    return t->strides[t->rank - 1] == 1 && t->strides[t->rank - 2] == cols;
}

int check_tensor(const chelis_gpu_tensor *t, chelis_dtype dt, const char *op) {
    if (!t) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in %s at i64", op);
    if (t->dtype != dt)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "%s: dtype %d where %d expected", op,
                         static_cast<int>(t->dtype), static_cast<int>(dt));
    return CHELIS_CUDA_OK;
}

int matmul_2d(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
              const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k, chelis_dtype dt) {
    const char *op = "matmul";
    CHELIS_TRY(check_tensor(a, dt, op));
    CHELIS_TRY(check_tensor(b, dt, op));
    CHELIS_TRY(check_tensor(out, dt, op));
    if (out->count == 0) return CHELIS_CUDA_OK;  // emit.rs:4806
    if (!slices_contiguous(a, k) || !slices_contiguous(b, n) || !slices_contiguous(out, n))
        return set_error(CHELIS_CUDA_ERR_DOMAIN,
                         "chelis_cuda gemm requires contiguous row-major matrix slices");
    if (dt == CHELIS_DTYPE_F32)
        return chelis_cuda_sgemm(0, 0, m, n, k, static_cast<const float *>(a->data), k, m * k,
                                 static_cast<const float *>(b->data), n, k * n,
                                 static_cast<float *>(out->data), n, m * n, 1);
    return chelis_cuda_dgemm(0, 0, m, n, k, static_cast<const double *>(a->data), k, m * k,
                             static_cast<const double *>(b->data), n, k * n,
                             static_cast<double *>(out->data), n, m * n, 1);
}

int matmul_strided(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                   const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k, int64_t batch,
                   int64_t sa, int64_t sb, int64_t so, chelis_dtype dt) {
    const char *op = "matmul";
    CHELIS_TRY(check_tensor(a, dt, op));
    CHELIS_TRY(check_tensor(b, dt, op));
    CHELIS_TRY(check_tensor(out, dt, op));
    if (out->count == 0 || batch == 0) return CHELIS_CUDA_OK;
    if (!slices_contiguous(a, k) || !slices_contiguous(b, n) || !slices_contiguous(out, n))
        return set_error(CHELIS_CUDA_ERR_DOMAIN,
                         "chelis_cuda gemm requires contiguous row-major matrix slices");
    if (dt == CHELIS_DTYPE_F32)
        return chelis_cuda_sgemm(0, 0, m, n, k, static_cast<const float *>(a->data), k, sa,
                                 static_cast<const float *>(b->data), n, sb,
                                 static_cast<float *>(out->data), n, so, batch);
    return chelis_cuda_dgemm(0, 0, m, n, k, static_cast<const double *>(a->data), k, sa,
                             static_cast<const double *>(b->data), n, sb,
                             static_cast<double *>(out->data), n, so, batch);
}

// batch stride of the leading axes of a batched operand (one uniform stride
// over the flattened batch, as the reference's per-batch loop assumes)
int64_t batch_stride(const chelis_gpu_tensor *t) {
    return t->rank >= 3 ? t->strides[t->rank - 3] : 0;
}

int check_owner_counts(chelis_device_rank n_in, chelis_device_rank want_in,
                       chelis_device_rank n_out, chelis_device_rank want_out, const char *what) {
    if (n_in != want_in || n_out != want_out)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "%s: expected %d inputs and %d outputs", what,
                         want_in, want_out);
    return CHELIS_CUDA_OK;
}

bool contiguous(const chelis_gpu_tensor *t) {
    int64_t expect = 1;
    for (int ax = t->rank - 1; ax >= 0; --ax) {
        if (t->shape[ax] != 1 && t->strides[ax] != expect) return false;
        expect *= t->shape[ax];
    }
    return true;
}

void release_all(chelis_device_tensor_owner **outs, int n) {
    for (int i = 0; i < n; ++i) {
        chelis_device_tensor_release(outs[i]);
        outs[i] = nullptr;
    }
}

}  // namespace

extern "C" {

int chelis_cuda_sgemm_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k) {
    return matmul_2d(a, b, out, m, n, k, CHELIS_DTYPE_F32);
}

int chelis_cuda_dgemm_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k) {
    return matmul_2d(a, b, out, m, n, k, CHELIS_DTYPE_F64);
}

int chelis_cuda_sgemm_batched_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                        const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                        int64_t k, int64_t batch_count) {
    if (!a || !b || !out) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    return matmul_strided(a, b, out, m, n, k, batch_count, batch_stride(a), batch_stride(b),
                          batch_stride(out), CHELIS_DTYPE_F32);
}

int chelis_cuda_sgemm_strided_batched_row_major(const chelis_gpu_tensor *a,
                                                const chelis_gpu_tensor *b,
                                                const chelis_gpu_tensor *out, int64_t m,
                                                int64_t n, int64_t k, int64_t batch_count,
                                                int64_t a_batch_stride, int64_t b_batch_stride,
                                                int64_t out_batch_stride) {
    return matmul_strided(a, b, out, m, n, k, batch_count, a_batch_stride, b_batch_stride,
                          out_batch_stride, CHELIS_DTYPE_F32);
}

int chelis_cuda_dgemm_batched_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                                        const chelis_gpu_tensor *out, int64_t m, int64_t n,
                                        int64_t k, int64_t batch_count) {
    if (!a || !b || !out) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    return matmul_strided(a, b, out, m, n, k, batch_count, batch_stride(a), batch_stride(b),
                          batch_stride(out), CHELIS_DTYPE_F64);
}

int chelis_cuda_dgemm_strided_batched_row_major(const chelis_gpu_tensor *a,
                                                const chelis_gpu_tensor *b,
                                                const chelis_gpu_tensor *out, int64_t m,
                                                int64_t n, int64_t k, int64_t batch_count,
                                                int64_t a_batch_stride, int64_t b_batch_stride,
                                                int64_t out_batch_stride) {
    return matmul_strided(a, b, out, m, n, k, batch_count, a_batch_stride, b_batch_stride,
                          out_batch_stride, CHELIS_DTYPE_F64);
}

// ---- generated-entry device ABI programs ----

int chelis_chain_fwd_device(const chelis_device_tensor_owner *const *inputs,
                            chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                            chelis_device_rank n_out) {
    CHELIS_TRY(check_owner_counts(n_in, 3, n_out, 1, "chain_fwd"));
    const chelis_gpu_tensor *x = chelis_device_tensor_view(inputs[0]);
    const chelis_gpu_tensor *g = chelis_device_tensor_view(inputs[1]);
    const chelis_gpu_tensor *b = chelis_device_tensor_view(inputs[2]);
    if (!x || !g || !b || x->rank != 2 || g->rank != 1 || b->rank != 1 ||
        x->dtype != CHELIS_DTYPE_F32 || g->dtype != CHELIS_DTYPE_F32 ||
        b->dtype != CHELIS_DTYPE_F32 || g->shape[0] != x->shape[1] ||
        b->shape[0] != x->shape[1] || !contiguous(x) || !contiguous(g) || !contiguous(b))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "chain_fwd: operand shapes or dtypes do not match");
    const int64_t rows = x->shape[0], hidden = x->shape[1];
    outputs[0] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F32, 1, &rows);
    if (!outputs[0]) return CHELIS_CUDA_ERR_CUDA;
    int st = chelis_cuda_chain_fwd(static_cast<const float *>(x->data),
                                   static_cast<const float *>(g->data),
                                   static_cast<const float *>(b->data), 1e-5f, 42u, 0.1f, rows,
                                   hidden, 0,
                                   static_cast<float *>(chelis_device_tensor_view(outputs[0])->data),
                                   nullptr);
    if (st) release_all(outputs, 1);
    return st;
}

int chelis_chain_grad_device(const chelis_device_tensor_owner *const *inputs,
                             chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                             chelis_device_rank n_out) {
    CHELIS_TRY(check_owner_counts(n_in, 3, n_out, 3, "chain_grad"));
    const chelis_gpu_tensor *x = chelis_device_tensor_view(inputs[0]);
    const chelis_gpu_tensor *g = chelis_device_tensor_view(inputs[1]);
    const chelis_gpu_tensor *b = chelis_device_tensor_view(inputs[2]);
    if (!x || !g || !b || x->rank != 2 || g->rank != 1 || b->rank != 1 ||
        x->dtype != CHELIS_DTYPE_F32 || g->dtype != CHELIS_DTYPE_F32 ||
        b->dtype != CHELIS_DTYPE_F32 || g->shape[0] != x->shape[1] ||
        b->shape[0] != x->shape[1] || !contiguous(x) || !contiguous(g) || !contiguous(b))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "chain_grad: operand shapes or dtypes do not match");
    const int64_t hidden = x->shape[1];
    outputs[0] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F32, 2, x->shape);
    outputs[1] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F32, 1, &hidden);
    outputs[2] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F32, 1, &hidden);
    if (!outputs[0] || !outputs[1] || !outputs[2]) {
        release_all(outputs, 3);
        return CHELIS_CUDA_ERR_CUDA;
    }
    int st = chelis_cuda_chain_bwd(
        static_cast<const float *>(x->data), static_cast<const float *>(g->data),
        static_cast<const float *>(b->data), 1e-5f, 42u, 0.1f, x->shape[0], hidden, 0, nullptr,
        static_cast<float *>(chelis_device_tensor_view(outputs[0])->data),
        static_cast<float *>(chelis_device_tensor_view(outputs[1])->data),
        static_cast<float *>(chelis_device_tensor_view(outputs[2])->data));
    if (st) release_all(outputs, 3);
    return st;
}

int chelis_portfolio_device(const chelis_device_tensor_owner *const *inputs,
                            chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                            chelis_device_rank n_out) {
    CHELIS_TRY(check_owner_counts(n_in, 2, n_out, 3, "portfolio"));
    const chelis_gpu_tensor *r = chelis_device_tensor_view(inputs[0]);
    const chelis_gpu_tensor *w = chelis_device_tensor_view(inputs[1]);
    if (!r || !w || r->rank != 3 || w->rank != 2 || r->dtype != CHELIS_DTYPE_F64 ||
        w->dtype != CHELIS_DTYPE_F64 || w->shape[0] != r->shape[0] || w->shape[1] != r->shape[2] ||
        !contiguous(r) || !contiguous(w))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "portfolio: operand shapes or dtypes do not match");
    const int64_t count = r->shape[0], t = r->shape[1], a = r->shape[2];
    const int64_t sshape[3] = {count, a, a};
    const int64_t cshape[2] = {count, t};
    outputs[0] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F64, 3, sshape);
    outputs[1] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F64, 1, &count);
    outputs[2] = chelis_device_tensor_alloc_shape(CHELIS_DTYPE_F64, 2, cshape);
    if (!outputs[0] || !outputs[1] || !outputs[2]) {
        release_all(outputs, 3);
        return CHELIS_CUDA_ERR_CUDA;
    }
    int st = chelis_cuda_portfolio_f64(
        static_cast<const double *>(r->data), static_cast<const double *>(w->data), count, t, a,
        static_cast<double *>(chelis_device_tensor_view(outputs[0])->data),
        static_cast<double *>(chelis_device_tensor_view(outputs[1])->data),
        static_cast<double *>(chelis_device_tensor_view(outputs[2])->data));
    if (st) release_all(outputs, 3);
    return st;
}

int chelis_matmul_device(const chelis_device_tensor_owner *const *inputs, chelis_device_rank n_in,
                         chelis_device_tensor_owner **outputs, chelis_device_rank n_out) {
    CHELIS_TRY(check_owner_counts(n_in, 2, n_out, 1, "matmul"));
    const chelis_gpu_tensor *a = chelis_device_tensor_view(inputs[0]);
    const chelis_gpu_tensor *b = chelis_device_tensor_view(inputs[1]);
    if (!a || !b || a->rank != b->rank || (a->rank != 2 && a->rank != 3) || a->dtype != b->dtype ||
        (a->dtype != CHELIS_DTYPE_F32 && a->dtype != CHELIS_DTYPE_F64))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "matmul: operand ranks or dtypes do not match");
    const int r = a->rank;
    const int64_t m = a->shape[r - 2], k = a->shape[r - 1], n = b->shape[r - 1];
    if (b->shape[r - 2] != k || (r == 3 && a->shape[0] != b->shape[0]))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "matmul: contraction extents differ");
    int64_t oshape[3];
    if (r == 3) {
        oshape[0] = a->shape[0];
        oshape[1] = m;
        oshape[2] = n;
    } else {
        oshape[0] = m;
        oshape[1] = n;
    }
    outputs[0] = chelis_device_tensor_alloc_shape(a->dtype, r, oshape);
    if (!outputs[0]) return CHELIS_CUDA_ERR_CUDA;
    const chelis_gpu_tensor *o = chelis_device_tensor_view(outputs[0]);
    int st;
    if (r == 2) {
        st = (a->dtype == CHELIS_DTYPE_F32) ? chelis_cuda_sgemm_row_major(a, b, o, m, n, k)
                                            : chelis_cuda_dgemm_row_major(a, b, o, m, n, k);
    } else {
        st = (a->dtype == CHELIS_DTYPE_F32)
                 ? chelis_cuda_sgemm_batched_row_major(a, b, o, m, n, k, a->shape[0])
                 : chelis_cuda_dgemm_batched_row_major(a, b, o, m, n, k, a->shape[0]);
    }
    if (st) release_all(outputs, 1);
    return st;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// bounded-wait self-test: a consumer waits on an mbarrier for a producer
// thread's arrival through the same mbar_wait_bounded every pipeline uses
// ---------------------------------------------------------------------------
namespace chelis {
namespace selftest {
__global__ void bounded_wait_probe_kernel(int skip_arrival) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 32 && !skip_arrival) mbar_arrive(&bar);  // the producer warp
    if (threadIdx.x == 0) (void)mbar_wait_bounded(&bar, 0, DEVERR_TIMEOUT_PRODUCER);
    __syncthreads();
}
}  // namespace selftest
}  // namespace chelis

extern "C" int chelis_cuda_selftest_bounded_wait(int skip_arrival) {
    selftest::bounded_wait_probe_kernel<<<1, 64, 0, current_stream()>>>(skip_arrival);
    g_launches++;
    CHELIS_LAUNCH_CHECK("bounded_wait_probe_kernel");
    return CHELIS_CUDA_OK;
}
