// activations.cu -- the row ops a generated entry calls one at a time:
// Relu / ReluAdjoint ([05-OP-43], dag.rs:957,965; adjoint grad.rs:2281-2294),
// gelu = m(x) * Phi(x) with the compensated Phi graph (spec 05 section 3.3,
// tier2.rs lower_gelu) and its adjoint, the layer_norm adjoint (AD of the
// tier2.rs:1248-1375 lowering) and the cross-entropy of spec 05 section 4.3
// (log of the row softmax, gather at the label, negate, mean) with its
// adjoint.  The transformer block and the MLP step run the same arithmetic
// inside their own kernels; these entries expose each op on its own.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gelu.cuh"
#include "crmath.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int scratch_alloc(void **ptr, size_t bytes, cudaStream_t stream);
void scratch_free(void *ptr, cudaStream_t stream);

namespace act {

using chain::canon;

// relu = max_elem(x, +0): a NaN keeps its bits, -0 stays -0 (the first
// operand wins ties), every negative value becomes +0.
template <typename T>
__device__ __forceinline__ T relu1(T x) {
    return (isnan(x) || x >= T(0)) ? x : T(0);
}

template <typename T>
__global__ void relu_kernel(const T *__restrict__ x, T *__restrict__ y, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = relu1(x[i]);
}

// ReluAdjoint: the cotangent's bits where 0 < x, exact +0 elsewhere (both
// zeros and NaN inputs included).
template <typename T>
__global__ void relu_adjoint_kernel(const T *__restrict__ x, const T *__restrict__ g,
                                    T *__restrict__ dx, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dx[i] = (T(0) < x[i]) ? g[i] : T(0);
}

__global__ void gelu_adjoint_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                    float *__restrict__ dx, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        dx[i] = canon(__fmul_rn(g[i], gelu::derivative(x[i])));
    }
}

// Cross-entropy, one thread per row: nl[r] = -log(s[r, label[r]]) from the
// row softmax s; an out-of-range label is the gather's index trap
// ([05-OP-52], recorded in the device error word).
__global__ void ce_nl_kernel(const float *__restrict__ s, const int64_t *__restrict__ labels,
                             int64_t rows, int64_t classes, float *__restrict__ nl, int exact) {
    for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < rows;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t label = labels[r];
        if (label < 0 || label >= classes) {
            report_device_error(DEVERR_BAD_INDEX);
            nl[r] = 0.0f;
            continue;
        }
        const float p = s[r * classes + label];
        nl[r] = -(exact ? crmath::logf_cr(p) : logf(p));  // EXACT: CORE-MATH's bits
    }
}

// loss = total / rows, finalized
__global__ void ce_mean_kernel(const float *__restrict__ total, int64_t rows, float *__restrict__ loss) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *loss = canon(__fdiv_rn(*total, static_cast<float>(rows)));
}

// Adjoint of the mean cross-entropy through mean, neg, gather and log, then
// the row softmax (grad.rs:2248-2280): the log adjoint is g_j = dlp_j / s_j
// with dlp = dsel = -1/rows at the label and +0 elsewhere, so g_j is NaN
// where s_j underflowed to 0; q = sum_j g_j * s_j (one nonzero leaf, exact,
// or NaN) and dz_j = s_j * (g_j - q).  ce_q_kernel: one warp per row.
__global__ void ce_q_kernel(const float *__restrict__ s, const int64_t *__restrict__ labels,
                            int64_t rows, int64_t classes, float dsel, float *__restrict__ q) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < rows;
         r += warps) {
        const float *sr = s + r * classes;
        bool bad = false;  // a zero or NaN probability: 0 / s_j or NaN enters the sum
        for (int64_t j = lane; j < classes; j += 32) bad |= !(sr[j] != 0.0f);
        bad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
            const int64_t label = labels[r];
            float v = __int_as_float(0x7fc00000);
            if (label >= 0 && label < classes && !bad) {
                const float sl = sr[label];
                v = __fmul_rn(__fdiv_rn(dsel, sl), sl);
            }
            q[r] = v;
        }
    }
}

__global__ void ce_grad_kernel(const float *__restrict__ s, const int64_t *__restrict__ labels,
                               const float *__restrict__ q, int64_t rows, int64_t classes,
                               float dsel, float *__restrict__ dz) {
    const int64_t n = rows * classes;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / classes, j = i - r * classes;
        const float sj = s[i];
        const float g = __fdiv_rn(j == labels[r] ? dsel : 0.0f, sj);
        dz[i] = canon(__fmul_rn(sj, __fsub_rn(g, q[r])));
    }
}

}  // namespace act

namespace {

unsigned act_grid(int64_t n) {
    const int64_t g = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    return static_cast<unsigned>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_relu(int32_t dtype, const void *x, void *y, int64_t n) {
    if (dtype != CHELIS_DTYPE_F32 && dtype != CHELIS_DTYPE_F64)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "relu admits f32 and f64");
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in relu at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    if (!x || !y) return set_error(CHELIS_CUDA_ERR_DOMAIN, "relu: null operand");
    cudaStream_t s = current_stream();
    if (dtype == CHELIS_DTYPE_F32)
        act::relu_kernel<float><<<act_grid(n), 256, 0, s>>>(static_cast<const float *>(x),
                                                            static_cast<float *>(y), n);
    else
        act::relu_kernel<double><<<act_grid(n), 256, 0, s>>>(static_cast<const double *>(x),
                                                             static_cast<double *>(y), n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("act::relu_kernel");
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_relu_adjoint(int32_t dtype, const void *x, const void *g, void *dx,
                                        int64_t n) {
    if (dtype != CHELIS_DTYPE_F32 && dtype != CHELIS_DTYPE_F64)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "relu_adjoint admits f32 and f64");
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in relu_adjoint at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    if (!x || !g || !dx) return set_error(CHELIS_CUDA_ERR_DOMAIN, "relu_adjoint: null operand");
    cudaStream_t s = current_stream();
    if (dtype == CHELIS_DTYPE_F32)
        act::relu_adjoint_kernel<float><<<act_grid(n), 256, 0, s>>>(
            static_cast<const float *>(x), static_cast<const float *>(g), static_cast<float *>(dx), n);
    else
        act::relu_adjoint_kernel<double><<<act_grid(n), 256, 0, s>>>(
            static_cast<const double *>(x), static_cast<const double *>(g), static_cast<double *>(dx), n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("act::relu_adjoint_kernel");
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_gelu_f32(const float *x, float *y, int64_t n) {
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in gelu at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    if (!x || !y) return set_error(CHELIS_CUDA_ERR_DOMAIN, "gelu: null operand");
    block::gelu_fwd_kernel<<<act_grid(n), 256, 0, current_stream()>>>(x, y, n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("block::gelu_fwd_kernel");
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_gelu_adjoint_f32(const float *x, const float *g, float *dx, int64_t n) {
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in gelu at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    if (!x || !g || !dx) return set_error(CHELIS_CUDA_ERR_DOMAIN, "gelu_adjoint: null operand");
    act::gelu_adjoint_kernel<<<act_grid(n), 256, 0, current_stream()>>>(x, g, dx, n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("act::gelu_adjoint_kernel");
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_layer_norm_bwd_f32(const float *x, const float *gamma, float eps,
                                              const float *dy, int64_t rows, int64_t hidden,
                                              float *dx, float *dgamma, float *dbeta) {
    if (rows < 0 || hidden < 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at i64");
    if (hidden > 8192)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "layer_norm adjoint admits rows of <= 8192");
    if (rows == 0 || hidden == 0) {
        cudaStream_t s = current_stream();
        if (hidden > 0 && dgamma) CHELIS_TRY(check_cuda(cudaMemsetAsync(dgamma, 0, hidden * 4, s), "memset"));
        if (hidden > 0 && dbeta) CHELIS_TRY(check_cuda(cudaMemsetAsync(dbeta, 0, hidden * 4, s), "memset"));
        return CHELIS_CUDA_OK;
    }
    if (!x || !gamma || !dy || !dx || !dgamma || !dbeta)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "layer_norm adjoint: null operand");
    cudaStream_t s = current_stream();
    int grid = ln_grid();
    if (grid > rows) grid = static_cast<int>(rows);
    const size_t stats_bytes = static_cast<size_t>(rows) * sizeof(float2);
    const size_t part_bytes = 2 * static_cast<size_t>(grid) * hidden * sizeof(float);
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, stats_bytes + part_bytes, s));
    float2 *st = static_cast<float2 *>(scratch);
    float *part = reinterpret_cast<float *>(static_cast<char *>(scratch) + stats_bytes);
    int rc = ln_fwd(x, gamma, gamma, eps, nullptr, st, rows, hidden, s);  // statistics only
    if (rc == CHELIS_CUDA_OK)
        rc = ln_bwd(x, dy, st, gamma, nullptr, dx, part, dgamma, dbeta, rows, hidden, s);
    scratch_free(scratch, s);
    return rc;
}

extern "C" int chelis_cuda_cross_entropy_f32(const float *logits, const int64_t *labels, int64_t rows,
                                             int64_t classes, float *loss, float *dlogits) {
    if (rows < 1 || classes < 1)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in cross_entropy at i64");
    if (!logits || !labels || !loss)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "cross_entropy: null operand");
    cudaStream_t s = current_stream();
    // scratch: the row softmax, nl[rows], q[rows], the row-sum total
    const size_t n = static_cast<size_t>(rows) * classes;
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, (n + 2 * static_cast<size_t>(rows) + 4) * sizeof(float), s));
    float *soft = static_cast<float *>(scratch);
    float *nl = soft + n, *q = nl + rows, *total = q + rows;
    int rc = chelis_cuda_softmax_rows_f32(logits, soft, rows, classes);
    if (rc == CHELIS_CUDA_OK) {
        act::ce_nl_kernel<<<act_grid(rows), 256, 0, s>>>(soft, labels, rows, classes, nl,
                                                         rows_mode() == CHELIS_CUDA_ROWS_EXACT);
        g_launches++;
        rc = check_cuda(cudaGetLastError(), "act::ce_nl_kernel");
    }
    if (rc == CHELIS_CUDA_OK) rc = chelis_cuda_row_sum_f32(nl, 1, rows, total);  // canonical tree over rows
    if (rc == CHELIS_CUDA_OK) {
        act::ce_mean_kernel<<<1, 32, 0, s>>>(total, rows, loss);
        g_launches++;
        rc = check_cuda(cudaGetLastError(), "act::ce_mean_kernel");
    }
    if (rc == CHELIS_CUDA_OK && dlogits) {
        const float dsel = -(1.0f / static_cast<float>(rows));  // mean adjoint, then neg
        act::ce_q_kernel<<<act_grid(rows * 32), 256, 0, s>>>(soft, labels, rows, classes, dsel, q);
        act::ce_grad_kernel<<<act_grid(static_cast<int64_t>(n)), 256, 0, s>>>(soft, labels, q, rows,
                                                                              classes, dsel, dlogits);
        g_launches += 2;
        rc = check_cuda(cudaGetLastError(), "act::ce_grad_kernel");
    }
    scratch_free(scratch, s);
    return rc;
}
