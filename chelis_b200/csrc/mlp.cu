// mlp.cu -- the 2-layer MLP training step (forward + reverse mode):
//   pre = x.W1 + b1; h = relu(pre); z = h.W2 + b2
//   loss = mean_b(-log(softmax(z)[b, label_b]))   (cross_entropy lowering,
//          spec/05-risc-primitives.md:5044-5063)
//   grads w.r.t. W1, b1, W2, b2 through the adjoint graphs of grad.rs
//   (Softmax :2248-2280, Relu -> ReluAdjoint, matmul = Sum(Mul(Expand)) ).
//
// The matmuls run on the canonical-tree CUDA-core GEMM, so every product and
// sum matches the C lane bit for bit; exp and log are CUDA's (the C lane
// uses CORE-MATH), which is where tolerance enters.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "crmath.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
template <typename T>
int launch_exact_gemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const T *a,
                      int64_t lda, int64_t stride_a, const T *b, int64_t ldb, int64_t stride_b,
                      T *c, int64_t ldc, int64_t stride_c, int64_t batch, cudaStream_t s);
int col_sum_into(const float *x, int64_t rows, int64_t cols, float *out, cudaStream_t s);

namespace mlp {

// pre += b1 (row broadcast); h = relu(pre) = max_elem(pre, 0) ([05-OP-43])
__global__ void bias_relu_kernel(float *__restrict__ pre, float *__restrict__ h,
                                 const float *__restrict__ bias, int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = __fadd_rn(pre[i], bias[i % cols]);
        pre[i] = v;
        h[i] = (v < 0.0f) ? 0.0f : v;
    }
}

// ReluAdjoint: g where 0 < x, exact +0 otherwise ([05-OP-43])
__global__ void relu_adjoint_kernel(const float *__restrict__ pre, float *__restrict__ g,
                                    int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        g[i] = (0.0f < pre[i]) ? g[i] : 0.0f;
}

// One warp per row (classes <= 32): z += b2; softmax; nl = -log(s[label]);
// dz = softmax adjoint of g = (onehot * (-1/B)) / s.
__global__ void ce_rows_kernel(float *__restrict__ z, const float *__restrict__ b2,
                               const int64_t *__restrict__ labels, int64_t rows, int classes,
                               float dsel, float *__restrict__ nl, float *__restrict__ dz) {
    const int lane = threadIdx.x & 31;
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (row >= rows) return;
    const bool valid = lane < classes;
    float v = valid ? __fadd_rn(z[row * classes + lane], b2[lane]) : -INFINITY;
    if (valid) z[row * classes + lane] = v;
    float m = v;
    bool nan = valid && isnan(v);
    m = warp_max(m);
    nan = __any_sync(0xffffffffu, nan);
    if (nan) m = __int_as_float(0x7fc00000);
    const float e = valid ? crmath::expf_cr(__fsub_rn(v, m)) : 0.0f;  // CORE-MATH's bits
    bool ve = valid;
    const float zsum = warp_tree(e, ve);
    const float s = __fdiv_rn(e, zsum);
    const int64_t label = labels[row];
    if (label < 0 || label >= classes) {
        // [05-OP-52] out-of-range gather index: recorded in the device error
        // word and reported by chelis_cuda_device_status (no host sync here)
        if (lane == 0) report_device_error(DEVERR_BAD_INDEX);
        return;
    }
    const float s_label = __shfl_sync(0xffffffffu, s, static_cast<int>(label));
    if (lane == 0) nl[row] = -crmath::logf_cr(s_label);
    const float dlp = (lane == label) ? dsel : 0.0f;
    const float g = valid ? __fdiv_rn(dlp, s) : 0.0f;
    bool vq = valid;
    const float q = warp_tree(__fmul_rn(g, s), vq);
    if (valid) dz[row * classes + lane] = __fmul_rn(s, __fsub_rn(g, q));
}

// loss = tree_b(nl) / B, one CTA
__global__ void mean_kernel(const float *__restrict__ nl, int64_t n, float *__restrict__ loss) {
    __shared__ float level[64];
    if (threadIdx.x != 0) return;
    int64_t count = 0;
    for (int64_t i = 0; i < n; ++i) {
        float carry = nl[i];
        int depth = 0;
        for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)
            carry = __fadd_rn(level[depth], carry);
        level[depth] = carry;
    }
    float total = 0.0f;
    bool found = false;
    int depth = 0;
    for (int64_t remaining = count; remaining; remaining >>= 1, ++depth)
        if (remaining & 1) {
            total = found ? __fadd_rn(level[depth], total) : level[depth];
            found = true;
        }
    *loss = __fdiv_rn(total, static_cast<float>(n));
}

// Column sums of a small [rows, cols] matrix, one warp per column: lane l
// takes row k0 + l of each aligned 32-row block (a subtree of the canonical
// tree over rows), the block sums go through lane 0's carry tree.  With
// `divide`, the total is divided by rows (the mean lowering).
__global__ void col_tree_warp_kernel(const float *__restrict__ x, int64_t rows, int64_t cols,
                                     float *__restrict__ out, bool divide) {
    const int lane = threadIdx.x & 31;
    const int64_t col = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    if (col >= cols) return;
    float level[40];
    int64_t count = 0;
    for (int64_t r0 = 0; r0 < rows; r0 += 32) {
        bool valid = r0 + lane < rows;
        float v = valid ? x[(r0 + lane) * cols + col] : 0.0f;
        v = warp_tree(v, valid);
        if (lane == 0) {
            float carry = v;
            int depth = 0;
            for (int64_t pending = count; pending & 1; pending >>= 1, ++depth)
                carry = __fadd_rn(level[depth], carry);
            level[depth] = carry;
        }
        ++count;
    }
    if (lane == 0) {
        float total = 0.0f;
        bool found = false;
        int depth = 0;
        for (int64_t remaining = count; remaining; remaining >>= 1, ++depth)
            if (remaining & 1) {
                total = found ? __fadd_rn(level[depth], total) : level[depth];
                found = true;
            }
        out[col] = divide ? __fdiv_rn(total, static_cast<float>(rows)) : total;
    }
}

// pre = tree over `nk` k-chunk partial sums (each an aligned power-of-two
// block of the contraction, so a subtree of the canonical tree) + bias;
// h = relu(pre).
__global__ void combine_bias_relu_kernel(const float *__restrict__ part, int nk, int64_t mn,
                                         const float *__restrict__ bias, int64_t cols,
                                         float *__restrict__ pre, float *__restrict__ h) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < mn;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float level[8];
        int count = 0;
        for (int c = 0; c < nk; ++c) {
            float carry = part[c * mn + i];
            int depth = 0;
            for (int pending = count++; pending & 1; pending >>= 1, ++depth)
                carry = __fadd_rn(level[depth], carry);
            level[depth] = carry;
        }
        float total = 0.0f;
        bool found = false;
        int depth = 0;
        for (int remaining = count; remaining; remaining >>= 1, ++depth)
            if (remaining & 1) {
                total = found ? __fadd_rn(level[depth], total) : level[depth];
                found = true;
            }
        const float v = __fadd_rn(total, bias[i % cols]);
        pre[i] = v;
        h[i] = (v < 0.0f) ? 0.0f : v;
    }
}

}  // namespace mlp
}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_mlp_step(const float *x, const int64_t *labels, const float *w1,
                                    const float *b1, const float *w2, const float *b2,
                                    int64_t batch, int64_t din, int64_t dh, int64_t dout,
                                    float *loss, float *dw1, float *db1, float *dw2,
                                    float *db2) {
    if (batch <= 0 || din <= 0 || dh <= 0 || dout <= 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in cross_entropy at i64");
    if (dout > 32)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "cross_entropy kernel admits <= 32 classes");
    cudaStream_t s = current_stream();
    // The first product (k = din) is split along k into aligned chunks of
    // KC leaves computed in parallel; every chunk is a subtree of the
    // canonical tree, so combining the chunk sums pass by pass gives the
    // same bits as one tree over k.
    constexpr int64_t KC = 256;
    const int64_t nk = (din + KC - 1) / KC;
    if (nk > 255)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "mlp input width beyond %lld", 255 * KC);
    // scratch: k-chunk partials; pre, h, dh [batch, dh]; z, dz [batch, dout]; nl [batch]
    const size_t bh = static_cast<size_t>(batch * dh), bo = static_cast<size_t>(batch * dout);
    const size_t bytes = (nk * bh + 3 * bh + 2 * bo + batch) * sizeof(float) + 16;
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, bytes, s));
    float *part = static_cast<float *>(scratch);
    float *pre = part + nk * bh;
    float *h = pre + bh;
    float *dhid = h + bh;
    float *z = dhid + bh;
    float *dz = z + bo;
    float *nl = dz + bo;
    int st = CHELIS_CUDA_OK;
    auto launch_blocks = [](int64_t n) {
        int64_t b = (n + 255) / 256;
        return static_cast<unsigned>(b > 148 * 8 ? 148 * 8 : (b < 1 ? 1 : b));
    };
    do {
        // forward: full chunks as one batched launch, the ragged tail apart
        const int64_t full = din / KC, tail = din - full * KC;
        if (full > 0) {
            st = launch_exact_gemm<float>(0, 0, batch, dh, KC, x, din, KC, w1, dh, KC * dh, part,
                                          dh, static_cast<int64_t>(bh), full, s);
            if (st) break;
        }
        if (tail > 0) {
            st = launch_exact_gemm<float>(0, 0, batch, dh, tail, x + full * KC, din, 0,
                                          w1 + full * KC * dh, dh, 0, part + full * bh, dh, 0, 1, s);
            if (st) break;
        }
        mlp::combine_bias_relu_kernel<<<launch_blocks(bh), 256, 0, s>>>(
            part, static_cast<int>(nk), static_cast<int64_t>(bh), b1, dh, pre, h);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "combine_bias_relu_kernel"))) break;
        st = launch_exact_gemm<float>(0, 0, batch, dout, dh, h, dh, 0, w2, dout, 0, z, dout, 0, 1, s);
        if (st) break;
        const float bf = static_cast<float>(batch);
        const float dnl = 1.0f / bf;
        mlp::ce_rows_kernel<<<static_cast<unsigned>((batch * 32 + 255) / 256), 256, 0, s>>>(
            z, b2, labels, batch, static_cast<int>(dout), -dnl, nl, dz);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "ce_rows_kernel"))) break;
        mlp::col_tree_warp_kernel<<<1, 32, 0, s>>>(nl, batch, 1, loss, true);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "col_tree_warp_kernel"))) break;
        // adjoint; the bias gradients are column trees over the batch
        const unsigned cbo = static_cast<unsigned>((dout * 32 + 255) / 256);
        mlp::col_tree_warp_kernel<<<cbo, 256, 0, s>>>(dz, batch, dout, db2, false);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "col_tree_warp_kernel"))) break;
        st = launch_exact_gemm<float>(1, 0, dh, dout, batch, h, dh, 0, dz, dout, 0, dw2, dout, 0, 1, s);
        if (st) break;
        st = launch_exact_gemm<float>(0, 1, batch, dh, dout, dz, dout, 0, w2, dout, 0, dhid, dh, 0, 1, s);
        if (st) break;
        mlp::relu_adjoint_kernel<<<launch_blocks(bh), 256, 0, s>>>(pre, dhid, bh);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "relu_adjoint_kernel"))) break;
        const unsigned cbh = static_cast<unsigned>((dh * 32 + 255) / 256);
        mlp::col_tree_warp_kernel<<<cbh, 256, 0, s>>>(dhid, batch, dh, db1, false);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "col_tree_warp_kernel"))) break;
        st = launch_exact_gemm<float>(1, 0, din, dh, batch, x, din, 0, dhid, dh, 0, dw1, dh, 0, 1, s);
        if (st) break;
    } while (0);
    scratch_free(scratch, s);
    return st;
}
