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
                               float dsel, float *__restrict__ nl, float *__restrict__ dz,
                               int *__restrict__ bad_label) {
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
    const float e = valid ? expf(__fsub_rn(v, m)) : 0.0f;
    bool ve = valid;
    const float zsum = warp_tree(e, ve);
    const float s = __fdiv_rn(e, zsum);
    const int64_t label = labels[row];
    if (label < 0 || label >= classes) {
        if (lane == 0) atomicExch(bad_label, 1);
        return;
    }
    const float s_label = __shfl_sync(0xffffffffu, s, static_cast<int>(label));
    if (lane == 0) nl[row] = -logf(s_label);
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
    // scratch: pre, h, dh [batch, dh]; z, dz [batch, dout]; nl [batch]; flag
    const size_t bh = static_cast<size_t>(batch * dh), bo = static_cast<size_t>(batch * dout);
    const size_t bytes = (3 * bh + 2 * bo + batch) * sizeof(float) + 16;
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, bytes, s));
    float *pre = static_cast<float *>(scratch);
    float *h = pre + bh;
    float *dhid = h + bh;
    float *z = dhid + bh;
    float *dz = z + bo;
    float *nl = dz + bo;
    int *bad = reinterpret_cast<int *>(nl + batch);
    int st = CHELIS_CUDA_OK;
    auto launch_blocks = [](int64_t n) {
        int64_t b = (n + 255) / 256;
        return static_cast<unsigned>(b > 148 * 8 ? 148 * 8 : (b < 1 ? 1 : b));
    };
    do {
        st = check_cuda(cudaMemsetAsync(bad, 0, sizeof(int), s), "memset");
        if (st) break;
        // forward
        st = launch_exact_gemm<float>(0, 0, batch, dh, din, x, din, 0, w1, dh, 0, pre, dh, 0, 1, s);
        if (st) break;
        mlp::bias_relu_kernel<<<launch_blocks(bh), 256, 0, s>>>(pre, h, b1, batch, dh);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "bias_relu_kernel"))) break;
        st = launch_exact_gemm<float>(0, 0, batch, dout, dh, h, dh, 0, w2, dout, 0, z, dout, 0, 1, s);
        if (st) break;
        const float bf = static_cast<float>(batch);
        const float dnl = 1.0f / bf;
        mlp::ce_rows_kernel<<<static_cast<unsigned>((batch * 32 + 255) / 256), 256, 0, s>>>(
            z, b2, labels, batch, static_cast<int>(dout), -dnl, nl, dz, bad);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "ce_rows_kernel"))) break;
        mlp::mean_kernel<<<1, 32, 0, s>>>(nl, batch, loss);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "mean_kernel"))) break;
        // adjoint
        if ((st = col_sum_into(dz, batch, dout, db2, s))) break;
        st = launch_exact_gemm<float>(1, 0, dh, dout, batch, h, dh, 0, dz, dout, 0, dw2, dout, 0, 1, s);
        if (st) break;
        st = launch_exact_gemm<float>(0, 1, batch, dh, dout, dz, dout, 0, w2, dout, 0, dhid, dh, 0, 1, s);
        if (st) break;
        mlp::relu_adjoint_kernel<<<launch_blocks(bh), 256, 0, s>>>(pre, dhid, bh);
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "relu_adjoint_kernel"))) break;
        if ((st = col_sum_into(dhid, batch, dh, db1, s))) break;
        st = launch_exact_gemm<float>(1, 0, din, dh, batch, x, din, 0, dhid, dh, 0, dw1, dh, 0, 1, s);
        if (st) break;
        int flag = 0;
        st = check_cuda(cudaMemcpyAsync(&flag, bad, sizeof(int), cudaMemcpyDeviceToHost, s), "copy flag");
        if (st) break;
        st = check_cuda(cudaStreamSynchronize(s), "sync");
        if (st) break;
        if (flag) st = set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in gather at i64");
    } while (0);
    scratch_free(scratch, s);
    return st;
}
