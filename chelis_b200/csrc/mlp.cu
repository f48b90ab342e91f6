// mlp.cu -- the 2-layer MLP training step (forward + reverse mode):
//   pre = x.W1 + b1; h = relu(pre); z = h.W2 + b2
//   loss = mean_b(-log(softmax(z)[b, label_b]))   (cross_entropy lowering,
//          spec/05-risc-primitives.md:5044-5063)
//   grads w.r.t. W1, b1, W2, b2 through the adjoint graphs of grad.rs
//   (Softmax :2248-2280, Relu -> ReluAdjoint, matmul = Sum(Mul(Expand)) ).
//
// The matmuls run on the canonical-tree CUDA-core GEMM, so every product and
// sum matches the C lane bit for bit, and exp / log are correctly rounded
// (crmath.cuh) as CORE-MATH's are in the C lane: the step is bit-identical.
//
// The step is a dozen small dependent launches, so a repeated call (same
// arguments and stream, as a training loop makes) runs as a CUDA graph:
// captured at the second call (with scratch of its own) and replayed from
// then on.  First calls, and callers that are capturing a graph of their
// own, get the launches enqueued directly.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

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

namespace chelis {
namespace mlp {

struct StepArgs {
    const float *x;
    const int64_t *labels;
    const float *w1, *b1, *w2, *b2;
    int64_t batch, din, dh, dout;
    float *loss, *dw1, *db1, *dw2, *db2;
    bool operator==(const StepArgs &o) const {
        return x == o.x && labels == o.labels && w1 == o.w1 && b1 == o.b1 && w2 == o.w2 &&
               b2 == o.b2 && batch == o.batch && din == o.din && dh == o.dh && dout == o.dout &&
               loss == o.loss && dw1 == o.dw1 && db1 == o.db1 && dw2 == o.dw2 && db2 == o.db2;
    }
};

// The first product (k = din) is split along k into aligned chunks of KC
// leaves computed in parallel; every chunk is a subtree of the canonical
// tree, so combining the chunk sums pass by pass gives the same bits as one
// tree over k.
constexpr int64_t KC = 256;

// scratch: k-chunk partials; pre, h, dh [batch, dh]; z, dz [batch, dout]; nl [batch]
size_t scratch_bytes(const StepArgs &a) {
    const int64_t nk = (a.din + KC - 1) / KC;
    const size_t bh = static_cast<size_t>(a.batch * a.dh), bo = static_cast<size_t>(a.batch * a.dout);
    return (nk * bh + 3 * bh + 2 * bo + a.batch) * sizeof(float) + 16;
}

// The step's launches on `s`, using `scratch` (scratch_bytes(a) bytes).
int enqueue(const StepArgs &a, void *scratch, cudaStream_t s) {
    const int64_t batch = a.batch, din = a.din, dh = a.dh, dout = a.dout;
    const int64_t nk = (din + KC - 1) / KC;
    const size_t bh = static_cast<size_t>(batch * dh), bo = static_cast<size_t>(batch * dout);
    float *part = static_cast<float *>(scratch);
    float *pre = part + nk * bh;
    float *h = pre + bh;
    float *dhid = h + bh;
    float *z = dhid + bh;
    float *dz = z + bo;
    float *nl = dz + bo;
    auto launch_blocks = [](int64_t n) {
        int64_t b = (n + 255) / 256;
        return static_cast<unsigned>(b > 148 * 8 ? 148 * 8 : (b < 1 ? 1 : b));
    };
    // forward: full chunks as one batched launch, the ragged tail apart
    const int64_t full = din / KC, tail = din - full * KC;
    if (full > 0)
        CHELIS_TRY(launch_exact_gemm<float>(0, 0, batch, dh, KC, a.x, din, KC, a.w1, dh, KC * dh, part,
                                            dh, static_cast<int64_t>(bh), full, s));
    if (tail > 0)
        CHELIS_TRY(launch_exact_gemm<float>(0, 0, batch, dh, tail, a.x + full * KC, din, 0,
                                            a.w1 + full * KC * dh, dh, 0, part + full * bh, dh, 0, 1, s));
    combine_bias_relu_kernel<<<launch_blocks(bh), 256, 0, s>>>(part, static_cast<int>(nk),
                                                               static_cast<int64_t>(bh), a.b1, dh, pre, h);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "combine_bias_relu_kernel"));
    CHELIS_TRY(launch_exact_gemm<float>(0, 0, batch, dout, dh, h, dh, 0, a.w2, dout, 0, z, dout, 0, 1, s));
    const float bf = static_cast<float>(batch);
    const float dnl = 1.0f / bf;
    ce_rows_kernel<<<static_cast<unsigned>((batch * 32 + 255) / 256), 256, 0, s>>>(
        z, a.b2, a.labels, batch, static_cast<int>(dout), -dnl, nl, dz);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "ce_rows_kernel"));
    col_tree_warp_kernel<<<1, 32, 0, s>>>(nl, batch, 1, a.loss, true);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "col_tree_warp_kernel"));
    // adjoint; the bias gradients are column trees over the batch
    const unsigned cbo = static_cast<unsigned>((dout * 32 + 255) / 256);
    col_tree_warp_kernel<<<cbo, 256, 0, s>>>(dz, batch, dout, a.db2, false);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "col_tree_warp_kernel"));
    CHELIS_TRY(launch_exact_gemm<float>(1, 0, dh, dout, batch, h, dh, 0, dz, dout, 0, a.dw2, dout, 0, 1, s));
    CHELIS_TRY(launch_exact_gemm<float>(0, 1, batch, dh, dout, dz, dout, 0, a.w2, dout, 0, dhid, dh, 0, 1, s));
    relu_adjoint_kernel<<<launch_blocks(bh), 256, 0, s>>>(pre, dhid, bh);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "relu_adjoint_kernel"));
    const unsigned cbh = static_cast<unsigned>((dh * 32 + 255) / 256);
    col_tree_warp_kernel<<<cbh, 256, 0, s>>>(dhid, batch, dh, a.db1, false);
    g_launches++;
    CHELIS_TRY(check_cuda(cudaGetLastError(), "col_tree_warp_kernel"));
    return launch_exact_gemm<float>(1, 0, din, dh, batch, a.x, din, 0, dhid, dh, 0, a.dw1, dh, 0, 1, s);
}

// Instantiated step graphs, least recently used evicted past kGraphs.
struct Graph {
    StepArgs key{};
    int device = -1;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    void *scratch = nullptr;
    uint64_t kernels = 0;
    uint64_t used = 0;
};
constexpr int kGraphs = 8;
std::mutex g_mu;
Graph g_graphs[kGraphs];
uint64_t g_tick = 0;
// Argument sets run once, directly: a set becomes a graph when it repeats
// (a capture costs more than the launches it saves on a one-off call).
struct Seen {
    StepArgs key{};
    int device = -1;
    cudaStream_t stream = nullptr;
};
constexpr int kSeen = 16;
Seen g_seen[kSeen];
int g_seen_next = 0;

// Destroy one cached graph and its scratch (on its device; the device is
// synchronised first, since a replay may still be in flight).
void drop(Graph &g) {
    if (!g.exec) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(g.device);
    cudaDeviceSynchronize();
    cudaGraphExecDestroy(g.exec);
    cudaFree(g.scratch);
    cudaSetDevice(prev);
    g = Graph{};
}

// Capture the step for (a, s) on a private stream and instantiate it.
int capture(const StepArgs &a, cudaStream_t s, int device, Graph *out) {
    Graph g;
    g.key = a;
    g.device = device;
    g.stream = s;
    CHELIS_TRY(check_cuda(cudaMalloc(&g.scratch, scratch_bytes(a)), "cudaMalloc(mlp step scratch)"));
    cudaStream_t cs = nullptr;
    int st = check_cuda(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "cudaStreamCreate");
    cudaGraph_t graph = nullptr;
    if (st == CHELIS_CUDA_OK) {
        st = check_cuda(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
        if (st == CHELIS_CUDA_OK) {
            const int est = enqueue(a, g.scratch, cs);
            const int cst = check_cuda(cudaStreamEndCapture(cs, &graph), "cudaStreamEndCapture");
            st = est != CHELIS_CUDA_OK ? est : cst;
        }
        if (st == CHELIS_CUDA_OK) {
            // kernels of the graph: counted each time it runs, not at capture
            size_t n = 0;
            st = check_cuda(cudaGraphGetNodes(graph, nullptr, &n), "cudaGraphGetNodes");
            cudaGraphNode_t nodes[64];
            if (st == CHELIS_CUDA_OK && n <= 64) {
                st = check_cuda(cudaGraphGetNodes(graph, nodes, &n), "cudaGraphGetNodes");
                for (size_t i = 0; st == CHELIS_CUDA_OK && i < n; ++i) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel)
                        ++g.kernels;
                }
            }
            g_launches -= g.kernels;
        }
        if (st == CHELIS_CUDA_OK)
            st = check_cuda(cudaGraphInstantiate(&g.exec, graph, 0), "cudaGraphInstantiate(mlp step)");
        if (graph) cudaGraphDestroy(graph);
        cudaStreamDestroy(cs);
    }
    if (st != CHELIS_CUDA_OK) {
        cudaFree(g.scratch);
        return st;
    }
    *out = g;
    return CHELIS_CUDA_OK;
}

}  // namespace mlp

// Release every cached step graph (chelis_cuda_shutdown).
void mlp_release_graphs() {
    std::lock_guard<std::mutex> lk(mlp::g_mu);
    for (mlp::Graph &g : mlp::g_graphs) mlp::drop(g);
}

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
    if ((din + mlp::KC - 1) / mlp::KC > 255)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "mlp input width beyond %lld", 255 * mlp::KC);
    const mlp::StepArgs a{x, labels, w1, b1, w2, b2, batch, din, dh, dout, loss, dw1, db1, dw2, db2};
    cudaStream_t s = current_stream();
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    CHELIS_TRY(check_cuda(cudaStreamIsCapturing(s, &cap), "cudaStreamIsCapturing"));
    if (cap != cudaStreamCaptureStatusNone) {
        // the caller is building a graph of its own: enqueue into it
        void *scratch = nullptr;
        CHELIS_TRY(scratch_alloc(&scratch, mlp::scratch_bytes(a), s));
        const int st = mlp::enqueue(a, scratch, s);
        scratch_free(scratch, s);
        return st;
    }
    int device = 0;
    CHELIS_TRY(current_device_checked(&device));
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;
    {
        std::lock_guard<std::mutex> lk(mlp::g_mu);
        mlp::Graph *hit = nullptr, *lru = &mlp::g_graphs[0];
        for (mlp::Graph &g : mlp::g_graphs) {
            if (g.exec && g.device == device && g.stream == s && g.key == a) hit = &g;
            if (g.used < lru->used) lru = &g;
        }
        if (!hit) {
            bool repeat = false;
            for (const mlp::Seen &q : mlp::g_seen)
                if (q.device == device && q.stream == s && q.key == a) repeat = true;
            if (!repeat) {
                mlp::g_seen[mlp::g_seen_next] = mlp::Seen{a, device, s};
                mlp::g_seen_next = (mlp::g_seen_next + 1) % mlp::kSeen;
                void *scratch = nullptr;
                CHELIS_TRY(scratch_alloc(&scratch, mlp::scratch_bytes(a), s));
                const int st = mlp::enqueue(a, scratch, s);
                scratch_free(scratch, s);
                return st;
            }
            mlp::drop(*lru);
            CHELIS_TRY(mlp::capture(a, s, device, lru));
            hit = lru;
        }
        hit->used = ++mlp::g_tick;
        exec = hit->exec;
        kernels = hit->kernels;
        // launched under the lock, so no other thread can evict (and free
        // the scratch of) this graph between lookup and launch
        CHELIS_TRY(check_cuda(cudaGraphLaunch(exec, s), "cudaGraphLaunch(mlp step)"));
    }
    g_launches += kernels;
    return CHELIS_CUDA_OK;
}
