// host_gemm.cu -- matmul on HOST buffers with the PCIe copies overlapped.
//
// The reference evaluates a matmul whose operands live in host arrays by
// uploading both, running the library GEMM and downloading the result, one
// step after the other (crates/chelis-backend-hip/src/lib.rs execute path ->
// chelis_hipblas_sgemm_row_major, runtime/chelis_hip_runtime.h:48-78).  Here
// the same call is a three-stream pipeline on the device:
//
//   upload stream    B in row chunks, then A in row panels (cudaMemcpy2DAsync)
//   compute stream   (the caller's stream) 3xTF32 split of each chunk as it
//                    lands, then one tcgen05 GEMM per row panel of C
//   download stream  each finished panel of C back to the host
//
// so the host link carries A while the tensor cores work on earlier panels
// and C streams back in the other direction.  Only the first operand chunk
// and the last panel's GEMM + read-back are exposed.  Host buffers should be
// page-locked for the copies to run asynchronously; pageable memory gives
// the same results with serialised copies.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace chelis {
namespace hostgemm {

struct DeviceStreams {
    bool ready = false;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev_start = nullptr, ev_up = nullptr, ev_comp = nullptr, ev_down = nullptr;
    std::mutex lock;
    struct Empty {};
    DeviceStreams &operator=(Empty) {  // back to the unset state (the lock is kept)
        ready = false;
        up = down = nullptr;
        ev_start = ev_up = ev_comp = ev_down = nullptr;
        return *this;
    }
};
DeviceStreams g_dev[64];

int streams_for_current(DeviceStreams **out) {
    int d = 0;
    CHELIS_TRY(current_device_checked(&d));
    if (d >= 64) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "device ordinal beyond 63");
    DeviceStreams &ds = g_dev[d];
    if (!ds.ready) {
        CHELIS_TRY(check_cuda(cudaStreamCreateWithFlags(&ds.up, cudaStreamNonBlocking),
                              "cudaStreamCreate(upload)"));
        CHELIS_TRY(check_cuda(cudaStreamCreateWithFlags(&ds.down, cudaStreamNonBlocking),
                              "cudaStreamCreate(download)"));
        cudaEvent_t *evs[4] = {&ds.ev_start, &ds.ev_up, &ds.ev_comp, &ds.ev_down};
        for (cudaEvent_t *e : evs)
            CHELIS_TRY(check_cuda(cudaEventCreateWithFlags(e, cudaEventDisableTiming),
                                  "cudaEventCreate"));
        ds.ready = true;
    }
    *out = &ds;
    return CHELIS_CUDA_OK;
}

// Destroy the upload / download streams and their events on every device.
void release_streams() {
    int prev = 0;
    cudaGetDevice(&prev);
    for (int d = 0; d < 64; ++d) {
        DeviceStreams &ds = g_dev[d];
        std::lock_guard<std::mutex> lock(ds.lock);
        if (!ds.ready) continue;
        cudaSetDevice(d);
        cudaStreamSynchronize(ds.up);
        cudaStreamSynchronize(ds.down);
        cudaStreamDestroy(ds.up);
        cudaStreamDestroy(ds.down);
        for (cudaEvent_t e : {ds.ev_start, ds.ev_up, ds.ev_comp, ds.ev_down}) cudaEventDestroy(e);
        ds = DeviceStreams::Empty();
    }
    cudaSetDevice(prev);
}

// `to` waits for everything enqueued on `from` so far (one reusable event:
// a wait captures the event's most recent record at enqueue time).
int order(cudaStream_t from, cudaStream_t to, cudaEvent_t ev) {
    CHELIS_TRY(check_cuda(cudaEventRecord(ev, from), "cudaEventRecord"));
    return check_cuda(cudaStreamWaitEvent(to, ev, 0), "cudaStreamWaitEvent");
}

template <typename T>
int upload_rows(T *dst, const T *src, int64_t ld_src, int64_t cols, int64_t r0, int64_t r1,
                cudaStream_t s) {
    if (r1 <= r0 || cols == 0) return CHELIS_CUDA_OK;
    return check_cuda(cudaMemcpy2DAsync(dst + r0 * cols, cols * sizeof(T), src + r0 * ld_src,
                                        ld_src * sizeof(T), cols * sizeof(T), r1 - r0,
                                        cudaMemcpyHostToDevice, s),
                      "cudaMemcpy2DAsync(upload)");
}

// 3xTF32 split of stored rows [r0, r1) of a dense device operand: both
// layouts map stored row r to split row r (K-major: operand rows; MN-major:
// k rows).
int split_range(const OperandPlan &p, const float *src, int64_t cols, int64_t r0, int64_t r1,
                float *hi, float *lo, cudaStream_t s) {
    if (r1 <= r0) return CHELIS_CUDA_OK;
    OperandPlan q = p;
    if (p.mn) {
        q.k = r1 - r0;
    } else {
        q.rows = r1 - r0;
    }
    // a dense stored row-major block with stride `cols`: K-major sources are
    // K-contiguous (sk = 1), MN-major sources MN-contiguous (sr = 1)
    const int64_t sr = p.mn ? 1 : cols, sk = p.mn ? cols : 1;
    return launch_split_plan(q, src + r0 * cols, sr, sk, 0, 1, hi + r0 * p.cp, lo + r0 * p.cp, s);
}

inline int64_t panel_rows_for(int64_t m) {
    // about 16 panels, each a whole number of 128-row GEMM tiles
    int64_t p = (m + 15) / 16;
    p = (p + 127) / 128 * 128;
    return p < m ? p : m;
}

template <typename T>
struct Panels;

// f32: 3xTF32 tensor-core path (or the exact-tree mode on the CUDA cores)
template <>
struct Panels<float> {
    GemmPlan g;
    bool exact;
    float *ahi = nullptr, *alo = nullptr, *bhi = nullptr, *blo = nullptr;
    size_t split_bytes(int ta, int tb, int64_t m, int64_t n, int64_t k) {
        exact = gemm_mode() == CHELIS_CUDA_GEMM_EXACT_TREE;
        g = plan_gemm(ta, tb, m, n, k, ta ? m : k, tb ? k : n, 1);
        return exact ? 0 : g.bytes();
    }
    void carve(float *base) {
        ahi = base;
        alo = ahi + g.a.floats;
        bhi = alo + g.a.floats;
        blo = bhi + g.b.floats;
    }
    int on_b_rows(const float *bd, int64_t cols, int64_t r0, int64_t r1, cudaStream_t s) {
        return exact ? CHELIS_CUDA_OK : split_range(g.b, bd, cols, r0, r1, bhi, blo, s);
    }
    int on_a_rows(const float *ad, int64_t cols, int64_t r0, int64_t r1, cudaStream_t s) {
        return exact ? CHELIS_CUDA_OK : split_range(g.a, ad, cols, r0, r1, ahi, alo, s);
    }
    int gemm_panel(int ta, int tb, int64_t m, int64_t n, int64_t k, const float *ad,
                   const float *bd, float *cd, int64_t m0, int64_t m1, cudaStream_t s) {
        const int64_t lda = ta ? m : k, ldb = tb ? k : n;
        const float *ap = ta ? ad + m0 : ad + m0 * k;
        if (exact)
            return launch_exact_gemm<float>(ta, tb, m1 - m0, n, k, ap, lda, 0, bd, ldb, 0,
                                            cd + m0 * n, n, 0, 1, s);
        OperandPlan pa = g.a;
        pa.rows = m1 - m0;
        // K-major A: rows m0.. of [m][kp]; MN-major A: columns m0.. of [k][mp]
        const int64_t off = g.a.mn ? m0 : m0 * g.a.cp;
        return sgemm_3xtf32_main(pa, ahi + off, alo + off, g.b, bhi, blo, m1 - m0, n, k,
                                 cd + m0 * n, n, 0, 1, s);
    }
};

// f64: DMMA tensor-core path (or the exact-tree mode)
template <>
struct Panels<double> {
    bool exact;
    size_t split_bytes(int, int, int64_t, int64_t, int64_t) {
        exact = gemm_mode() == CHELIS_CUDA_GEMM_EXACT_TREE;
        return 0;
    }
    void carve(double *) {}
    int on_b_rows(const double *, int64_t, int64_t, int64_t, cudaStream_t) { return CHELIS_CUDA_OK; }
    int on_a_rows(const double *, int64_t, int64_t, int64_t, cudaStream_t) { return CHELIS_CUDA_OK; }
    int gemm_panel(int ta, int tb, int64_t m, int64_t n, int64_t k, const double *ad,
                   const double *bd, double *cd, int64_t m0, int64_t m1, cudaStream_t s) {
        const int64_t lda = ta ? m : k, ldb = tb ? k : n;
        const double *ap = ta ? ad + m0 : ad + m0 * k;
        if (exact)
            return launch_exact_gemm<double>(ta, tb, m1 - m0, n, k, ap, lda, 0, bd, ldb, 0,
                                             cd + m0 * n, n, 0, 1, s);
        return launch_dgemm_dmma(ta, tb, m1 - m0, n, k, ap, lda, 0, bd, ldb, 0, cd + m0 * n, n, 0,
                                 1, s);
    }
};

template <typename T>
int pipeline_one(DeviceStreams &ds, Panels<T> &pl, int ta, int tb, int64_t m, int64_t n, int64_t k,
                 const T *a, int64_t lda, const T *b, int64_t ldb, T *c, int64_t ldc, T *ad,
                 T *bd, T *cd, cudaStream_t s) {
    // stored shapes of the host operands
    const int64_t ra = ta ? k : m, ca = ta ? m : k;
    const int64_t rb = tb ? n : k, cb = tb ? k : n;
    // B in 8 row chunks, each split as soon as it lands
    const int64_t bchunk = (rb + 7) / 8;
    for (int64_t r0 = 0; r0 < rb; r0 += bchunk) {
        const int64_t r1 = r0 + bchunk < rb ? r0 + bchunk : rb;
        CHELIS_TRY(upload_rows(bd, b, ldb, cb, r0, r1, ds.up));
        CHELIS_TRY(order(ds.up, s, ds.ev_up));
        CHELIS_TRY(pl.on_b_rows(bd, cb, r0, r1, s));
    }
    const int64_t pr = panel_rows_for(m);
    if (ta) {
        // stored A is k x m: its rows are k, so every panel needs all of it
        const int64_t achunk = (ra + 7) / 8;
        for (int64_t r0 = 0; r0 < ra; r0 += achunk) {
            const int64_t r1 = r0 + achunk < ra ? r0 + achunk : ra;
            CHELIS_TRY(upload_rows(ad, a, lda, ca, r0, r1, ds.up));
            CHELIS_TRY(order(ds.up, s, ds.ev_up));
            CHELIS_TRY(pl.on_a_rows(ad, ca, r0, r1, s));
        }
    }
    for (int64_t m0 = 0; m0 < m; m0 += pr) {
        const int64_t m1 = m0 + pr < m ? m0 + pr : m;
        if (!ta) {
            CHELIS_TRY(upload_rows(ad, a, lda, ca, m0, m1, ds.up));
            CHELIS_TRY(order(ds.up, s, ds.ev_up));
            CHELIS_TRY(pl.on_a_rows(ad, ca, m0, m1, s));
        }
        CHELIS_TRY(pl.gemm_panel(ta, tb, m, n, k, ad, bd, cd, m0, m1, s));
        CHELIS_TRY(order(s, ds.down, ds.ev_comp));
        CHELIS_TRY(check_cuda(cudaMemcpy2DAsync(c + m0 * ldc, ldc * sizeof(T), cd + m0 * n,
                                                n * sizeof(T), n * sizeof(T), m1 - m0,
                                                cudaMemcpyDeviceToHost, ds.down),
                              "cudaMemcpy2DAsync(download)"));
    }
    return CHELIS_CUDA_OK;
}

template <typename T>
int gemm_host(int ta, int tb, int64_t m, int64_t n, int64_t k, const T *a, int64_t lda,
              int64_t stride_a, const T *b, int64_t ldb, int64_t stride_b, T *c, int64_t ldc,
              int64_t stride_c, int64_t batch) {
    CHELIS_TRY(validate_gemm_args(m, n, k, lda, ldb, ldc, batch, ta, tb));
    if (m == 0 || n == 0 || batch == 0) return CHELIS_CUDA_OK;
    if ((m > 0 && !c) || (k > 0 && (!a || !b)))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    cudaStream_t s = current_stream();
    if (k == 0) {
        // empty contraction: exact zero, written once earlier stream work is done
        CHELIS_TRY(check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize"));
        for (int64_t bb = 0; bb < batch; ++bb)
            for (int64_t i = 0; i < m; ++i)
                for (int64_t j = 0; j < n; ++j) c[bb * stride_c + i * ldc + j] = T(0);
        return CHELIS_CUDA_OK;
    }
    DeviceStreams *dsp = nullptr;
    CHELIS_TRY(streams_for_current(&dsp));
    DeviceStreams &ds = *dsp;
    std::lock_guard<std::mutex> guard(ds.lock);

    Panels<T> pl;
    const size_t a_bytes = static_cast<size_t>(m * k) * sizeof(T);
    const size_t b_bytes = static_cast<size_t>(k * n) * sizeof(T);
    const size_t c_bytes = static_cast<size_t>(m * n) * sizeof(T);
    const size_t round = 256;
    auto up256 = [&](size_t x) { return (x + round - 1) / round * round; };
    const size_t split = pl.split_bytes(ta, tb, m, n, k);
    void *buf = nullptr;
    CHELIS_TRY(scratch_alloc(&buf, up256(a_bytes) + up256(b_bytes) + up256(c_bytes) + split, s));
    unsigned char *p = static_cast<unsigned char *>(buf);
    T *ad = reinterpret_cast<T *>(p);
    T *bd = reinterpret_cast<T *>(p + up256(a_bytes));
    T *cd = reinterpret_cast<T *>(p + up256(a_bytes) + up256(b_bytes));
    pl.carve(reinterpret_cast<T *>(p + up256(a_bytes) + up256(b_bytes) + up256(c_bytes)));

    int st = CHELIS_CUDA_OK;
    for (int64_t bb = 0; bb < batch && st == CHELIS_CUDA_OK; ++bb) {
        // the upload stream may overwrite the device operands only after the
        // compute stream is done with the previous item (and with the
        // allocation); the compute stream may overwrite C only after the
        // previous read-back
        st = order(s, ds.up, ds.ev_start);
        if (st == CHELIS_CUDA_OK) st = order(ds.down, s, ds.ev_down);
        if (st == CHELIS_CUDA_OK)
            st = pipeline_one<T>(ds, pl, ta, tb, m, n, k, a + bb * stride_a, lda,
                                 b + bb * stride_b, ldb, c + bb * stride_c, ldc, ad, bd, cd, s);
    }
    // join: the caller's stream completes only after every copy; the buffer
    // is released in stream order after that (also on an error path)
    order(ds.up, s, ds.ev_up);
    order(ds.down, s, ds.ev_down);
    scratch_free(buf, s);
    return st;
}

}  // namespace hostgemm
}  // namespace chelis

extern "C" int chelis_cuda_sgemm_host(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                                      const float *a, int64_t lda, int64_t stride_a,
                                      const float *b, int64_t ldb, int64_t stride_b, float *c,
                                      int64_t ldc, int64_t stride_c, int64_t batch) {
    return chelis::hostgemm::gemm_host<float>(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb,
                                              stride_b, c, ldc, stride_c, batch);
}

extern "C" int chelis_cuda_dgemm_host(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                                      const double *a, int64_t lda, int64_t stride_a,
                                      const double *b, int64_t ldb, int64_t stride_b, double *c,
                                      int64_t ldc, int64_t stride_c, int64_t batch) {
    return chelis::hostgemm::gemm_host<double>(trans_a, trans_b, m, n, k, a, lda, stride_a, b,
                                               ldb, stride_b, c, ldc, stride_c, batch);
}
