// portfolio.cu -- the vmap'd covariance / risk program in f64.
//
// vectorize_axis0 (crates/chelis-ir-core/src/vmap.rs:9-56) gives every node
// of the per-portfolio graph a leading batch axis; per portfolio p:
//   mean[a]  = sum_t R[t,a] / T              (tier2.rs:1183-1245)
//   C        = R - mean
//   Sigma    = matmul(transpose(C), C) / (T-1)
//   risk     = sqrt(matmul(w, matmul(Sigma, w)))
//   cum[t]   = cumsum_t(matmul(R, w))         ([05-OP-53])
//
// One CTA (256 threads) owns one portfolio at a time.  Pass 1 streams R in
// 64-row chunks (coalesced 16-double-per-thread loads) to form the column
// sums (canonical tree over t: aligned 64-row chunks are subtrees) and the
// row dot products R.w (canonical tree over a).  Pass 2 re-streams R (an
// L2 hit: the CTA read the same 129 KiB moments before), centres each
// chunk into shared memory and accumulates C^T C on the FP64 tensor path
// (mma.sync m16n8k4 .f64), 8 warps x (16 x 32) of the 64 x 64 result.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;

namespace portfolio {

constexpr int THREADS = 256;
constexpr int A = 64;       // assets (the kernel is specialised to 64)
constexpr int CH = 64;      // rows of R per chunk
constexpr int PER_T = CH * A / THREADS;  // 16 doubles per thread per chunk

__device__ __forceinline__ int sw(int k, int a) { return k * A + (a ^ ((k & 3) << 2)); }

__device__ __forceinline__ void dmma(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%0,%1,%2,%3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

__device__ __forceinline__ double canon(double x) {
    return isnan(x) ? __longlong_as_double(0x7ff8000000000000ll) : x;
}

__global__ void __launch_bounds__(THREADS, 2)
    portfolio_kernel(const double *__restrict__ r_all, const double *__restrict__ w_all,
                     int64_t count, int t_len, double *__restrict__ sigma_all,
                     double *__restrict__ risk_all, double *__restrict__ cum_all) {
    __shared__ __align__(16) double tile[CH * A];   // staged chunk (raw or centred)
    __shared__ double wv[A];
    __shared__ double mean[A];
    __shared__ double colsum[8][A];                 // per-chunk column subtree sums
    __shared__ double rw[256 + 4];                  // R.w per t (t_len <= 256)
    __shared__ double u[A];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int nchunks = (t_len + CH - 1) / CH;
    const double tf = static_cast<double>(t_len), tm1 = static_cast<double>(t_len - 1);

    for (int64_t p = blockIdx.x; p < count; p += gridDim.x) {
        const double *R = r_all + p * t_len * A;
        if (tid < A) wv[tid] = w_all[p * A + tid];
        __syncthreads();

        // ---------------- pass 1: column sums and R.w ----------------
        for (int q = 0; q < nchunks; ++q) {
            const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
            const double *src = R + static_cast<int64_t>(q) * CH * A;
#pragma unroll
            for (int j = 0; j < PER_T; ++j) {
                const int e = tid + j * THREADS;
                tile[e] = (e / A) < rows ? __ldg(src + e) : 0.0;
            }
            __syncthreads();
            if (tid < A) {
                // carry tree over this chunk's rows (aligned block: a subtree)
                double lv[7];
                int cnt = 0;
                for (int k = 0; k < rows; ++k) {
                    double carry = tile[k * A + tid];
                    bool active = true;
#pragma unroll
                    for (int d = 0; d < 7; ++d) {
                        if (active) {
                            if ((cnt >> d) & 1) carry = __dadd_rn(lv[d], carry);
                            else { lv[d] = carry; active = false; }
                        }
                    }
                    ++cnt;
                }
                double tot = 0.0;
                bool found = false;
#pragma unroll
                for (int d = 0; d < 7; ++d)
                    if ((cnt >> d) & 1) { tot = found ? __dadd_rn(lv[d], tot) : lv[d]; found = true; }
                colsum[q][tid] = tot;
            }
            // R.w for each row of the chunk: lane l holds a = 2l, 2l+1
            for (int k = warp; k < rows; k += THREADS / 32) {
                const double p0 = __dmul_rn(tile[k * A + 2 * lane], wv[2 * lane]);
                const double p1 = __dmul_rn(tile[k * A + 2 * lane + 1], wv[2 * lane + 1]);
                double s = __dadd_rn(p0, p1);
                s = warp_tree_full(s);
                if (lane == 0) rw[q * CH + k] = s;
            }
            __syncthreads();
        }
        if (tid < A) {
            // canonical tree over the chunk sums (pass by pass)
            double c[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) c[q] = q < nchunks ? colsum[q][tid] : 0.0;
#pragma unroll
            for (int width = 1; width < 8; width <<= 1)
#pragma unroll
                for (int i = 0; i + width < 8; i += 2 * width)
                    c[i] = tree_pair(c[i], i < nchunks, c[i + width], i + width < nchunks);
            mean[tid] = __ddiv_rn(c[0], tf);
        }
        if (tid == A) {
            // sequential prefix ([05-OP-53]): the first input is the first prefix
            double acc = rw[0];
            double *cum = cum_all + p * t_len;
            cum[0] = canon(acc);
            for (int k = 1; k < t_len; ++k) {
                acc = __dadd_rn(acc, rw[k]);
                cum[k] = canon(acc);
            }
        }
        __syncthreads();

        // ---------------- pass 2: Sigma = C^T C ----------------
        const int mi = warp >> 1;        // 16-row block of Sigma (a index)
        const int nj0 = (warp & 1) * 4;  // first of 4 8-column blocks
        double acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] = 0.0;
        for (int q = 0; q < nchunks; ++q) {
            const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
            const double *src = R + static_cast<int64_t>(q) * CH * A;
#pragma unroll
            for (int j = 0; j < PER_T; ++j) {
                const int e = tid + j * THREADS;
                const int k = e / A, a = e % A;
                tile[sw(k, a)] = k < rows ? __dsub_rn(__ldg(src + e), mean[a]) : 0.0;
            }
            __syncthreads();
            const int ksteps = (rows + 3) / 4;
            for (int ks = 0; ks < ksteps; ++ks) {
                const int k = ks * 4 + tq;
                const double a0 = tile[sw(k, mi * 16 + g)];
                const double a1 = tile[sw(k, mi * 16 + g + 8)];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const double b0 = tile[sw(k, (nj0 + j) * 8 + g)];
                    dmma(acc[j], a0, a1, b0);
                }
            }
            __syncthreads();
        }
        // Sigma / (T-1): to global and to shared memory (for Sigma.w)
        double *S = sigma_all + p * A * A;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = (nj0 + j) * 8 + 2 * tq;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = mi * 16 + g + h * 8;
                const double v0 = canon(__ddiv_rn(acc[j][2 * h], tm1));
                const double v1 = canon(__ddiv_rn(acc[j][2 * h + 1], tm1));
                *reinterpret_cast<double2 *>(S + row * A + col) = make_double2(v0, v1);
                tile[row * A + col] = v0;
                tile[row * A + col + 1] = v1;
            }
        }
        __syncthreads();
        // u = Sigma.w (tree over j), then w.u (tree over i), risk = sqrt
        for (int i = warp; i < A; i += THREADS / 32) {
            const double p0 = __dmul_rn(tile[i * A + 2 * lane], wv[2 * lane]);
            const double p1 = __dmul_rn(tile[i * A + 2 * lane + 1], wv[2 * lane + 1]);
            double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) u[i] = s;
        }
        __syncthreads();
        if (warp == 0) {
            const double p0 = __dmul_rn(wv[2 * lane], u[2 * lane]);
            const double p1 = __dmul_rn(wv[2 * lane + 1], u[2 * lane + 1]);
            const double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) risk_all[p] = canon(__dsqrt_rn(s));
        }
        __syncthreads();
    }
}

}  // namespace portfolio
}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_portfolio_f64(const double *r, const double *w, int64_t count,
                                         int64_t t, int64_t a, double *sigma, double *risk,
                                         double *cum) {
    if (count < 0 || t < 0 || a < 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in portfolio at i64");
    if (a != portfolio::A || t < 2 || t > 256)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                         "portfolio kernel admits a = 64 assets and 2 <= t <= 256 (got a=%lld t=%lld)",
                         static_cast<long long>(a), static_cast<long long>(t));
    if (count == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    int64_t grid = static_cast<int64_t>(sm_count()) * 2;
    if (grid > count) grid = count;
    portfolio::portfolio_kernel<<<static_cast<unsigned>(grid), portfolio::THREADS, 0, s>>>(
        r, w, count, static_cast<int>(t), sigma, risk, cum);
    g_launches++;
    CHELIS_LAUNCH_CHECK("portfolio_kernel");
    return CHELIS_CUDA_OK;
}
