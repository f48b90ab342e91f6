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
// One CTA owns one portfolio at a time: 10 "compute" warps and 1 "serial"
// warp.  Pass 1 streams R in 64-row chunks (coalesced loads, the next
// chunk prefetched into registers while the current one is reduced) to form
// the column sums (canonical tree over t: aligned 64-row chunks are
// subtrees) and the row dot products R.w (canonical tree over a).  Pass 2
// re-streams R (an L2 hit: the CTA read the same 129 KiB moments before),
// centres each chunk into shared memory and accumulates C^T C on the FP64
// tensor path (mma.sync m16n8k4 .f64).  Sigma is symmetric, so only the 20
// m16n8 tiles that touch the upper triangle are computed (two per compute
// warp, sharing their A fragment) and mirrored: 37.5 % fewer DMMAs.  The
// serial warp runs the sequential cumsum of R.w concurrently with pass 2;
// the compute warps synchronise among themselves with a named barrier.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;

namespace portfolio {

constexpr int A = 64;         // assets (the kernel is specialised to 64)
constexpr int CH = 64;        // rows of R per chunk
constexpr int CW = 10;        // compute warps
constexpr int CT = CW * 32;   // compute threads
constexpr int THREADS = CT + 32;
constexpr int PER_T = (CH * A + CT - 1) / CT;  // 13 doubles per compute thread per chunk

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

// barrier among the compute warps only (named barrier 1)
__device__ __forceinline__ void compute_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory");
}

// The upper-triangle tiles: warp w owns tiles (mi, nj) and (mi, nj + 1).
__device__ __forceinline__ void warp_tiles(int w, int &mi, int &nj) {
    // mi = 0: nj 0,2,4,6 | mi = 1: nj 2,4,6 | mi = 2: nj 4,6 | mi = 3: nj 6
    if (w < 4) { mi = 0; nj = 2 * w; }
    else if (w < 7) { mi = 1; nj = 2 * (w - 4) + 2; }
    else if (w < 9) { mi = 2; nj = 2 * (w - 7) + 4; }
    else { mi = 3; nj = 6; }
}

__global__ void __launch_bounds__(THREADS, 2)
    portfolio_kernel(const double *__restrict__ r_all, const double *__restrict__ w_all,
                     int64_t count, int t_len, double *__restrict__ sigma_all,
                     double *__restrict__ risk_all, double *__restrict__ cum_all) {
    extern __shared__ __align__(16) double tiles[];  // 2 x [CH * A]: staged chunks
    double *tile = tiles;                           // pass 1, Sigma.w: buffer 0
    __shared__ double wv[A];
    __shared__ double mean[A];
    __shared__ double colsum[4][A];                 // per-chunk column subtree sums
    __shared__ double segsum[4][A];                 // 16-row segment sums of a chunk
    __shared__ bool segvalid[4][A];
    __shared__ double rw[256 + 4];                  // R.w per t (t_len <= 256)
    __shared__ double u[A];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool serial = warp == CW;
    const int g = lane >> 2, tq = lane & 3;
    const int nchunks = (t_len + CH - 1) / CH;
    const double tf = static_cast<double>(t_len), tm1 = static_cast<double>(t_len - 1);
    int mi = 0, nj = 0;
    if (!serial) warp_tiles(warp, mi, nj);

    for (int64_t p = blockIdx.x; p < count; p += gridDim.x) {
        const double *R = r_all + p * t_len * A;
        __syncthreads();  // all warps: the previous portfolio is finished
        if (tid < A) wv[tid] = w_all[p * A + tid];  // read after pass 1's first barrier

        if (!serial) {
            // ---------------- pass 1: column sums and R.w ----------------
            double nxt[PER_T];
#pragma unroll
            for (int j = 0; j < PER_T; ++j) {
                const int e = tid + j * CT;
                nxt[j] = (e < CH * A && e / A < t_len) ? __ldcs(R + e) : 0.0;
            }
            for (int q = 0; q < nchunks; ++q) {
                const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
#pragma unroll
                for (int j = 0; j < PER_T; ++j) {
                    const int e = tid + j * CT;
                    if (e < CH * A) tile[e] = nxt[j];
                }
                compute_sync();
                if (q + 1 < nchunks) {
                    const double *src = R + static_cast<int64_t>(q + 1) * CH * A;
                    const int rows2 = (t_len - (q + 1) * CH) < CH ? (t_len - (q + 1) * CH) : CH;
#pragma unroll
                    for (int j = 0; j < PER_T; ++j) {
                        const int e = tid + j * CT;
                        nxt[j] = (e < CH * A && e / A < rows2) ? __ldcs(src + e) : 0.0;
                    }
                }
                if (tid < 4 * A) {
                    // column a, rows [16*seg, 16*seg + 16): an aligned 16-leaf
                    // subtree of the chunk's canonical tree, reduced pairwise
                    // (rows past the chunk end are absent leaves)
                    const int a = tid & (A - 1), seg = tid >> 6;
                    double v[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = tile[(seg * 16 + i) * A + a];
                    const int nv = rows - seg * 16;  // valid leaves of this segment
#pragma unroll
                    for (int width = 1; width < 16; width <<= 1)
#pragma unroll
                        for (int i = 0; i + width < 16; i += 2 * width)
                            v[i] = tree_pair(v[i], i < nv, v[i + width], i + width < nv);
                    segsum[seg][a] = v[0];
                    segvalid[seg][a] = nv > 0;
                }
                compute_sync();
                if (tid < A) {
                    double s4[4];
                    bool v4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) { s4[i] = segsum[i][tid]; v4[i] = segvalid[i][tid]; }
                    const double lo = tree_pair(s4[0], v4[0], s4[1], v4[1]);
                    const double hi = tree_pair(s4[2], v4[2], s4[3], v4[3]);
                    colsum[q][tid] = tree_pair(lo, v4[0], hi, v4[2]);
                }
                // R.w for each row of the chunk: lane l holds a = 2l, 2l+1
                for (int k = warp; k < rows; k += CW) {
                    const double p0 = __dmul_rn(tile[k * A + 2 * lane], wv[2 * lane]);
                    const double p1 = __dmul_rn(tile[k * A + 2 * lane + 1], wv[2 * lane + 1]);
                    const double s = warp_tree_full(__dadd_rn(p0, p1));
                    if (lane == 0) rw[q * CH + k] = s;
                }
                compute_sync();
            }
            if (tid < A) {
                double c[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) c[q] = q < nchunks ? colsum[q][tid] : 0.0;
#pragma unroll
                for (int width = 1; width < 4; width <<= 1)
#pragma unroll
                    for (int i = 0; i + width < 4; i += 2 * width)
                        c[i] = tree_pair(c[i], i < nchunks, c[i + width], i + width < nchunks);
                mean[tid] = __ddiv_rn(c[0], tf);
            }
        }
        __syncthreads();  // rw and mean complete

        if (serial) {
            // sequential prefix ([05-OP-53]): the first input is the first
            // prefix; runs while the compute warps do pass 2
            if (lane == 0) {
                double acc = rw[0];
                double *cum = cum_all + p * t_len;
                cum[0] = canon(acc);
                for (int k = 1; k < t_len; ++k) {
                    acc = __dadd_rn(acc, rw[k]);
                    cum[k] = canon(acc);
                }
            }
            continue;  // joins the next portfolio's first __syncthreads
        }

        // ---------------- pass 2: upper tiles of Sigma = C^T C ----------------
        double acc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] = 0.0;
        double nxt[PER_T];
#pragma unroll
        for (int j = 0; j < PER_T; ++j) {
            const int e = tid + j * CT;
            nxt[j] = (e < CH * A && e / A < t_len) ? __ldg(R + e) : 0.0;
        }
        // centred chunk q into buffer q & 1 (rows past the end are zeros, so
        // the k loop can always run all CH / 4 steps: they add exact zeros)
        auto stage = [&](int q) {
            const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
            double *buf = tiles + (q & 1) * CH * A;
#pragma unroll
            for (int j = 0; j < PER_T; ++j) {
                const int e = tid + j * CT;
                if (e < CH * A) {
                    const int k = e / A, a = e % A;
                    buf[sw(k, a)] = k < rows ? __dsub_rn(nxt[j], mean[a]) : 0.0;
                }
            }
        };
        auto fetch = [&](int q) {
            const double *src = R + static_cast<int64_t>(q) * CH * A;
            const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
#pragma unroll
            for (int j = 0; j < PER_T; ++j) {
                const int e = tid + j * CT;
                nxt[j] = (e < CH * A && e / A < rows) ? __ldg(src + e) : 0.0;
            }
        };
        stage(0);
        compute_sync();
        for (int q = 0; q < nchunks; ++q) {
            if (q + 1 < nchunks) fetch(q + 1);
            const double *buf = tiles + (q & 1) * CH * A;
#pragma unroll
            for (int ks = 0; ks < CH / 4; ++ks) {
                const int k = ks * 4 + tq;
                const double a0 = buf[sw(k, mi * 16 + g)];
                const double a1 = buf[sw(k, mi * 16 + g + 8)];
                const double b0 = buf[sw(k, nj * 8 + g)];
                const double b1 = buf[sw(k, (nj + 1) * 8 + g)];
                dmma(acc[0], a0, a1, b0);
                dmma(acc[1], a0, a1, b1);
            }
            // the other buffer was last read before the previous barrier
            if (q + 1 < nchunks) stage(q + 1);
            compute_sync();
        }
        // Sigma / (T-1) for the upper entries (row <= col), mirrored
        double *S = sigma_all + p * A * A;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = mi * 16 + g + h * 8;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int col = (nj + j) * 8 + 2 * tq + e;
                    if (row <= col) {
                        const double v = canon(__ddiv_rn(acc[j][2 * h + e], tm1));
                        S[row * A + col] = v;
                        S[col * A + row] = v;
                        tile[row * A + col] = v;
                        tile[col * A + row] = v;
                    }
                }
            }
        }
        compute_sync();
        // u = Sigma.w (tree over j), then w.u (tree over i), risk = sqrt
        for (int i = warp; i < A; i += CW) {
            const double p0 = __dmul_rn(tile[i * A + 2 * lane], wv[2 * lane]);
            const double p1 = __dmul_rn(tile[i * A + 2 * lane + 1], wv[2 * lane + 1]);
            const double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) u[i] = s;
        }
        compute_sync();
        if (warp == 0) {
            const double p0 = __dmul_rn(wv[2 * lane], u[2 * lane]);
            const double p1 = __dmul_rn(wv[2 * lane + 1], u[2 * lane + 1]);
            const double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) risk_all[p] = canon(__dsqrt_rn(s));
        }
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
    constexpr int smem = 2 * portfolio::CH * portfolio::A * sizeof(double);
    CHELIS_TRY(check_cuda(cudaFuncSetAttribute(portfolio::portfolio_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "cudaFuncSetAttribute(portfolio_kernel)"));
    portfolio::portfolio_kernel<<<static_cast<unsigned>(grid), portfolio::THREADS, smem, s>>>(
        r, w, count, static_cast<int>(t), sigma, risk, cum);
    g_launches++;
    CHELIS_LAUNCH_CHECK("portfolio_kernel");
    return CHELIS_CUDA_OK;
}
