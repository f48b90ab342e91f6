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
// One CTA carries two portfolios at a time on two warp groups.  The 4
// "stream" warps run pass 1 of portfolio p+1: the column sums (one thread per
// asset, 16 rows at a time from HBM, each aligned 16-row run a subtree of the
// canonical tree over t, pushed through a carry tree), the row dot products
// R.w (one warp per row, canonical tree over a) and then the sequential
// cumsum of R.w ([05-OP-53]).  Meanwhile the 10 "tensor" warps run pass 2 of
// portfolio p: they re-stream R (an L2 hit: pass 1 read it one portfolio
// earlier), centre each 64-row chunk into shared memory and accumulate C^T C
// on the FP64 tensor path (mma.sync m16n8k4 .f64).  Sigma is symmetric, so
// only the 20 m16n8 tiles that touch the upper triangle are computed (two per
// tensor warp, sharing their A fragment) and mirrored: 37.5 % fewer DMMAs.
// The groups meet once per portfolio (__syncthreads); the tensor warps
// synchronise among themselves with named barrier 1, the stream warps with
// named barrier 2.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;

namespace portfolio {

constexpr int A = 64;         // assets (the kernel is specialised to 64)
constexpr int CH = 32;        // rows of R per ring slot
constexpr int NST = 4;        // ring slots (CH * A doubles each)
constexpr int CW = 10;        // tensor warps
constexpr int CT = CW * 32;   // tensor threads
constexpr int SW = 4;         // stream warps
constexpr int THREADS = CT + SW * 32;
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

// barriers among the tensor warps only (1) and among the stream warps only (2)
__device__ __forceinline__ void tensor_sync() { asm volatile("bar.sync 1, %0;" ::"n"(CT) : "memory"); }
__device__ __forceinline__ void stream_sync() { asm volatile("bar.sync 2, %0;" ::"n"(SW * 32) : "memory"); }

// The upper-triangle tiles: warp w owns tiles (mi, nj) and (mi, nj + 1).
__device__ __forceinline__ void warp_tiles(int w, int &mi, int &nj) {
    // mi = 0: nj 0,2,4,6 | mi = 1: nj 2,4,6 | mi = 2: nj 4,6 | mi = 3: nj 6
    if (w < 4) { mi = 0; nj = 2 * w; }
    else if (w < 7) { mi = 1; nj = 2 * (w - 4) + 2; }
    else if (w < 9) { mi = 2; nj = 2 * (w - 7) + 4; }
    else { mi = 3; nj = 6; }
}

constexpr int BR = 16;  // rows of a stream block

struct Shared {
    double mean[2][A];   // per portfolio slot (portfolio i uses slot i & 1)
    double wv[2][A];
    double rw[2][256];   // R.w halves of the portfolio in pass 1: assets [0, 32) and [32, 64)
    double colpart[A];   // column sums of rows [128, t)
    double u[A];
    double ring[2][2][BR * A];  // [half][stage]: blocks of R in flight for pass 1
};

// barriers of one half of the stream warps (ids 3 and 4, 64 threads)
__device__ __forceinline__ void half_sync(int half) {
    if (half) asm volatile("bar.sync 4, 64;" ::: "memory");
    else asm volatile("bar.sync 3, 64;" ::: "memory");
}

// Pass 1 of portfolio p on the stream warps: mean, w, R.w and its cumsum.
// Threads st and st + 64 take asset a = st & 63; the first 64 threads rows
// [0, 128), the others rows [128, t) -- the aligned 128-leaf subtree of the
// canonical tree over t and the rest of the tree -- 16 rows at a time,
// copied into shared memory asynchronously (cp.async) one block ahead.  The
// same rows give R.w: the products of row t over a warp's 32 assets pair up
// by the xor butterfly (aligned subtrees of the tree over a), and the two
// warps' halves meet in the cumsum.
__device__ __forceinline__ void stream_pass(const double *__restrict__ R, const double *__restrict__ w,
                                            int t_len, double *__restrict__ cum, Shared &sh, int slot,
                                            int st) {
    const int lane = st & 31, a = st & (A - 1), half = st >> 6, wa = a >> 5, hs = st & 63;
    if (st < A) sh.wv[slot][st] = w[st];
    stream_sync();  // wv visible
    const double wa_v = sh.wv[slot][a];
    const int split = t_len > 128 ? 128 : t_len;
    const int r0 = half ? split : 0, r1 = half ? t_len : split;
    // copy rows [t0, t0 + BR) (those below r1) into ring stage `stg`: 16-byte
    // pieces, 8 per thread of the half
    auto copy = [&](int t0, int stg) {
        double *dst = sh.ring[half][stg];
#pragma unroll
        for (int j = 0; j < BR * A / 2 / 64; ++j) {
            const int e = hs + j * 64;           // 16-byte piece
            const int row = e / (A / 2), col = (e % (A / 2)) * 2;
            const bool ok = t0 + row < r1;
            dmma::cp_async16(dst + row * A + col, ok ? R + (t0 + row) * A + col : R, ok);
        }
        dmma::cp_async_commit();
    };
    double level[8];
    int64_t count = 0;
    double tail = 0.0;
    bool has_tail = false;
    if (r0 < r1) copy(r0, 0);
    for (int t0 = r0, stg = 0; t0 < r1; t0 += BR, stg ^= 1) {
        const int nv = (r1 - t0) < BR ? (r1 - t0) : BR;
        dmma::cp_async_wait<0>();
        half_sync(half);  // block t0 landed for every thread; stage stg ^ 1 is free
        if (t0 + BR < r1) copy(t0 + BR, stg ^ 1);
        const double *blk = sh.ring[half][stg];
        double v[BR];
#pragma unroll
        for (int i = 0; i < BR; ++i) v[i] = blk[i * A + a];
        // R.w of rows t0 .. t0 + BR: this warp's 32 products per row, tree
        // over a by recursive halving -- at level L a lane keeps BR >> L rows
        // and adds its partner's (lane ^ 2^(L-1)) aligned 2^L-lane subtree
        // of them; after four levels lane l holds row l & 15, and one more
        // xor-16 step completes the 32-lane subtree.
        {
            double q[BR];
#pragma unroll
            for (int i = 0; i < BR; ++i) q[i] = __dmul_rn(v[i], wa_v);
#pragma unroll
            for (int lvl = 0; lvl < 4; ++lvl) {
                const int off = 1 << lvl, n = BR >> (lvl + 1);  // rows kept after this level
                const bool upper = (lane & off) != 0;          // keeps the upper half of its rows
#pragma unroll
                for (int i = 0; i < n; ++i) {
                    const double send = upper ? q[i] : q[i + n];
                    const double mine = upper ? q[i + n] : q[i];
                    q[i] = __dadd_rn(mine, __shfl_xor_sync(0xffffffffu, send, off));
                }
            }
            const double s = __dadd_rn(q[0], __shfl_xor_sync(0xffffffffu, q[0], 16));
            // lane l now holds the row whose index bits are lane bits 0..3
            // (each level kept the half named by that lane bit)
            const int row = ((lane & 1) << 3) | ((lane & 2) << 1) | ((lane & 4) >> 1) | ((lane & 8) >> 3);
            if (lane < 16 && row < nv) sh.rw[wa][t0 + row] = s;
        }
        // column subtree of these rows (pairwise, absent rows pass through)
#pragma unroll
        for (int width = 1; width < BR; width <<= 1)
#pragma unroll
            for (int i = 0; i + width < BR; i += 2 * width)
                v[i] = tree_pair(v[i], i < nv, v[i + width], i + width < nv);
        if (nv == BR) {
            double carry = v[0];
            int depth = 0;
            for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)
                carry = __dadd_rn(level[depth], carry);
            level[depth] = carry;
        } else {
            tail = v[0];
            has_tail = true;
        }
    }
    double total = tail;
    bool found = has_tail;
    int depth = 0;
    for (int64_t remaining = count; remaining; remaining >>= 1, ++depth)
        if (remaining & 1) {
            total = found ? __dadd_rn(level[depth], total) : level[depth];
            found = true;
        }
    if (half) sh.colpart[a] = total;
    stream_sync();  // colpart and both R.w halves complete; the ring is idle
    if (half == 0) {
        // rows [0, 128) are a complete subtree when t > 128: on the left
        const double s = t_len > 128 ? __dadd_rn(total, sh.colpart[a]) : total;
        sh.mean[slot][a] = __ddiv_rn(s, static_cast<double>(t_len));
    } else if (hs == 0) {
        // sequential prefix of R.w = (assets [0,32) + assets [32,64)) per row
        double acc = __dadd_rn(sh.rw[0][0], sh.rw[1][0]);
        cum[0] = canon(acc);
        for (int k = 1; k < t_len; ++k) {
            acc = __dadd_rn(acc, __dadd_rn(sh.rw[0][k], sh.rw[1][k]));
            cum[k] = canon(acc);
        }
    }
}

__global__ void __launch_bounds__(THREADS, 2)
    portfolio_kernel(const double *__restrict__ r_all, const double *__restrict__ w_all,
                     int64_t count, int t_len, double *__restrict__ sigma_all,
                     double *__restrict__ risk_all, double *__restrict__ cum_all) {
    extern __shared__ __align__(16) double tiles[];  // NST x [CH * A]: the pass-2 ring
    __shared__ Shared sh;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool tensor = warp < CW;
    const int g = lane >> 2, tq = lane & 3;
    const int nchunks = (t_len + CH - 1) / CH;
    const double tm1 = static_cast<double>(t_len - 1);
    int mi = 0, nj = 0;
    if (tensor) warp_tiles(warp, mi, nj);
    const int64_t stride = gridDim.x;

    // portfolio i of this CTA is blockIdx.x + i * gridDim.x; pass 1 of
    // portfolio i + 1 overlaps pass 2 of portfolio i
    int64_t p = blockIdx.x;
    if (!tensor && p < count)
        stream_pass(r_all + p * t_len * A, w_all + p * A, t_len, cum_all + p * t_len, sh, 0, tid - CT);
    __syncthreads();
    for (int slot = 0; p < count; p += stride, slot ^= 1) {
        if (!tensor) {
            const int64_t pn = p + stride;
            if (pn < count)
                stream_pass(r_all + pn * t_len * A, w_all + pn * A, t_len, cum_all + pn * t_len, sh,
                            slot ^ 1, tid - CT);
            __syncthreads();
            continue;
        }
        const double *R = r_all + p * t_len * A;
        const double *mean = sh.mean[slot];
        const double *wv = sh.wv[slot];
        // ---------------- pass 2: upper tiles of Sigma = C^T C ----------------
        // R streams through a ring of NST chunks of CH rows in shared memory
        // by cp.async (an L2 hit: pass 1 read it one portfolio earlier), NST - 1
        // chunks in flight; the fragments are centred as they are read
        // (C = R - mean, the same one rounding as a centred copy), rows past
        // t are exact zeros.
        double acc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[j][q] = 0.0;
        const int ca0 = mi * 16 + g, ca1 = ca0 + 8, cb0 = nj * 8 + g, cb1 = cb0 + 8;
        const double m0 = mean[ca0], m1 = mean[ca1], n0 = mean[cb0], n1 = mean[cb1];
        auto copy = [&](int q) {  // chunk q into ring slot q % NST (empty group past the end)
            if (q < nchunks) {
                double *dst = tiles + (q % NST) * CH * A;
                const int rows = (t_len - q * CH) < CH ? (t_len - q * CH) : CH;
                const double *src = R + static_cast<int64_t>(q) * CH * A;
#pragma unroll
                for (int j = 0; j < (CH * A / 2 + CT - 1) / CT; ++j) {
                    const int e = tid + j * CT;  // 16-byte piece
                    if (e < CH * A / 2) {
                        const int k = e / (A / 2), c = (e % (A / 2)) * 2;
                        const bool ok = k < rows;
                        dmma::cp_async16(dst + sw(k, c), ok ? src + k * A + c : src, ok);
                    }
                }
            }
            dmma::cp_async_commit();
        };
#pragma unroll
        for (int q = 0; q < NST - 1; ++q) copy(q);
        for (int q = 0; q < nchunks; ++q) {
            dmma::cp_async_wait<NST - 2>();
            tensor_sync();  // chunk q landed for all; slot (q - 1) % NST is free
            copy(q + NST - 1);
            const double *buf = tiles + (q % NST) * CH * A;
            const int k0 = q * CH;
#pragma unroll
            for (int ks = 0; ks < CH / 4; ++ks) {
                const int k = ks * 4 + tq;
                const bool in = k0 + k < t_len;
                const double a0 = in ? __dsub_rn(buf[sw(k, ca0)], m0) : 0.0;
                const double a1 = in ? __dsub_rn(buf[sw(k, ca1)], m1) : 0.0;
                const double b0 = in ? __dsub_rn(buf[sw(k, cb0)], n0) : 0.0;
                const double b1 = in ? __dsub_rn(buf[sw(k, cb1)], n1) : 0.0;
                dmma(acc[0], a0, a1, b0);
                dmma(acc[1], a0, a1, b1);
            }
        }
        dmma::cp_async_wait<0>();
        tensor_sync();  // every warp is done with the ring: Sigma may take slots 0 and 1
        // Sigma / (T-1) for the upper entries (row <= col), mirrored
        double *S = sigma_all + p * A * A;
        double *tile = tiles;  // Sigma, for Sigma.w (ring slots 0 and 1)
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
        tensor_sync();
        // u = Sigma.w (tree over j), then w.u (tree over i), risk = sqrt
        for (int i = warp; i < A; i += CW) {
            const double p0 = __dmul_rn(tile[i * A + 2 * lane], wv[2 * lane]);
            const double p1 = __dmul_rn(tile[i * A + 2 * lane + 1], wv[2 * lane + 1]);
            const double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) sh.u[i] = s;
        }
        tensor_sync();
        if (warp == 0) {
            const double p0 = __dmul_rn(wv[2 * lane], sh.u[2 * lane]);
            const double p1 = __dmul_rn(wv[2 * lane + 1], sh.u[2 * lane + 1]);
            const double s = warp_tree_full(__dadd_rn(p0, p1));
            if (lane == 0) risk_all[p] = canon(__dsqrt_rn(s));
        }
        __syncthreads();  // both groups: portfolio p done, p + stride's pass 1 done
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
    constexpr int smem = portfolio::NST * portfolio::CH * portfolio::A * sizeof(double);
    CHELIS_TRY(check_cuda(cudaFuncSetAttribute(portfolio::portfolio_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "cudaFuncSetAttribute(portfolio_kernel)"));
    portfolio::portfolio_kernel<<<static_cast<unsigned>(grid), portfolio::THREADS, smem, s>>>(
        r, w, count, static_cast<int>(t), sigma, risk, cum);
    g_launches++;
    CHELIS_LAUNCH_CHECK("portfolio_kernel");
    return CHELIS_CUDA_OK;
}
