// gemm_f64.cu -- f64 GEMM for the matmul lowering with an f64 accumulator
// (spec/05-risc-primitives.md:4962-5000) on the FP64 tensor path (DMMA,
// mma.sync m16n8k4 .f64) or the CUDA cores' FP64 FMA pipe (FFMA), chosen per
// product (dgemm_pick).  Replaces chelis_hipblas_dgemm_*_row_major
// (chelis_hip_runtime.h:271-404).
//
// DMMA kernels:
// CTA tile 128 x 128, k-slab 16, 256 threads = 8 warps in a 2 x 4 grid,
// warp tile 64 x 32 = 4 x 4 m16n8 accumulators (64 doubles per thread).
// Tiles are staged global -> registers -> shared memory with one slab of
// register prefetch (double-buffered shared memory), so any layout, leading
// dimension and ragged edge is handled by the same code path.  Shared
// memory rows are XOR-swizzled at 16-byte granularity so that the DMMA
// fragment reads of a half-warp hit 16 distinct bank pairs.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int gemm_mode();
int dgemm_kernel_choice();
template <typename T>
int launch_exact_gemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const T *a,
                      int64_t lda, int64_t stride_a, const T *b, int64_t ldb, int64_t stride_b,
                      T *c, int64_t ldc, int64_t stride_c, int64_t batch, cudaStream_t s);
int validate_gemm_args(int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                       int64_t batch, int trans_a, int trans_b);

namespace dmma {

constexpr int BM = 128, BN = 128, BK = 16, THREADS = 256;
constexpr int LOADS = BM * BK / THREADS;  // 8 doubles per thread per operand
constexpr int SMEM_BYTES = 2 * (BM * BK + BK * BN) * 8;  // 64 KiB, double-buffered

// element offsets inside the swizzled tiles
__device__ __forceinline__ int a_off(int r, int k) { return r * BK + (k ^ ((r & 3) << 2)); }
__device__ __forceinline__ int b_off(int k, int n) { return k * BN + (n ^ ((k & 3) << 2)); }

__device__ __forceinline__ void dmma_16x8x4(double (&d)[4], double a0, double a1, double b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, "
        "{%0,%1,%2,%3};"
        : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
        : "d"(a0), "d"(a1), "d"(b0));
}

__global__ void __launch_bounds__(THREADS, 1)
    dgemm_kernel(int64_t m, int64_t n, int64_t k, const double *__restrict__ a, int64_t sa_r,
                 int64_t sa_k, int64_t sa_b, const double *__restrict__ b, int64_t sb_k,
                 int64_t sb_n, int64_t sb_b, double *__restrict__ c, int64_t ldc,
                 int64_t sc_b) {
    extern __shared__ __align__(16) double dsmem[];
    double (*As)[BM * BK] = reinterpret_cast<double (*)[BM * BK]>(dsmem);
    double (*Bs)[BK * BN] = reinterpret_cast<double (*)[BK * BN]>(dsmem + 2 * BM * BK);

    const int64_t bz = blockIdx.z;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    a += bz * sa_b;
    b += bz * sb_b;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2;  // 0..1 -> 64-row half
    const int wn = warp & 3;   // 0..3 -> 32-col quarter
    const int g = lane >> 2, t = lane & 3;
    const bool a_kfast = (sa_k == 1);
    const bool b_nfast = (sb_n == 1);

    double ra[LOADS], rb[LOADS];
    auto load_slab = [&](int64_t k0) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            const int64_t gr = m0 + r, gk = k0 + kk;
            ra[j] = (gr < m && gk < k) ? a[gr * sa_r + gk * sa_k] : 0.0;
        }
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int kk, nn;
            if (b_nfast) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            const int64_t gk = k0 + kk, gn = n0 + nn;
            rb[j] = (gk < k && gn < n) ? b[gk * sb_k + gn * sb_n] : 0.0;
        }
    };
    auto store_slab = [&](int buf) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            As[buf][a_off(r, kk)] = ra[j];
        }
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int kk, nn;
            if (b_nfast) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            Bs[buf][b_off(kk, nn)] = rb[j];
        }
    };

    double acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0;

    const int64_t nslab = (k + BK - 1) / BK;
    load_slab(0);
    store_slab(0);
    __syncthreads();
    for (int64_t s = 0; s < nslab; ++s) {
        const int buf = static_cast<int>(s & 1);
        if (s + 1 < nslab) load_slab((s + 1) * BK);
        const double *Ab = As[buf];
        const double *Bb = Bs[buf];
#pragma unroll
        for (int kk = 0; kk < BK; kk += 4) {
            double af[4][2], bf[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = wm * 64 + i * 16 + g;
                af[i][0] = Ab[a_off(r, kk + t)];
                af[i][1] = Ab[a_off(r + 8, kk + t)];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[j] = Bb[b_off(kk + t, wn * 32 + j * 8 + g)];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_16x8x4(acc[i][j], af[i][0], af[i][1], bf[j]);
        }
        if (s + 1 < nslab) {
            store_slab(buf ^ 1);
        }
        __syncthreads();
    }

    double *cb = c + bz * sc_b;
    const bool vec = ((ldc & 1) == 0) && ((reinterpret_cast<uintptr_t>(cb) & 15) == 0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + wn * 32 + j * 8 + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t row = m0 + wm * 64 + i * 16 + g + h * 8;
                if (row >= m) continue;
                double *dst = cb + row * ldc + col;
                const double v0 = acc[i][j][2 * h], v1 = acc[i][j][2 * h + 1];
                if (vec && col + 1 < n) {
                    *reinterpret_cast<double2 *>(dst) = make_double2(v0, v1);
                } else {
                    if (col < n) dst[0] = v0;
                    if (col + 1 < n) dst[1] = v1;
                }
            }
        }
    }
}


// ---------------------------------------------------------------------------
// Row-major fast path: both operands contiguous along their tile rows (A
// along k, B along n), even extents and leading dimensions, 16-byte aligned
// bases.  Slabs stream global -> shared memory with cp.async (16-byte
// chunks, zero-filled past the matrix edge) through a 4-deep ring, so three
// slabs are in flight while the DMMAs consume the fourth; no registers are
// spent on staging.  Same tile, swizzle and fragment code as dgemm_kernel.
// ---------------------------------------------------------------------------
constexpr int ASTAGES = 4;
constexpr int ASYNC_SMEM_BYTES = ASTAGES * (BM * BK + BK * BN) * 8;  // 128 KiB

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    dgemm_async_kernel(int64_t m, int64_t n, int64_t k, const double *__restrict__ a, int64_t lda,
                       int64_t sa_b, const double *__restrict__ b, int64_t ldb, int64_t sb_b,
                       double *__restrict__ c, int64_t ldc, int64_t sc_b) {
    extern __shared__ __align__(16) double dsmem[];
    double *As = dsmem;                          // [ASTAGES][BM * BK]
    double *Bs = dsmem + ASTAGES * BM * BK;      // [ASTAGES][BK * BN]

    const int64_t bz = blockIdx.z;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    a += bz * sa_b;
    b += bz * sb_b;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;
    const int g = lane >> 2, t = lane & 3;

    // 16-byte chunks per slab: A 128 rows x 8 chunks, B 16 rows x 64 chunks
    auto issue = [&](int64_t slab, int buf) {
        const int64_t k0 = slab * BK;
        double *as = As + buf * BM * BK;
        double *bs = Bs + buf * BK * BN;
#pragma unroll
        for (int j = 0; j < (BM * BK / 2) / THREADS; ++j) {
            const int e = tid + j * THREADS;
            const int r = e >> 3, kk = (e & 7) * 2;
            const int64_t gr = m0 + r, gk = k0 + kk;
            const bool ok = gr < m && gk < k;
            cp_async16(as + a_off(r, kk), ok ? a + gr * lda + gk : a, ok);
        }
#pragma unroll
        for (int j = 0; j < (BK * BN / 2) / THREADS; ++j) {
            const int e = tid + j * THREADS;
            const int kk = e >> 6, nn = (e & 63) * 2;
            const int64_t gk = k0 + kk, gn = n0 + nn;
            const bool ok = gk < k && gn < n;
            cp_async16(bs + b_off(kk, nn), ok ? b + gk * ldb + gn : b, ok);
        }
    };

    double acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0;

    const int64_t nslab = (k + BK - 1) / BK;
#pragma unroll
    for (int s = 0; s < ASTAGES - 1; ++s) {
        if (s < nslab) issue(s, s);
        cp_async_commit();
    }
    for (int64_t s = 0; s < nslab; ++s) {
        cp_async_wait<ASTAGES - 2>();  // slab s has landed (this thread's chunks)
        __syncthreads();               // ... everyone's; and slab s - 1 is consumed
        if (s + ASTAGES - 1 < nslab) issue(s + ASTAGES - 1, static_cast<int>((s + ASTAGES - 1) % ASTAGES));
        cp_async_commit();
        const int buf = static_cast<int>(s % ASTAGES);
        const double *Ab = As + buf * BM * BK;
        const double *Bb = Bs + buf * BK * BN;
#pragma unroll
        for (int kk = 0; kk < BK; kk += 4) {
            double af[4][2], bf[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = wm * 64 + i * 16 + g;
                af[i][0] = Ab[a_off(r, kk + t)];
                af[i][1] = Ab[a_off(r + 8, kk + t)];
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) bf[j] = Bb[b_off(kk + t, wn * 32 + j * 8 + g)];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) dmma_16x8x4(acc[i][j], af[i][0], af[i][1], bf[j]);
        }
    }
    cp_async_wait<0>();

    double *cb = c + bz * sc_b;
    const bool vec = ((ldc & 1) == 0) && ((reinterpret_cast<uintptr_t>(cb) & 15) == 0);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + wn * 32 + j * 8 + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t row = m0 + wm * 64 + i * 16 + g + h * 8;
                if (row >= m) continue;
                double *dst = cb + row * ldc + col;
                const double v0 = acc[i][j][2 * h], v1 = acc[i][j][2 * h + 1];
                if (vec && col + 1 < n) {
                    *reinterpret_cast<double2 *>(dst) = make_double2(v0, v1);
                } else {
                    if (col < n) dst[0] = v0;
                    if (col + 1 < n) dst[1] = v1;
                }
            }
        }
    }
}

}  // namespace dmma

// ---------------------------------------------------------------------------
// FFMA path: the FP64 FMA pipe of the CUDA cores (on B200 its peak equals
// the DMMA pipe's).  CTA tile BM x BN, k-slab 8, each thread a TM x TN
// register tile split into four quadrants (rows r0 + i and r0 + BM/2 + i,
// columns likewise) so that the shared-memory reads of a warp are
// broadcasts (A) and 16-byte vectors over consecutive columns (B).  Slabs
// are staged global -> registers -> shared memory with one slab of register
// prefetch, any layout and ragged edge, as the DMMA register-staged path.
// Each output is one chain of fma over k in increasing k.
// ---------------------------------------------------------------------------
namespace ffma {

constexpr int BK = 8;
constexpr int PAD = 2;  // doubles of padding per shared row (transposing stores)

template <int BM, int BN, int TM, int TN>
struct Cfg {
    static constexpr int TX = BN / TN, TY = BM / TM, THREADS = TX * TY;
    static constexpr int A_LOADS = BM * BK / THREADS, B_LOADS = BK * BN / THREADS;
    static constexpr int SMEM_BYTES = 2 * BK * ((BM + PAD) + (BN + PAD)) * 8;
    static_assert(TM % 2 == 0 && TN % 2 == 0, "quadrant split needs even micro tiles");
    static_assert(A_LOADS * THREADS == BM * BK && B_LOADS * THREADS == BK * BN, "load split");
};

template <int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(Cfg<BM, BN, TM, TN>::THREADS)
    dgemm_kernel(int64_t m, int64_t n, int64_t k, const double *__restrict__ a, int64_t sa_r,
                 int64_t sa_k, int64_t sa_b, const double *__restrict__ b, int64_t sb_k,
                 int64_t sb_n, int64_t sb_b, double *__restrict__ c, int64_t ldc,
                 int64_t sc_b) {
    using C = Cfg<BM, BN, TM, TN>;
    constexpr int AS = BM + PAD, BS = BN + PAD;
    constexpr int HM = TM / 2, HN = TN / 2;
    __shared__ __align__(16) double As[2][BK * AS];
    __shared__ __align__(16) double Bs[2][BK * BS];

    const int64_t bz = blockIdx.z;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    a += bz * sa_b;
    b += bz * sb_b;
    const int tid = threadIdx.x;
    const int tx = tid % C::TX, ty = tid / C::TX;
    const bool a_kfast = (sa_k == 1);
    const bool b_nfast = (sb_n == 1);

    double ra[C::A_LOADS], rb[C::B_LOADS];
    auto load_slab = [&](int64_t k0) {
#pragma unroll
        for (int j = 0; j < C::A_LOADS; ++j) {
            const int e = tid + j * C::THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            const int64_t gr = m0 + r, gk = k0 + kk;
            ra[j] = (gr < m && gk < k) ? a[gr * sa_r + gk * sa_k] : 0.0;
        }
#pragma unroll
        for (int j = 0; j < C::B_LOADS; ++j) {
            const int e = tid + j * C::THREADS;
            int kk, nn;
            if (b_nfast) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            const int64_t gk = k0 + kk, gn = n0 + nn;
            rb[j] = (gk < k && gn < n) ? b[gk * sb_k + gn * sb_n] : 0.0;
        }
    };
    auto store_slab = [&](int buf) {
#pragma unroll
        for (int j = 0; j < C::A_LOADS; ++j) {
            const int e = tid + j * C::THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            As[buf][kk * AS + r] = ra[j];
        }
#pragma unroll
        for (int j = 0; j < C::B_LOADS; ++j) {
            const int e = tid + j * C::THREADS;
            int kk, nn;
            if (b_nfast) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
            Bs[buf][kk * BS + nn] = rb[j];
        }
    };

    double acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0;

    const int ra0 = ty * HM, rb0 = BM / 2 + ty * HM;  // this thread's two row groups
    const int ca0 = tx * HN, cb0 = BN / 2 + tx * HN;  // and two column groups
    const int64_t nslab = (k + BK - 1) / BK;
    load_slab(0);
    store_slab(0);
    __syncthreads();
    for (int64_t s = 0; s < nslab; ++s) {
        const int buf = static_cast<int>(s & 1);
        if (s + 1 < nslab) load_slab((s + 1) * BK);
        const double *Ab = As[buf];
        const double *Bb = Bs[buf];
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            double av[TM], bv[TN];
#pragma unroll
            for (int i = 0; i < HM; i += 2) {
                const double2 lo = *reinterpret_cast<const double2 *>(&Ab[kk * AS + ra0 + i]);
                const double2 hi = *reinterpret_cast<const double2 *>(&Ab[kk * AS + rb0 + i]);
                av[i] = lo.x; av[i + 1] = lo.y;
                av[HM + i] = hi.x; av[HM + i + 1] = hi.y;
            }
#pragma unroll
            for (int j = 0; j < HN; j += 2) {
                const double2 lo = *reinterpret_cast<const double2 *>(&Bb[kk * BS + ca0 + j]);
                const double2 hi = *reinterpret_cast<const double2 *>(&Bb[kk * BS + cb0 + j]);
                bv[j] = lo.x; bv[j + 1] = lo.y;
                bv[HN + j] = hi.x; bv[HN + j + 1] = hi.y;
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fma(av[i], bv[j], acc[i][j]);
        }
        if (s + 1 < nslab) store_slab(buf ^ 1);
        __syncthreads();
    }

    double *cb = c + bz * sc_b;
    const bool vec = ((ldc & 1) == 0) && ((reinterpret_cast<uintptr_t>(cb) & 15) == 0);
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int64_t row = m0 + (i < HM ? ra0 + i : rb0 + i - HM);
        if (row >= m) continue;
#pragma unroll
        for (int jh = 0; jh < 2; ++jh) {
#pragma unroll
            for (int j = 0; j < HN; j += 2) {
                const int64_t col = n0 + (jh ? cb0 : ca0) + j;
                double *dst = cb + row * ldc + col;
                const double v0 = acc[i][jh * HN + j], v1 = acc[i][jh * HN + j + 1];
                if (vec && col + 1 < n) {
                    *reinterpret_cast<double2 *>(dst) = make_double2(v0, v1);
                } else {
                    if (col < n) dst[0] = v0;
                    if (col + 1 < n) dst[1] = v1;
                }
            }
        }
    }
}

}  // namespace ffma

// FFMA launch: 128 x 128 tiles where they fill the GPU, else 64 x 64.
int launch_dgemm_ffma(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const double *a,
                      int64_t lda, int64_t stride_a, const double *b, int64_t ldb,
                      int64_t stride_b, double *c, int64_t ldc, int64_t stride_c, int64_t batch,
                      cudaStream_t s) {
    const int64_t sa_r = trans_a ? 1 : lda, sa_k = trans_a ? lda : 1;
    const int64_t sb_k = trans_b ? 1 : ldb, sb_n = trans_b ? ldb : 1;
    const int64_t big_tiles = ((m + 127) / 128) * ((n + 127) / 128) * batch;
    if (big_tiles >= sm_count()) {
        using C = ffma::Cfg<128, 128, 8, 8>;
        dim3 grid(static_cast<unsigned>((n + 127) / 128), static_cast<unsigned>((m + 127) / 128),
                  static_cast<unsigned>(batch));
        ffma::dgemm_kernel<128, 128, 8, 8><<<grid, C::THREADS, 0, s>>>(
            m, n, k, a, sa_r, sa_k, stride_a, b, sb_k, sb_n, stride_b, c, ldc, stride_c);
        g_launches++;
        CHELIS_LAUNCH_CHECK("ffma::dgemm_kernel<128,128>");
        return CHELIS_CUDA_OK;
    }
    using C = ffma::Cfg<64, 64, 4, 4>;
    dim3 grid(static_cast<unsigned>((n + 63) / 64), static_cast<unsigned>((m + 63) / 64),
              static_cast<unsigned>(batch));
    ffma::dgemm_kernel<64, 64, 4, 4><<<grid, C::THREADS, 0, s>>>(
        m, n, k, a, sa_r, sa_k, stride_a, b, sb_k, sb_n, stride_b, c, ldc, stride_c);
    g_launches++;
    CHELIS_LAUNCH_CHECK("ffma::dgemm_kernel<64,64>");
    return CHELIS_CUDA_OK;
}

// True when the DMMA streaming path (cp.async slab ring) takes the product.
bool dmma_streams(int trans_a, int trans_b, int64_t n, int64_t k, const double *a, int64_t lda,
                  int64_t stride_a, const double *b, int64_t ldb, int64_t stride_b,
                  int64_t batch) {
    return !trans_a && !trans_b && (k % 2 == 0) && (n % 2 == 0) && (lda % 2 == 0) &&
           (ldb % 2 == 0) && (batch == 1 || (stride_a % 2 == 0 && stride_b % 2 == 0)) &&
           (reinterpret_cast<uintptr_t>(a) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0;
}

// Kernel for one f64 product: the calling thread's / process's choice, and
// under CHELIS_CUDA_DGEMM_AUTO the per-shape rule.  Measured on B200 (one
// GPU, TFLOP/s): the FFMA pipe tops out at half the DMMA pipe (FFMA 18.0,
// DMMA 32.1 at 8192^3; transposed A at 4096^3: DMMA register-staged 27.5,
// FFMA 18.0), so DMMA takes every product whose 128 x 128 tiles number at
// least the SM count; below that FFMA's 64 x 64 tiles (four times the CTAs)
// win (512^3: FFMA 4.4, DMMA 3.2; 256 x 256 x 4096: 1.21 vs 0.87; 777 x 1333
// x 999: 12.9 vs 11.0).
int dgemm_pick(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const double *a,
               int64_t lda, int64_t stride_a, const double *b, int64_t ldb, int64_t stride_b,
               int64_t batch) {
    (void)trans_a, (void)trans_b, (void)k, (void)a, (void)lda, (void)stride_a, (void)b, (void)ldb,
        (void)stride_b;
    const int choice = dgemm_kernel_choice();
    if (choice != CHELIS_CUDA_DGEMM_AUTO) return choice;
    const int64_t tiles = ((m + 127) / 128) * ((n + 127) / 128) * batch;
    return tiles >= sm_count() ? CHELIS_CUDA_DGEMM_DMMA : CHELIS_CUDA_DGEMM_FFMA;
}

int launch_dgemm_dmma(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const double *a,
                      int64_t lda, int64_t stride_a, const double *b, int64_t ldb,
                      int64_t stride_b, double *c, int64_t ldc, int64_t stride_c, int64_t batch,
                      cudaStream_t s) {
    const int64_t sa_r = trans_a ? 1 : lda, sa_k = trans_a ? lda : 1;
    const int64_t sb_k = trans_b ? 1 : ldb, sb_n = trans_b ? ldb : 1;
    dim3 grid(static_cast<unsigned>((n + dmma::BN - 1) / dmma::BN),
              static_cast<unsigned>((m + dmma::BM - 1) / dmma::BM),
              static_cast<unsigned>(batch));
    const bool fast =
        dmma_streams(trans_a, trans_b, n, k, a, lda, stride_a, b, ldb, stride_b, batch);
    if (fast) {
        static uint64_t done = 0;
        CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(dmma::dgemm_async_kernel),
                                    dmma::ASYNC_SMEM_BYTES, &done,
                                    "cudaFuncSetAttribute(dgemm_async_kernel)"));
        dmma::dgemm_async_kernel<<<grid, dmma::THREADS, dmma::ASYNC_SMEM_BYTES, s>>>(
            m, n, k, a, lda, stride_a, b, ldb, stride_b, c, ldc, stride_c);
        g_launches++;
        CHELIS_LAUNCH_CHECK("dgemm_async_kernel(dmma)");
        return CHELIS_CUDA_OK;
    }
    static uint64_t done_sync = 0;
    CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(dmma::dgemm_kernel), dmma::SMEM_BYTES,
                                &done_sync, "cudaFuncSetAttribute(dgemm_kernel)"));
    dmma::dgemm_kernel<<<grid, dmma::THREADS, dmma::SMEM_BYTES, s>>>(m, n, k, a, sa_r, sa_k, stride_a, b, sb_k,
                                                       sb_n, stride_b, c, ldc, stride_c);
    g_launches++;
    CHELIS_LAUNCH_CHECK("dgemm_kernel(dmma)");
    return CHELIS_CUDA_OK;
}

}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_dgemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                                 const double *a, int64_t lda, int64_t stride_a, const double *b,
                                 int64_t ldb, int64_t stride_b, double *c, int64_t ldc,
                                 int64_t stride_c, int64_t batch) {
    CHELIS_TRY(validate_gemm_args(m, n, k, lda, ldb, ldc, batch, trans_a, trans_b));
    if (m == 0 || n == 0 || batch == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (k == 0) {
        for (int64_t bb = 0; bb < batch; ++bb)
            CHELIS_TRY(check_cuda(cudaMemset2DAsync(c + bb * stride_c, ldc * sizeof(double), 0,
                                                    n * sizeof(double), m, s),
                                  "cudaMemset2DAsync"));
        return CHELIS_CUDA_OK;
    }
    if (gemm_mode() == CHELIS_CUDA_GEMM_EXACT_TREE)
        return launch_exact_gemm<double>(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb,
                                         stride_b, c, ldc, stride_c, batch, s);
    if (dgemm_pick(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb, stride_b, batch) ==
        CHELIS_CUDA_DGEMM_FFMA)
        return launch_dgemm_ffma(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb, stride_b, c,
                                 ldc, stride_c, batch, s);
    return launch_dgemm_dmma(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb, stride_b, c,
                             ldc, stride_c, batch, s);
}

extern "C" int chelis_cuda_dgemm_kernel_for(int trans_a, int trans_b, int64_t m, int64_t n,
                                            int64_t k, int64_t batch) {
    const int64_t lda = trans_a ? m : k, ldb = trans_b ? k : n;
    return dgemm_pick(trans_a, trans_b, m, n, k, nullptr, lda, m * k, nullptr, ldb, k * n, batch);
}
