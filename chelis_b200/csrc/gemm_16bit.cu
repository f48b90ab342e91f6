// gemm_16bit.cu -- bf16 / f16 GEMM with an f32 accumulator: C = round16(A . B)
// with A, B and C in the same 16-bit storage type, the products and the sum
// over k in f32, the result rounded to the storage type once (nearest-even).
// Replaces chelis_hipblas_bf16_gemm_f32_acc_row_major and
// chelis_hipblas_f16_gemm_f32_acc_row_major
// (crates/chelis-backend-hip/runtime/chelis_hip_runtime.h:92-165, which call
// hipblasGemmEx with HIPBLAS_COMPUTE_32F; spec section 5.7.1).  No benchmark
// configuration runs 16-bit matmuls; this path keeps the helper surface
// complete with warp-level tensor-core MMAs (mma.sync m16n8k16, f32
// accumulate).
//
// CTA tile 128 x 128, k-slab 32, 256 threads (8 warps, 2 x 4), warp tile
// 64 x 32 = 4 x 4 m16n8 accumulators.  Slabs go global -> registers ->
// shared memory with one slab of register prefetch; A is staged [row][k],
// B transposed to [col][k], so both fragments are 32-bit pairs along k.
// Any layout (transposes, leading dimensions, ragged edges) takes the same
// path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;

namespace g16 {

constexpr int BM = 128, BN = 128, BK = 32, THREADS = 256;
constexpr int SK = BK + 8;  // shared row length in halves (pad: conflict-free fragment reads)
constexpr int LOADS = BM * BK / THREADS;  // 16 halves per thread per operand

template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
    if constexpr (BF16)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool BF16>
__device__ __forceinline__ uint16_t round16(float v) {
    if constexpr (BF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return __half_as_ushort(__float2half_rn(v));
}

// element (r, kk) of A at a[r * sa_r + kk * sa_k]; (kk, c) of B at
// b[kk * sb_k + c * sb_n]; batch item z at + z * s*_b
template <bool BF16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm16_kernel(int64_t m, int64_t n, int64_t k, const uint16_t *__restrict__ a, int64_t sa_r,
                  int64_t sa_k, int64_t sa_b, const uint16_t *__restrict__ b, int64_t sb_k,
                  int64_t sb_n, int64_t sb_b, uint16_t *__restrict__ c, int64_t ldc, int64_t sc_b) {
    __shared__ __align__(16) uint16_t As[2][BM * SK];
    __shared__ __align__(16) uint16_t Bs[2][BN * SK];
    const int64_t z = blockIdx.z;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    a += z * sa_b;
    b += z * sb_b;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;
    const int g = lane >> 2, t = lane & 3;
    const bool a_kfast = sa_k == 1;
    const bool b_nfast = sb_n == 1;

    uint16_t ra[LOADS], rb[LOADS];
    auto load = [&](int64_t k0) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            const int64_t gr = m0 + r, gk = k0 + kk;
            ra[j] = (gr < m && gk < k) ? a[gr * sa_r + gk * sa_k] : uint16_t(0);
        }
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int cc, kk;
            if (b_nfast) { kk = e / BN; cc = e % BN; } else { cc = e / BK; kk = e % BK; }
            const int64_t gk = k0 + kk, gc = n0 + cc;
            rb[j] = (gk < k && gc < n) ? b[gk * sb_k + gc * sb_n] : uint16_t(0);
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int r, kk;
            if (a_kfast) { r = e / BK; kk = e % BK; } else { kk = e / BM; r = e % BM; }
            As[buf][r * SK + kk] = ra[j];
        }
#pragma unroll
        for (int j = 0; j < LOADS; ++j) {
            const int e = tid + j * THREADS;
            int cc, kk;
            if (b_nfast) { kk = e / BN; cc = e % BN; } else { cc = e / BK; kk = e % BK; }
            Bs[buf][cc * SK + kk] = rb[j];
        }
    };

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[i][j][q] = 0.0f;

    const int64_t nslab = (k + BK - 1) / BK;
    load(0);
    store(0);
    __syncthreads();
    for (int64_t sl = 0; sl < nslab; ++sl) {
        const int buf = static_cast<int>(sl & 1);
        if (sl + 1 < nslab) load((sl + 1) * BK);
        const uint16_t *Ab = As[buf];
        const uint16_t *Bb = Bs[buf];
#pragma unroll
        for (int kk = 0; kk < BK; kk += 16) {
            uint32_t af[4][4], bf[4][2];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = wm * 64 + i * 16 + g;
                af[i][0] = *reinterpret_cast<const uint32_t *>(&Ab[r * SK + kk + 2 * t]);
                af[i][1] = *reinterpret_cast<const uint32_t *>(&Ab[(r + 8) * SK + kk + 2 * t]);
                af[i][2] = *reinterpret_cast<const uint32_t *>(&Ab[r * SK + kk + 8 + 2 * t]);
                af[i][3] = *reinterpret_cast<const uint32_t *>(&Ab[(r + 8) * SK + kk + 8 + 2 * t]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int cc = wn * 32 + j * 8 + g;
                bf[j][0] = *reinterpret_cast<const uint32_t *>(&Bb[cc * SK + kk + 2 * t]);
                bf[j][1] = *reinterpret_cast<const uint32_t *>(&Bb[cc * SK + kk + 8 + 2 * t]);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) mma_16816<BF16>(acc[i][j], af[i], bf[j][0], bf[j][1]);
        }
        if (sl + 1 < nslab) store(buf ^ 1);
        __syncthreads();
    }

    uint16_t *cb = c + z * sc_b;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t col = n0 + wn * 32 + j * 8 + 2 * t;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int64_t row = m0 + wm * 64 + i * 16 + g + h * 8;
                if (row >= m) continue;
                if (col < n) cb[row * ldc + col] = round16<BF16>(acc[i][j][2 * h]);
                if (col + 1 < n) cb[row * ldc + col + 1] = round16<BF16>(acc[i][j][2 * h + 1]);
            }
        }
}

}  // namespace g16

int validate_gemm_args(int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                       int64_t batch, int trans_a, int trans_b);

}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_gemm16(int32_t dtype, int trans_a, int trans_b, int64_t m, int64_t n,
                                  int64_t k, const void *a, int64_t lda, int64_t stride_a,
                                  const void *b, int64_t ldb, int64_t stride_b, void *c,
                                  int64_t ldc, int64_t stride_c, int64_t batch) {
    if (dtype != CHELIS_DTYPE_BF16 && dtype != CHELIS_DTYPE_F16)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "16-bit GEMM takes bf16 or f16");
    CHELIS_TRY(validate_gemm_args(m, n, k, lda, ldb, ldc, batch, trans_a, trans_b));
    if (m == 0 || n == 0 || batch == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (batch > 65535)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "16-bit GEMM batch above 65535");
    const int64_t sa_r = trans_a ? 1 : lda, sa_k = trans_a ? lda : 1;
    const int64_t sb_k = trans_b ? 1 : ldb, sb_n = trans_b ? ldb : 1;
    dim3 grid(static_cast<unsigned>((n + g16::BN - 1) / g16::BN),
              static_cast<unsigned>((m + g16::BM - 1) / g16::BM), static_cast<unsigned>(batch));
    auto A = static_cast<const uint16_t *>(a);
    auto B = static_cast<const uint16_t *>(b);
    auto C = static_cast<uint16_t *>(c);
    if (dtype == CHELIS_DTYPE_BF16)
        g16::gemm16_kernel<true><<<grid, g16::THREADS, 0, s>>>(m, n, k, A, sa_r, sa_k, stride_a, B,
                                                              sb_k, sb_n, stride_b, C, ldc, stride_c);
    else
        g16::gemm16_kernel<false><<<grid, g16::THREADS, 0, s>>>(m, n, k, A, sa_r, sa_k, stride_a, B,
                                                               sb_k, sb_n, stride_b, C, ldc, stride_c);
    g_launches++;
    CHELIS_LAUNCH_CHECK("g16::gemm16_kernel");
    return CHELIS_CUDA_OK;
}

namespace {
int gemm16_row_major(const chelis_gpu_tensor *a, const chelis_gpu_tensor *b,
                     const chelis_gpu_tensor *out, int64_t m, int64_t n, int64_t k, chelis_dtype dt) {
    if (!a || !b || !out) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    if (a->dtype != dt || b->dtype != dt || out->dtype != dt)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "16-bit GEMM: operand dtypes differ from %d", dt);
    if (out->count == 0) return CHELIS_CUDA_OK;  // emit.rs:4806
    auto dense = [](const chelis_gpu_tensor *t, int64_t cols) {
        return t->rank >= 2 && t->strides[t->rank - 1] == 1 && t->strides[t->rank - 2] == cols;
    };
    if (!dense(a, k) || !dense(b, n) || !dense(out, n))
        return set_error(CHELIS_CUDA_ERR_DOMAIN,
                         "chelis_cuda gemm requires contiguous row-major matrix slices");
    return chelis_cuda_gemm16(dt, 0, 0, m, n, k, a->data, k, m * k, b->data, n, k * n, out->data, n,
                              m * n, 1);
}
}  // namespace

extern "C" int chelis_cuda_bf16_gemm_f32_acc_row_major(const chelis_gpu_tensor *a,
                                                       const chelis_gpu_tensor *b,
                                                       const chelis_gpu_tensor *out, int64_t m,
                                                       int64_t n, int64_t k) {
    return gemm16_row_major(a, b, out, m, n, k, CHELIS_DTYPE_BF16);
}

extern "C" int chelis_cuda_f16_gemm_f32_acc_row_major(const chelis_gpu_tensor *a,
                                                      const chelis_gpu_tensor *b,
                                                      const chelis_gpu_tensor *out, int64_t m,
                                                      int64_t n, int64_t k) {
    return gemm16_row_major(a, b, out, m, n, k, CHELIS_DTYPE_F16);
}
