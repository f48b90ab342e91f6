// crmath.cu -- entry points of the correctly rounded binary32 exp / log
// (crmath.cuh): over an array, and over a range of bit patterns (the
// exhaustive comparison with CORE-MATH walks all 2^32 inputs this way).
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "crmath.cuh"

namespace chelis {
extern std::atomic<uint64_t> g_launches;
namespace crmath {

__device__ __forceinline__ float apply(int op, float x) {
    return op == CHELIS_CRMATH_EXP ? expf_cr(x) : logf_cr(x);
}

__global__ void array_kernel(int op, const float *__restrict__ x, float *__restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = apply(op, x[i]);
}

__global__ void sweep_kernel(int op, uint32_t start, float *__restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = apply(op, __uint_as_float(start + static_cast<uint32_t>(i)));
}

}  // namespace crmath
}  // namespace chelis

using namespace chelis;

namespace {
unsigned crmath_grid(int64_t n) {
    int64_t b = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}
}  // namespace

extern "C" int chelis_cuda_crmath_f32(int32_t op, const float *x, float *y, int64_t n) {
    if (op != CHELIS_CRMATH_EXP && op != CHELIS_CRMATH_LOG)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "crmath: unknown op %d", op);
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "crmath: negative count");
    if (n == 0) return CHELIS_CUDA_OK;
    crmath::array_kernel<<<crmath_grid(n), 256, 0, current_stream()>>>(op, x, y, n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("crmath::array_kernel");
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_crmath_sweep_f32(int32_t op, uint32_t start, int64_t n, float *y) {
    if (op != CHELIS_CRMATH_EXP && op != CHELIS_CRMATH_LOG)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "crmath: unknown op %d", op);
    if (n < 0 || n > (int64_t(1) << 32))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "crmath: count outside [0, 2^32]");
    if (n == 0) return CHELIS_CUDA_OK;
    crmath::sweep_kernel<<<crmath_grid(n), 256, 0, current_stream()>>>(op, start, y, n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("crmath::sweep_kernel");
    return CHELIS_CUDA_OK;
}
