// chain_noalloc.cu -- the fused-chain adjoint without any device allocation.
//
// chelis_cuda_chain_bwd needs scratch for its per-CTA dgamma / dbeta
// partials and takes it from the library's stream-ordered pool.  Some
// callers cannot let a library allocate: a host that sized its device arena
// up front from the program's peak-bytes figure and hands every buffer out
// itself, or one running under a driver-allocation ban.  For them this entry
// keeps the scratch in one file-scope device array of fixed size, so a call
// allocates nothing: no cudaMalloc / cudaMallocAsync / cudaFree, no pool,
// no torch allocator.
//
// Limits and rules (also in include/chelis_cuda.h):
//  * hidden <= 4096 (the array holds the partials of up to 296 CTAs, two per
//    SM of a 148-SM B200, for rows of up to 4096 floats); larger rows are
//    rejected.  The grid is two CTAs per SM, capped at 296: on a 148-SM B200
//    it is the allocating entry's grid, so dgamma / dbeta come out bit for
//    bit as chelis_cuda_chain_bwd's; on a GPU with more SMs the cap keeps
//    the grid at 296 and dgamma / dbeta group their rows differently (they
//    then agree within f32 rounding).
//  * The array lives in every GPU that loads the library until the process
//    exits (10 MiB each).
//  * Every call shares the one array per device.  Calls that overlap on the
//    GPU (two streams, or two host threads) race on it and must be ordered
//    by the caller.  Each call overwrites all of the scratch it reads, so
//    nothing has to start at zero and nothing carries over between calls.
//  * The first call on a device looks up the array's device address with
//    that device current (cudaGetSymbolAddress); make that first call before
//    any stream capture.  The address is kept for the life of the process: a
//    device reset (cudaDeviceReset, or anything else that tears down the
//    primary context) invalidates it, so do not call this entry on a device
//    after resetting it.
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace chelis {
namespace noalloc {

constexpr int kGrid = 296;                                    // most adjoint CTAs per call
constexpr int64_t kMaxHidden = 4096;                          // widest admitted row
constexpr int64_t kScratchFloats = 10ll * 1024 * 1024 / 4;    // 10 MiB
constexpr int64_t kRB = rows::COL_RB;                         // column-block height
// partials for dgamma and dbeta, then one level of column-block sums
static_assert(2 * kGrid * kMaxHidden + ((kGrid + kRB - 1) / kRB) * kMaxHidden <= kScratchFloats,
              "scratch array too small for its stated limits");
static_assert((kGrid + kRB - 1) / kRB <= kRB, "two column-block levels must cover the grid");

static __device__ __align__(256) float g_chain_bwd_scratch[kScratchFloats];

// Host-side device address of the array, per device, resolved once per
// device (std::call_once, so concurrent first calls from several host
// threads do not race).  In host code the symbol's name is only a host
// stand-in, never a device address.
static float *g_scratch_ptr[64] = {};
static int g_scratch_status[64] = {};
static std::once_flag g_scratch_once[64];

static int scratch_for_current_device(float **out) {
    int dev = 0;
    CHELIS_TRY(current_device_checked(&dev));
    if (dev >= 64) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "device index %d", dev);
    std::call_once(g_scratch_once[dev], [dev] {
        void *p = nullptr;
        g_scratch_status[dev] = check_cuda(cudaGetSymbolAddress(&p, g_chain_bwd_scratch),
                                           "cudaGetSymbolAddress(chain_bwd scratch)");
        g_scratch_ptr[dev] = static_cast<float *>(p);
    });
    if (g_scratch_status[dev] != CHELIS_CUDA_OK || !g_scratch_ptr[dev])
        return set_error(CHELIS_CUDA_ERR_CUDA,
                         "chain_bwd_noalloc: device address of the scratch array unavailable");
    *out = g_scratch_ptr[dev];
    return CHELIS_CUDA_OK;
}

// Canonical column sums of a [rows, cols] block (rows <= kRB * kRB) through
// caller scratch `tmp` of ceil(rows / kRB) * cols floats: aligned blocks of
// kRB rows, then one block over the block sums (every aligned power-of-two
// block is a subtree of the canonical tree, so the result is the same as
// the allocating path's).
static int col_sum_scratch(const float *x, int64_t rows, int64_t cols, float *out, float *tmp,
                           cudaStream_t s) {
    const unsigned cb = static_cast<unsigned>((cols + 127) / 128);
    if (rows <= kRB) {
        rows::col_block_kernel<<<dim3(cb, 1), 128, 0, s>>>(x, rows, cols, rows, out);
        g_launches++;
        CHELIS_LAUNCH_CHECK("col_block_kernel");
        return CHELIS_CUDA_OK;
    }
    const int64_t nb = (rows + kRB - 1) / kRB;
    rows::col_block_kernel<<<dim3(cb, static_cast<unsigned>(nb)), 128, 0, s>>>(
        x, rows, cols, kRB, tmp);
    g_launches++;
    CHELIS_LAUNCH_CHECK("col_block_kernel");
    rows::col_block_kernel<<<dim3(cb, 1), 128, 0, s>>>(tmp, nb, cols, nb, out);
    g_launches++;
    CHELIS_LAUNCH_CHECK("col_block_kernel");
    return CHELIS_CUDA_OK;
}

}  // namespace noalloc
}  // namespace chelis

extern "C" int chelis_cuda_chain_bwd_noalloc(const float *x, const float *gamma,
                                             const float *beta, float eps, uint64_t key,
                                             float rate, int64_t rows, int64_t hidden,
                                             int64_t index_base, const float *row_stats,
                                             float *dx, float *dgamma, float *dbeta) {
    using namespace chelis;
    using namespace chelis::noalloc;
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    CHELIS_TRY(check_rate(rate));
    if (hidden == 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    if (hidden > kMaxHidden)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                         "chelis_cuda_chain_bwd_noalloc admits hidden <= %lld (got %lld); use "
                         "chelis_cuda_chain_bwd",
                         static_cast<long long>(kMaxHidden), static_cast<long long>(hidden));
    float *scratch = nullptr;
    CHELIS_TRY(scratch_for_current_device(&scratch));
    cudaStream_t s = current_stream();
    if (rows == 0) {
        CHELIS_TRY(check_cuda(cudaMemsetAsync(dgamma, 0, hidden * sizeof(float), s), "memset"));
        return check_cuda(cudaMemsetAsync(dbeta, 0, hidden * sizeof(float), s), "memset");
    }
    // two CTAs per SM (the allocating entry's grid), at most kGrid
    const int64_t cap = std::min<int64_t>(static_cast<int64_t>(sm_count()) * 2, kGrid);
    const int grid = static_cast<int>(rows < cap ? rows : cap);
    ChainParams p = make_chain_params(x, gamma, beta, eps, key, rate, rows, hidden, index_base);
    p.stats_in = row_stats;
    p.dx = dx;
    p.dgamma_part = scratch;
    p.dbeta_part = scratch + static_cast<int64_t>(grid) * hidden;
    p.rows_per_cta = static_cast<int>((rows + grid - 1) / grid);
    float *tmp = scratch + 2 * static_cast<int64_t>(grid) * hidden;
    CHELIS_TRY(launch_chain_bwd<kRowThreads>(p, grid, s));
    CHELIS_TRY(col_sum_scratch(p.dgamma_part, grid, hidden, dgamma, tmp, s));
    CHELIS_TRY(col_sum_scratch(p.dbeta_part, grid, hidden, dbeta, tmp, s));
    return CHELIS_CUDA_OK;
}
