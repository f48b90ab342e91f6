// shutdown.cu -- chelis_cuda_shutdown: give back everything the library
// created on its own (the reference's runtime has no counterpart: its HIP
// entries create and destroy a hipBLAS handle and JIT modules on every
// call, chelis_hip_runtime.h:171-267, 409-485).
#include "common.cuh"

namespace chelis {
int release_pools();
namespace fusedjit { int release_all(); }
namespace hostgemm { void release_streams(); }
void mlp_release_graphs();
}  // namespace chelis
namespace grad_reduce { void release_events(); }
namespace block_timing { void release(); }

extern "C" int chelis_cuda_shutdown(void) {
    using namespace chelis;
    int st = CHELIS_CUDA_OK;
    auto keep_first = [&st](int s) {
        if (st == CHELIS_CUDA_OK && s != CHELIS_CUDA_OK) st = s;
    };
    keep_first(chelis_cuda_dp_finalize(0));
    block_timing::release();
    mlp_release_graphs();
    grad_reduce::release_events();
    hostgemm::release_streams();
    keep_first(fusedjit::release_all());
    keep_first(release_pools());
    return st;
}
