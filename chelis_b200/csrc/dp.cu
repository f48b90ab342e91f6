// dp.cu -- data-parallel plumbing behind the C ABI: one NCCL communicator
// per process (one process per GPU), the sum all-reduce of a flat gradient
// buffer on the caller's stream, and the contiguous batch shard of a vmap'd
// or data-parallel program.  The reference has no multi-GPU lane; the shard
// rule follows its vmap axis (crates/chelis-ir-core/src/vmap.rs:9-56).
//
// NCCL is opened at run time (dlopen of libnccl.so.2; the process's already
// loaded copy when torch brought one), so the library itself links no NCCL
// and every other entry works where NCCL is absent; the dp entries then
// return CHELIS_CUDA_ERR_UNSUPPORTED.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace chelis {
namespace {

struct Nccl {
    bool tried = false, ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = -1, device = -1;
};

std::mutex g_dp_mu;
Nccl g_nccl;

int nccl_load() {
    if (g_nccl.tried) {
        return g_nccl.ok ? CHELIS_CUDA_OK
                         : set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
    }
    g_nccl.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "NCCL (libnccl.so.2) is not available");
    auto sym = [&](const char *name) { return dlsym(h, name); };
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(sym("ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(sym("ncclCommInitRank"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(sym("ncclAllReduce"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(sym("ncclCommDestroy"));
    g_nccl.comm_abort = reinterpret_cast<decltype(g_nccl.comm_abort)>(sym("ncclCommAbort"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(sym("ncclGetErrorString"));
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_reduce &&
                g_nccl.comm_destroy && g_nccl.comm_abort && g_nccl.error_string;
    return g_nccl.ok ? CHELIS_CUDA_OK
                     : set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "libnccl.so.2 lacks an entry this library calls");
}

int nccl_check(ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return CHELIS_CUDA_OK;
    return set_error(CHELIS_CUDA_ERR_CUDA, "%s: %s", what, g_nccl.error_string ? g_nccl.error_string(r) : "?");
}

}  // namespace

// ---------------------------------------------------------------------------
// Library-internal entry points for programs that reduce their gradients as
// they produce them (chelis_cuda_block_step_dp): the communicator's size and
// an f32 sum all-reduce on a given stream.  The communication stream is
// created once per process, on the communicator's device, non-blocking with
// respect to the legacy default stream.
// ---------------------------------------------------------------------------
cudaStream_t g_comm_stream = nullptr;

int dp_nranks() {
    std::lock_guard<std::mutex> lock(g_dp_mu);
    return g_nccl.comm ? g_nccl.nranks : 1;
}

int dp_comm_stream(cudaStream_t *out) {
    std::lock_guard<std::mutex> lock(g_dp_mu);
    if (!g_nccl.comm) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp: no communicator (dp_init)");
    if (!g_comm_stream) {
        int prio_lo = 0, prio_hi = 0;
        CHELIS_TRY(check_cuda(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi),
                              "cudaDeviceGetStreamPriorityRange"));
        CHELIS_TRY(check_cuda(cudaStreamCreateWithPriority(&g_comm_stream, cudaStreamNonBlocking,
                                                           prio_hi),
                              "cudaStreamCreateWithPriority(dp comm)"));
    }
    *out = g_comm_stream;
    return CHELIS_CUDA_OK;
}

int dp_allreduce_f32_on(float *buf, int64_t count, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(g_dp_mu);
    if (!g_nccl.comm) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_allreduce: no communicator (dp_init)");
    if (count <= 0) return CHELIS_CUDA_OK;
    return nccl_check(g_nccl.all_reduce(buf, buf, static_cast<size_t>(count), ncclFloat32, ncclSum,
                                        g_nccl.comm, s),
                      "ncclAllReduce");
}

}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_dp_shard(int64_t n, int32_t nranks, int32_t rank, int64_t *start,
                                    int64_t *stop) {
    if (n < 0 || nranks < 1 || rank < 0 || rank >= nranks || !start || !stop)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_shard: n %lld over %d ranks, rank %d",
                         static_cast<long long>(n), nranks, rank);
    const int64_t base = n / nranks, extra = n % nranks;
    *start = rank * base + (rank < extra ? rank : extra);
    *stop = *start + base + (rank < extra ? 1 : 0);
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_dp_unique_id(uint8_t *id) {
    if (!id) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_unique_id: null output");
    std::lock_guard<std::mutex> lock(g_dp_mu);
    CHELIS_TRY(nccl_load());
    ncclUniqueId u;
    CHELIS_TRY(nccl_check(g_nccl.get_unique_id(&u), "ncclGetUniqueId"));
    std::memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_dp_init(int32_t nranks, int32_t rank, const uint8_t *id) {
    if (nranks < 1 || rank < 0 || rank >= nranks || !id)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_init: rank %d of %d", rank, nranks);
    std::lock_guard<std::mutex> lock(g_dp_mu);
    CHELIS_TRY(nccl_load());
    if (g_nccl.comm) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_init: a communicator is already open");
    int device = 0;
    CHELIS_TRY(check_cuda(cudaGetDevice(&device), "cudaGetDevice"));
    ncclUniqueId u;
    std::memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t comm = nullptr;
    CHELIS_TRY(nccl_check(g_nccl.comm_init_rank(&comm, nranks, u, rank), "ncclCommInitRank"));
    g_nccl.comm = comm;
    g_nccl.nranks = nranks;
    g_nccl.rank = rank;
    g_nccl.device = device;
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_dp_allreduce_sum(int32_t dtype, void *buf, int64_t count) {
    ncclDataType_t t;
    switch (dtype) {
        case CHELIS_DTYPE_F32: t = ncclFloat32; break;
        case CHELIS_DTYPE_F64: t = ncclFloat64; break;
        case CHELIS_DTYPE_I64: t = ncclInt64; break;
        case CHELIS_DTYPE_I32: t = ncclInt32; break;
        default: return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "dp_allreduce admits f32, f64, i32, i64");
    }
    if (count < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in dp_allreduce at i64");
    std::lock_guard<std::mutex> lock(g_dp_mu);
    if (!g_nccl.comm) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_allreduce: no communicator (dp_init)");
    if (count == 0) return CHELIS_CUDA_OK;
    if (!buf) return set_error(CHELIS_CUDA_ERR_DOMAIN, "dp_allreduce: null buffer");
    return nccl_check(g_nccl.all_reduce(buf, buf, static_cast<size_t>(count), t, ncclSum, g_nccl.comm,
                                        current_stream()),
                      "ncclAllReduce");
}

extern "C" int chelis_cuda_dp_world(int32_t *nranks, int32_t *rank) {
    std::lock_guard<std::mutex> lock(g_dp_mu);
    if (nranks) *nranks = g_nccl.comm ? g_nccl.nranks : 1;
    if (rank) *rank = g_nccl.comm ? g_nccl.rank : 0;
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_dp_finalize(int32_t abort) {
    std::lock_guard<std::mutex> lock(g_dp_mu);
    if (!g_nccl.comm) return CHELIS_CUDA_OK;
    ncclComm_t comm = g_nccl.comm;
    g_nccl.comm = nullptr;
    g_nccl.nranks = 0;
    g_nccl.rank = -1;
    if (g_comm_stream) {
        cudaStreamSynchronize(g_comm_stream);
        cudaStreamDestroy(g_comm_stream);
        g_comm_stream = nullptr;
    }
    return nccl_check(abort ? g_nccl.comm_abort(comm) : g_nccl.comm_destroy(comm),
                      abort ? "ncclCommAbort" : "ncclCommDestroy");
}
