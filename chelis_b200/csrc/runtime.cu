// runtime.cu -- status, streams, scratch and the device tensor owner.
//
// Replaces crates/chelis-backend-hip/runtime/chelis_device_owner.cpp
// (allocation, borrow, import, clone, release, host copies) and the
// abort-on-error helpers of chelis_hip_runtime.h:20-44 with status codes.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace chelis {

namespace {
thread_local char t_error[512] = "";
thread_local cudaStream_t t_stream = nullptr;
// process defaults, and the calling thread's overrides (-1 = the default)
std::atomic<int> g_gemm_mode{CHELIS_CUDA_GEMM_3XTF32};
std::atomic<int> g_rows_mode{CHELIS_CUDA_ROWS_FAST};
std::atomic<int> g_dgemm_kernel{CHELIS_CUDA_DGEMM_AUTO};
thread_local int t_gemm_mode = -1;
thread_local int t_rows_mode = -1;
thread_local int t_dgemm_kernel = -1;
int g_sm_count[64] = {0};
}  // namespace

std::atomic<uint64_t> g_launches{0};

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_error, sizeof(t_error), fmt, ap);
    va_end(ap);
    return status;
}

int check_cuda(cudaError_t err, const char *what) {
    if (err == cudaSuccess) return CHELIS_CUDA_OK;
    return set_error(CHELIS_CUDA_ERR_CUDA, "CUDA error in %s: %s", what, cudaGetErrorString(err));
}

cudaStream_t current_stream() { return t_stream; }

int current_device_checked(int *device) {
    int d = -1;
    CHELIS_TRY(check_cuda(cudaGetDevice(&d), "cudaGetDevice"));
    if (d < 0) return set_error(CHELIS_CUDA_ERR_NO_DEVICE, "no current CUDA device");
    *device = d;
    return CHELIS_CUDA_OK;
}

int sm_count() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return 148;
    if (g_sm_count[d] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
        g_sm_count[d] = n > 0 ? n : 148;
    }
    return g_sm_count[d];
}

// The library's own stream-ordered pool per device.  Freed scratch stays
// mapped (release threshold = unlimited) so repeated calls reuse it instead
// of re-mapping physical memory at every synchronisation point; the
// process's default pool is left as it is.
static cudaMemPool_t g_pools[64] = {};

static int library_pool(cudaMemPool_t *out) {
    cudaMemPool_t *pools = g_pools;
    int d = 0;
    CHELIS_TRY(check_cuda(cudaGetDevice(&d), "cudaGetDevice"));
    if (d < 0 || d >= 64) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "device index %d", d);
    if (!pools[d]) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = d;
        cudaMemPool_t pool;
        CHELIS_TRY(check_cuda(cudaMemPoolCreate(&pool, &props), "cudaMemPoolCreate"));
        uint64_t threshold = UINT64_MAX;
        CHELIS_TRY(check_cuda(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold),
                              "cudaMemPoolSetAttribute"));
        pools[d] = pool;
    }
    *out = pools[d];
    return CHELIS_CUDA_OK;
}

int scratch_alloc(void **ptr, size_t bytes, cudaStream_t stream) {
    *ptr = nullptr;
    if (bytes == 0) return CHELIS_CUDA_OK;
    cudaMemPool_t pool;
    CHELIS_TRY(library_pool(&pool));
    return check_cuda(cudaMallocFromPoolAsync(ptr, bytes, pool, stream), "cudaMallocFromPoolAsync(scratch)");
}

void scratch_free(void *ptr, cudaStream_t stream) {
    if (ptr) cudaFreeAsync(ptr, stream);
}

// Destroy the library's pools (each device synchronised first, so every
// stream-ordered free has happened and the pool's memory goes back).
int release_pools() {
    int st = CHELIS_CUDA_OK, prev = 0;
    cudaGetDevice(&prev);
    for (int d = 0; d < 64; ++d) {
        if (!g_pools[d]) continue;
        cudaSetDevice(d);
        if (cudaDeviceSynchronize() != cudaSuccess || cudaMemPoolDestroy(g_pools[d]) != cudaSuccess)
            st = set_error(CHELIS_CUDA_ERR_CUDA, "releasing the scratch pool of device %d failed", d);
        g_pools[d] = nullptr;
    }
    cudaSetDevice(prev);
    return st;
}

int gemm_mode() { return t_gemm_mode >= 0 ? t_gemm_mode : g_gemm_mode.load(); }
int rows_mode() { return t_rows_mode >= 0 ? t_rows_mode : g_rows_mode.load(); }
int dgemm_kernel_choice() { return t_dgemm_kernel >= 0 ? t_dgemm_kernel : g_dgemm_kernel.load(); }

namespace {
bool valid_gemm_mode(int m) { return m == CHELIS_CUDA_GEMM_3XTF32 || m == CHELIS_CUDA_GEMM_EXACT_TREE; }
bool valid_rows_mode(int m) { return m == CHELIS_CUDA_ROWS_EXACT || m == CHELIS_CUDA_ROWS_FAST; }
bool valid_dgemm_kernel(int m) {
    return m == CHELIS_CUDA_DGEMM_AUTO || m == CHELIS_CUDA_DGEMM_DMMA || m == CHELIS_CUDA_DGEMM_FFMA;
}
// The calling thread's modes for the lifetime of one call.
struct ThreadModeScope {
    int g, r, d;
    ThreadModeScope(int gemm, int dgemm) : g(t_gemm_mode), r(t_rows_mode), d(t_dgemm_kernel) {
        t_gemm_mode = gemm;
        if (dgemm >= 0) t_dgemm_kernel = dgemm;
    }
    ~ThreadModeScope() {
        t_gemm_mode = g;
        t_rows_mode = r;
        t_dgemm_kernel = d;
    }
};
}  // namespace

// ---------------------------------------------------------------------------
// strided gather used by clone (one kernel instead of one memcpy per element)
// ---------------------------------------------------------------------------
struct StrideInfo {
    int32_t rank;
    int64_t shape[8];
    int64_t strides[8];
};

__global__ void gather_strided_kernel(const unsigned char *__restrict__ src,
                                      unsigned char *__restrict__ dst, int64_t count, int width,
                                      StrideInfo info) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, off = 0;
        for (int ax = info.rank - 1; ax >= 0; --ax) {
            int64_t idx = rem % info.shape[ax];
            rem /= info.shape[ax];
            off += idx * info.strides[ax];
        }
        const unsigned char *s = src + off * width;
        unsigned char *d = dst + i * width;
        for (int b = 0; b < width; ++b) d[b] = s[b];
    }
}

int dtype_width(chelis_dtype dt) {
    switch (dt) {
        case CHELIS_DTYPE_F32: return 4;
        case CHELIS_DTYPE_F64: return 8;
        case CHELIS_DTYPE_I32: return 4;
        case CHELIS_DTYPE_BOOL: return 1;
        case CHELIS_DTYPE_I64: return 8;
        case CHELIS_DTYPE_BF16: return 2;
        case CHELIS_DTYPE_F16: return 2;
        case CHELIS_DTYPE_I8: return 1;
        case CHELIS_DTYPE_I16: return 2;
        case CHELIS_DTYPE_KEY: return 8;
        default: return 0;
    }
}

}  // namespace chelis

using namespace chelis;

// ---------------------------------------------------------------------------
// device tensor owner
// ---------------------------------------------------------------------------
struct chelis_device_tensor_owner {
    std::vector<int64_t> shape;
    std::vector<int64_t> strides;
    void *allocation = nullptr;  // owned storage (null when borrowed or empty)
    int32_t device = 0;
    chelis_gpu_tensor packet{};
};

namespace {

// Overflow-checked canonical metadata (the Rust metadata plan's job in the
// reference: chelis_device_owner.cpp:101-160).
int canonical_metadata(chelis_dtype dtype, int32_t rank, const int64_t *shape,
                       std::vector<int64_t> &sh, std::vector<int64_t> &st, int64_t &count,
                       int64_t &bytes) {
    int width = dtype_width(dtype);
    if (width == 0 || rank < 0 || rank > 8 || (rank > 0 && !shape))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    sh.assign(shape, shape + rank);
    st.assign(rank, 1);
    count = 1;
    for (int ax = rank - 1; ax >= 0; --ax) {
        if (sh[ax] < 0)
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
        st[ax] = count;
        if (sh[ax] != 0 && count > INT64_MAX / sh[ax])
            return set_error(CHELIS_CUDA_ERR_OVERFLOW,
                             "numeric trap: overflow in metadata_plan at i64");
        count *= sh[ax];
    }
    if (count > INT64_MAX / width)
        return set_error(CHELIS_CUDA_ERR_OVERFLOW, "numeric trap: overflow in metadata_plan at i64");
    bytes = count * width;
    return CHELIS_CUDA_OK;
}

void fill_packet(chelis_device_tensor_owner *o, void *data, int64_t count, int64_t capacity,
                 chelis_dtype dtype, bool owned) {
    o->packet.data = data;
    o->packet.shape = o->shape.data();
    o->packet.strides = o->strides.data();
    o->packet.count = count;
    o->packet.byte_capacity = capacity;
    o->packet.rank = static_cast<int32_t>(o->shape.size());
    o->packet.dtype = dtype;
    o->packet.ownership = owned ? 1 : 0;
    o->packet.reserved[0] = o->packet.reserved[1] = 0;
}

bool canonical_strides(const chelis_device_tensor_owner *o) {
    int64_t expect = 1;
    for (int ax = static_cast<int>(o->shape.size()) - 1; ax >= 0; --ax) {
        if (o->shape[ax] != 1 && o->strides[ax] != expect) return false;
        expect *= o->shape[ax];
    }
    return true;
}

int validate_device_pointer(const void *data, int32_t device) {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, data) != cudaSuccess) {
        cudaGetLastError();
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    }
    if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) ||
        attr.device != device)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    return CHELIS_CUDA_OK;
}

}  // namespace

namespace chelis {
namespace {
std::mutex g_fail_mu;
std::unordered_map<uint32_t, std::string> g_fail_messages;
uint32_t g_fail_next = 1;
}  // namespace
uint32_t register_fail_message(const char *message) {
    std::lock_guard<std::mutex> lk(g_fail_mu);
    const uint32_t id = g_fail_next++;
    g_fail_messages[id] = message;
    return id;
}
void unregister_fail_message(uint32_t id) {
    std::lock_guard<std::mutex> lk(g_fail_mu);
    g_fail_messages.erase(id);
}
// the registered message of guard `id` (a default text if it was released)
std::string fail_message(uint32_t id) {
    std::lock_guard<std::mutex> lk(g_fail_mu);
    const auto it = g_fail_messages.find(id);
    return it != g_fail_messages.end() ? it->second : std::string("a guarded abort fired");
}
}  // namespace chelis

extern "C" {

int chelis_cuda_version(void) { return 1; }

const char *chelis_cuda_last_error(void) { return t_error; }

int chelis_cuda_init(int32_t device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return set_error(CHELIS_CUDA_ERR_NO_DEVICE, "no CUDA device visible");
    }
    if (device < 0 || device >= n)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "device %d out of range (%d devices)", device, n);
    CHELIS_TRY(check_cuda(cudaSetDevice(device), "cudaSetDevice"));
    CHELIS_TRY(check_cuda(cudaFree(nullptr), "context init"));
    cudaDeviceProp prop{};
    CHELIS_TRY(check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties"));
    if (prop.major != 10)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                         "device %d is sm_%d%d; this library is built for sm_100a only", device,
                         prop.major, prop.minor);
    return CHELIS_CUDA_OK;
}

int chelis_cuda_set_stream(void *cuda_stream) {
    t_stream = static_cast<cudaStream_t>(cuda_stream);
    return CHELIS_CUDA_OK;
}

void *chelis_cuda_get_stream(void) { return t_stream; }

int chelis_cuda_synchronize(void) {
    return check_cuda(cudaStreamSynchronize(t_stream), "cudaStreamSynchronize");
}

int chelis_cuda_device_status(void) {
    CHELIS_TRY(check_cuda(cudaStreamSynchronize(t_stream), "cudaStreamSynchronize"));
    unsigned int word = 0, zero = 0;
    CHELIS_TRY(check_cuda(cudaMemcpyFromSymbol(&word, g_device_error, sizeof(word)),
                          "read device error word"));
    if (word) {
        CHELIS_TRY(check_cuda(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)),
                              "clear device error word"));
        if (word & DEVERR_TIMEOUTS)
            return set_error(CHELIS_CUDA_ERR_TIMEOUT,
                             "a bounded device wait gave up (error word 0x%x)", word);
        if (word & DEVERR_FAIL) {
            unsigned int id = 0;
            CHELIS_TRY(check_cuda(cudaMemcpyFromSymbol(&id, g_fail_id, sizeof(id)), "read fail id"));
            CHELIS_TRY(check_cuda(cudaMemcpyToSymbol(g_fail_id, &zero, sizeof(zero)), "clear fail id"));
            return set_error(CHELIS_CUDA_ERR_FAIL, "%s", fail_message(id).c_str());
        }
        if (word & DEVERR_BAD_INDEX)
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in gather at i64");
        if (word & (DEVERR_DROPOUT_F32 | DEVERR_DROPOUT_F64))
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in dropout at %s",
                             (word & DEVERR_DROPOUT_F32) ? "f32" : "f64");
        if (word & DEVERR_SHIFT) {
            unsigned long long bits = 0, zero64 = 0;
            CHELIS_TRY(check_cuda(cudaMemcpyFromSymbol(&bits, g_shift_count, sizeof(bits)), "read shift count"));
            CHELIS_TRY(check_cuda(cudaMemcpyToSymbol(g_shift_count, &zero64, sizeof(zero64)), "clear shift count"));
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "shift amount must be non-negative, got %lld",
                             static_cast<long long>(bits));
        }
        unsigned int code = 0;
        CHELIS_TRY(check_cuda(cudaMemcpyFromSymbol(&code, g_trap_code, sizeof(code)), "read trap code"));
        CHELIS_TRY(check_cuda(cudaMemcpyToSymbol(g_trap_code, &zero, sizeof(zero)), "clear trap code"));
        static const char *const kinds[] = {"overflow", "domain", "division by zero"};
        static const char *const ops[] = {"add", "sub", "mul", "trunc_div", "floor_div", "mod", "neg", "abs", "cast",
                                          "cast_trunc", "cast_saturate",
                                          "uniform_like", "range",
                                          "reduce_window_sum", "gather", "scatter_add", "scatter",
                                          "scatter_elements"};
        static const char *const dtypes[] = {"f32", "f64", "i32", "bool", "i64", "bf16", "f16", "i8", "i16", "key"};
        constexpr unsigned int n_ops = sizeof(ops) / sizeof(ops[0]);
        const unsigned int c = code ? code - 1 : 0, k = c >> 16, o = (c >> 8) & 0xff, d = c & 0xff;
        const char *op = o < n_ops ? ops[o] : "?";
        if (o >= TRAP_OP_GATHER && o < n_ops) {
            // the reference's sparse-index failure: the index line, then the trap line
            long long at[3] = {0, 0, 0};
            CHELIS_TRY(check_cuda(cudaMemcpyFromSymbol(at, g_trap_index, sizeof(at)), "read trap index"));
            return set_error(CHELIS_CUDA_ERR_DOMAIN,
                             "%s index %lld out of bounds at axis %lld of extent %lld\nnumeric trap: domain in %s at i64",
                             op, at[0], at[1], at[2], op);
        }
        return set_error(k == 0 ? CHELIS_CUDA_ERR_OVERFLOW : CHELIS_CUDA_ERR_DOMAIN,
                         "numeric trap: %s in %s at %s", k < 3 ? kinds[k] : "?", op, d < 10 ? dtypes[d] : "?");
    }
    return CHELIS_CUDA_OK;
}

uint64_t chelis_cuda_launch_count(void) { return g_launches.load(); }

int chelis_cuda_set_wait_limit(uint32_t tries) {
    const uint32_t v = tries ? tries : kMaxTries;
    return check_cuda(cudaMemcpyToSymbol(g_wait_tries, &v, sizeof(v)), "set wait limit");
}

uint32_t chelis_cuda_get_wait_limit(void) {
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, g_wait_tries, sizeof(v)) != cudaSuccess) return 0;
    return v;
}

int chelis_cuda_set_gemm_mode(int mode) {
    if (!valid_gemm_mode(mode))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown GEMM mode %d", mode);
    g_gemm_mode.store(mode);
    return CHELIS_CUDA_OK;
}
int chelis_cuda_get_gemm_mode(void) { return g_gemm_mode.load(); }

int chelis_cuda_set_rows_mode(int mode) {
    if (!valid_rows_mode(mode))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown rows mode %d", mode);
    g_rows_mode.store(mode);
    return CHELIS_CUDA_OK;
}
int chelis_cuda_get_rows_mode(void) { return g_rows_mode.load(); }

int chelis_cuda_set_dgemm_kernel(int kernel) {
    if (!valid_dgemm_kernel(kernel))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown f64 GEMM kernel %d", kernel);
    g_dgemm_kernel.store(kernel);
    return CHELIS_CUDA_OK;
}
int chelis_cuda_get_dgemm_kernel(void) { return g_dgemm_kernel.load(); }

int chelis_cuda_set_thread_modes(int gemm_mode, int rows_mode, int dgemm_kernel) {
    if ((gemm_mode != -1 && !valid_gemm_mode(gemm_mode)) ||
        (rows_mode != -1 && !valid_rows_mode(rows_mode)) ||
        (dgemm_kernel != -1 && !valid_dgemm_kernel(dgemm_kernel)))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown mode (%d, %d, %d)", gemm_mode, rows_mode,
                         dgemm_kernel);
    t_gemm_mode = gemm_mode;
    t_rows_mode = rows_mode;
    t_dgemm_kernel = dgemm_kernel;
    return CHELIS_CUDA_OK;
}

int chelis_cuda_get_thread_modes(int *gemm_mode, int *rows_mode, int *dgemm_kernel) {
    if (gemm_mode) *gemm_mode = chelis::gemm_mode();
    if (rows_mode) *rows_mode = chelis::rows_mode();
    if (dgemm_kernel) *dgemm_kernel = chelis::dgemm_kernel_choice();
    return CHELIS_CUDA_OK;
}

int chelis_cuda_sgemm_ex(int gemm_mode, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                         const float *a, int64_t lda, int64_t stride_a, const float *b,
                         int64_t ldb, int64_t stride_b, float *c, int64_t ldc, int64_t stride_c,
                         int64_t batch) {
    if (!valid_gemm_mode(gemm_mode))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown GEMM mode %d", gemm_mode);
    ThreadModeScope scope(gemm_mode, -1);
    return chelis_cuda_sgemm(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb, stride_b, c,
                             ldc, stride_c, batch);
}

int chelis_cuda_dgemm_ex(int gemm_mode, int dgemm_kernel, int trans_a, int trans_b, int64_t m,
                         int64_t n, int64_t k, const double *a, int64_t lda, int64_t stride_a,
                         const double *b, int64_t ldb, int64_t stride_b, double *c, int64_t ldc,
                         int64_t stride_c, int64_t batch) {
    if (!valid_gemm_mode(gemm_mode) || !valid_dgemm_kernel(dgemm_kernel))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "unknown GEMM mode %d / f64 kernel %d", gemm_mode,
                         dgemm_kernel);
    ThreadModeScope scope(gemm_mode, dgemm_kernel);
    return chelis_cuda_dgemm(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb, stride_b, c,
                             ldc, stride_c, batch);
}

chelis_device_tensor_owner *chelis_device_tensor_alloc_shape(chelis_dtype dtype, int32_t rank,
                                                             const int64_t *shape) {
    int device = 0;
    if (current_device_checked(&device) != CHELIS_CUDA_OK) return nullptr;
    auto *o = new (std::nothrow) chelis_device_tensor_owner();
    if (!o) {
        set_error(CHELIS_CUDA_ERR_OVERFLOW, "host allocation failed");
        return nullptr;
    }
    int64_t count = 0, bytes = 0;
    if (canonical_metadata(dtype, rank, shape, o->shape, o->strides, count, bytes) !=
        CHELIS_CUDA_OK) {
        delete o;
        return nullptr;
    }
    o->device = device;
    if (bytes) {
        cudaStream_t s = current_stream();
        if (check_cuda(cudaMallocAsync(&o->allocation, bytes, s), "cudaMallocAsync") !=
                CHELIS_CUDA_OK ||
            check_cuda(cudaMemsetAsync(o->allocation, 0, bytes, s), "cudaMemsetAsync") !=
                CHELIS_CUDA_OK) {
            if (o->allocation) cudaFreeAsync(o->allocation, s);
            delete o;
            return nullptr;
        }
    }
    fill_packet(o, o->allocation, count, bytes, dtype, true);
    return o;
}

chelis_device_tensor_owner *chelis_device_tensor_borrow_shape(chelis_dtype dtype, int32_t rank,
                                                              const int64_t *shape, void *data,
                                                              int64_t byte_capacity) {
    int device = 0;
    if (current_device_checked(&device) != CHELIS_CUDA_OK) return nullptr;
    auto *o = new (std::nothrow) chelis_device_tensor_owner();
    if (!o) return nullptr;
    int64_t count = 0, bytes = 0;
    if (canonical_metadata(dtype, rank, shape, o->shape, o->strides, count, bytes) !=
        CHELIS_CUDA_OK) {
        delete o;
        return nullptr;
    }
    if (byte_capacity < bytes ||
        (count && (!data || reinterpret_cast<uintptr_t>(data) % dtype_width(dtype))) ||
        (count && validate_device_pointer(data, device) != CHELIS_CUDA_OK)) {
        set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
        delete o;
        return nullptr;
    }
    o->device = device;
    fill_packet(o, data, count, byte_capacity, dtype, false);
    return o;
}

chelis_device_tensor_owner *chelis_device_tensor_import(const chelis_gpu_tensor *packet) {
    int device = 0;
    if (current_device_checked(&device) != CHELIS_CUDA_OK) return nullptr;
    if (!packet || packet->ownership != 0 || packet->reserved[0] || packet->reserved[1] ||
        packet->rank < 0 || packet->rank > 8 || dtype_width(packet->dtype) == 0 ||
        (packet->rank > 0 && (!packet->shape || !packet->strides))) {
        set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
        return nullptr;
    }
    auto *o = new (std::nothrow) chelis_device_tensor_owner();
    if (!o) return nullptr;
    o->shape.assign(packet->shape, packet->shape + packet->rank);
    o->strides.assign(packet->strides, packet->strides + packet->rank);
    int64_t count = 1, max_off = 0;
    for (int ax = 0; ax < packet->rank; ++ax) {
        if (o->shape[ax] < 0 || o->strides[ax] < 0) {
            set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
            delete o;
            return nullptr;
        }
        count *= o->shape[ax];
        if (o->shape[ax] > 0) max_off += (o->shape[ax] - 1) * o->strides[ax];
    }
    int width = dtype_width(packet->dtype);
    if (count != packet->count ||
        (count && (max_off + 1) * width > packet->byte_capacity) ||
        (count && validate_device_pointer(packet->data, device) != CHELIS_CUDA_OK)) {
        set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
        delete o;
        return nullptr;
    }
    o->device = device;
    fill_packet(o, packet->data, count, packet->byte_capacity, packet->dtype, false);
    return o;
}

const chelis_gpu_tensor *chelis_device_tensor_view(const chelis_device_tensor_owner *owner) {
    if (!owner) return nullptr;
    return &owner->packet;
}

int32_t chelis_device_tensor_device(const chelis_device_tensor_owner *owner) {
    return owner ? owner->device : -1;
}

chelis_device_tensor_owner *chelis_device_tensor_clone(const chelis_device_tensor_owner *source) {
    if (!source) return nullptr;
    chelis_device_tensor_owner *dst = chelis_device_tensor_alloc_shape(
        source->packet.dtype, source->packet.rank, source->shape.data());
    if (!dst || source->packet.count == 0) return dst;
    int width = dtype_width(source->packet.dtype);
    cudaStream_t s = current_stream();
    if (canonical_strides(source)) {
        if (check_cuda(cudaMemcpyAsync(dst->packet.data, source->packet.data,
                                       source->packet.count * width, cudaMemcpyDeviceToDevice, s),
                       "clone copy") != CHELIS_CUDA_OK) {
            chelis_device_tensor_release(dst);
            return nullptr;
        }
        return dst;
    }
    StrideInfo info{};
    info.rank = source->packet.rank;
    for (int ax = 0; ax < info.rank; ++ax) {
        info.shape[ax] = source->shape[ax];
        info.strides[ax] = source->strides[ax];
    }
    int64_t blocks = (source->packet.count + 255) / 256;
    if (blocks > 4 * 148 * 8) blocks = 4 * 148 * 8;
    gather_strided_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const unsigned char *>(source->packet.data),
        static_cast<unsigned char *>(dst->packet.data), source->packet.count, width, info);
    g_launches++;
    if (check_cuda(cudaGetLastError(), "gather_strided_kernel") != CHELIS_CUDA_OK) {
        chelis_device_tensor_release(dst);
        return nullptr;
    }
    return dst;
}

void chelis_device_tensor_release(chelis_device_tensor_owner *owner) {
    if (!owner) return;
    if (owner->allocation) cudaFreeAsync(owner->allocation, current_stream());
    delete owner;
}

int chelis_device_tensor_copy_from_host_bytes(chelis_device_tensor_owner *destination,
                                              const void *host, int64_t bytes) {
    if (!destination || !destination->allocation || !canonical_strides(destination))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    int64_t need = destination->packet.count * dtype_width(destination->packet.dtype);
    if (bytes != need)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    if (!bytes) return CHELIS_CUDA_OK;
    return check_cuda(cudaMemcpyAsync(destination->packet.data, host, bytes,
                                      cudaMemcpyHostToDevice, current_stream()),
                      "copy_from_host");
}

int chelis_device_tensor_copy_to_host_bytes(void *host, int64_t bytes,
                                            const chelis_device_tensor_owner *source) {
    if (!source) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    int64_t need = source->packet.count * dtype_width(source->packet.dtype);
    if (bytes != need)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in metadata_plan at i64");
    if (!bytes) return CHELIS_CUDA_OK;
    if (canonical_strides(source))
        return check_cuda(cudaMemcpyAsync(host, source->packet.data, bytes, cudaMemcpyDeviceToHost,
                                          current_stream()),
                          "copy_to_host");
    chelis_device_tensor_owner *tmp = chelis_device_tensor_clone(source);
    if (!tmp) return CHELIS_CUDA_ERR_CUDA;
    int st = check_cuda(cudaMemcpyAsync(host, tmp->packet.data, bytes, cudaMemcpyDeviceToHost,
                                        current_stream()),
                        "copy_to_host");
    if (st == CHELIS_CUDA_OK) st = check_cuda(cudaStreamSynchronize(current_stream()), "sync");
    chelis_device_tensor_release(tmp);
    return st;
}

}  // extern "C"
