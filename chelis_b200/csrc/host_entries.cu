// host_entries.cu -- the device owner under the reference's own names and
// argument types, and the generated-entry host-array ABI of the shipped
// programs.
//
// Device owner (crates/chelis-backend-hip/runtime/chelis_device_owner.h:16-24,
// chelis_device_owner.cpp:184-274): metadata plans in, host tensors and host
// write guards for the copies.  The plain names fail as the reference does:
// a metadata or argument error prints the runtime's "numeric trap: domain in
// metadata_plan at i64" line and exits with status 1; a CUDA failure prints
// "CUDA device owner failure: <error>" and aborts.  Each has a `_status`
// twin that returns a CHELIS_CUDA_* code instead (message in
// chelis_cuda_last_error()).  Copies and allocation run on the calling
// thread's library stream; every entry returns with its work complete, as
// the reference's hipDeviceSynchronize does.
//
// Host-array entries (crates/chelis-backend-hip/src/emit.rs:660-800):
// `void f(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int
// n_out)` uploads the host inputs into device owners, runs the `f_device`
// program, and returns newly allocated host tensors (chelis_alloc + write
// guard + copy_to_host), exactly the sequence the generated code runs.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "chelis_host_runtime.h"
#include "common.cuh"

using namespace chelis;

namespace {

constexpr const char *kPlanDomain = "numeric trap: domain in metadata_plan at i64";

// A status code turned into the reference's failure behaviour.
void fail_like_reference(int status) {
    if (status == CHELIS_CUDA_OK) return;
    if (status == CHELIS_CUDA_ERR_DOMAIN || status == CHELIS_CUDA_ERR_OVERFLOW ||
        status == CHELIS_CUDA_ERR_UNSUPPORTED) {
        std::fprintf(stderr, "%s\n", chelis_cuda_last_error());
        std::fflush(stdout);
        std::fflush(stderr);
        std::exit(1);
    }
    std::fprintf(stderr, "CUDA device owner failure: %s\n", chelis_cuda_last_error());
    std::fflush(stderr);
    std::abort();
}

int plan_domain_error() { return set_error(CHELIS_CUDA_ERR_DOMAIN, "%s", kPlanDomain); }

// Bytes a plan's elements reach: (largest element offset + 1) * width, 0
// when empty (the capacity rule of chelis_metadata_plan_check_capacity).
int plan_span_bytes(const chelis_metadata_plan *plan, int64_t *span) {
    const int32_t rank = chelis_metadata_plan_rank(plan);
    const int64_t count = chelis_metadata_plan_count(plan);
    const int width = dtype_width(chelis_metadata_plan_dtype(plan));
    if (width == 0) return plan_domain_error();
    if (count == 0) {
        *span = 0;
        return CHELIS_CUDA_OK;
    }
    const int64_t *shape = chelis_metadata_plan_shape(plan);
    const int64_t *strides = chelis_metadata_plan_strides(plan);
    int64_t largest = 0;
    for (int32_t ax = 0; ax < rank; ++ax) {
        if (strides[ax] < 0) return plan_domain_error();
        const int64_t e = shape[ax] - 1;
        if (strides[ax] != 0 && e > INT64_MAX / strides[ax])
            return set_error(CHELIS_CUDA_ERR_OVERFLOW, "numeric trap: overflow in metadata_plan at i64");
        largest += e * strides[ax];
    }
    *span = (largest + 1) * width;
    return CHELIS_CUDA_OK;
}

chelis_device_tensor_owner *owner_from_plan(const chelis_metadata_plan *plan, void *data,
                                            int64_t capacity, bool owned, int32_t device) {
    auto *o = new (std::nothrow) chelis_device_tensor_owner();
    if (!o) return nullptr;
    const int32_t rank = chelis_metadata_plan_rank(plan);
    const int64_t *shape = chelis_metadata_plan_shape(plan);
    const int64_t *strides = chelis_metadata_plan_strides(plan);
    o->shape.assign(shape, shape + rank);
    o->strides.assign(strides, strides + rank);
    o->device = device;
    o->allocation = owned ? data : nullptr;
    o->packet.data = data;
    o->packet.shape = o->shape.data();
    o->packet.strides = o->strides.data();
    o->packet.count = chelis_metadata_plan_count(plan);
    o->packet.byte_capacity = capacity;
    o->packet.rank = rank;
    o->packet.dtype = chelis_metadata_plan_dtype(plan);
    o->packet.ownership = owned ? 1 : 0;
    o->packet.reserved[0] = o->packet.reserved[1] = 0;
    return o;
}

bool owner_canonical(const chelis_device_tensor_owner *o) {
    int64_t expect = 1;
    for (int ax = static_cast<int>(o->shape.size()) - 1; ax >= 0; --ax) {
        if (o->shape[ax] != 1 && o->strides[ax] != expect) return false;
        expect *= o->shape[ax];
    }
    return true;
}

int require_current(const chelis_device_tensor_owner *o) {
    if (!o) return plan_domain_error();
    int device = 0;
    CHELIS_TRY(current_device_checked(&device));
    if (device != o->device) return plan_domain_error();
    return CHELIS_CUDA_OK;
}

template <class View>
int require_matching(const View &host, const chelis_gpu_tensor &dev) {
    if (host.count != dev.count || host.dtype != dev.dtype) return plan_domain_error();
    for (uint8_t b : host.reserved)
        if (b) return plan_domain_error();
    return CHELIS_CUDA_OK;
}

}  // namespace

extern "C" {

// ---- device owner, reference names ----

int chelis_device_tensor_alloc_status(chelis_metadata_plan *plan,
                                      chelis_device_tensor_owner **out) {
    if (!out) return plan_domain_error();
    *out = nullptr;
    if (!plan) return plan_domain_error();
    int64_t span = 0;
    int st = plan_span_bytes(plan, &span);
    const int64_t bytes = chelis_metadata_plan_byte_count(plan);
    if (st == CHELIS_CUDA_OK && span > bytes) st = plan_domain_error();
    int device = 0;
    if (st == CHELIS_CUDA_OK) st = current_device_checked(&device);
    void *data = nullptr;
    cudaStream_t s = current_stream();
    if (st == CHELIS_CUDA_OK && bytes) {
        st = check_cuda(cudaMallocAsync(&data, static_cast<size_t>(bytes), s), "cudaMallocAsync");
        if (st == CHELIS_CUDA_OK)
            st = check_cuda(cudaMemsetAsync(data, 0, static_cast<size_t>(bytes), s), "cudaMemsetAsync");
        if (st == CHELIS_CUDA_OK) st = check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    }
    if (st == CHELIS_CUDA_OK) {
        *out = owner_from_plan(plan, data, bytes, true, device);
        if (!*out) st = set_error(CHELIS_CUDA_ERR_OVERFLOW, "host allocation failed");
    }
    if (st != CHELIS_CUDA_OK && data) cudaFreeAsync(data, s);
    chelis_metadata_plan_release(plan);  // the plan transfers to the owner (owner.h:13-15)
    return st;
}

chelis_device_tensor_owner *chelis_device_tensor_alloc(chelis_metadata_plan *plan) {
    chelis_device_tensor_owner *o = nullptr;
    fail_like_reference(chelis_device_tensor_alloc_status(plan, &o));
    return o;
}

int chelis_device_tensor_borrow_status(chelis_metadata_plan *plan, void *data,
                                       chelis_scalar byte_capacity,
                                       chelis_device_tensor_owner **out) {
    if (!out) return plan_domain_error();
    *out = nullptr;
    if (!plan) return plan_domain_error();
    int st = CHELIS_CUDA_OK;
    int64_t capacity = 0, span = 0;
    bool canonical_capacity = byte_capacity.dtype == CHELIS_DTYPE_I64;
    for (uint8_t b : byte_capacity.reserved) canonical_capacity = canonical_capacity && b == 0;
    if (canonical_capacity) std::memcpy(&capacity, &byte_capacity.bits, sizeof(capacity));
    if (!canonical_capacity || capacity < 0) st = plan_domain_error();
    if (st == CHELIS_CUDA_OK) st = plan_span_bytes(plan, &span);
    if (st == CHELIS_CUDA_OK && span > capacity) st = plan_domain_error();
    int device = 0;
    if (st == CHELIS_CUDA_OK) st = current_device_checked(&device);
    const int64_t count = chelis_metadata_plan_count(plan);
    const int width = dtype_width(chelis_metadata_plan_dtype(plan));
    if (st == CHELIS_CUDA_OK && count &&
        (!data || reinterpret_cast<uintptr_t>(data) % static_cast<uintptr_t>(width)))
        st = plan_domain_error();
    if (st == CHELIS_CUDA_OK && count) {
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, data) != cudaSuccess) {
            cudaGetLastError();
            st = plan_domain_error();
        } else if ((attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) ||
                   attr.device != device) {
            st = plan_domain_error();
        }
    }
    if (st == CHELIS_CUDA_OK) {
        *out = owner_from_plan(plan, data, capacity, false, device);
        if (!*out) st = set_error(CHELIS_CUDA_ERR_OVERFLOW, "host allocation failed");
    }
    chelis_metadata_plan_release(plan);
    return st;
}

chelis_device_tensor_owner *chelis_device_tensor_borrow(chelis_metadata_plan *plan, void *data,
                                                        chelis_scalar byte_capacity) {
    chelis_device_tensor_owner *o = nullptr;
    fail_like_reference(chelis_device_tensor_borrow_status(plan, data, byte_capacity, &o));
    return o;
}

int chelis_device_tensor_copy_from_host_status(chelis_device_tensor_owner *destination,
                                               const chelis_tensor *source) {
    CHELIS_TRY(require_current(destination));
    if (!source) return plan_domain_error();
    const chelis_read_view in = chelis_tensor_read_view(source);
    CHELIS_TRY(require_matching(in, destination->packet));
    if (!destination->allocation && destination->packet.count) return plan_domain_error();
    if (destination->packet.ownership != 1 || !owner_canonical(destination))
        return plan_domain_error();
    const int64_t bytes = destination->packet.count * dtype_width(destination->packet.dtype);
    if (!bytes) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    CHELIS_TRY(check_cuda(cudaMemcpyAsync(destination->packet.data, in.data,
                                          static_cast<size_t>(bytes), cudaMemcpyHostToDevice, s),
                          "copy_from_host"));
    return check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
}

void chelis_device_tensor_copy_from_host(chelis_device_tensor_owner *destination,
                                         const chelis_tensor *source) {
    fail_like_reference(chelis_device_tensor_copy_from_host_status(destination, source));
}

int chelis_device_tensor_copy_to_host_status(chelis_tensor_write *destination,
                                             const chelis_device_tensor_owner *source) {
    CHELIS_TRY(require_current(source));
    if (!destination) return plan_domain_error();
    const chelis_write_view out = chelis_tensor_write_view(destination);
    CHELIS_TRY(require_matching(out, source->packet));
    const int64_t bytes = source->packet.count * dtype_width(source->packet.dtype);
    if (!bytes) return CHELIS_CUDA_OK;
    // strided sources are gathered on the device first (one kernel), then
    // copied in one transfer
    CHELIS_TRY(chelis_device_tensor_copy_to_host_bytes(out.data, bytes, source));
    return check_cuda(cudaStreamSynchronize(current_stream()), "cudaStreamSynchronize");
}

void chelis_device_tensor_copy_to_host(chelis_tensor_write *destination,
                                       const chelis_device_tensor_owner *source) {
    fail_like_reference(chelis_device_tensor_copy_to_host_status(destination, source));
}

}  // extern "C"

// ---- host-array program entries ----

namespace {

using DeviceEntry = int (*)(const chelis_device_tensor_owner *const *, chelis_device_rank,
                            chelis_device_tensor_owner **, chelis_device_rank);

// Inputs must carry `dtypes[i]` (or, where dtypes[i] < 0, the dtype of
// input 0, which must be f32 or f64).
int run_host_entry(const char *name, DeviceEntry entry, const int *dtypes, int want_in,
                   int want_out, chelis_tensor **inputs, int n_in, chelis_tensor **outputs,
                   int n_out) {
    if (n_in != want_in || n_out != want_out)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "%s: expected %d inputs and %d outputs, got %d and %d",
                         name, want_in, want_out, n_in, n_out);
    if (!inputs || !outputs) return set_error(CHELIS_CUDA_ERR_DOMAIN, "%s: null argument array", name);
    for (int i = 0; i < n_out; ++i) outputs[i] = nullptr;
    std::vector<chelis_device_tensor_owner *> din(n_in, nullptr), dout(n_out, nullptr);
    int st = CHELIS_CUDA_OK;
    chelis_dtype first = 0;
    for (int i = 0; i < n_in && st == CHELIS_CUDA_OK; ++i) {
        if (!inputs[i]) {
            st = set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
            break;
        }
        const chelis_read_view v = chelis_tensor_read_view(inputs[i]);
        if (i == 0) first = v.dtype;
        const bool ok = dtypes[i] >= 0 ? v.dtype == dtypes[i]
                                       : (v.dtype == first && (first == CHELIS_DTYPE_F32 ||
                                                               first == CHELIS_DTYPE_F64));
        if (!ok) {  // emit.rs:1112
            st = set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
            break;
        }
        const int32_t rank = chelis_tensor_rank(inputs[i]);
        std::vector<int64_t> shape(rank);
        for (int32_t ax = 0; ax < rank; ++ax) shape[ax] = chelis_tensor_shape(inputs[i], ax);
        din[i] = chelis_device_tensor_alloc_shape(v.dtype, rank, shape.data());
        if (!din[i]) {
            st = CHELIS_CUDA_ERR_CUDA;
            break;
        }
        if (v.count)
            st = chelis_device_tensor_copy_from_host_bytes(din[i], v.data,
                                                           v.count * dtype_width(v.dtype));
    }
    if (st == CHELIS_CUDA_OK) st = entry(din.data(), n_in, dout.data(), n_out);
    for (int i = 0; i < n_out && st == CHELIS_CUDA_OK; ++i) {
        const chelis_gpu_tensor *d = chelis_device_tensor_view(dout[i]);
        outputs[i] = chelis_alloc(d->rank, d->shape, d->dtype);
        chelis_tensor_write *guard = chelis_tensor_begin_write(outputs[i]);
        st = chelis_device_tensor_copy_to_host_status(guard, dout[i]);
        chelis_tensor_end_write(guard);
    }
    if (st == CHELIS_CUDA_OK) st = check_cuda(cudaStreamSynchronize(current_stream()), "sync");
    for (auto *o : din) chelis_device_tensor_release(o);
    for (auto *o : dout) chelis_device_tensor_release(o);
    if (st != CHELIS_CUDA_OK) {
        for (int i = 0; i < n_out; ++i)
            if (outputs[i]) {
                chelis_tensor_release(outputs[i]);
                outputs[i] = nullptr;
            }
    }
    return st;
}

// Count errors abort with the generated code's message (emit.rs:677-693);
// everything else fails like the owner.
void host_entry_or_fail(const char *name, DeviceEntry entry, const int *dtypes, int want_in,
                        int want_out, chelis_tensor **inputs, int n_in, chelis_tensor **outputs,
                        int n_out) {
    if (n_in != want_in) {
        std::fprintf(stderr, "%s: expected %d inputs, got %d\n", name, want_in, n_in);
        std::abort();
    }
    if (n_out != want_out) {
        std::fprintf(stderr, "%s: expected %d outputs, got %d\n", name, want_out, n_out);
        std::abort();
    }
    fail_like_reference(
        run_host_entry(name, entry, dtypes, want_in, want_out, inputs, n_in, outputs, n_out));
}

constexpr int kChainDtypes[3] = {CHELIS_DTYPE_F32, CHELIS_DTYPE_F32, CHELIS_DTYPE_F32};
constexpr int kPortfolioDtypes[2] = {CHELIS_DTYPE_F64, CHELIS_DTYPE_F64};
constexpr int kMatmulDtypes[2] = {-1, -1};

}  // namespace

extern "C" {

int chelis_chain_fwd_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    return run_host_entry("chelis_chain_fwd", chelis_chain_fwd_device, kChainDtypes, 3, 1, inputs,
                          n_in, outputs, n_out);
}
void chelis_chain_fwd(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    host_entry_or_fail("chelis_chain_fwd", chelis_chain_fwd_device, kChainDtypes, 3, 1, inputs,
                       n_in, outputs, n_out);
}

int chelis_chain_grad_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    return run_host_entry("chelis_chain_grad", chelis_chain_grad_device, kChainDtypes, 3, 3, inputs,
                          n_in, outputs, n_out);
}
void chelis_chain_grad(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    host_entry_or_fail("chelis_chain_grad", chelis_chain_grad_device, kChainDtypes, 3, 3, inputs,
                       n_in, outputs, n_out);
}

int chelis_portfolio_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    return run_host_entry("chelis_portfolio", chelis_portfolio_device, kPortfolioDtypes, 2, 3,
                          inputs, n_in, outputs, n_out);
}
void chelis_portfolio(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    host_entry_or_fail("chelis_portfolio", chelis_portfolio_device, kPortfolioDtypes, 2, 3, inputs,
                       n_in, outputs, n_out);
}

int chelis_matmul_status(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    return run_host_entry("chelis_matmul", chelis_matmul_device, kMatmulDtypes, 2, 1, inputs, n_in,
                          outputs, n_out);
}
void chelis_matmul(chelis_tensor **inputs, int n_in, chelis_tensor **outputs, int n_out) {
    host_entry_or_fail("chelis_matmul", chelis_matmul_device, kMatmulDtypes, 2, 1, inputs, n_in,
                       outputs, n_out);
}

}  // extern "C"
