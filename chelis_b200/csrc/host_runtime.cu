// host_runtime.cu -- weak stand-ins for the Chelis host runtime functions the
// device owner and the host-array program entries call (tagged scalars, the
// metadata plan, host tensors with read views and write guards).
//
// The reference implements these in Rust (crates/chelis-runtime/src/lib.rs:
// chelis_alloc :2155, chelis_tensor_entry_borrow :2275, read view :2370,
// write guard :2460-2534, metadata plan :3022-3138; the plan arithmetic is
// crates/chelis-abi/src/metadata.rs).  Every definition here is weak: a
// process that links the real runtime uses the runtime's definitions, and
// this file only serves a process without it.  Failures print the runtime's
// message and exit(1), as its runtime_fail! / numeric_trap! macros do
// (lib.rs:321-354).
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "chelis_host_runtime.h"

#define CHELIS_WEAK extern "C" __attribute__((weak, visibility("default")))

namespace chelis {
namespace hostrt {

[[noreturn]] void fail_line(const char *line) {
    std::fprintf(stderr, "%s\n", line);
    std::fflush(stdout);
    std::fflush(stderr);
    std::exit(1);
}
[[noreturn]] void plan_domain() { fail_line("numeric trap: domain in metadata_plan at i64"); }
[[noreturn]] void plan_overflow() { fail_line("numeric trap: overflow in metadata_plan at i64"); }

int64_t width_of(chelis_dtype dt) {
    switch (dt) {
        case CHELIS_DTYPE_F32: case CHELIS_DTYPE_I32: return 4;
        case CHELIS_DTYPE_F64: case CHELIS_DTYPE_I64: case CHELIS_DTYPE_KEY: return 8;
        case CHELIS_DTYPE_BOOL: case CHELIS_DTYPE_I8: return 1;
        case CHELIS_DTYPE_BF16: case CHELIS_DTYPE_F16: case CHELIS_DTYPE_I16: return 2;
        default: return 0;
    }
}

// A canonical tagged i64 (lib.rs:4310-4321 affine_scalar).
int64_t tagged_i64(chelis_scalar v) {
    if (v.dtype != CHELIS_DTYPE_I64) plan_domain();
    for (uint8_t b : v.reserved)
        if (b) plan_domain();
    int64_t out;
    std::memcpy(&out, &v.bits, sizeof(out));
    return out;
}

// The exemplar names the element dtype (lib.rs:4152-4175
// reduction_exemplar): a known id, never a key, reserved bytes zero, no
// bits beyond the dtype's width.
chelis_dtype exemplar_dtype(chelis_scalar v) {
    const int64_t w = width_of(v.dtype);
    if (w == 0 || v.dtype == CHELIS_DTYPE_KEY) plan_domain();
    for (uint8_t b : v.reserved)
        if (b) plan_domain();
    if (w < 8 && (v.bits >> (8 * w)) != 0) plan_domain();
    if (v.dtype == CHELIS_DTYPE_BOOL && v.bits > 1) plan_domain();
    return v.dtype;
}

int32_t plan_rank(chelis_scalar rank) {
    const int64_t r = tagged_i64(rank);
    if (r < 0) plan_domain();
    if (r > INT32_MAX) plan_overflow();
    return static_cast<int32_t>(r);
}

void preflight(const chelis_scalar *values, int32_t rank) {
    if (rank != 0 && (!values || reinterpret_cast<uintptr_t>(values) % alignof(chelis_scalar)))
        plan_domain();
}

// Element count and logical bytes of a shape (metadata.rs CheckedDomain):
// negative extents are a domain error, products past i64 an overflow.
void checked_domain(const std::vector<int64_t> &shape, int64_t width, int64_t *count,
                    int64_t *bytes) {
    int64_t c = 1;
    for (int64_t e : shape) {
        if (e < 0) plan_domain();
        if (e != 0 && c > INT64_MAX / e) plan_overflow();
        c *= e;
    }
    if (c > INT64_MAX / width) plan_overflow();
    *count = c;
    *bytes = c * width;
}

}  // namespace hostrt
}  // namespace chelis

using namespace chelis::hostrt;

struct chelis_metadata_plan {
    chelis_dtype dtype;
    bool strided;
    std::vector<int64_t> shape;
    std::vector<int64_t> strides;  // in elements
    int64_t count;
    int64_t bytes;       // logical bytes: count * width
    int64_t span_bytes;  // bytes a view reaches: (largest offset + 1) * width
};

struct chelis_tensor_write {
    chelis_tensor *tensor;
};

struct chelis_tensor {
    std::atomic<int64_t> refs{1};
    std::atomic<int> writing{0};
    chelis_dtype dtype = 0;
    std::vector<int64_t> shape;
    int64_t count = 0;
    int64_t bytes = 0;
    void *data = nullptr;
    bool owned = false;
    chelis_tensor_write guard{nullptr};
};

namespace {

const chelis_metadata_plan &plan_ref(const chelis_metadata_plan *p) {
    if (!p || reinterpret_cast<uintptr_t>(p) % alignof(chelis_metadata_plan)) plan_domain();
    return *p;
}

chelis_tensor &tensor_ref(const chelis_tensor *t, const char *site) {
    if (!t || reinterpret_cast<uintptr_t>(t) % alignof(chelis_tensor)) {
        std::fprintf(stderr, "Domain: %s: null or misaligned tensor\n", site);
        std::fflush(stderr);
        std::exit(1);
    }
    return *const_cast<chelis_tensor *>(t);
}

[[noreturn]] void runtime_fail(const char *site, const char *what) {
    std::fprintf(stderr, "Domain: %s %s\n", site, what);
    std::fflush(stdout);
    std::fflush(stderr);
    std::exit(1);
}

// checked_tensor_metadata (lib.rs:2155-2170): rank, shape and dtype of a
// host tensor request.
std::vector<int64_t> host_shape(int32_t rank, const int64_t *shape, chelis_dtype dtype,
                                const char *site, int64_t *count, int64_t *bytes) {
    const int64_t w = width_of(dtype);
    if (w == 0) runtime_fail(site, "unknown dtype");
    if (rank < 0 || (rank > 0 && !shape)) runtime_fail(site, "invalid rank or shape");
    std::vector<int64_t> sh(shape, shape + rank);
    checked_domain(sh, w, count, bytes);
    return sh;
}

}  // namespace

CHELIS_WEAK chelis_scalar chelis_scalar_from_bits(chelis_dtype dtype, uint64_t bits) {
    chelis_scalar s{};
    s.dtype = dtype;
    s.bits = bits;
    return s;
}

CHELIS_WEAK int64_t chelis_dtype_size(chelis_dtype dtype) { return width_of(dtype); }

CHELIS_WEAK chelis_metadata_plan *chelis_metadata_plan_new(chelis_scalar rank,
                                                           const chelis_scalar *shape,
                                                           chelis_scalar exemplar) {
    const int32_t r = plan_rank(rank);
    preflight(shape, r);
    const chelis_dtype dt = exemplar_dtype(exemplar);
    auto *p = new chelis_metadata_plan();
    p->dtype = dt;
    p->strided = false;
    for (int32_t ax = 0; ax < r; ++ax) p->shape.push_back(tagged_i64(shape[ax]));
    checked_domain(p->shape, width_of(dt), &p->count, &p->bytes);
    // suffix products, zero after a zero extent (metadata.rs:1263-1278)
    p->strides.assign(r, 1);
    int64_t run = 1;
    for (int32_t ax = r - 1; ax >= 0; --ax) {
        p->strides[ax] = run;
        if (p->shape[ax] != 0 && run > INT64_MAX / p->shape[ax]) plan_overflow();
        run *= p->shape[ax];
    }
    p->span_bytes = p->bytes;
    return p;
}

CHELIS_WEAK chelis_metadata_plan *chelis_metadata_plan_view(chelis_scalar rank,
                                                            const chelis_scalar *shape,
                                                            const chelis_scalar *strides,
                                                            chelis_scalar exemplar,
                                                            chelis_scalar byte_capacity) {
    const int32_t r = plan_rank(rank);
    preflight(shape, r);
    preflight(strides, r);
    const chelis_dtype dt = exemplar_dtype(exemplar);
    const int64_t capacity = tagged_i64(byte_capacity);
    if (capacity < 0) plan_domain();
    auto *p = new chelis_metadata_plan();
    p->dtype = dt;
    p->strided = true;
    for (int32_t ax = 0; ax < r; ++ax) p->shape.push_back(tagged_i64(shape[ax]));
    for (int32_t ax = 0; ax < r; ++ax) p->strides.push_back(tagged_i64(strides[ax]));
    for (int64_t s : p->strides)
        if (s < 0) {  // forward views only (metadata.rs:93-98)
            delete p;
            plan_domain();
        }
    const int64_t w = width_of(dt);
    checked_domain(p->shape, w, &p->count, &p->bytes);
    int64_t largest = 0;
    if (p->count != 0) {
        for (int32_t ax = 0; ax < r; ++ax) {
            const int64_t e = p->shape[ax] - 1, s = p->strides[ax];
            if (s != 0 && e > INT64_MAX / s) plan_overflow();
            if (largest > INT64_MAX - e * s) plan_overflow();
            largest += e * s;
        }
    }
    const int64_t span = p->count ? largest + 1 : 0;
    if (span > INT64_MAX / w) plan_overflow();
    p->span_bytes = span * w;
    if (p->span_bytes > capacity) {
        delete p;
        plan_domain();
    }
    return p;
}

CHELIS_WEAK int32_t chelis_metadata_plan_rank(const chelis_metadata_plan *plan) {
    return static_cast<int32_t>(plan_ref(plan).shape.size());
}

CHELIS_WEAK const int64_t *chelis_metadata_plan_shape(const chelis_metadata_plan *plan) {
    const auto &p = plan_ref(plan);
    return p.shape.empty() ? nullptr : p.shape.data();
}

CHELIS_WEAK const int64_t *chelis_metadata_plan_strides(const chelis_metadata_plan *plan) {
    const auto &p = plan_ref(plan);
    return p.strides.empty() ? nullptr : p.strides.data();
}

CHELIS_WEAK int64_t chelis_metadata_plan_count(const chelis_metadata_plan *plan) {
    return plan_ref(plan).count;
}

CHELIS_WEAK int64_t chelis_metadata_plan_byte_count(const chelis_metadata_plan *plan) {
    return plan_ref(plan).bytes;
}

CHELIS_WEAK int64_t chelis_metadata_plan_byte_offset(const chelis_metadata_plan *plan,
                                                     chelis_scalar linear_index) {
    const auto &p = plan_ref(plan);
    const int64_t index = tagged_i64(linear_index);
    if (index < 0 || index >= p.count) plan_domain();
    int64_t rem = index, off = 0;
    for (int ax = static_cast<int>(p.shape.size()) - 1; ax >= 0; --ax) {
        off += (rem % p.shape[ax]) * p.strides[ax];
        rem /= p.shape[ax];
    }
    return off * width_of(p.dtype);
}

CHELIS_WEAK chelis_dtype chelis_metadata_plan_dtype(const chelis_metadata_plan *plan) {
    return plan_ref(plan).dtype;
}

CHELIS_WEAK void chelis_metadata_plan_check_capacity(const chelis_metadata_plan *plan,
                                                     chelis_scalar byte_capacity) {
    const auto &p = plan_ref(plan);
    const int64_t capacity = tagged_i64(byte_capacity);
    if (capacity < 0 || p.span_bytes > capacity) plan_domain();
}

CHELIS_WEAK void chelis_metadata_plan_release(chelis_metadata_plan *plan) {
    plan_ref(plan);
    delete plan;
}

CHELIS_WEAK chelis_tensor *chelis_alloc(int32_t rank, const int64_t *shape, chelis_dtype dtype) {
    int64_t count = 0, bytes = 0;
    auto sh = host_shape(rank, shape, dtype, "chelis_alloc", &count, &bytes);
    void *data = nullptr;
    if (bytes) {
        if (posix_memalign(&data, 32, static_cast<size_t>(bytes)) != 0 || !data)
            runtime_fail("chelis_alloc", "tensor allocation failed");
        std::memset(data, 0, static_cast<size_t>(bytes));
    }
    auto *t = new chelis_tensor();
    t->dtype = dtype;
    t->shape = std::move(sh);
    t->count = count;
    t->bytes = bytes;
    t->data = data;
    t->owned = true;
    t->guard.tensor = t;
    return t;
}

CHELIS_WEAK chelis_tensor *chelis_tensor_entry_borrow(int32_t rank, const int64_t *shape,
                                                      chelis_dtype dtype, const void *data,
                                                      int64_t byte_capacity) {
    const char *site = "chelis_tensor_entry_borrow";
    int64_t count = 0, bytes = 0;
    auto sh = host_shape(rank, shape, dtype, site, &count, &bytes);
    if (byte_capacity < bytes) runtime_fail(site, "capacity below the tensor's bytes");
    if (count && (!data || reinterpret_cast<uintptr_t>(data) % width_of(dtype)))
        runtime_fail(site, "null or misaligned data");
    auto *t = new chelis_tensor();
    t->dtype = dtype;
    t->shape = std::move(sh);
    t->count = count;
    t->bytes = bytes;
    t->data = const_cast<void *>(data);
    t->owned = false;
    t->guard.tensor = t;
    return t;
}

CHELIS_WEAK void chelis_tensor_retain(const chelis_tensor *tensor) {
    tensor_ref(tensor, "chelis_tensor_retain").refs.fetch_add(1);
}

CHELIS_WEAK void chelis_tensor_release(const chelis_tensor *tensor) {
    auto &t = tensor_ref(tensor, "chelis_tensor_release");
    if (t.refs.fetch_sub(1) == 1) {
        if (t.owned) std::free(t.data);
        delete &t;
    }
}

CHELIS_WEAK chelis_read_view chelis_tensor_read_view(const chelis_tensor *tensor) {
    auto &t = tensor_ref(tensor, "chelis_tensor_read_view");
    if (t.writing.load()) runtime_fail("chelis_tensor_read_view:", "tensor has a live write guard");
    chelis_read_view v{};
    v.data = t.count ? t.data : nullptr;
    v.count = t.count;
    v.dtype = t.dtype;
    return v;
}

CHELIS_WEAK chelis_tensor_write *chelis_tensor_begin_write(chelis_tensor *tensor) {
    auto &t = tensor_ref(tensor, "chelis_tensor_begin_write");
    if (t.refs.load() != 1)
        runtime_fail("chelis_tensor_begin_write", "requires a unique tensor owner");
    if (!t.owned) runtime_fail("chelis_tensor_begin_write", "requires runtime-owned storage");
    int idle = 0;
    if (!t.writing.compare_exchange_strong(idle, 1))
        runtime_fail("chelis_tensor_begin_write", "tensor already has a write guard");
    return &t.guard;
}

CHELIS_WEAK chelis_write_view chelis_tensor_write_view(const chelis_tensor_write *guard) {
    if (!guard || !guard->tensor || guard != &guard->tensor->guard)
        runtime_fail("chelis_tensor_write_view:", "invalid tensor write guard");
    const chelis_tensor &t = *guard->tensor;
    if (!t.writing.load()) runtime_fail("chelis_tensor_write_view:", "tensor write guard has ended");
    chelis_write_view v{};
    v.data = t.count ? t.data : nullptr;
    v.count = t.count;
    v.dtype = t.dtype;
    return v;
}

CHELIS_WEAK void chelis_tensor_end_write(chelis_tensor_write *guard) {
    if (!guard || !guard->tensor || guard != &guard->tensor->guard)
        runtime_fail("chelis_tensor_end_write:", "invalid tensor write guard");
    int writing = 1;
    if (!guard->tensor->writing.compare_exchange_strong(writing, 0))
        runtime_fail("chelis_tensor_end_write:", "tensor write guard has ended");
}

CHELIS_WEAK int32_t chelis_tensor_rank(const chelis_tensor *tensor) {
    return static_cast<int32_t>(tensor_ref(tensor, "chelis_tensor_rank").shape.size());
}

CHELIS_WEAK int64_t chelis_tensor_shape(const chelis_tensor *tensor, int32_t axis) {
    auto &t = tensor_ref(tensor, "chelis_tensor_shape");
    if (axis < 0 || axis >= static_cast<int32_t>(t.shape.size()))
        fail_line("numeric trap: domain in shape at i64");
    return t.shape[axis];
}

CHELIS_WEAK int64_t chelis_tensor_numel(const chelis_tensor *tensor) {
    return tensor_ref(tensor, "chelis_tensor_numel").count;
}

CHELIS_WEAK int64_t chelis_tensor_byte_count(const chelis_tensor *tensor) {
    return tensor_ref(tensor, "chelis_tensor_byte_count").bytes;
}
