// common.cuh -- shared device helpers for the Chelis sm_100a backend.
//
// * status / device error word used by every kernel that waits on an
//   mbarrier (bounded waits report a timeout instead of hanging);
// * inline-PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, never with
//   .multicast::cluster) and tcgen05 (alloc / mma / commit / ld);
// * the canonical adjacent-pair tree in warp / block form;
// * the keyed RNG of [05-RNG-1/2].
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "chelis_cuda.h"

namespace chelis {

// ---------------------------------------------------------------------------
// host-side status helpers (runtime.cu)
// ---------------------------------------------------------------------------
int set_error(int status, const char *fmt, ...);
int check_cuda(cudaError_t err, const char *what);
cudaStream_t current_stream();
int current_device_checked(int *device);
// Stream-ordered scratch from the library's pool.
int scratch_alloc(void **ptr, size_t bytes, cudaStream_t stream);
void scratch_free(void *ptr, cudaStream_t stream);
int sm_count();
// GuardedFail messages, by id, for chelis_cuda_device_status (runtime.cu)
uint32_t register_fail_message(const char *message);
void unregister_fail_message(uint32_t id);
// data-parallel communicator (dp.cu): its size (1 when none is open), the
// library's communication stream, an f32 sum all-reduce on a given stream
int dp_nranks();
int dp_comm_stream(cudaStream_t *out);
int dp_allreduce_f32_on(float *buf, int64_t count, cudaStream_t s);

#define CHELIS_TRY(expr)                   \
    do {                                   \
        int _st = (expr);                  \
        if (_st != CHELIS_CUDA_OK) return _st; \
    } while (0)

#define CHELIS_LAUNCH_CHECK(name) \
    CHELIS_TRY(::chelis::check_cuda(cudaGetLastError(), name))

// Device error word: one bit per kind of bounded wait that gave up.  Read
// and cleared by chelis_cuda_device_status().  The library is built as one
// translation unit (libchelis_cuda.cu), so this is its only definition.
__device__ unsigned int g_device_error = 0;

enum : unsigned int {
    DEVERR_TIMEOUT_PRODUCER = 1u,
    DEVERR_TIMEOUT_MMA = 2u,
    DEVERR_TIMEOUT_EPILOGUE = 4u,
    DEVERR_TIMEOUTS = 7u,
    DEVERR_BAD_INDEX = 8u,  // an index operand outside its axis ([05-OP-52])
    DEVERR_DROPOUT_F32 = 16u,  // a dropout rate outside [0, 1) ([05-OP-37]), f32 draw
    DEVERR_DROPOUT_F64 = 32u,  // the same, f64 draw
    DEVERR_TRAP = 64u,         // a numeric trap recorded in g_trap_code (first one wins)
    DEVERR_SHIFT = 128u,       // a negative shift count, recorded in g_shift_count
    DEVERR_FAIL = 256u,        // a GuardedFail fired: its message id in g_fail_id
};
__device__ unsigned int g_fail_id = 0;  // the first fired guard's registered message id
__device__ unsigned long long g_shift_count = 0;  // the first negative count reported (its bits)

// A numeric trap raised on the device: kind, operation and dtype packed as
// 1 + (kind << 16 | op << 8 | dtype), kept for the first trap only, read and
// cleared with the error word; chelis_cuda_device_status() renders it as
// "numeric trap: <kind> in <op> at <dtype>".
__device__ unsigned int g_trap_code = 0;
enum : unsigned int { TRAP_OVERFLOW = 0u, TRAP_DOMAIN = 1u, TRAP_DIVZERO = 2u };
enum : unsigned int {
    TRAP_OP_ADD = 0u, TRAP_OP_SUB, TRAP_OP_MUL, TRAP_OP_TRUNC_DIV, TRAP_OP_FLOOR_DIV, TRAP_OP_MOD,
    TRAP_OP_NEG, TRAP_OP_ABS, TRAP_OP_CAST, TRAP_OP_CAST_TRUNC, TRAP_OP_CAST_SATURATE, TRAP_OP_UNIFORM_LIKE,
    TRAP_OP_RANGE, TRAP_OP_REDUCE_WINDOW_SUM, TRAP_OP_GATHER, TRAP_OP_SCATTER_ADD, TRAP_OP_SCATTER,
    TRAP_OP_SCATTER_ELEMENTS
};
// The offending index of a sparse-index trap ([05-SPARSE-1]): index, axis and
// the axis extent, written by the thread whose trap was recorded first.
__device__ long long g_trap_index[3] = {0, 0, 0};
enum : unsigned int { TRAP_DTYPE_I64 = 4u };

__device__ __forceinline__ void report_device_error(unsigned int code) {
    atomicOr(&g_device_error, code);
}
__device__ __forceinline__ void report_trap(unsigned int kind, unsigned int op, unsigned int dtype) {
    atomicCAS(&g_trap_code, 0u, 1u + ((kind << 16) | (op << 8) | dtype));
    atomicOr(&g_device_error, static_cast<unsigned int>(DEVERR_TRAP));
}
// An index outside [0, extent) of a gather or scatter: a domain trap at i64
// that also keeps the offending index for the message.
__device__ __forceinline__ void report_index_trap(unsigned int op, int64_t index, int axis, int64_t extent) {
    if (atomicCAS(&g_trap_code, 0u, 1u + ((TRAP_DOMAIN << 16) | (op << 8) | TRAP_DTYPE_I64)) == 0u) {
        g_trap_index[0] = index;
        g_trap_index[1] = axis;
        g_trap_index[2] = extent;
    }
    atomicOr(&g_device_error, static_cast<unsigned int>(DEVERR_TRAP));
}

// ---------------------------------------------------------------------------
// shared-memory addresses
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait with a suspend-time hint of 1 us: the thread sleeps at most that
// long before the probe reports "not yet".
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}
// try_wait that acquires at cluster scope: pairs with arrivals that other
// CTAs of the cluster make with release.cluster (mbar_arrive_cluster).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
        : "memory");
    return ok != 0;
}
// Arrive (release, cluster scope) on an mbarrier given by its
// shared::cluster address, in this CTA or another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// Bounded wait: at most kMaxTries probes of at most ~1 us each (a few
// seconds), far beyond any legal stall of these kernels (a whole CTA tile
// main loop is well under 100 ms even at k = 10^6).  On timeout the error bit
// is recorded and false is returned: the caller skips its remaining work and
// proceeds to teardown.
// The limit is a device variable (default kMaxTries) that the host may
// lower with chelis_cuda_set_wait_limit, so a test can make a wait run out
// in about a millisecond and check the reported status.
constexpr uint32_t kMaxTries = 1u << 22;
__device__ uint32_t g_wait_tries = kMaxTries;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  unsigned int err_code) {
    const uint32_t tries = *static_cast<volatile uint32_t *>(&g_wait_tries);
    for (uint32_t i = 0; i < tries; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    report_device_error(err_code);
    return false;
}
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity,
                                                          unsigned int err_code) {
    const uint32_t tries = *static_cast<volatile uint32_t *>(&g_wait_tries);
    for (uint32_t i = 0; i < tries; ++i)
        if (mbar_try_wait_cluster(bar, parity)) return true;
    report_device_error(err_code);
    return false;
}

// ---------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// row (lane base + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2).  The pair is the two CTAs
// whose %cluster_ctarank differs in bit 0; rank 0 issues the MMAs, each CTA
// holds half of A (along M) and half of B (along N) in its own shared memory
// and its half of the accumulator rows in its own TMEM.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the variable at the same offset in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
    return r;
}
// Tiled TMA loads into this CTA's shared memory whose completion bytes go to
// an mbarrier that may live in the pair's other CTA (`bar` is a
// shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar,
                                                 int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// TMEM allocation for the pair: one warp (same warp index) in each CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D[tmem of both CTAs] (+)= A . B, kind::tf32, M = 256 across the pair;
// issued by one thread of rank 0.
__device__ __forceinline__ void mma_tf32_ss_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the mbarrier at this offset in every CTA of `cta_mask`
// when the pair MMAs issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::tf32, one CTA.  A is M x K with
// row m in TMEM lane m and element k in column (a + k).
__device__ __forceinline__ void mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers: thread t of the
// warp writes row (lane base + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte swizzle layout that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N.
//   bits  0-13  start address >> 4
//   bits 16-29  leading byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45  stride byte offset >> 4 (1024 bytes between 8-row groups)
//   bits 46-47  descriptor version (1 on sm_100)
//   bits 49-51  base offset (0: atoms are 1024-byte aligned)
//   bits 61-63  layout (2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for kind::tf32 with f32 accumulation, both operands
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4)                                   // D format f32
           | (2u << 7)                                 // A format tf32
           | (2u << 10)                                // B format tf32
           | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
           | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

// ---------------------------------------------------------------------------
// canonical adjacent-pair tree (spec/05-risc-primitives.md:452-466,515-531)
// ---------------------------------------------------------------------------
// The pass-by-pass adjacent-pair tree over a prefix of valid leaves equals
// the xor butterfly over aligned power-of-two groups in which an absent
// operand passes the other through unchanged.  IEEE addition is commutative,
// so which partner sits on the left does not change a single sum.
template <typename T>
__device__ __forceinline__ T tree_pair(T a, bool va, T b, bool vb) {
    return va ? (vb ? a + b : a) : b;
}
template <typename T>
__device__ __forceinline__ T warp_tree(T v, bool &valid) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        T o = __shfl_xor_sync(0xffffffffu, v, off);
        bool ov = __shfl_xor_sync(0xffffffffu, valid ? 1 : 0, off) != 0;
        bool left = ((threadIdx.x & 31) & off) == 0;
        // left partner holds the lower group; the sum is the same either way
        T s = left ? tree_pair(v, valid, o, ov) : tree_pair(o, ov, v, valid);
        valid = valid || ov;
        v = s;
    }
    return v;
}
// Full-warp butterfly when every lane is valid.
__device__ __forceinline__ float warp_tree_full(float v) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
__device__ __forceinline__ double warp_tree_full(double v) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

// ---------------------------------------------------------------------------
// keyed RNG (crates/chelis-numeric-core/src/dtype_semantics.rs:4508-4540)
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint64_t splitmix64(uint64_t v) {
    v += 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
    return v ^ (v >> 31);
}
__host__ __device__ __forceinline__ uint64_t rng_word(uint64_t key, uint64_t index) {
    uint64_t s = splitmix64(index);
    return splitmix64(key ^ ((s << 41) | (s >> 23)));
}
// Keep decision of PreparedDropout::apply for an f32 draw: keep iff
// round_f32(unit) >= rate.  round_f32(unit) = RN_f32(w >> 11) * 2^-53 exactly
// (a power-of-two scale commutes with rounding), and RN_f32 is monotone, so
// the test is (w >> 11) >= threshold with threshold the least 53-bit integer
// whose f32 rounding reaches rate * 2^53 (computed exactly on the host by
// dropout_threshold()).
//
// (w >> 11) >= threshold  <=>  w >= lim = threshold << 11 (threshold < 2^53).
// The last splitmix64 step is w = z ^ (z >> 31) with z = u * C2 mod 2^64, so
// the top 32 bits of w are zh ^ (zh >> 31), zh = hi32(z) =
// umulhi(lo(u), lo(C2)) + lo(u) hi(C2) + hi(u) lo(C2) mod 2^32.  Those bits
// decide the comparison unless they equal the top 32 bits of lim (once in
// 2^32 draws), when the full word is formed.
__host__ __device__ __forceinline__ uint32_t mulhi_u32(uint32_t a, uint32_t b) {
#ifdef __CUDA_ARCH__
    return __umulhi(a, b);
#else
    return static_cast<uint32_t>((static_cast<uint64_t>(a) * b) >> 32);
#endif
}
__host__ __device__ __forceinline__ bool dropout_keep(uint64_t key, uint64_t index, uint64_t threshold) {
    constexpr uint64_t C2 = 0x94d049bb133111ebull;
    constexpr uint32_t C2L = static_cast<uint32_t>(C2), C2H = static_cast<uint32_t>(C2 >> 32);
    const uint64_t s = splitmix64(index);
    uint64_t v = (key ^ ((s << 41) | (s >> 23))) + 0x9e3779b97f4a7c15ull;
    v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
    v ^= v >> 27;
    const uint64_t lim = threshold << 11;
    const uint32_t ul = static_cast<uint32_t>(v), uh = static_cast<uint32_t>(v >> 32);
    const uint32_t zh = mulhi_u32(ul, C2L) + ul * C2H + uh * C2L;
    const uint32_t wh = zh ^ (zh >> 31), lh = static_cast<uint32_t>(lim >> 32);
    if (wh != lh) return wh > lh;
    const uint64_t z = v * C2;
    return (z ^ (z >> 31)) >= lim;
}

}  // namespace chelis
