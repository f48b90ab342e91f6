// gemm_tf32x3.cu -- f32 GEMM on the sm_100a tensor cores with 3xTF32
// split-accumulate, plus the bit-exact CUDA-core "canonical tree" GEMM.
//
// Replaces chelis_hipblas_sgemm_*_row_major
// (crates/chelis-backend-hip/runtime/chelis_hip_runtime.h:48-267).
//
// 3xTF32: each f32 operand x is split into hi = RN_tf32(x) and
// lo = RN_tf32(x - hi) (x - hi is exact in f32).  The product a.b is then
// accumulated as a_lo.b_hi + a_hi.b_lo + a_hi.b_hi in the f32 accumulator
// of tcgen05.mma kind::tf32; the dropped a_lo.b_lo term is below 2^-22
// relative.  The split runs as a pre-pass in the operand's own orientation
// (one streaming read, two writes): a K-contiguous operand becomes K-major
// [rows][Kp] (Kp = K rounded up to 32), an MN-contiguous one (row-major B,
// transposed A) MN-major [K][MNp] (MNp = MN rounded up to 4), both zero
// padded; only operands with neither stride 1 go through a transposing
// tile kernel.  The main kernel streams four tiles per stage with TMA
// (128-byte swizzle) and tells tcgen05.mma each operand's major-ness.
//
// Main kernel (one 128 x 256 output tile per CTA, or 256 x 256 per CTA
// pair, 320 threads per CTA):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2-9   epilogue: fold the accumulator chunks (below) into f32
//               registers, then store the 128 x 256 tile rows to C
//
// Chunked accumulation.  The tensor core's f32 accumulator does not add like
// a chain of IEEE additions: kept over a long K in one TMEM accumulator, the
// error grows linearly with K (measured against float64: normwise 2e-6 at
// K = 256, 5.8e-5 at K = 8192, 16x cuBLAS's FFMA GEMM there).  So every
// accumulator covers CHUNK_KB k-blocks (128 of K) from a fresh start,
// alternating between two 256-column TMEM buffers, and the eight epilogue
// warps fold each finished chunk into f32 registers with IEEE additions
// (two warps per TMEM lane quadrant, 128 columns each) while the MMAs fill
// the other buffer.  Error then grows like an f32 sum of K/128 terms.
// Every mbarrier wait is bounded (common.cuh) so a fault in the pipeline
// reports CHELIS_CUDA_ERR_TIMEOUT instead of hanging the GPU.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int gemm_mode();
// 1: 3xTF32 products with more than 128 rows run on CTA pairs (default);
// 0: one CTA per 128 x 256 tile everywhere
std::atomic<int> g_pair_tiles{1};

namespace tf32x3 {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 32;  // 32 f32 = 128 bytes = one swizzle row
constexpr int STAGES = 2;
constexpr int A_TILE_BYTES = BM * BK * 4;  // 16 KiB
constexpr int B_TILE_BYTES = BN * BK * 4;  // 32 KiB
constexpr int STAGE_BYTES = 2 * A_TILE_BYTES + 2 * B_TILE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int EPI_WARPS = 8;                 // warps 2..9
constexpr int THREADS = 64 + 32 * EPI_WARPS;  // 320
// k-blocks per fresh accumulator.  Measured at 8192^3 (normwise error vs
// float64, main kernel ms): 2 -> 8.6e-7, 4.53; 4 -> 9.9e-7, 4.20; 8 ->
// 1.8e-6, 4.58; 16 -> 3.9e-6, 4.48; one accumulator -> 6.5e-5, 4.36.
constexpr int CHUNK_KB = 4;
constexpr uint32_t ACC_COLS = 256;            // one 128 x 256 f32 accumulator
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;  // two, alternating by chunk
constexpr int MN_BOX = 32;                  // MN-major TMA box: 32 (MN) x 32 (K) f32
constexpr int MN_BOX_BYTES = MN_BOX * BK * 4;  // 4 KiB

struct Params {
    int64_t m, n, batch;
    int64_t pairs_m, tiles_n;  // pair kernel: 256-row tile count, 256-column tile count
    int32_t num_kb;       // ceil(K / BK)
    int64_t a_rows_per_batch, b_rows_per_batch;  // K-major split buffers: rows per batch item
    float *c;
    int64_t ldc, stride_c;
    // pair kernel split-K: blockIdx.z = batch * splits + split; split s covers
    // k-blocks [s * kb_per_split, (s + 1) * kb_per_split) and writes its
    // partial product to part[blockIdx.z] ([m][n], dense) when splits > 1
    int32_t splits, kb_per_split;
    float *part;
    int32_t chunk_kb;  // k-blocks per fresh accumulator (CHUNK_KB)
    // fused epilogue (EPI_*): epi_in is indexed like C
    int32_t epi;
    const float *epi_in;
};

// Work folded into the store of a finished C value v at index i of C's
// layout: EPI_ADD, C = v + in[i] (a residual add; in shares C's layout).
// Elementwise work heavier than an add does not belong here: the epilogue
// runs on one CTA's eight warps per SM after the tile's last MMA, so an erfc
// per element (gelu) leaves the tensor pipe idle for its latency.  Measured:
// gelu and its adjoint folded into the block step's epilogues (with scalar
// stores of the tf32 splits) took the step from 10.8 to 15.0 ms at batch 8.
enum Epi : int32_t { EPI_NONE = 0, EPI_ADD = 1 };
struct EpiArgs {
    int32_t op = EPI_NONE;
    const float *in = nullptr;
};

// Operand layouts in shared memory (both written by TMA):
//  K-major  (operand stored [rows][K]): one box of `rows` x 32 K, 128-byte
//           swizzle of 16-byte chunks; 128-byte rows along K, 8-row atoms
//           1024 B apart; an MMA K-step of 8 moves the start 32 B along the
//           swizzled row.
//  MN-major (operand stored [K][rows]): rows/32 boxes of 32 (MN) x 32 (K),
//           4 KiB apart; inside a box one 128-byte row along MN per k.  For
//           32-bit operands tcgen05 reads MN-major data only in the
//           "128-byte span, 32-byte chunk" swizzle (descriptor layout 1,
//           TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B), whose atom is 4 rows
//           (512 B).  LBO = 4096 (next 32 MN), SBO = 512 (next 4 k); an MMA
//           K-step of 8 moves the start 1024 B.
__device__ __forceinline__ uint64_t sw128a32_mnmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(MN_BOX_BYTES >> 4) << 16;  // leading byte offset
    d |= static_cast<uint64_t>(512u >> 4) << 32;          // stride byte offset
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(1u) << 61;                 // 128B swizzle, 32B atoms
    return d;
}
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, int kk) {
    return MN ? sw128a32_mnmajor_desc(tile + kk * 1024) : sw128_kmajor_desc(tile + kk * 32);
}

// Load one operand's tile for k-block `kb` into `dst`.
template <bool MN, int ROWS>
__device__ __forceinline__ void load_operand(unsigned char *dst, const CUtensorMap *map,
                                             uint64_t *bar, int kb, int32_t row0, int32_t y_kmaj,
                                             int32_t batch) {
    if (MN) {
#pragma unroll
        for (int j = 0; j < ROWS / MN_BOX; ++j)
            tma_load_3d(dst + j * MN_BOX_BYTES, map, bar, row0 + j * MN_BOX, kb * BK, batch);
    } else {
        tma_load_2d(dst, map, bar, kb * BK, y_kmaj);
    }
}

// Epilogue warps (2..9): fold the tile's accumulator chunks into `run` (this
// thread's row, this warp's 128 columns), releasing each buffer to the MMA
// issuer once read.  Chunks are numbered from the kernel's start (c0 is this
// tile's first): chunk c sits in TMEM buffer c & 1 and is that buffer's
// (c >> 1)-th use.  In a CTA pair the release goes to rank 0's barrier (the
// issuer's), from both CTAs.  False on a timeout or an aborted pipeline.
template <bool PAIR>
__device__ __forceinline__ bool fold_chunks(uint32_t tmem_base, int c0, int nchunks,
                                            uint64_t *chunk_full, uint64_t *chunk_empty, int warp,
                                            int lane, float (&run)[128],
                                            volatile uint32_t *abort_flag) {
    const int quad = warp & 3;          // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;   // warps 2-5: columns 0..127, 6-9: 128..255
    const uint32_t lanes = static_cast<uint32_t>(quad * 32) << 16;
    for (int c = c0; c < c0 + nchunks; ++c) {
        const int b = c & 1;
        if (!mbar_wait_bounded(&chunk_full[b], (c >> 1) & 1, DEVERR_TIMEOUT_EPILOGUE)) {
            *abort_flag = 1;
            return false;
        }
        tc_fence_after();
        if (*abort_flag) return false;
        const uint32_t base = tmem_base + lanes + static_cast<uint32_t>(b) * ACC_COLS +
                              static_cast<uint32_t>(half * 128);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(base + j * 32, r);
            tmem_wait_ld();
            if (c == c0) {
#pragma unroll
                for (int t = 0; t < 32; ++t) run[j * 32 + t] = __uint_as_float(r[t]);
            } else {
#pragma unroll
                for (int t = 0; t < 32; ++t)
                    run[j * 32 + t] = __fadd_rn(run[j * 32 + t], __uint_as_float(r[t]));
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            if (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&chunk_empty[b]), 0));
            else mbar_arrive(&chunk_empty[b]);
        }
    }
    return true;
}

// This thread's row (m0 + lane quadrant row), this warp's 128 columns, to C.
__device__ __forceinline__ void store_run(const float (&run)[128], int warp, int lane, int64_t m0,
                                          int64_t n0, int64_t batch, const Params &p) {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int64_t row = m0 + quad * 32 + lane;
    if (row >= p.m) return;
    const int64_t rbase = batch * p.stride_c + row * p.ldc;
    float *crow = p.c + rbase;
    const float *irow = p.epi == EPI_ADD ? p.epi_in + rbase : nullptr;
    const int64_t col0 = n0 + half * 128;
    const bool vec_ok = ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.c) & 15) == 0) &&
                        ((p.stride_c & 3) == 0) &&
                        (!irow || (reinterpret_cast<uintptr_t>(p.epi_in) & 15) == 0);
    if (vec_ok && col0 + 128 <= p.n) {
        if (irow) {
#pragma unroll
            for (int j = 0; j < 128; j += 4) {
                const float4 a = *reinterpret_cast<const float4 *>(irow + col0 + j);
                *reinterpret_cast<float4 *>(crow + col0 + j) =
                    make_float4(__fadd_rn(run[j], a.x), __fadd_rn(run[j + 1], a.y),
                                __fadd_rn(run[j + 2], a.z), __fadd_rn(run[j + 3], a.w));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 128; j += 4)
                *reinterpret_cast<float4 *>(crow + col0 + j) =
                    make_float4(run[j], run[j + 1], run[j + 2], run[j + 3]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 128; ++j)
            if (col0 + j < p.n) crow[col0 + j] = irow ? __fadd_rn(run[j], irow[col0 + j]) : run[j];
    }
}

template <bool AMN, bool BMN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_ahi,
                const __grid_constant__ CUtensorMap map_alo,
                const __grid_constant__ CUtensorMap map_bhi,
                const __grid_constant__ CUtensorMap map_blo, Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment for the swizzle atoms
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *chunk_full = empty + STAGES;   // [2]: MMA commit of a chunk
    uint64_t *chunk_empty = chunk_full + 2;  // [2]: epilogue warps have read it
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(chunk_empty + 2);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile int32_t *consumed = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);
    int32_t issued = 0;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
    const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;
    const int64_t batch = blockIdx.z;
    const int nchunks = (p.num_kb + p.chunk_kb - 1) / p.chunk_kb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&chunk_full[b], 1);
            mbar_init(&chunk_empty[b], EPI_WARPS);
        }
        *abort_flag = 0;
        *consumed = 0;
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&map_ahi);
        prefetch_tensormap(&map_alo);
        prefetch_tensormap(&map_bhi);
        prefetch_tensormap(&map_blo);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const int32_t ya = static_cast<int32_t>(batch * p.a_rows_per_batch + m0);
            const int32_t yb = static_cast<int32_t>(batch * p.b_rows_per_batch + n0);
            const int32_t z = static_cast<int32_t>(batch);
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int s = kb % STAGES;
                const uint32_t phase = (kb / STAGES) & 1;
                if (!mbar_wait_bounded(&empty[s], phase ^ 1, DEVERR_TIMEOUT_PRODUCER)) {
                    *abort_flag = 1;
                    break;
                }
                unsigned char *st = smem + s * STAGE_BYTES;
                mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
                load_operand<AMN, BM>(st, &map_ahi, &full[s], kb, static_cast<int32_t>(m0), ya, z);
                load_operand<AMN, BM>(st + A_TILE_BYTES, &map_alo, &full[s], kb,
                                      static_cast<int32_t>(m0), ya, z);
                load_operand<BMN, BN>(st + 2 * A_TILE_BYTES, &map_bhi, &full[s], kb,
                                      static_cast<int32_t>(n0), yb, z);
                load_operand<BMN, BN>(st + 2 * A_TILE_BYTES + B_TILE_BYTES, &map_blo, &full[s],
                                      kb, static_cast<int32_t>(n0), yb, z);
                issued = kb + 1;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_tf32(BM, BN) | (AMN ? (1u << 15) : 0u) |
                                       (BMN ? (1u << 16) : 0u);
            int cur = 0;  // accumulator buffer of the chunk in progress
            for (int kb = 0; kb < p.num_kb; ++kb) {
                const int c = kb / p.chunk_kb;
                const bool first = (kb % p.chunk_kb) == 0;
                cur = c & 1;
                // buffer `cur` last held chunk c - 2: wait until it was folded
                if (first && c >= 2) {
                    if (!mbar_wait_bounded(&chunk_empty[cur], ((c >> 1) - 1) & 1,
                                           DEVERR_TIMEOUT_MMA)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                }
                const int s = kb % STAGES;
                const uint32_t phase = (kb / STAGES) & 1;
                if (!mbar_wait_bounded(&full[s], phase, DEVERR_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * STAGE_BYTES);
                const uint32_t ahi = st, alo = st + A_TILE_BYTES;
                const uint32_t bhi = st + 2 * A_TILE_BYTES;
                const uint32_t blo = bhi + B_TILE_BYTES;
                const uint32_t d = tmem_base + static_cast<uint32_t>(cur) * ACC_COLS;
#pragma unroll
                for (int kk = 0; kk < BK / 8; ++kk) {
                    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
                    mma_tf32_ss(d, operand_desc<AMN>(alo, kk), operand_desc<BMN>(bhi, kk), idesc,
                                acc);
                    mma_tf32_ss(d, operand_desc<AMN>(ahi, kk), operand_desc<BMN>(blo, kk), idesc,
                                1u);
                    mma_tf32_ss(d, operand_desc<AMN>(ahi, kk), operand_desc<BMN>(bhi, kk), idesc,
                                1u);
                }
                mma_commit(&empty[s]);
                *consumed = kb + 1;
                if ((kb % p.chunk_kb) == p.chunk_kb - 1 || kb == p.num_kb - 1)
                    mma_commit(&chunk_full[cur]);
            }
            // on abort, release the epilogue waiting for the unfinished chunk
            if (*abort_flag) mma_commit(&chunk_full[cur]);
        }
    } else {
        // ---------------- epilogue (warps 2..9) ----------------
        float run[128];
#pragma unroll
        for (int j = 0; j < 128; ++j) run[j] = 0.0f;  // K = 0: the empty sum
        if (fold_chunks<false>(tmem_base, 0, nchunks, chunk_full, chunk_empty, warp, lane, run,
                               abort_flag))
            store_run(run, warp, lane, m0, n0, batch, p);
    }

    tc_fence_before();
    __syncthreads();
    // On an aborted pipeline, let TMA copies that were issued but never
    // consumed land before the CTA exits (bounded as well).
    if (warp == 0 && lane == 0 && *abort_flag) {
        for (int kb = *consumed; kb < issued; ++kb)
            mbar_wait_bounded(&full[kb % STAGES], (kb / STAGES) & 1, DEVERR_TIMEOUT_PRODUCER);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair main kernel: 256 x 256 output tiles on clusters of 2 CTAs
// (tcgen05 cta_group::2, M = 256), persistent: cluster c takes tiles c,
// c + clusters, ... (tiles numbered batch/split-major, grouped order inside),
// and the stage ring and the two accumulator buffers run on across tiles,
// so the MMAs of a tile's first chunks overlap the previous tile's last fold
// and its stores.  Each CTA stages its 128 rows of A and
// its 128 rows of B^T (half of the tile's columns), so one pair MMA reads
// 8 KiB of operands per SM per K-step of 8 instead of 12 KiB: the shared
// memory port stays below its limit with the TMA writes included, and the
// tensor pipe, not shared memory, bounds the main loop.  Rank 0 issues the
// MMAs; both CTAs' TMA loads report to rank 0's `full` barriers; the MMA
// commits release both CTAs' `empty` barriers and both accumulators.
// ---------------------------------------------------------------------------
constexpr int P_STAGES = 3;
constexpr int P_ROWS = 128;  // A rows and B rows per CTA
constexpr int P_TILE_BYTES = P_ROWS * BK * 4;   // 16 KiB
constexpr int P_STAGE_BYTES = 4 * P_TILE_BYTES;  // A hi, A lo, B hi, B lo
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;
constexpr uint64_t P_DRAIN_NS = 200000;  // bounded drain of an aborted rank 1
constexpr int P_GROUP = 8;                // pair-rows per group of the tile order
// Persistent launches for tiles of at most this many k-blocks (K <= 2048 per
// split).  Measured: K = 1024 products of the transformer block 8-10 %
// faster persistent; 8192^3 (256 k-blocks per tile) 4 % slower, where a
// static round-robin of ~14 tiles per cluster loses the hardware's dynamic
// hand-out of tiles to clusters that finish early.
constexpr int P_PERSIST_KB = 64;

template <bool MN>
__device__ __forceinline__ void load_operand_pair(unsigned char *dst, const CUtensorMap *map,
                                                  uint32_t bar, int kb, int32_t row0,
                                                  int32_t y_kmaj, int32_t batch) {
    if (MN) {
#pragma unroll
        for (int j = 0; j < P_ROWS / MN_BOX; ++j)
            tma_load_3d_pair(dst + j * MN_BOX_BYTES, map, bar, row0 + j * MN_BOX, kb * BK, batch);
    } else {
        tma_load_2d_pair(dst, map, bar, kb * BK, y_kmaj);
    }
}

// Tile L of a pair launch: its rows (this CTA's 128 of A), columns (this
// CTA's 128 of B^T), batch item, split and k-block range.  Within one batch
// item and split, consecutive tiles walk P_GROUP pair-rows down one column of
// tiles before moving right, so the ~74 pairs in flight share a few A and B
// panels in L2 instead of streaming all of A.
struct PairTile {
    int64_t m0, n0, nb0, zz, batch;
    int kb_lo, nk, nchunks;
};
__device__ __forceinline__ PairTile pair_tile(const Params &p, int64_t L, uint32_t rank) {
    PairTile t;
    const int64_t tiles_mn = p.pairs_m * p.tiles_n;
    const int64_t pid = L % tiles_mn;
    t.zz = L / tiles_mn;
    const int64_t per_group = static_cast<int64_t>(P_GROUP) * p.tiles_n;
    const int64_t first = (pid / per_group) * P_GROUP;
    const int64_t rem = p.pairs_m - first;
    const int64_t gsize = rem < P_GROUP ? rem : P_GROUP;
    const int64_t in = pid % per_group;
    const int64_t pm = first + in % gsize, pn = in / gsize;
    t.m0 = pm * (2 * P_ROWS) + rank * P_ROWS;
    t.n0 = pn * BN;
    t.nb0 = t.n0 + rank * P_ROWS;
    const int split = static_cast<int>(t.zz % p.splits);
    t.batch = t.zz / p.splits;
    t.kb_lo = split * p.kb_per_split;
    t.nk = (p.num_kb - t.kb_lo < p.kb_per_split) ? p.num_kb - t.kb_lo : p.kb_per_split;
    t.nchunks = (t.nk + p.chunk_kb - 1) / p.chunk_kb;
    return t;
}

template <bool AMN, bool BMN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_ahi,
                     const __grid_constant__ CUtensorMap map_alo,
                     const __grid_constant__ CUtensorMap map_bhi,
                     const __grid_constant__ CUtensorMap map_blo, Params p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // The dynamic shared window starts at the same offset in both CTAs, so
    // the aligned tiles and barriers below do too (the pair MMA and the
    // multicast commits address the peer by offset).
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + P_STAGES * P_STAGE_BYTES);
    uint64_t *empty = full + P_STAGES;
    uint64_t *chunk_full = empty + P_STAGES;  // [2]: MMA commit of a chunk (both CTAs)
    uint64_t *chunk_empty = chunk_full + 2;   // [2]: rank 0's; both CTAs' epilogues arrive
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(chunk_empty + 2);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile int32_t *consumed = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);
    int32_t issued = 0;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int64_t total_tiles = p.pairs_m * p.tiles_n * p.batch * p.splits;
    const int64_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&chunk_full[b], 1);
            mbar_init(&chunk_empty[b], 2 * EPI_WARPS);
        }
        *abort_flag = 0;
        *consumed = 0;
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&map_ahi);
        prefetch_tensormap(&map_alo);
        prefetch_tensormap(&map_bhi);
        prefetch_tensormap(&map_blo);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, TMEM_COLS);
        tmem_relinquish_pair();
    }
    // barrier inits of both CTAs are visible cluster-wide before any remote
    // arrival (TMA bytes from rank 1, multicast commits from rank 0, chunk
    // releases from rank 1's epilogue)
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (lane == 0) {
            int32_t it = 0;  // k-blocks issued since the kernel started
            bool ok = true;
            for (int64_t L = cluster; ok && L < total_tiles; L += clusters) {
                const PairTile t = pair_tile(p, L, rank);
                const int32_t ya = static_cast<int32_t>(t.batch * p.a_rows_per_batch + t.m0);
                const int32_t yb = static_cast<int32_t>(t.batch * p.b_rows_per_batch + t.nb0);
                const int32_t z = static_cast<int32_t>(t.batch);
                for (int i = 0; i < t.nk; ++i, ++it) {
                    const int kb = t.kb_lo + i;
                    const int s = it % P_STAGES;
                    const uint32_t phase = (it / P_STAGES) & 1;
                    if (!mbar_wait_bounded(&empty[s], phase ^ 1, DEVERR_TIMEOUT_PRODUCER)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * P_STAGE_BYTES);
                    unsigned char *st = smem + s * P_STAGE_BYTES;
                    load_operand_pair<AMN>(st, &map_ahi, bar, kb, static_cast<int32_t>(t.m0), ya, z);
                    load_operand_pair<AMN>(st + P_TILE_BYTES, &map_alo, bar, kb,
                                           static_cast<int32_t>(t.m0), ya, z);
                    load_operand_pair<BMN>(st + 2 * P_TILE_BYTES, &map_bhi, bar, kb,
                                           static_cast<int32_t>(t.nb0), yb, z);
                    load_operand_pair<BMN>(st + 3 * P_TILE_BYTES, &map_blo, bar, kb,
                                           static_cast<int32_t>(t.nb0), yb, z);
                    issued = it + 1;
                }
                if (*abort_flag) ok = false;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (rank 0 only) ----------------
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_tf32(2 * P_ROWS, BN) | (AMN ? (1u << 15) : 0u) |
                                       (BMN ? (1u << 16) : 0u);
            int32_t it = 0;  // k-blocks consumed since the kernel started
            int cc = 0;      // chunks started since the kernel started
            int cur = 0;     // accumulator buffer of the chunk in progress
            bool ok = true;
            for (int64_t L = cluster; ok && L < total_tiles; L += clusters) {
                const PairTile t = pair_tile(p, L, rank);
                for (int i = 0; i < t.nk; ++i, ++it) {
                    const bool first = (i % p.chunk_kb) == 0;
                    if (first) {
                        cur = cc & 1;
                        // buffer `cur` last held chunk cc - 2: wait until both
                        // CTAs have folded it (their epilogues arrive at
                        // cluster scope)
                        if (cc >= 2) {
                            if (!mbar_wait_cluster_bounded(&chunk_empty[cur], ((cc >> 1) - 1) & 1,
                                                           DEVERR_TIMEOUT_MMA)) {
                                *abort_flag = 1;
                                ok = false;
                                break;
                            }
                            tc_fence_after();
                        }
                    }
                    const int s = it % P_STAGES;
                    const uint32_t phase = (it / P_STAGES) & 1;
                    if (!mbar_wait_bounded(&full[s], phase, DEVERR_TIMEOUT_MMA)) {
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + s * P_STAGE_BYTES);
                    const uint32_t ahi = st, alo = st + P_TILE_BYTES;
                    const uint32_t bhi = st + 2 * P_TILE_BYTES, blo = st + 3 * P_TILE_BYTES;
                    const uint32_t d = tmem_base + static_cast<uint32_t>(cur) * ACC_COLS;
#pragma unroll
                    for (int kk = 0; kk < BK / 8; ++kk) {
                        const uint32_t acc = (first && kk == 0) ? 0u : 1u;
                        mma_tf32_ss_pair(d, operand_desc<AMN>(alo, kk), operand_desc<BMN>(bhi, kk),
                                         idesc, acc);
                        mma_tf32_ss_pair(d, operand_desc<AMN>(ahi, kk), operand_desc<BMN>(blo, kk),
                                         idesc, 1u);
                        mma_tf32_ss_pair(d, operand_desc<AMN>(ahi, kk), operand_desc<BMN>(bhi, kk),
                                         idesc, 1u);
                    }
                    mma_commit_pair(&empty[s], 0x3);
                    *consumed = it + 1;
                    if ((i % p.chunk_kb) == p.chunk_kb - 1 || i == t.nk - 1) {
                        mma_commit_pair(&chunk_full[cur], 0x3);
                        ++cc;
                    }
                }
                if (*abort_flag) ok = false;
            }
            // on abort, release both epilogues waiting for the unfinished
            // chunk; rank 0 skips its stores
            if (*abort_flag) mma_commit_pair(&chunk_full[cur], 0x3);
        }
    } else {
        // ---------------- epilogue (warps 2..9, both CTAs) ----------------
        int cc = 0;  // chunks folded since the kernel started
        for (int64_t L = cluster; L < total_tiles; L += clusters) {
            const PairTile t = pair_tile(p, L, rank);
            float run[128];
#pragma unroll
            for (int j = 0; j < 128; ++j) run[j] = 0.0f;  // K = 0: the empty sum
            if (!fold_chunks<true>(tmem_base, cc, t.nchunks, chunk_full, chunk_empty, warp, lane,
                                   run, abort_flag))
                break;
            cc += t.nchunks;
            if (p.splits > 1) {
                Params q = p;
                q.c = p.part;
                q.ldc = p.n;
                q.stride_c = p.m * p.n;
                q.epi = EPI_NONE;  // the reduction applies it to the sums
                store_run(run, warp, lane, t.m0, t.n0, t.zz, q);
            } else {
                store_run(run, warp, lane, t.m0, t.n0, t.batch, p);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && *abort_flag) {
        if (rank == 0) {
            // loads this CTA issued land on its own `full` barriers
            for (int kb = *consumed; kb < issued; ++kb)
                mbar_wait_bounded(&full[kb % P_STAGES], (kb / P_STAGES) & 1,
                                  DEVERR_TIMEOUT_PRODUCER);
        } else if (issued > 0) {
            // rank 1's loads report to rank 0's barriers: give any still in
            // flight a bounded time to land before the pair retires
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < P_DRAIN_NS) __nanosleep(1000);
        }
    }
    // neither CTA frees TMEM or exits while the other may still read its
    // shared memory or TMEM
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// C[b][i][j] = sum over s of part[b * splits + s][i][j], in split order
__global__ void splitk_reduce_kernel(const float *__restrict__ part, int splits, int64_t m,
                                     int64_t n, int64_t batch, float *__restrict__ c, int64_t ldc,
                                     int64_t stride_c) {
    const int64_t mn = m * n, total = batch * mn;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / mn, e = i % mn, row = e / n, col = e % n;
        const float *src = part + b * splits * mn + e;
        float acc = src[0];
        for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, src[s * mn]);
        c[b * stride_c + row * ldc + col] = acc;
    }
}

// The same sum for a dense C (ldc == n, batch items back to back) whose
// element count is a multiple of 4: four outputs per thread, 16-byte loads
// and stores, no index arithmetic beyond the flat offset.
// The fused epilogue (p.epi, p.c, p.epi_*) applies to the sums.
__global__ void splitk_reduce_dense4_kernel(const float4 *__restrict__ part, int splits,
                                            int64_t mn4, int64_t batch, Params p) {
    const int64_t total = batch * mn4;
    float4 *c = reinterpret_cast<float4 *>(p.c);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = batch == 1 ? 0 : i / mn4;
        const float4 *src = part + b * splits * mn4 + (i - b * mn4);
        float4 acc = src[0];
        for (int s = 1; s < splits; ++s) {
            const float4 v = src[s * mn4];
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (p.epi == EPI_ADD) {
            const float4 a = reinterpret_cast<const float4 *>(p.epi_in)[i];
            acc = make_float4(__fadd_rn(acc.x, a.x), __fadd_rn(acc.y, a.y), __fadd_rn(acc.z, a.z),
                              __fadd_rn(acc.w, a.w));
        }
        c[i] = acc;
    }
}

// ---------------------------------------------------------------------------
// split pre-pass kernels.  hi = RN_tf32(x), lo = RN_tf32(x - hi) (x - hi is
// exact in f32); non-finite x gets lo = 0.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rna_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// General strides: element (r, kk) at src[b*sb + r*sr + kk*sk] ->
// hi/lo[b][r][kk] (K-major, row stride kp), zero for kk >= K.  A 32 x 32
// tile goes through shared memory so both the read and the write coalesce.
__global__ void split_kernel(const float *__restrict__ src, int64_t rows, int64_t k,
                             int64_t sr, int64_t sk, int64_t sb, int64_t kp,
                             float *__restrict__ hi, float *__restrict__ lo) {
    __shared__ float tile[32][33];
    const int64_t b = blockIdx.z;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32;
    const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
    const float *s = src + b * sb;
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    if (sk == 1) {
        for (int i = ty; i < 32; i += 8) {
            int64_t r = r0 + i, kk = k0 + tx;
            tile[i][tx] = (r < rows && kk < k) ? s[r * sr + kk] : 0.0f;
        }
    } else {
        for (int i = ty; i < 32; i += 8) {
            int64_t r = r0 + tx, kk = k0 + i;
            tile[tx][i] = (r < rows && kk < k) ? s[r * sr + kk * sk] : 0.0f;
        }
    }
    __syncthreads();
    float *h = hi + b * rows * kp;
    float *l = lo + b * rows * kp;
    for (int i = ty; i < 32; i += 8) {
        int64_t r = r0 + i, kk = k0 + tx;
        if (r < rows && kk < kp) {
            float x = tile[i][tx];
            float xh = rna_tf32(x);
            float xl = isfinite(x) ? rna_tf32(__fsub_rn(x, xh)) : 0.0f;
            h[r * kp + kk] = xh;
            l[r * kp + kk] = xl;
        }
    }
}

// Row-contiguous source: the split streams, one float4 in and two float4
// out per step; row r of `rows` has `cols` valid entries at src[b*sb +
// r*sr + c] and the output row stride is `cp` (columns [cols, cp) zero).
// Used for both layouts: K-major (rows = MN, cols = K) and MN-major
// (rows = K, cols = MN).
__global__ void split_rows_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                  int64_t sr, int64_t sb, int64_t cp, float *__restrict__ hi,
                                  float *__restrict__ lo) {
    const int64_t b = blockIdx.y;
    const float *s = src + b * sb;
    float *h = hi + b * rows * cp;
    float *l = lo + b * rows * cp;
    const int64_t q = cp / 4;  // float4 per output row
    const bool vec = (cols % 4 == 0) && (sr % 4 == 0) && ((reinterpret_cast<uintptr_t>(s) & 15) == 0);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows * q;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / q, c0 = (i % q) * 4;
        float x[4];
        if (vec && c0 + 3 < cols) {
            const float4 v = __ldcs(reinterpret_cast<const float4 *>(s + r * sr + c0));
            x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) x[j] = (c0 + j < cols) ? s[r * sr + c0 + j] : 0.0f;
        }
        float xh[4], xl[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            xh[j] = rna_tf32(x[j]);
            xl[j] = isfinite(x[j]) ? rna_tf32(__fsub_rn(x[j], xh[j])) : 0.0f;
        }
        *reinterpret_cast<float4 *>(h + r * cp + c0) = make_float4(xh[0], xh[1], xh[2], xh[3]);
        *reinterpret_cast<float4 *>(l + r * cp + c0) = make_float4(xl[0], xl[1], xl[2], xl[3]);
    }
}


typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// K-major split buffer [total_rows][kp] -> box 32 (K) x box_rows
int make_kmajor_map(CUtensorMap *map, const float *base, int64_t rows, int64_t kp, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kp), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kp) * 4};
    cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CHELIS_CUDA_OK;
}

// MN-major split buffer [batch][k][mnp] -> box 32 (MN) x 32 (K) x 1; rows
// past k and columns past mn read as zeros (per batch item: 3-D map)
int make_mnmajor_map(CUtensorMap *map, const float *base, int64_t mn, int64_t mnp, int64_t k,
                     int64_t batch) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(mn), static_cast<cuuint64_t>(k),
                          static_cast<cuuint64_t>(batch)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(mnp) * 4, static_cast<cuuint64_t>(mnp * k) * 4};
    cuuint32_t box[3] = {MN_BOX, BK, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled(3d) failed (%d)", (int)r);
    return CHELIS_CUDA_OK;
}

}  // namespace tf32x3

// ---------------------------------------------------------------------------
// exact canonical-tree GEMM on CUDA cores (bit-identical to the C lane's
// inlined product sum, crates/chelis-backend-c/src/emit.rs:8431-8640).
// A CTA is 8 warps; warp w owns output row r0 + w and 32 columns.  For each
// aligned block of 32 leaves (k0 .. k0+31, a complete subtree of the
// canonical tree over k) lane l forms the 32 products a[r, k0+l]*b[k0+l, j]
// and a halving warp butterfly reduces them: adjacent leaves pair first, as
// the tree requires, and every lane ends holding the block sum of one
// column.  Block sums (and a ragged last block, the tree of its prefix)
// then enter that lane's outer carry tree, whose levels live in registers.
// ---------------------------------------------------------------------------
namespace exact {

constexpr int RW = 8, TN = 32, TK = 32, THREADS = 256;
constexpr int MAXD = 14;  // outer levels: up to 2^14 blocks of 32 (k <= 524288)

template <typename T>
struct Carry {
    T level[MAXD];
};

template <typename T>
__device__ __forceinline__ T add_rn(T a, T b);
template <>
__device__ __forceinline__ float add_rn<float>(float a, float b) { return __fadd_rn(a, b); }
template <>
__device__ __forceinline__ double add_rn<double>(double a, double b) { return __dadd_rn(a, b); }
template <typename T>
__device__ __forceinline__ T mul_rn(T a, T b);
template <>
__device__ __forceinline__ float mul_rn<float>(float a, float b) { return __fmul_rn(a, b); }
template <>
__device__ __forceinline__ double mul_rn<double>(double a, double b) { return __dmul_rn(a, b); }

// push `carry` as leaf number `count` of the outer tree
template <typename T>
__device__ __forceinline__ void push(Carry<T> &t, uint32_t count, T carry) {
    bool active = true;
#pragma unroll
    for (int d = 0; d < MAXD; ++d) {
        const bool bit = (count >> d) & 1u;
        if (active) {
            if (bit) {
                carry = add_rn(t.level[d], carry);
            } else {
                t.level[d] = carry;
                active = false;
            }
        }
    }
}
template <typename T>
__device__ __forceinline__ T total(const Carry<T> &t, uint32_t count) {
    T tot = T(0);
    bool found = false;
#pragma unroll
    for (int d = 0; d < MAXD; ++d) {
        if ((count >> d) & 1u) {
            tot = found ? add_rn(t.level[d], tot) : t.level[d];
            found = true;
        }
    }
    return tot;
}

// Halving butterfly over 32 values per lane.  `valid` marks the lane's leaf
// as present (lanes holding leaves past the end of k are absent: the tree of
// a prefix).  Returns the lane's block sum; `col` = the column it belongs to.
template <typename T, bool FULL>
__device__ __forceinline__ T block_butterfly(T (&v)[TN], int lane, bool valid, int &col) {
    col = 0;
    bool vs = valid;
#pragma unroll
    for (int cnt = TN, off = 1; cnt > 1; cnt >>= 1, off <<= 1) {
        const bool bit = (lane & off) != 0;
        const bool vp = FULL ? true : (__shfl_xor_sync(0xffffffffu, vs ? 1 : 0, off) != 0);
#pragma unroll
        for (int j = 0; j < cnt / 2; ++j) {
            const T send = bit ? v[j] : v[j + cnt / 2];
            const T keep = bit ? v[j + cnt / 2] : v[j];
            const T recv = __shfl_xor_sync(0xffffffffu, send, off);
            v[j] = FULL ? add_rn(keep, recv) : tree_pair(keep, vs, recv, vp);
        }
        vs = vs || vp;
        if (bit) col += cnt / 2;
    }
    return v[0];
}

template <typename T>
__global__ void __launch_bounds__(THREADS)
    gemm_exact_kernel(int64_t m, int64_t n, int64_t k, const T *__restrict__ a, int64_t sa_r,
                      int64_t sa_k, int64_t sa_b, const T *__restrict__ b, int64_t sb_k,
                      int64_t sb_c, int64_t sb_b, T *__restrict__ c, int64_t ldc,
                      int64_t sc_b) {
    __shared__ T bs[TK][TN + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bb = blockIdx.z;
    const int64_t row = static_cast<int64_t>(blockIdx.y) * RW + warp;
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * TN;
    a += bb * sa_b;
    b += bb * sb_b;
    Carry<T> tree;
    uint32_t blocks = 0;
    int col = lane;
    // block k0's B tile and A leaf are loaded into registers one block ahead,
    // so their global-memory latency overlaps the previous block's butterfly
    // (small grids -- a few warps per SM -- are otherwise bound by it)
    constexpr int PER = TK * TN / THREADS;
    T bnext[PER], anext;
    auto fetch = [&](int64_t k0) {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = threadIdx.x + j * THREADS;
            const int kk = i / TN, cc = i % TN;
            const int64_t gk = k0 + kk, gc = c0 + cc;
            bnext[j] = (gc < n && gk < k) ? b[gk * sb_k + gc * sb_c] : T(0);
        }
        anext = (row < m && k0 + lane < k) ? a[row * sa_r + (k0 + lane) * sa_k] : T(0);
    };
    if (k > 0) fetch(0);
    for (int64_t k0 = 0; k0 < k; k0 += TK) {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int i = threadIdx.x + j * THREADS;
            bs[i / TN][i % TN] = bnext[j];
        }
        const T av = anext;
        __syncthreads();
        if (k0 + TK < k) fetch(k0 + TK);
        const int64_t valid = (k - k0) < TK ? (k - k0) : TK;
        const bool lv = lane < valid;
        T v[TN];
#pragma unroll
        for (int j = 0; j < TN; ++j) v[j] = mul_rn(av, bs[lane][j]);
        const T s = (valid == TK) ? block_butterfly<T, true>(v, lane, lv, col)
                                  : block_butterfly<T, false>(v, lane, lv, col);
        push(tree, blocks, s);
        ++blocks;
        __syncthreads();
    }
    const int64_t gc = c0 + col;
    if (row < m && gc < n) c[bb * sc_b + row * ldc + gc] = k > 0 ? total(tree, blocks) : T(0);
}

}  // namespace exact

template <typename T>
int launch_exact_gemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const T *a,
                      int64_t lda, int64_t stride_a, const T *b, int64_t ldb, int64_t stride_b,
                      T *c, int64_t ldc, int64_t stride_c, int64_t batch, cudaStream_t s) {
    if (k > static_cast<int64_t>(exact::TK) << exact::MAXD)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "exact-tree matmul admits k <= %lld",
                         static_cast<long long>(exact::TK) << exact::MAXD);
    int64_t sa_r = trans_a ? 1 : lda, sa_k = trans_a ? lda : 1;
    int64_t sb_k = trans_b ? 1 : ldb, sb_c = trans_b ? ldb : 1;
    dim3 grid(static_cast<unsigned>((n + exact::TN - 1) / exact::TN),
              static_cast<unsigned>((m + exact::RW - 1) / exact::RW),
              static_cast<unsigned>(batch));
    exact::gemm_exact_kernel<T><<<grid, exact::THREADS, 0, s>>>(
        m, n, k, a, sa_r, sa_k, stride_a, b, sb_k, sb_c, stride_b, c, ldc, stride_c);
    g_launches++;
    CHELIS_LAUNCH_CHECK("gemm_exact_kernel");
    return CHELIS_CUDA_OK;
}
template int launch_exact_gemm<float>(int, int, int64_t, int64_t, int64_t, const float *, int64_t,
                                      int64_t, const float *, int64_t, int64_t, float *, int64_t,
                                      int64_t, int64_t, cudaStream_t);
template int launch_exact_gemm<double>(int, int, int64_t, int64_t, int64_t, const double *,
                                       int64_t, int64_t, const double *, int64_t, int64_t,
                                       double *, int64_t, int64_t, int64_t, cudaStream_t);

// ---------------------------------------------------------------------------
// operand plans: how one operand of op(A) . op(B) is split and loaded
// ---------------------------------------------------------------------------
// The operand is viewed as `rows` x k (rows = m for A, n for B) with element
// (r, kk) at src[b*sb + r*sr + kk*sk].  K-contiguous sources (sk == 1) split
// K-major; MN-contiguous ones (sr == 1) split MN-major; anything else goes
// through the transposing tile kernel into K-major.
struct OperandPlan {
    bool mn;             // MN-major layout
    int64_t rows, k;
    int64_t cp;          // padded inner extent of the split buffer
    int64_t floats;      // floats of one of hi / lo, all batch items
};

OperandPlan plan_operand(int64_t rows, int64_t k, int64_t sr, int64_t sk, int64_t batch) {
    using namespace tf32x3;
    OperandPlan p;
    p.rows = rows;
    p.k = k;
    p.mn = (sk != 1) && (sr == 1);
    if (p.mn) {
        p.cp = (rows + 3) / 4 * 4;
        p.floats = batch * k * p.cp;
    } else {
        p.cp = (k + BK - 1) / BK * BK;
        p.floats = batch * rows * p.cp;
    }
    return p;
}

int launch_split_plan(const OperandPlan &p, const float *src, int64_t sr, int64_t sk, int64_t sb,
                      int64_t batch, float *hi, float *lo, cudaStream_t s) {
    using namespace tf32x3;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (p.mn || sk == 1) {
        // streaming: MN-major rows are k (stride sk), K-major rows are `rows` (stride sr)
        const int64_t out_rows = p.mn ? p.k : p.rows;
        const int64_t cols = p.mn ? p.rows : p.k;
        const int64_t row_stride = p.mn ? sk : sr;
        int64_t blocks = (out_rows * (p.cp / 4) + 255) / 256;
        if (blocks > cap) blocks = cap;
        if (blocks < 1) blocks = 1;
        split_rows_kernel<<<dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(batch)), 256,
                            0, s>>>(src, out_rows, cols, row_stride, sb, p.cp, hi, lo);
        g_launches++;
        CHELIS_LAUNCH_CHECK("split_rows_kernel");
        return CHELIS_CUDA_OK;
    }
    dim3 grid(static_cast<unsigned>(p.cp / 32), static_cast<unsigned>((p.rows + 31) / 32),
              static_cast<unsigned>(batch));
    split_kernel<<<grid, dim3(32, 8), 0, s>>>(src, p.rows, p.k, sr, sk, sb, p.cp, hi, lo);
    g_launches++;
    CHELIS_LAUNCH_CHECK("split_kernel");
    return CHELIS_CUDA_OK;
}

int make_operand_map(CUtensorMap *map, const OperandPlan &p, const float *buf, int64_t batch,
                     int box_rows) {
    if (p.mn) return tf32x3::make_mnmajor_map(map, buf, p.rows, p.cp, p.k, batch);
    return tf32x3::make_kmajor_map(map, buf, batch * p.rows, p.cp, box_rows);
}

// Large dynamic shared memory is a per-device function attribute: set it
// once per (kernel, device).
int ensure_smem_attr(const void *fn, int bytes, uint64_t *done_mask, const char *what) {
    int d = 0;
    CHELIS_TRY(current_device_checked(&d));
    const uint64_t bit = 1ull << (d & 63);
    if (*done_mask & bit) return CHELIS_CUDA_OK;
    CHELIS_TRY(check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               bytes),
                          what));
    *done_mask |= bit;
    return CHELIS_CUDA_OK;
}

// Clusters of the pair kernel that fit on the device at once (its shared
// memory allows one CTA per SM, and a pair needs two SMs of one GPC), once
// per (kernel, device); the persistent grid launches no more than this.
template <bool AMN, bool BMN>
int pair_clusters(int *out) {
    using namespace tf32x3;
    static std::atomic<int> cached[64];
    int d = 0;
    CHELIS_TRY(current_device_checked(&d));
    if (d < 64) {
        const int c = cached[d].load(std::memory_order_relaxed);
        if (c > 0) {
            *out = c;
            return CHELIS_CUDA_OK;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * static_cast<unsigned>(sm_count()), 1, 1);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    CHELIS_TRY(check_cuda(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<AMN, BMN>, &cfg),
                          "cudaOccupancyMaxActiveClusters(gemm_pair_kernel)"));
    if (n < 1) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "no CTA pair of the matmul kernel fits");
    if (d < 64) cached[d].store(n, std::memory_order_relaxed);
    *out = n;
    return CHELIS_CUDA_OK;
}

template <bool AMN, bool BMN>
int launch_main(const CUtensorMap &ahi, const CUtensorMap &alo, const CUtensorMap &bhi,
                const CUtensorMap &blo, const tf32x3::Params &p, bool pair, cudaStream_t s) {
    using namespace tf32x3;
    if (pair) {
        static uint64_t done = 0;
        CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(gemm_pair_kernel<AMN, BMN>),
                                    P_SMEM_BYTES, &done, "cudaFuncSetAttribute(gemm_pair_kernel)"));
        cudaLaunchConfig_t cfg = {};
        Params q = p;
        q.pairs_m = (p.m + 2 * P_ROWS - 1) / (2 * P_ROWS);
        q.tiles_n = (p.n + BN - 1) / BN;
        const int64_t tiles = q.pairs_m * q.tiles_n * p.batch * p.splits;
        if (tiles == 0) return CHELIS_CUDA_OK;
        // Short tiles (few k-blocks) run persistently, so one tile's setup and
        // stores overlap the next one's MMAs; long tiles get one cluster
        // each, so the hardware hands tiles to clusters as they free up.
        int64_t clusters = tiles;
        if (p.kb_per_split <= P_PERSIST_KB) {
            int max_clusters = 0;
            CHELIS_TRY((pair_clusters<AMN, BMN>(&max_clusters)));
            if (clusters > max_clusters) clusters = max_clusters;
        }
        if (2 * clusters > INT32_MAX)
            return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "matmul tile count beyond 2^30");
        cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters), 1, 1);
        cfg.blockDim = dim3(THREADS);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CHELIS_TRY(check_cuda(cudaLaunchKernelEx(&cfg, gemm_pair_kernel<AMN, BMN>, ahi, alo, bhi,
                                                 blo, q),
                              "cudaLaunchKernelEx(gemm_pair_kernel)"));
        g_launches++;
        CHELIS_LAUNCH_CHECK("gemm_pair_kernel(3xtf32)");
        return CHELIS_CUDA_OK;
    }
    static uint64_t done = 0;
    CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(gemm_kernel<AMN, BMN>), SMEM_BYTES,
                                &done, "cudaFuncSetAttribute(gemm_kernel)"));
    dim3 grid(static_cast<unsigned>((p.n + BN - 1) / BN), static_cast<unsigned>((p.m + BM - 1) / BM),
              static_cast<unsigned>(p.batch));
    gemm_kernel<AMN, BMN><<<grid, THREADS, SMEM_BYTES, s>>>(ahi, alo, bhi, blo, p);
    g_launches++;
    CHELIS_LAUNCH_CHECK("gemm_kernel(3xtf32)");
    return CHELIS_CUDA_OK;
}

// Main kernel on split operands.  CTA pairs (256-row tiles) whenever the
// product has more than one 128-row tile; a single CTA per 128 x 256 tile
// otherwise.
int sgemm_3xtf32_main(const OperandPlan &pa, const float *ahi, const float *alo,
                      const OperandPlan &pb, const float *bhi, const float *blo, int64_t m,
                      int64_t n, int64_t k, float *c, int64_t ldc, int64_t stride_c, int64_t batch,
                      cudaStream_t s, const tf32x3::EpiArgs &epi = tf32x3::EpiArgs()) {
    using namespace tf32x3;
    const bool pair = m > BM && g_pair_tiles.load();
    const int b_box = pair ? P_ROWS : BN;
    CUtensorMap mahi, malo, mbhi, mblo;
    CHELIS_TRY(make_operand_map(&mahi, pa, ahi, batch, BM));
    CHELIS_TRY(make_operand_map(&malo, pa, alo, batch, BM));
    CHELIS_TRY(make_operand_map(&mbhi, pb, bhi, batch, b_box));
    CHELIS_TRY(make_operand_map(&mblo, pb, blo, batch, b_box));
    Params p;
    p.m = m;
    p.n = n;
    p.batch = batch;
    p.pairs_m = 0;
    p.tiles_n = 0;
    p.num_kb = static_cast<int32_t>((k + BK - 1) / BK);
    p.a_rows_per_batch = m;
    p.b_rows_per_batch = n;
    p.c = c;
    p.ldc = ldc;
    p.stride_c = stride_c;
    p.splits = 1;
    p.kb_per_split = p.num_kb;
    p.part = nullptr;
    p.chunk_kb = CHUNK_KB;
    p.epi = epi.op;
    p.epi_in = epi.in;
    // Split-K when the tile grid fills the GPU poorly.  Each candidate split
    // count is costed as (waves of CTA pairs) x (time of one tile: its
    // k-blocks plus a fixed prologue / epilogue) plus the HBM traffic of the
    // partial products (written by the epilogues, read by the reduction, and
    // the reduced result written); the cheapest wins, each split keeping at
    // least 4 k-blocks.  Times in microseconds at the tf32 pipe's pace
    // (three MMAs of K = 8, four per 32-wide k-block, ~1.15 us per k-block).
    // a fused epilogue on a split product runs in the 16-byte reduction only
    const bool dense_c = ldc == n && (batch == 1 || stride_c == m * n) && (m * n) % 4 == 0 &&
                         (reinterpret_cast<uintptr_t>(c) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(epi.in) & 15) == 0;
    if (pair && (epi.op == tf32x3::EPI_NONE || dense_c)) {
        const int64_t clusters = sm_count() / 2;
        const int64_t pairs = ((m + 2 * P_ROWS - 1) / (2 * P_ROWS)) * ((n + BN - 1) / BN) * batch;
        if (pairs < 2 * clusters && p.num_kb >= 8) {
            constexpr double kTileK = 1.15, kTileFixed = 5.0, kBytesPerUs = 5.0e6;
            double best = 0.0;
            int best_s = 1;
            for (int sp = 1; sp <= 16 && p.num_kb / sp >= 4; ++sp) {
                const int64_t kbs = (p.num_kb + sp - 1) / sp;
                const int64_t waves = (pairs * sp + clusters - 1) / clusters;
                double t = static_cast<double>(waves) * (kbs * kTileK + kTileFixed);
                if (sp > 1)
                    t += static_cast<double>(2 * sp + 1) * static_cast<double>(batch * m * n) * 4.0 /
                         kBytesPerUs;
                if (sp == 1 || t < best) {
                    best = t;
                    best_s = sp;
                }
            }
            if (best_s > 1) {
                p.kb_per_split = (p.num_kb + best_s - 1) / best_s;
                p.splits = (p.num_kb + p.kb_per_split - 1) / p.kb_per_split;
            }
        }
    }
    void *part = nullptr;
    if (p.splits > 1) {
        CHELIS_TRY(scratch_alloc(&part, static_cast<size_t>(p.splits * batch * m * n) * sizeof(float), s));
        p.part = static_cast<float *>(part);
    }
    int st;
    if (pa.mn) {
        if (pb.mn) st = launch_main<true, true>(mahi, malo, mbhi, mblo, p, pair, s);
        else st = launch_main<true, false>(mahi, malo, mbhi, mblo, p, pair, s);
    } else {
        if (pb.mn) st = launch_main<false, true>(mahi, malo, mbhi, mblo, p, pair, s);
        else st = launch_main<false, false>(mahi, malo, mbhi, mblo, p, pair, s);
    }
    if (st == CHELIS_CUDA_OK && p.splits > 1) {
        const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
        const int64_t mn = m * n;
        const bool dense4 = ldc == n && (batch == 1 || stride_c == mn) && mn % 4 == 0 &&
                            (reinterpret_cast<uintptr_t>(c) & 15) == 0;
        if (dense4) {
            int64_t blocks = (batch * mn / 4 + 255) / 256;
            if (blocks > cap) blocks = cap;
            splitk_reduce_dense4_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
                reinterpret_cast<const float4 *>(p.part), p.splits, mn / 4, batch, p);
        } else {
            int64_t blocks = (batch * mn + 255) / 256;
            if (blocks > cap) blocks = cap;
            splitk_reduce_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
                p.part, p.splits, m, n, batch, c, ldc, stride_c);
        }
        g_launches++;
        st = check_cuda(cudaGetLastError(), "splitk_reduce_kernel");
    }
    if (part) scratch_free(part, s);
    return st;
}


struct GemmPlan {
    OperandPlan a, b;
    int64_t sar, sak, sbr, sbk;
    size_t bytes() const { return static_cast<size_t>(2 * (a.floats + b.floats)) * sizeof(float); }
};

GemmPlan plan_gemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, int64_t lda,
                   int64_t ldb, int64_t batch) {
    GemmPlan g;
    // op(A)[i, kk] = a[i*lda + kk] (no trans) or a[kk*lda + i] (trans)
    g.sar = trans_a ? 1 : lda;
    g.sak = trans_a ? lda : 1;
    // op(B)[kk, j] as the n x k operand: element (j, kk) = b[kk*ldb + j] (no
    // trans) or b[j*ldb + kk] (trans)
    g.sbr = trans_b ? ldb : 1;
    g.sbk = trans_b ? 1 : ldb;
    g.a = plan_operand(m, k, g.sar, g.sak, batch);
    g.b = plan_operand(n, k, g.sbr, g.sbk, batch);
    return g;
}

// Split both operands into caller-provided scratch (GemmPlan::bytes()) and
// run the tcgen05 kernel.
int sgemm_3xtf32_with_scratch(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                              const float *a, int64_t lda, int64_t stride_a, const float *b,
                              int64_t ldb, int64_t stride_b, float *c, int64_t ldc,
                              int64_t stride_c, int64_t batch, float *scratch, cudaStream_t s) {
    const GemmPlan g = plan_gemm(trans_a, trans_b, m, n, k, lda, ldb, batch);
    float *ahi = scratch;
    float *alo = ahi + g.a.floats;
    float *bhi = alo + g.a.floats;
    float *blo = bhi + g.b.floats;
    CHELIS_TRY(launch_split_plan(g.a, a, g.sar, g.sak, stride_a, batch, ahi, alo, s));
    CHELIS_TRY(launch_split_plan(g.b, b, g.sbr, g.sbk, stride_b, batch, bhi, blo, s));
    return sgemm_3xtf32_main(g.a, ahi, alo, g.b, bhi, blo, m, n, k, c, ldc, stride_c, batch, s);
}

int validate_gemm_args(int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                       int64_t batch, int trans_a, int trans_b) {
    if (m < 0 || n < 0 || k < 0 || batch < 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "matmul extent beyond 2^30");
    const int64_t a_cols = trans_a ? m : k, b_cols = trans_b ? k : n;
    if ((a_cols > 0 && lda < a_cols) || (b_cols > 0 && ldb < b_cols) || (n > 0 && ldc < n))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    return CHELIS_CUDA_OK;
}

}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_tf32x3_split(int trans, int layout, int64_t rows, int64_t k,
                                        const float *src, int64_t ld, int64_t stride,
                                        int64_t batch, float *hi, float *lo) {
    if (rows < 0 || k < 0 || batch < 0 || (layout & ~1))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    const int64_t sr = trans ? 1 : ld, sk = trans ? ld : 1;
    OperandPlan p = plan_operand(rows, k, sr, sk, batch);
    if (layout == 1 && !p.mn)
        return set_error(CHELIS_CUDA_ERR_DOMAIN,
                         "MN-major split needs an MN-contiguous source (trans = 1)");
    if (layout == 0 && p.mn) {  // force K-major through the transposing kernel
        p.mn = false;
        p.cp = (k + tf32x3::BK - 1) / tf32x3::BK * tf32x3::BK;
    }
    if (rows == 0 || batch == 0 || k == 0) return CHELIS_CUDA_OK;
    return launch_split_plan(p, src, sr, sk, stride, batch, hi, lo, current_stream());
}

extern "C" int chelis_cuda_sgemm_tf32x3_presplit(int64_t m, int64_t n, int64_t k, int64_t batch,
                                                 int a_layout, const float *a_hi,
                                                 const float *a_lo, int b_layout,
                                                 const float *b_hi, const float *b_lo, float *c,
                                                 int64_t ldc, int64_t stride_c) {
    if (m < 0 || n < 0 || k <= 0 || batch < 0 || ldc < n || (a_layout & ~1) || (b_layout & ~1))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    if (m == 0 || n == 0 || batch == 0) return CHELIS_CUDA_OK;
    OperandPlan pa = plan_operand(m, k, a_layout ? 1 : 2, a_layout ? 2 : 1, batch);
    OperandPlan pb = plan_operand(n, k, b_layout ? 1 : 2, b_layout ? 2 : 1, batch);
    return sgemm_3xtf32_main(pa, a_hi, a_lo, pb, b_hi, b_lo, m, n, k, c, ldc, stride_c, batch,
                             current_stream());
}

namespace chelis {
// The presplit product with a fused epilogue (tf32x3::EPI_ADD: a residual
// added as C is stored), for the transformer block step; C dense (ldc = n),
// one batch item.
int sgemm_presplit_epi(int64_t m, int64_t n, int64_t k, int a_layout, const float *a_hi,
                       const float *a_lo, int b_layout, const float *b_hi, const float *b_lo,
                       float *c, const tf32x3::EpiArgs &epi) {
    if (m <= 0 || n <= 0 || k <= 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in matmul at i64");
    OperandPlan pa = plan_operand(m, k, a_layout ? 1 : 2, a_layout ? 2 : 1, 1);
    OperandPlan pb = plan_operand(n, k, b_layout ? 1 : 2, b_layout ? 2 : 1, 1);
    return sgemm_3xtf32_main(pa, a_hi, a_lo, pb, b_hi, b_lo, m, n, k, c, n, m * n, 1,
                             current_stream(), epi);
}
}  // namespace chelis

extern "C" int chelis_cuda_sgemm(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k,
                                 const float *a, int64_t lda, int64_t stride_a, const float *b,
                                 int64_t ldb, int64_t stride_b, float *c, int64_t ldc,
                                 int64_t stride_c, int64_t batch) {
    CHELIS_TRY(validate_gemm_args(m, n, k, lda, ldb, ldc, batch, trans_a, trans_b));
    if (m == 0 || n == 0 || batch == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (k == 0) {
        // empty contraction: exact zero (the empty Sum, [05-OP-30])
        for (int64_t bb = 0; bb < batch; ++bb)
            CHELIS_TRY(check_cuda(cudaMemset2DAsync(c + bb * stride_c, ldc * sizeof(float), 0,
                                                    n * sizeof(float), m, s),
                                  "cudaMemset2DAsync"));
        return CHELIS_CUDA_OK;
    }
    if (gemm_mode() == CHELIS_CUDA_GEMM_EXACT_TREE)
        return launch_exact_gemm<float>(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb,
                                        stride_b, c, ldc, stride_c, batch, s);
    if (batch * (m > n ? m : n) > INT32_MAX)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "batched matmul rows beyond 2^31");
    const GemmPlan g = plan_gemm(trans_a, trans_b, m, n, k, lda, ldb, batch);
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, g.bytes(), s));
    int st = sgemm_3xtf32_with_scratch(trans_a, trans_b, m, n, k, a, lda, stride_a, b, ldb,
                                       stride_b, c, ldc, stride_c, batch,
                                       static_cast<float *>(scratch), s);
    scratch_free(scratch, s);
    return st;
}

extern "C" int chelis_cuda_set_gemm_pairs(int enable) {
    if (enable != 0 && enable != 1)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "gemm pair mode must be 0 or 1");
    g_pair_tiles.store(enable);
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_get_gemm_pairs(void) { return g_pair_tiles.load(); }

