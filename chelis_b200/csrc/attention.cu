// attention.cu -- causal softmax attention without the [S, S] scores in HBM.
//
// The reference evaluates attention as its graph spells it: scores
// (q.k^T)*scale, where(causal, ., -inf), softmax over the last axis, then
// probabilities . v (spec 05 section 4.7; tier2.rs attention lowering), every
// step a separate tensor.  Here one kernel keeps a 128-row query tile's
// scores, probabilities and output accumulator in tensor memory and streams
// the keys and values through shared memory in blocks of 64, combining the
// blocks with the running-maximum form of softmax:
//
//   m_j = max(m_{j-1}, rowmax(s_j)),  p_j = exp(s_j - m_j),
//   l_j = l_{j-1} exp(m_{j-1} - m_j) + rowsum(p_j),
//   o_j = o_{j-1} exp(m_{j-1} - m_j) + p_j . v_j,   out = o_J / l_J.
//
// Every product is 3xTF32 on tcgen05 (hi/lo split of both operands, three
// MMAs), so the f32 result carries f32-level error like the rest of the
// block; the query tile and the probabilities are the MMA's A operand
// straight from tensor memory, the keys and values the B operand from
// shared memory (TMA, 128-byte swizzle).
//
// Roles (384 threads): warps 0 / 11 load key / value blocks with TMA, warp 1
// issues the score MMAs and warp 10 the output MMAs (independent streams, so
// neither waits behind the other), warps 2-9 own the query rows (two
// threads per TMEM lane, each half of the columns).
// Every wait is bounded; a timeout sets the device error word and the CTA
// winds down.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;

namespace attn {

constexpr int BQ = 128;      // query rows per CTA (TMEM lanes)
constexpr int BKV = 64;      // keys per block
constexpr int THREADS = 384;  // 0 key TMA, 1 score MMA, 2-9 rows, 10 output MMA, 11 value TMA
constexpr int THREADS_BWD = 320;  // 0 TMA, 1 MMA, 2-9 rows
constexpr int MN_BOX_BYTES = 32 * 32 * 4;  // MN-major TMA box 32 x 32 f32

template <int DH>
struct Fwd {
    static_assert(DH == 32 || DH == 64, "flash attention path covers head dims 32 and 64");
    static constexpr int KCH = DH / 32;                 // 128-byte chunks along the head dim
    static constexpr int K_TILE = BKV * DH * 4;          // one of hi / lo
    static constexpr int V_TILE = BKV * DH * 4;
    static constexpr int STAGE = 2 * K_TILE + 2 * V_TILE;
    static constexpr int STAGES = 2;
    // at least ~116 KiB so that one CTA (holding all 512 TMEM columns) runs per SM
    static constexpr int SMEM_USED = STAGES * STAGE + 1024 + 256 + 10 * BQ * 4;
    static constexpr int SMEM = SMEM_USED > 118784 ? SMEM_USED : 118784;
    // tensor-memory columns
    // Score block j lands in S[j % 2]; its probabilities overwrite it (hi)
    // and PLO[j % 2] (lo), so block j + 1's scores and block j's P . V never
    // share columns.
    static constexpr uint32_t C_QHI = 0, C_QLO = DH;
    static constexpr uint32_t C_S0 = 2 * DH, C_S1 = 2 * DH + BKV;
    static constexpr uint32_t C_PLO0 = 2 * DH + 2 * BKV, C_PLO1 = C_PLO0 + BKV;
    static constexpr uint32_t C_O0 = C_PLO1 + BKV, C_O1 = C_O0 + DH;
    static constexpr uint32_t COLS = 512;
    static_assert(C_O1 + DH <= COLS, "tensor memory budget");
};

struct FwdParams {
    const float *q;                  // f32 query rows (split in the kernel)
    int64_t q_row, q_b, q_h;         // element strides: row, batch item, head
    float *o;                        // output rows
    int64_t o_row, o_b, o_h;
    float *lse;                      // [BH][S] log-sum-exp of the scaled scores (may be null)
    int heads, seq;
    float scale;
    int n_qblocks;
};

// Round a finite f32 to the nearest tf32 (ties away from zero), the value
// cvt.rna.tf32.f32 gives, with two integer ops instead of a conversion-pipe
// instruction: add half an ulp of the 10-bit mantissa to the magnitude bits
// and clear the 13 dropped bits (a carry into the exponent is the correct
// rounding up).
__device__ __forceinline__ uint32_t rna_tf32_bits(uint32_t b) { return (b + 0x1000u) & 0xFFFFE000u; }
// hi = RN_tf32(x), lo = RN_tf32(x - hi) (x - hi is exact); non-finite x
// passes through as hi with lo = 0.
__device__ __forceinline__ void split_tf32(float x, uint32_t &hi, uint32_t &lo) {
    if (isfinite(x)) {
        hi = rna_tf32_bits(__float_as_uint(x));
        lo = rna_tf32_bits(__float_as_uint(__fsub_rn(x, __uint_as_float(hi))));
    } else {
        hi = __float_as_uint(x);
        lo = 0u;
    }
}

// 2^x (MUFU), flushing subnormal results; x <= 0 here, ex2(-inf) = +0
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// acc = acc * alpha + O, O the OH accumulator columns at `taddr`
template <int OH>
__device__ __forceinline__ void fold_o(float (&acc)[OH], uint32_t taddr, float alpha) {
    if constexpr (OH >= 32) {
#pragma unroll
        for (int c = 0; c < OH / 32; ++c) {
            uint32_t ov[32];
            tmem_ld_32x32b_x32(taddr + c * 32, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) acc[c * 32 + i] = fmaf(acc[c * 32 + i], alpha, __uint_as_float(ov[i]));
        }
    } else {
        uint32_t ov[16];
        tmem_ld_32x32b_x16(taddr, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = fmaf(acc[i], alpha, __uint_as_float(ov[i]));
    }
}

// K-major 128-byte-swizzle operand (rows x 32-float chunks), K-step kk of 8
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, int rows, int kk) {
    return sw128_kmajor_desc(tile + (kk >> 2) * rows * 128 + (kk & 3) * 32);
}
// MN-major 128-byte / 32-byte-atom operand made of 32 x 32 boxes laid out
// [k-chunk][mn-chunk]; K-step kk of 8 (LBO 4 KiB to the next 32 of MN,
// SBO 512 B to the next 4 k)
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, int mn_chunks, int kk) {
    const uint32_t a = tile + (kk >> 2) * mn_chunks * MN_BOX_BYTES + (kk & 3) * 1024;
    uint64_t d = 0;
    d |= static_cast<uint64_t>((a >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(MN_BOX_BYTES >> 4) << 16;
    d |= static_cast<uint64_t>(512u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(1u) << 61;
    return d;
}

template <int DH>
__global__ void __launch_bounds__(THREADS, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap map_khi,
               const __grid_constant__ CUtensorMap map_klo,
               const __grid_constant__ CUtensorMap map_vhi,
               const __grid_constant__ CUtensorMap map_vlo, FwdParams p) {
    using C = Fwd<DH>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE);
    uint64_t *k_full = bars;          // [2]
    uint64_t *v_full = bars + 2;      // [2]
    uint64_t *k_empty = bars + 4;     // [2]
    uint64_t *s_full = bars + 6;      // [2]
    uint64_t *s_free = bars + 8;      // [2]
    uint64_t *o_full = bars + 10;     // [2]
    uint64_t *o_free = bars + 12;     // [2]
    uint64_t *p_full = bars + 14;     // [2]
    uint64_t *q_ready = bars + 16;
    uint64_t *s_done = bars + 17;
    uint64_t *v_empty = bars + 18;    // [2]
    uint64_t *pv_done = bars + 20;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 21);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile int32_t *k_used = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);
    volatile int32_t *v_used = reinterpret_cast<volatile int32_t *>(tmem_slot + 3);
    float *red = reinterpret_cast<float *>(tmem_slot + 8);  // [6][BQ] row-half maxima / sums
    volatile int *stop = reinterpret_cast<volatile int *>(red + 6 * BQ);  // [4][BQ] stop flags

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // heads vary fastest in launch order, so every head's longest tiles run
    // before any shorter one (longest-first scheduling of the causal work)
    const int bh = blockIdx.x;
    const int qb = p.n_qblocks - 1 - static_cast<int>(blockIdx.y);  // longest rows first
    const int q0 = qb * BQ;
    int last_key = q0 + BQ - 1;
    if (last_key > p.seq - 1) last_key = p.seq - 1;
    const int nkb = last_key / BKV + 1;  // key blocks up to the diagonal

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 1);
            mbar_init(&o_full[i], 1);
            mbar_init(&o_free[i], 8);
            mbar_init(&p_full[i], 8);
        }
        mbar_init(q_ready, 8);
        mbar_init(s_done, 1);
        mbar_init(pv_done, 1);
        *abort_flag = 0;
        *k_used = 0;
        *v_used = 0;
        fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&map_khi);
        prefetch_tensormap(&map_klo);
        prefetch_tensormap(&map_vhi);
        prefetch_tensormap(&map_vlo);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    int32_t issued = 0;

    if (warp == 0 || warp == 11) {
        // ---------------- TMA producers: warp 0 keys, warp 11 values ----------------
        if (lane == 0) {
            const bool keys = warp == 0;
            uint64_t *full = keys ? k_full : v_full;
            uint64_t *empty = keys ? k_empty : v_empty;
            for (int j = 0; j < nkb; ++j) {
                const int s = j & 1;
                if (*abort_flag ||
                    !mbar_wait_bounded(&empty[s], ((j >> 1) & 1) ^ 1, DEVERR_TIMEOUT_PRODUCER)) {
                    *abort_flag = 1;
                    break;
                }
                unsigned char *st = smem + s * C::STAGE;
                if (keys) {
                    mbar_arrive_expect_tx(&full[s], 2 * C::K_TILE);
#pragma unroll
                    for (int c = 0; c < C::KCH; ++c) {
                        tma_load_3d(st + c * BKV * 128, &map_khi, &full[s], c * 32, j * BKV, bh);
                        tma_load_3d(st + C::K_TILE + c * BKV * 128, &map_klo, &full[s], c * 32,
                                    j * BKV, bh);
                    }
                } else {
                    unsigned char *sv = st + 2 * C::K_TILE;
                    mbar_arrive_expect_tx(&full[s], 2 * C::V_TILE);
#pragma unroll
                    for (int kc = 0; kc < BKV / 32; ++kc)
#pragma unroll
                        for (int dc = 0; dc < C::KCH; ++dc) {
                            const int off = (kc * C::KCH + dc) * MN_BOX_BYTES;
                            tma_load_3d(sv + off, &map_vhi, &full[s], dc * 32, j * BKV + kc * 32, bh);
                            tma_load_3d(sv + C::V_TILE + off, &map_vlo, &full[s], dc * 32,
                                        j * BKV + kc * 32, bh);
                        }
                }
                issued = j + 1;
            }
        }
    } else if (warp == 1) {
        // ---------------- score MMAs: S_j = Q . K_j^T ----------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(BQ, BKV);
            bool ok = mbar_wait_bounded(q_ready, 0, DEVERR_TIMEOUT_MMA);
            if (!ok) *abort_flag = 1;
            for (int j = 0; ok && j < nkb; ++j) {
                const int s = j & 1;
                if (*abort_flag || !mbar_wait_bounded(&k_full[s], (j >> 1) & 1, DEVERR_TIMEOUT_MMA) ||
                    !mbar_wait_bounded(&s_free[s], ((j >> 1) & 1) ^ 1, DEVERR_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                *k_used = j + 1;
                tc_fence_after();
                const uint32_t kt = smem_u32(smem + s * C::STAGE);
                const uint32_t d = tm + (s ? C::C_S1 : C::C_S0);
#pragma unroll
                for (int kk = 0; kk < DH / 8; ++kk) {
                    const uint64_t bhi = kmajor_desc(kt, BKV, kk);
                    const uint64_t blo = kmajor_desc(kt + C::K_TILE, BKV, kk);
                    mma_tf32_ts(d, tm + C::C_QLO + 8 * kk, bhi, idesc_s, kk ? 1u : 0u);
                    mma_tf32_ts(d, tm + C::C_QHI + 8 * kk, blo, idesc_s, 1u);
                    mma_tf32_ts(d, tm + C::C_QHI + 8 * kk, bhi, idesc_s, 1u);
                }
                mma_commit(&s_full[s]);
                mma_commit(&k_empty[s]);
            }
            // no MMA of this thread may still run when tensor memory is released
            mma_commit(s_done);
            mbar_wait_bounded(s_done, 0, DEVERR_TIMEOUT_MMA);
        }
    } else if (warp == 10) {
        // ---------------- output MMAs: O_j = P_j . V_j ----------------
        if (lane == 0) {
            constexpr uint32_t idesc_o = idesc_tf32(BQ, DH) | (1u << 16);  // B (values) MN-major
            for (int j = 0; j < nkb; ++j) {
                const int s = j & 1;
                if (*abort_flag || !mbar_wait_bounded(&p_full[s], (j >> 1) & 1, DEVERR_TIMEOUT_MMA) ||
                    !mbar_wait_bounded(&v_full[s], (j >> 1) & 1, DEVERR_TIMEOUT_MMA) ||
                    !mbar_wait_bounded(&o_free[s], ((j >> 1) & 1) ^ 1, DEVERR_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                *v_used = j + 1;
                tc_fence_after();
                const uint32_t vt = smem_u32(smem + s * C::STAGE + 2 * C::K_TILE);
                const uint32_t d = tm + (s ? C::C_O1 : C::C_O0);
#pragma unroll
                for (int kk = 0; kk < BKV / 8; ++kk) {
                    const uint64_t bhi = mnmajor_desc(vt, C::KCH, kk);
                    const uint64_t blo = mnmajor_desc(vt + C::V_TILE, C::KCH, kk);
                    const uint32_t phi = tm + (s ? C::C_S1 : C::C_S0) + 8 * kk;
                    const uint32_t plo = tm + (s ? C::C_PLO1 : C::C_PLO0) + 8 * kk;
                    mma_tf32_ts(d, plo, bhi, idesc_o, kk ? 1u : 0u);
                    mma_tf32_ts(d, phi, blo, idesc_o, 1u);
                    mma_tf32_ts(d, phi, bhi, idesc_o, 1u);
                }
                mma_commit(&o_full[s]);
                mma_commit(&s_free[s]);  // S[s] / PLO[s] reusable for block j + 2
                mma_commit(&v_empty[s]);
            }
            mma_commit(pv_done);
            mbar_wait_bounded(pv_done, 0, DEVERR_TIMEOUT_MMA);
        }
    } else {
        // ---------------- rows: 8 warps, two per TMEM lane quadrant ----------------
        // Thread (half, r) owns query row r = quad * 32 + lane and columns
        // [half * 32, half * 32 + 32) of each score block and
        // [half * DH / 2, (half + 1) * DH / 2) of the output.  The two halves
        // of a row exchange their block maxima through shared memory; their
        // partial row sums combine once at the end.
        const int quad = warp & 3;
        const int half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int qrow = q0 + r;
        const bool live = qrow < p.seq;
        const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
        const int b = bh / p.heads, h = bh % p.heads;
        constexpr int OH = DH / 2;  // output columns per thread
        // scores are kept in the base-2 domain: x = s * scale * log2(e)
        const float c2 = __fmul_rn(p.scale, 1.4426950408889634f);
        // query row half -> hi / lo in tensor memory
        {
            const float *qr = p.q + b * p.q_b + h * p.q_h + static_cast<int64_t>(qrow) * p.q_row +
                              half * OH;
#pragma unroll
            for (int c = 0; c < OH / 32; ++c) {  // DH = 64: one 32-column chunk per half
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (live) v = *reinterpret_cast<const float4 *>(qr + c * 32 + i);
                    split_tf32(v.x, hi[i], lo[i]);
                    split_tf32(v.y, hi[i + 1], lo[i + 1]);
                    split_tf32(v.z, hi[i + 2], lo[i + 2]);
                    split_tf32(v.w, hi[i + 3], lo[i + 3]);
                }
                tmem_st_32x32b_x32(tm + lane_base + C::C_QHI + half * OH + c * 32, hi);
                tmem_st_32x32b_x32(tm + lane_base + C::C_QLO + half * OH + c * 32, lo);
            }
            if constexpr (OH < 32) {
                // DH = 32: 16 columns per half
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int i = 0; i < 16; i += 4) {
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (live) v = *reinterpret_cast<const float4 *>(qr + i);
                    split_tf32(v.x, hi[i], lo[i]);
                    split_tf32(v.y, hi[i + 1], lo[i + 1]);
                    split_tf32(v.z, hi[i + 2], lo[i + 2]);
                    split_tf32(v.w, hi[i + 3], lo[i + 3]);
                }
                tmem_st_32x32b_x16(tm + lane_base + C::C_QHI + half * OH, hi);
                tmem_st_32x32b_x16(tm + lane_base + C::C_QLO + half * OH, lo);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(q_ready);
        }
        float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
        float acc[OH];
#pragma unroll
        for (int i = 0; i < OH; ++i) acc[i] = 0.0f;
        bool ok = true;
        // The two halves of a row pass the exchange barrier below the same
        // number of times: a failed wait only clears `ok`, and the loop ends
        // at the exchange when either half has stopped.
        for (int j = 0; j < nkb; ++j) {
            const int s = j & 1;
            if (ok && (*abort_flag ||
                       !mbar_wait_bounded(&s_full[s], (j >> 1) & 1, DEVERR_TIMEOUT_EPILOGUE))) {
                *abort_flag = 1;
                ok = false;
            }
            uint32_t sr[32];
            if (ok) {
                tc_fence_after();
                tmem_ld_32x32b_x32(tm + lane_base + (s ? C::C_S1 : C::C_S0) + half * 32, sr);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) sr[c] = 0u;
            }
            // scale into the base-2 domain, causal mask, running maximum
            const int key0 = j * BKV + half * 32;
            const bool full_block = key0 + 31 <= q0 && key0 + 31 < p.seq;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const int key = key0 + c;
                float x = __fmul_rn(__uint_as_float(sr[c]), c2);
                if (!full_block && !(key <= qrow && key < p.seq)) x = -INFINITY;
                sr[c] = __float_as_uint(x);
                mx = fmaxf(mx, x);
            }
            const int slot = (j & 1) * 2;
            red[(slot + half) * BQ + r] = mx;
            stop[(slot + half) * BQ + r] = (!ok || *abort_flag) ? 1 : 0;
            named_bar_sync(1 + quad, 64);
            if (stop[(slot + half) * BQ + r] | stop[(slot + (half ^ 1)) * BQ + r]) {
                ok = false;
                break;
            }
            mx = fmaxf(mx, red[(slot + (half ^ 1)) * BQ + r]);
            const float m_new = fmaxf(m, mx);
            const float alpha = ex2_approx(__fsub_rn(m, m_new));
            // probabilities -> tensor memory (over this block's scores; the
            // output MMA of block j - 2, the last reader of PLO[s], finished
            // before this block's scores were computed)
            if (ok) {
                float rs = 0.0f;
                uint32_t phi[32], plo[32];
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    // e in [0, 1]: finite, so the split needs no special cases
                    const float e = ex2_approx(__fsub_rn(__uint_as_float(sr[c]), m_new));
                    rs = __fadd_rn(rs, e);
                    phi[c] = rna_tf32_bits(__float_as_uint(e));
                    plo[c] = rna_tf32_bits(__float_as_uint(__fsub_rn(e, __uint_as_float(phi[c]))));
                }
                tmem_st_32x32b_x32(tm + lane_base + (s ? C::C_S1 : C::C_S0) + half * 32, phi);
                tmem_st_32x32b_x32(tm + lane_base + (s ? C::C_PLO1 : C::C_PLO0) + half * 32, plo);
                l = fmaf(l, alpha, rs);
                m = m_new;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[s]);
            }
            // fold in the previous block's P . V
            if (ok && j >= 1) {
                const int jj = j - 1, so = jj & 1;
                if (!mbar_wait_bounded(&o_full[so], (jj >> 1) & 1, DEVERR_TIMEOUT_EPILOGUE)) {
                    *abort_flag = 1;
                    ok = false;
                } else {
                    tc_fence_after();
                    fold_o<OH>(acc, tm + lane_base + (so ? C::C_O1 : C::C_O0) + half * OH, alpha_prev);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_free[so]);
                }
            }
            alpha_prev = alpha;
        }
        // partial row sums of the two halves
        red[(4 + half) * BQ + r] = l;
        named_bar_sync(1 + quad, 64);
        l = __fadd_rn(red[(4 + half) * BQ + r], red[(4 + (half ^ 1)) * BQ + r]);
        if (ok) {
            const int jj = nkb - 1, so = jj & 1;
            if (!*abort_flag && mbar_wait_bounded(&o_full[so], (jj >> 1) & 1, DEVERR_TIMEOUT_EPILOGUE)) {
                tc_fence_after();
                fold_o<OH>(acc, tm + lane_base + (so ? C::C_O1 : C::C_O0) + half * OH, alpha_prev);
                if (live) {
                    float *orow = p.o + b * p.o_b + h * p.o_h + static_cast<int64_t>(qrow) * p.o_row +
                                  half * OH;
#pragma unroll
                    for (int i = 0; i < OH; i += 4)
                        *reinterpret_cast<float4 *>(orow + i) =
                            make_float4(__fdiv_rn(acc[i], l), __fdiv_rn(acc[i + 1], l),
                                        __fdiv_rn(acc[i + 2], l), __fdiv_rn(acc[i + 3], l));
                    if (p.lse && half == 0)
                        p.lse[static_cast<int64_t>(bh) * p.seq + qrow] =
                            __fadd_rn(__fmul_rn(m, 0.6931471805599453f), logf(l));
                }
            } else {
                *abort_flag = 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if ((warp == 0 || warp == 11) && lane == 0 && *abort_flag) {
        // let issued key / value loads land before the CTA retires
        uint64_t *full = warp == 0 ? k_full : v_full;
        for (int j = warp == 0 ? *k_used : *v_used; j < issued; ++j)
            mbar_wait_bounded(&full[j & 1], (j >> 1) & 1, DEVERR_TIMEOUT_PRODUCER);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, C::COLS);
    }
}

// hi / lo of a flat f32 array (a [BH][S][DH] head tensor with DH a multiple
// of 32 is its own K-major split layout)
__global__ void split_flat_kernel(const float *__restrict__ x, float *__restrict__ hi,
                                  float *__restrict__ lo, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        uint32_t h[4], l[4];
        split_tf32(v.x, h[0], l[0]);
        split_tf32(v.y, h[1], l[1]);
        split_tf32(v.z, h[2], l[2]);
        split_tf32(v.w, h[3], l[3]);
        reinterpret_cast<uint4 *>(hi)[i] = make_uint4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<uint4 *>(lo)[i] = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// ===========================================================================
// Reverse mode.  With P = softmax(S) saved only as the per-row log-sum-exp L
// and D = rowsum(dO * O) (= rowsum(dP * P)):
//   P = exp(S*scale - L),  dP = dO . V^T,  dS = P * (dP - D) * scale,
//   dV = P^T . dO,  dK = dS^T . Q,  dQ = dS . K.
// Two kernels, each owning its accumulators in tensor memory (no atomics,
// so the gradients are deterministic):
//   dkv_kernel: a 128-key tile in the TMEM lanes; streams 32-query blocks
//               from the diagonal down, S^T and dP^T per block, then
//               dV += P^T . dO and dK += dS^T . Q;
//   dq_kernel:  a 128-query tile in the lanes; streams 64-key blocks up to
//               the diagonal, S and dP per block, then dQ += dS . K.
// All products are 3xTF32.  Both kernels run one issuing thread (the
// scores of block n + 1 reuse block n's tensor-memory columns) and 8 row
// warps, two threads per lane, each with half of the block's columns.
// ===========================================================================
constexpr int BQ2 = 32;   // query block of dkv_kernel
constexpr int BK2 = 64;   // key block of dq_kernel

struct BwdParams {
    const float *q, *k, *v, *dout;   // f32 rows (strided like FwdParams)
    int64_t q_row, q_b, q_h;         // strides of q, k, v ([BH][S][DH] layout in the block)
    int64_t d_row, d_b, d_h;         // strides of dout
    const float *lse, *dsum;         // [BH][S]
    float *dq, *dk, *dv;             // outputs, strides below
    int64_t g_row, g_b, g_h;
    // 0: the gradients as f32; else their tf32 split, hi at dq / dk / dv and
    // lo split_lo floats further on (a matmul reads them only split)
    int64_t split_lo;
    int heads, seq;
    float scale;
    int n_blocks;
};

// One row half (DH / 2 floats at `src`) -> hi / lo columns of this lane.
template <int DH>
__device__ __forceinline__ void stage_row_split(const float *src, bool live, uint32_t thi,
                                                uint32_t tlo) {
    constexpr int HALF = DH / 2;
    if constexpr (HALF >= 32) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (live) v = *reinterpret_cast<const float4 *>(src + i);
            split_tf32(v.x, hi[i], lo[i]);
            split_tf32(v.y, hi[i + 1], lo[i + 1]);
            split_tf32(v.z, hi[i + 2], lo[i + 2]);
            split_tf32(v.w, hi[i + 3], lo[i + 3]);
        }
        tmem_st_32x32b_x32(thi, hi);
        tmem_st_32x32b_x32(tlo, lo);
    } else {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (live) v = *reinterpret_cast<const float4 *>(src + i);
            split_tf32(v.x, hi[i], lo[i]);
            split_tf32(v.y, hi[i + 1], lo[i + 1]);
            split_tf32(v.z, hi[i + 2], lo[i + 2]);
            split_tf32(v.w, hi[i + 3], lo[i + 3]);
        }
        tmem_st_32x32b_x16(thi, hi);
        tmem_st_32x32b_x16(tlo, lo);
    }
}

// acc += the DH / 2 accumulator columns of this lane at `taddr`
template <int DH>
__device__ __forceinline__ void add_row_half(float (&acc)[DH / 2], uint32_t taddr) {
    constexpr int HALF = DH / 2;
    if constexpr (HALF >= 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(taddr, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(v[i]));
    } else {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = __fadd_rn(acc[i], __uint_as_float(v[i]));
    }
}
template <int DH>
__device__ __forceinline__ void write_row_half(const float (&acc)[DH / 2], float *dst) {
#pragma unroll
    for (int i = 0; i < DH / 2; i += 4)
        *reinterpret_cast<float4 *>(dst + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
}
// The same row half as its tf32 split: hi = RN_tf32(v) at dst, lo =
// RN_tf32(v - hi) at dst + lo_off (lo = 0 for non-finite v); lo_off = 0
// writes the f32 values.
template <int DH>
__device__ __forceinline__ void write_row_half_out(const float (&acc)[DH / 2], float *dst, int64_t lo_off) {
    if (lo_off == 0) {
        write_row_half<DH>(acc, dst);
        return;
    }
#pragma unroll
    for (int i = 0; i < DH / 2; i += 4) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) split_tf32(acc[i + j], h[j], l[j]);
        *reinterpret_cast<uint4 *>(dst + i) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(dst + lo_off + i) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

template <int DH>
struct Dkv {
    static constexpr int KCH = DH / 32;
    static constexpr int T = BQ2 * DH * 4;          // one query tile (hi or lo), 8 KiB at DH 64
    // stage: Q and dO as K-major (for S^T, dP^T) and MN-major (for dK, dV)
    static constexpr int O_QK = 0, O_DOK = 2 * T, O_QM = 4 * T, O_DOM = 6 * T;
    static constexpr int STAGE = 8 * T;
    static constexpr int STAGES = 2;
    static constexpr int VT = BQ * DH * 4;          // the CTA's values, hi or lo (32 KiB at DH 64)
    static constexpr int O_V = STAGES * STAGE;      // values hi, then lo (K-major A operand)
    static constexpr int SMEM_USED = O_V + 2 * VT + 1024 + 256;
    static constexpr int SMEM = SMEM_USED > 118784 ? SMEM_USED : 118784;
    // TMEM: K (A operand of S^T), dK and dV of one block, then two score
    // buffers, each S^T (-> P^T hi), dP^T (-> dS^T hi), P^T lo, dS^T lo
    static constexpr uint32_t C_KHI = 0, C_KLO = DH, C_DK = 2 * DH, C_DV = 3 * DH;
    static constexpr uint32_t C_BUF = 4 * DH, BUF = 4 * BQ2;
    static constexpr uint32_t O_ST = 0, O_DPT = BQ2, O_PLO = 2 * BQ2, O_DSLO = 3 * BQ2;
    static constexpr uint32_t COLS = 512;
    static_assert(C_BUF + 2 * BUF <= COLS, "tensor memory budget");
    static_assert(SMEM_USED <= 232448, "shared memory budget");
};

template <int DH>
__global__ void __launch_bounds__(THREADS_BWD, 1)
    dkv_kernel(const __grid_constant__ CUtensorMap m_qhi, const __grid_constant__ CUtensorMap m_qlo,
               const __grid_constant__ CUtensorMap m_dhi, const __grid_constant__ CUtensorMap m_dlo,
               const __grid_constant__ CUtensorMap n_qhi, const __grid_constant__ CUtensorMap n_qlo,
               const __grid_constant__ CUtensorMap n_dhi, const __grid_constant__ CUtensorMap n_dlo,
               const __grid_constant__ CUtensorMap m_vhi, const __grid_constant__ CUtensorMap m_vlo,
               BwdParams p) {
    using C = Dkv<DH>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::O_V + 2 * C::VT);
    uint64_t *t_full = bars, *t_empty = bars + 2;   // [2] query tiles
    uint64_t *s_full = bars + 4, *p_full = bars + 6, *s_free = bars + 8;  // [2] score buffers
    uint64_t *kv_ready = bars + 10, *v_full = bars + 11, *acc_full = bars + 12, *acc_done = bars + 13;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 14);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile int32_t *t_used = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);
    volatile int32_t *v_used = reinterpret_cast<volatile int32_t *>(tmem_slot + 3);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x;           // heads fastest: longest tiles of every head first
    const int kb = blockIdx.y;           // key tile; tile 0 has the most query blocks
    const int k0 = kb * BQ;
    const int i0 = k0 / BQ2;             // first query block on or below the diagonal
    const int nq = (p.seq + BQ2 - 1) / BQ2;
    const int nblk = nq - i0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 8);
            mbar_init(&s_free[i], 1);
        }
        mbar_init(kv_ready, 8);
        mbar_init(v_full, 1);
        mbar_init(acc_full, 1);
        mbar_init(acc_done, 1);
        *abort_flag = 0;
        *t_used = 0;
        *v_used = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    int32_t issued = 0;

    if (warp == 0) {
        if (lane == 0) {
            // the CTA's values (A operand of dP^T), once
            mbar_arrive_expect_tx(v_full, 2 * C::VT);
#pragma unroll
            for (int c = 0; c < C::KCH; ++c) {
                tma_load_3d(smem + C::O_V + c * BQ * 128, &m_vhi, v_full, c * 32, k0, bh);
                tma_load_3d(smem + C::O_V + C::VT + c * BQ * 128, &m_vlo, v_full, c * 32, k0, bh);
            }
            for (int n = 0; n < nblk; ++n) {
                const int s = n & 1, q0 = (i0 + n) * BQ2;
                if (*abort_flag ||
                    !mbar_wait_bounded(&t_empty[s], ((n >> 1) & 1) ^ 1, DEVERR_TIMEOUT_PRODUCER)) {
                    *abort_flag = 1;
                    break;
                }
                unsigned char *st = smem + s * C::STAGE;
                mbar_arrive_expect_tx(&t_full[s], 8 * C::T);
#pragma unroll
                for (int c = 0; c < C::KCH; ++c) {
                    const int ko = c * BQ2 * 128;
                    tma_load_3d(st + C::O_QK + ko, &m_qhi, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_QK + C::T + ko, &m_qlo, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_DOK + ko, &m_dhi, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_DOK + C::T + ko, &m_dlo, &t_full[s], c * 32, q0, bh);
                    const int mo = c * MN_BOX_BYTES;  // one 32-query chunk: boxes [dh-chunk]
                    tma_load_3d(st + C::O_QM + mo, &n_qhi, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_QM + C::T + mo, &n_qlo, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_DOM + mo, &n_dhi, &t_full[s], c * 32, q0, bh);
                    tma_load_3d(st + C::O_DOM + C::T + mo, &n_dlo, &t_full[s], c * 32, q0, bh);
                }
                issued = n + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(BQ, BQ2);                 // S^T, dP^T
            constexpr uint32_t idesc_g = idesc_tf32(BQ, DH) | (1u << 16);     // dV, dK (B MN-major)
            const uint32_t vt = smem_u32(smem + C::O_V);
            bool ok = mbar_wait_bounded(kv_ready, 0, DEVERR_TIMEOUT_MMA) &&
                      mbar_wait_bounded(v_full, 0, DEVERR_TIMEOUT_MMA);
            if (!ok) *abort_flag = 1;
            if (ok) *v_used = 1;
            // scores of block n (S^T = K . Q^T, dP^T = V . dO^T) into buffer n % 2
            auto scores = [&](int n) -> bool {
                const int s = n & 1;
                if (*abort_flag || !mbar_wait_bounded(&t_full[s], (n >> 1) & 1, DEVERR_TIMEOUT_MMA) ||
                    !mbar_wait_bounded(&s_free[s], ((n >> 1) & 1) ^ 1, DEVERR_TIMEOUT_MMA))
                    return false;
                *t_used = n + 1;
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * C::STAGE);
                const uint32_t buf = tm + C::C_BUF + s * C::BUF;
#pragma unroll
                for (int kk = 0; kk < DH / 8; ++kk) {
                    const uint64_t qh = kmajor_desc(st + C::O_QK, BQ2, kk);
                    const uint64_t ql = kmajor_desc(st + C::O_QK + C::T, BQ2, kk);
                    const uint64_t dh = kmajor_desc(st + C::O_DOK, BQ2, kk);
                    const uint64_t dl = kmajor_desc(st + C::O_DOK + C::T, BQ2, kk);
                    const uint64_t vh = kmajor_desc(vt, BQ, kk);
                    const uint64_t vl = kmajor_desc(vt + C::VT, BQ, kk);
                    const uint32_t a = 8 * kk, acc = kk ? 1u : 0u;
                    mma_tf32_ts(buf + C::O_ST, tm + C::C_KLO + a, qh, idesc_s, acc);
                    mma_tf32_ts(buf + C::O_ST, tm + C::C_KHI + a, ql, idesc_s, 1u);
                    mma_tf32_ts(buf + C::O_ST, tm + C::C_KHI + a, qh, idesc_s, 1u);
                    mma_tf32_ss(buf + C::O_DPT, vl, dh, idesc_s, acc);
                    mma_tf32_ss(buf + C::O_DPT, vh, dl, idesc_s, 1u);
                    mma_tf32_ss(buf + C::O_DPT, vh, dh, idesc_s, 1u);
                }
                mma_commit(&s_full[s]);
                return true;
            };
            if (ok && nblk > 0) ok = scores(0);
            for (int n = 0; ok && n < nblk; ++n) {
                const int s = n & 1;
                // the next block's scores run while the rows work on this one
                if (n + 1 < nblk && !scores(n + 1)) {
                    ok = false;
                    break;
                }
                if (!mbar_wait_bounded(&p_full[s], (n >> 1) & 1, DEVERR_TIMEOUT_MMA)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * C::STAGE);
                const uint32_t buf = tm + C::C_BUF + s * C::BUF;
#pragma unroll
                for (int kk = 0; kk < BQ2 / 8; ++kk) {
                    const uint64_t dh = mnmajor_desc(st + C::O_DOM, C::KCH, kk);
                    const uint64_t dl = mnmajor_desc(st + C::O_DOM + C::T, C::KCH, kk);
                    const uint64_t qh = mnmajor_desc(st + C::O_QM, C::KCH, kk);
                    const uint64_t ql = mnmajor_desc(st + C::O_QM + C::T, C::KCH, kk);
                    const uint32_t a = 8 * kk, acc = kk ? 1u : 0u;  // fresh per block
                    mma_tf32_ts(tm + C::C_DV, buf + C::O_PLO + a, dh, idesc_g, acc);
                    mma_tf32_ts(tm + C::C_DV, buf + C::O_ST + a, dl, idesc_g, 1u);
                    mma_tf32_ts(tm + C::C_DV, buf + C::O_ST + a, dh, idesc_g, 1u);
                    mma_tf32_ts(tm + C::C_DK, buf + C::O_DSLO + a, qh, idesc_g, acc);
                    mma_tf32_ts(tm + C::C_DK, buf + C::O_DPT + a, ql, idesc_g, 1u);
                    mma_tf32_ts(tm + C::C_DK, buf + C::O_DPT + a, qh, idesc_g, 1u);
                }
                mma_commit(acc_full);       // this block's dK, dV ready to fold
                mma_commit(&s_free[s]);     // score buffer s reusable for block n + 2
                mma_commit(&t_empty[s]);    // query tiles of stage s reusable
            }
            if (!ok) *abort_flag = 1;
            mma_commit(acc_done);
            mbar_wait_bounded(acc_done, 0, DEVERR_TIMEOUT_MMA);
        }
    } else {
        // rows: thread (half, r) owns key row k0 + r and queries [half*16, half*16 + 16)
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int key = k0 + r;
        const bool live = key < p.seq;
        const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
        const int b = bh / p.heads, h = bh % p.heads;
        const int64_t row_off = b * p.q_b + h * p.q_h + static_cast<int64_t>(key) * p.q_row;
        stage_row_split<DH>(p.k + row_off + half * (DH / 2), live,
                            tm + lane_base + C::C_KHI + half * (DH / 2),
                            tm + lane_base + C::C_KLO + half * (DH / 2));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(kv_ready);
        const float c2 = __fmul_rn(p.scale, 1.4426950408889634f);
        const float *lse = p.lse + static_cast<int64_t>(bh) * p.seq;
        const float *dsum = p.dsum + static_cast<int64_t>(bh) * p.seq;
        float dk_acc[DH / 2], dv_acc[DH / 2];
#pragma unroll
        for (int i = 0; i < DH / 2; ++i) dk_acc[i] = dv_acc[i] = 0.0f;
        bool ok = true;
        // Block n's dK / dV contributions are folded into f32 registers
        // (rounded additions; each block is 12 tensor-core accumulations)
        // after the rows have turned block n + 1's scores into P and dS, so
        // the gradient MMAs of block n run while the rows work on block n + 1.
        // The accumulators are reused by block n + 1's gradient MMAs, which
        // wait for this thread's p_full arrival of block n + 1: the fold of
        // block n comes before that arrival.
        // (every wait's outcome is made warp-uniform, so the warp's lanes
        // stay converged for the shuffles and __syncwarp below)
        auto fold_block = [&](int n) -> bool {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(acc_full, n & 1, DEVERR_TIMEOUT_EPILOGUE)))
                return false;
            tc_fence_after();
            add_row_half<DH>(dk_acc, tm + lane_base + C::C_DK + half * (DH / 2));
            add_row_half<DH>(dv_acc, tm + lane_base + C::C_DV + half * (DH / 2));
            tc_fence_before();
            return true;
        };
        for (int n = 0; n < nblk; ++n) {
            const int s = n & 1;
            const uint32_t buf = tm + lane_base + C::C_BUF + s * C::BUF;
            // this half's 16 queries: lane c < 16 holds lse, lane 16 + c dsum
            // of query qb0 + c (one load per lane, issued before the wait)
            const int qb0 = (i0 + n) * BQ2 + half * 16;
            const int ql = qb0 + (lane & 15);
            const int qlc = ql < p.seq ? ql : p.seq - 1;
            const float stat = lane < 16 ? __fmul_rn(lse[qlc], 1.4426950408889634f) : dsum[qlc];
            const bool go = !*abort_flag &&
                            mbar_wait_bounded(&s_full[s], (n >> 1) & 1, DEVERR_TIMEOUT_EPILOGUE);
            if (!__all_sync(0xffffffffu, go)) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sv[16], dv[16];
            tmem_ld_32x32b_x16(buf + C::O_ST + half * 16, sv);
            tmem_ld_32x32b_x16(buf + C::O_DPT + half * 16, dv);
            tmem_wait_ld();
            uint32_t ph[16], pl[16], dh[16], dl[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int qi = qb0 + c;
                const bool valid = live && key <= qi && qi < p.seq;
                const float L2 = __shfl_sync(0xffffffffu, stat, c);
                const float Dq = __shfl_sync(0xffffffffu, stat, 16 + c);
                const float pr = valid ? ex2_approx(__fsub_rn(__fmul_rn(__uint_as_float(sv[c]), c2), L2)) : 0.0f;
                const float ds = __fmul_rn(__fmul_rn(pr, __fsub_rn(__uint_as_float(dv[c]), Dq)), p.scale);
                split_tf32(pr, ph[c], pl[c]);
                split_tf32(ds, dh[c], dl[c]);
            }
            tmem_st_32x32b_x16(buf + C::O_ST + half * 16, ph);
            tmem_st_32x32b_x16(buf + C::O_PLO + half * 16, pl);
            tmem_st_32x32b_x16(buf + C::O_DPT + half * 16, dh);
            tmem_st_32x32b_x16(buf + C::O_DSLO + half * 16, dl);
            tmem_wait_st();
            tc_fence_before();
            if (n > 0 && !fold_block(n - 1)) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[s]);
        }
        if (ok && nblk > 0) {
            const bool aborted = __any_sync(0xffffffffu, *abort_flag != 0);
            if (aborted || !fold_block(nblk - 1)) {
                *abort_flag = 1;
                ok = false;
            }
        }
        if (ok && !*abort_flag && live) {
            const int64_t g = b * p.g_b + h * p.g_h + static_cast<int64_t>(key) * p.g_row +
                              half * (DH / 2);
            write_row_half_out<DH>(dk_acc, p.dk + g, p.split_lo);
            write_row_half_out<DH>(dv_acc, p.dv + g, p.split_lo);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && *abort_flag) {
        for (int n = *t_used; n < issued; ++n)
            mbar_wait_bounded(&t_full[n & 1], (n >> 1) & 1, DEVERR_TIMEOUT_PRODUCER);
        if (!*v_used) mbar_wait_bounded(v_full, 0, DEVERR_TIMEOUT_PRODUCER);
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, C::COLS);
    }
}

template <int DH>
struct Dq {
    static constexpr int KCH = DH / 32;
    static constexpr int T = BK2 * DH * 4;          // one key tile (hi or lo), 16 KiB at DH 64
    // stage: K as K-major (for S) and MN-major (for dQ), V K-major (for dP)
    static constexpr int O_KK = 0, O_VK = 2 * T, O_KM = 4 * T;
    static constexpr int STAGE = 6 * T;
    static constexpr int STAGES = 2;
    static constexpr int SMEM = STAGES * STAGE + 1024 + 256;
    static constexpr uint32_t C_QHI = 0, C_QLO = DH, C_OHI = 2 * DH, C_OLO = 3 * DH;
    static constexpr uint32_t C_DQ = 4 * DH, C_S = 5 * DH, C_DP = C_S + BK2, C_DSLO = C_DP + BK2;
    static constexpr uint32_t COLS = 512;
    static_assert(C_DSLO + BK2 <= COLS, "tensor memory budget");
};

template <int DH>
__global__ void __launch_bounds__(THREADS_BWD, 1)
    dq_kernel(const __grid_constant__ CUtensorMap m_khi, const __grid_constant__ CUtensorMap m_klo,
              const __grid_constant__ CUtensorMap m_vhi, const __grid_constant__ CUtensorMap m_vlo,
              const __grid_constant__ CUtensorMap n_khi, const __grid_constant__ CUtensorMap n_klo,
              BwdParams p) {
    using C = Dq<DH>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE);
    uint64_t *t_full = bars, *t_empty = bars + 2;
    uint64_t *qo_ready = bars + 4, *s_full = bars + 5, *p_full = bars + 6, *s_free = bars + 7;
    uint64_t *acc_done = bars + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 9);
    volatile uint32_t *abort_flag = tmem_slot + 1;
    volatile int32_t *t_used = reinterpret_cast<volatile int32_t *>(tmem_slot + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x;                                        // heads fastest
    const int qb = p.n_blocks - 1 - static_cast<int>(blockIdx.y);  // longest rows first
    const int q0 = qb * BQ;
    int last_key = q0 + BQ - 1;
    if (last_key > p.seq - 1) last_key = p.seq - 1;
    const int nkb = last_key / BK2 + 1;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&t_full[i], 1);
            mbar_init(&t_empty[i], 1);
        }
        mbar_init(qo_ready, 8);
        mbar_init(s_full, 1);
        mbar_init(p_full, 8);
        mbar_init(s_free, 1);
        mbar_init(acc_done, 1);
        *abort_flag = 0;
        *t_used = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tm = *tmem_slot;
    int32_t issued = 0;

    if (warp == 0) {
        if (lane == 0) {
            for (int j = 0; j < nkb; ++j) {
                const int s = j & 1;
                if (*abort_flag ||
                    !mbar_wait_bounded(&t_empty[s], ((j >> 1) & 1) ^ 1, DEVERR_TIMEOUT_PRODUCER)) {
                    *abort_flag = 1;
                    break;
                }
                unsigned char *st = smem + s * C::STAGE;
                mbar_arrive_expect_tx(&t_full[s], 6 * C::T);
#pragma unroll
                for (int c = 0; c < C::KCH; ++c) {
                    const int ko = c * BK2 * 128;
                    tma_load_3d(st + C::O_KK + ko, &m_khi, &t_full[s], c * 32, j * BK2, bh);
                    tma_load_3d(st + C::O_KK + C::T + ko, &m_klo, &t_full[s], c * 32, j * BK2, bh);
                    tma_load_3d(st + C::O_VK + ko, &m_vhi, &t_full[s], c * 32, j * BK2, bh);
                    tma_load_3d(st + C::O_VK + C::T + ko, &m_vlo, &t_full[s], c * 32, j * BK2, bh);
                }
#pragma unroll
                for (int kc = 0; kc < BK2 / 32; ++kc)
#pragma unroll
                    for (int dc = 0; dc < C::KCH; ++dc) {
                        const int off = (kc * C::KCH + dc) * MN_BOX_BYTES;
                        tma_load_3d(st + C::O_KM + off, &n_khi, &t_full[s], dc * 32, j * BK2 + kc * 32, bh);
                        tma_load_3d(st + C::O_KM + C::T + off, &n_klo, &t_full[s], dc * 32,
                                    j * BK2 + kc * 32, bh);
                    }
                issued = j + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(BQ, BK2);
            constexpr uint32_t idesc_g = idesc_tf32(BQ, DH) | (1u << 16);
            bool ok = mbar_wait_bounded(qo_ready, 0, DEVERR_TIMEOUT_MMA);
            if (!ok) *abort_flag = 1;
            for (int j = 0; ok && j < nkb; ++j) {
                const int s = j & 1;
                if (*abort_flag || !mbar_wait_bounded(&t_full[s], (j >> 1) & 1, DEVERR_TIMEOUT_MMA) ||
                    !mbar_wait_bounded(s_free, (j & 1) ^ 1, DEVERR_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                *t_used = j + 1;
                tc_fence_after();
                const uint32_t st = smem_u32(smem + s * C::STAGE);
#pragma unroll
                for (int kk = 0; kk < DH / 8; ++kk) {
                    const uint64_t kh = kmajor_desc(st + C::O_KK, BK2, kk);
                    const uint64_t kl = kmajor_desc(st + C::O_KK + C::T, BK2, kk);
                    const uint64_t vh = kmajor_desc(st + C::O_VK, BK2, kk);
                    const uint64_t vl = kmajor_desc(st + C::O_VK + C::T, BK2, kk);
                    const uint32_t a = 8 * kk, acc = kk ? 1u : 0u;
                    mma_tf32_ts(tm + C::C_S, tm + C::C_QLO + a, kh, idesc_s, acc);
                    mma_tf32_ts(tm + C::C_S, tm + C::C_QHI + a, kl, idesc_s, 1u);
                    mma_tf32_ts(tm + C::C_S, tm + C::C_QHI + a, kh, idesc_s, 1u);
                    mma_tf32_ts(tm + C::C_DP, tm + C::C_OLO + a, vh, idesc_s, acc);
                    mma_tf32_ts(tm + C::C_DP, tm + C::C_OHI + a, vl, idesc_s, 1u);
                    mma_tf32_ts(tm + C::C_DP, tm + C::C_OHI + a, vh, idesc_s, 1u);
                }
                mma_commit(s_full);
                if (!mbar_wait_bounded(p_full, j & 1, DEVERR_TIMEOUT_MMA)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < BK2 / 8; ++kk) {
                    const uint64_t kh = mnmajor_desc(st + C::O_KM, C::KCH, kk);
                    const uint64_t kl = mnmajor_desc(st + C::O_KM + C::T, C::KCH, kk);
                    const uint32_t a = 8 * kk, acc = kk ? 1u : 0u;  // fresh per block
                    mma_tf32_ts(tm + C::C_DQ, tm + C::C_DSLO + a, kh, idesc_g, acc);
                    mma_tf32_ts(tm + C::C_DQ, tm + C::C_DP + a, kl, idesc_g, 1u);
                    mma_tf32_ts(tm + C::C_DQ, tm + C::C_DP + a, kh, idesc_g, 1u);
                }
                mma_commit(s_free);
                mma_commit(&t_empty[s]);
            }
            mma_commit(acc_done);
            mbar_wait_bounded(acc_done, 0, DEVERR_TIMEOUT_MMA);
        }
    } else {
        // rows: thread (half, r) owns query row q0 + r and keys [half*32, half*32 + 32)
        const int quad = warp & 3, half = (warp - 2) >> 2;
        const int r = quad * 32 + lane;
        const int qrow = q0 + r;
        const bool live = qrow < p.seq;
        const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
        const int b = bh / p.heads, h = bh % p.heads;
        stage_row_split<DH>(p.q + b * p.q_b + h * p.q_h + static_cast<int64_t>(qrow) * p.q_row + half * (DH / 2),
                            live, tm + lane_base + C::C_QHI + half * (DH / 2),
                            tm + lane_base + C::C_QLO + half * (DH / 2));
        stage_row_split<DH>(p.dout + b * p.d_b + h * p.d_h + static_cast<int64_t>(qrow) * p.d_row + half * (DH / 2),
                            live, tm + lane_base + C::C_OHI + half * (DH / 2),
                            tm + lane_base + C::C_OLO + half * (DH / 2));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(qo_ready);
        const float c2 = __fmul_rn(p.scale, 1.4426950408889634f);
        const int64_t ro = static_cast<int64_t>(bh) * p.seq + (live ? qrow : 0);
        const float L2 = __fmul_rn(p.lse[ro], 1.4426950408889634f);
        const float Dr = p.dsum[ro];
        float dq_acc[DH / 2];
#pragma unroll
        for (int i = 0; i < DH / 2; ++i) dq_acc[i] = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkb; ++j) {
            if (*abort_flag || !mbar_wait_bounded(s_full, j & 1, DEVERR_TIMEOUT_EPILOGUE)) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sv[32], dv[32];
            tmem_ld_32x32b_x32(tm + lane_base + C::C_S + half * 32, sv);
            tmem_ld_32x32b_x32(tm + lane_base + C::C_DP + half * 32, dv);
            tmem_wait_ld();
            const int kb0 = j * BK2 + half * 32;
            uint32_t dh[32], dl[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const int key = kb0 + c;
                const bool valid = live && key <= qrow;
                const float pr = valid ? ex2_approx(__fsub_rn(__fmul_rn(__uint_as_float(sv[c]), c2), L2)) : 0.0f;
                const float ds = __fmul_rn(__fmul_rn(pr, __fsub_rn(__uint_as_float(dv[c]), Dr)), p.scale);
                split_tf32(ds, dh[c], dl[c]);
            }
            tmem_st_32x32b_x32(tm + lane_base + C::C_DP + half * 32, dh);
            tmem_st_32x32b_x32(tm + lane_base + C::C_DSLO + half * 32, dl);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full);
            if (!mbar_wait_bounded(s_free, j & 1, DEVERR_TIMEOUT_EPILOGUE)) {
                *abort_flag = 1;
                ok = false;
                break;
            }
            tc_fence_after();
            add_row_half<DH>(dq_acc, tm + lane_base + C::C_DQ + half * (DH / 2));
            tc_fence_before();
        }
        if (ok && !*abort_flag && live)
            write_row_half_out<DH>(dq_acc, p.dq + b * p.g_b + h * p.g_h +
                                               static_cast<int64_t>(qrow) * p.g_row + half * (DH / 2),
                                   p.split_lo);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0 && lane == 0 && *abort_flag)
        for (int j = *t_used; j < issued; ++j)
            mbar_wait_bounded(&t_full[j & 1], (j >> 1) & 1, DEVERR_TIMEOUT_PRODUCER);
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tm, C::COLS);
    }
}

// D[bh][s] = sum_d dout[s][d] * o[s][d] (sequential over d), one warp per 32 rows
__global__ void dsum_kernel(const float *__restrict__ dout, int64_t d_row, int64_t d_b,
                            int64_t d_h, const float *__restrict__ o, int64_t o_row, int64_t o_b,
                            int64_t o_h, float *__restrict__ dsum, int heads, int seq, int dh,
                            int64_t rows) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t bh = i / seq;
        const int s = static_cast<int>(i % seq);
        const int b = static_cast<int>(bh / heads), h = static_cast<int>(bh % heads);
        const float *dr = dout + b * d_b + h * d_h + static_cast<int64_t>(s) * d_row;
        const float *orow = o + b * o_b + h * o_h + static_cast<int64_t>(s) * o_row;
        float acc = 0.0f;
        for (int d = 0; d < dh; d += 4) {
            const float4 x = *reinterpret_cast<const float4 *>(dr + d);
            const float4 y = *reinterpret_cast<const float4 *>(orow + d);
            acc = fmaf(x.x, y.x, acc);
            acc = fmaf(x.y, y.y, acc);
            acc = fmaf(x.z, y.z, acc);
            acc = fmaf(x.w, y.w, acc);
        }
        dsum[i] = acc;
    }
}

}  // namespace attn

namespace {

typedef CUresult (*EncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                             const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                             const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// [BH][S][DH] head tensor -> 3-D map {DH, S, BH}; box {32, rows, 1}.  Rows
// past S read as zeros (per head).
int head_map(CUtensorMap *map, const float *base, int64_t bh, int64_t s, int dh, int box_rows,
             bool mn_major) {
    EncodeFn fn = reinterpret_cast<EncodeFn>(tf32x3::encode_fn());
    if (!fn) return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(dh), static_cast<cuuint64_t>(s),
                          static_cast<cuuint64_t>(bh)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(dh) * 4, static_cast<cuuint64_t>(s * dh) * 4};
    cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(CHELIS_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled(head) failed (%d)", (int)r);
    return CHELIS_CUDA_OK;
}

}  // namespace

bool flash_attention_supported(int64_t dh) { return dh == 32 || dh == 64; }

int split_flat(const float *x, float *hi, float *lo, int64_t n, cudaStream_t s) {
    const int64_t n4 = n / 4;
    int64_t blocks = (n4 + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    attn::split_flat_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, hi, lo, n4);
    g_launches++;
    CHELIS_LAUNCH_CHECK("split_flat_kernel");
    return CHELIS_CUDA_OK;
}

// Causal attention forward on split keys / values ([BH][S][DH] hi / lo,
// contiguous) and f32 queries addressed by strides; output rows addressed
// the same way; lse [BH][S] optional.
int flash_fwd(int64_t bh, int64_t heads, int64_t seq, int64_t dh, float scale, const float *q,
              int64_t q_row, int64_t q_b, int64_t q_h, const float *k_hi, const float *k_lo,
              const float *v_hi, const float *v_lo, float *o, int64_t o_row, int64_t o_b,
              int64_t o_h, float *lse, cudaStream_t s) {
    if (!flash_attention_supported(dh))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "flash attention covers head dims 32, 64");
    if (bh > 65535 || seq > (1 << 24))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "attention extents beyond the grid");
    CUtensorMap mkh, mkl, mvh, mvl;
    CHELIS_TRY(head_map(&mkh, k_hi, bh, seq, static_cast<int>(dh), attn::BKV, false));
    CHELIS_TRY(head_map(&mkl, k_lo, bh, seq, static_cast<int>(dh), attn::BKV, false));
    CHELIS_TRY(head_map(&mvh, v_hi, bh, seq, static_cast<int>(dh), 32, true));
    CHELIS_TRY(head_map(&mvl, v_lo, bh, seq, static_cast<int>(dh), 32, true));
    attn::FwdParams p;
    p.q = q;
    p.q_row = q_row;
    p.q_b = q_b;
    p.q_h = q_h;
    p.o = o;
    p.o_row = o_row;
    p.o_b = o_b;
    p.o_h = o_h;
    p.lse = lse;
    p.heads = static_cast<int>(heads);
    p.seq = static_cast<int>(seq);
    p.scale = scale;
    p.n_qblocks = static_cast<int>((seq + attn::BQ - 1) / attn::BQ);
    if (p.n_qblocks > 65535) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "attention: sequence too long");
    dim3 grid(static_cast<unsigned>(bh), static_cast<unsigned>(p.n_qblocks));
    auto launch = [&](auto kern, int smem) -> int {
        static uint64_t done[2] = {0, 0};
        CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(kern), smem,
                                    &done[dh == 64 ? 1 : 0], "cudaFuncSetAttribute(attn fwd)"));
        kern<<<grid, attn::THREADS, smem, s>>>(mkh, mkl, mvh, mvl, p);
        g_launches++;
        CHELIS_LAUNCH_CHECK("attn::fwd_kernel");
        return CHELIS_CUDA_OK;
    };
    if (dh == 64) return launch(attn::fwd_kernel<64>, attn::Fwd<64>::SMEM);
    return launch(attn::fwd_kernel<32>, attn::Fwd<32>::SMEM);
}


// Causal attention reverse mode.  q, k, v: f32 rows addressed by (q_row,
// q_b, q_h) strides; dout, o likewise by their own strides; lse [BH][S]
// from the forward; *_hi / *_lo: split copies of q, k, v, dout as contiguous
// [BH][S][DH]; dsum: [BH][S] scratch; gradients written through (g_row,
// g_b, g_h) strides.
int flash_bwd(int64_t bh, int64_t heads, int64_t seq, int64_t dh, float scale, const float *q,
              const float *k, const float *v, int64_t q_row, int64_t q_b, int64_t q_h,
              const float *dout, int64_t d_row, int64_t d_b, int64_t d_h, const float *o,
              int64_t o_row, int64_t o_b, int64_t o_h, const float *lse, const float *q_hi,
              const float *q_lo, const float *k_hi, const float *k_lo, const float *v_hi,
              const float *v_lo, const float *do_hi, const float *do_lo, float *dsum, float *dq,
              float *dk, float *dv, int64_t g_row, int64_t g_b, int64_t g_h, cudaStream_t s,
              int64_t split_lo = 0) {
    if (!flash_attention_supported(dh))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "flash attention covers head dims 32, 64");
    if (bh > 65535 || seq > (1 << 24))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "attention extents beyond the grid");
    const int d = static_cast<int>(dh);
    {
        const int64_t rows = bh * seq;
        int64_t blocks = (rows + 255) / 256;
        const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
        if (blocks > cap) blocks = cap;
        attn::dsum_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
            dout, d_row, d_b, d_h, o, o_row, o_b, o_h, dsum, static_cast<int>(heads),
            static_cast<int>(seq), d, rows);
        g_launches++;
        CHELIS_LAUNCH_CHECK("attn::dsum_kernel");
    }
    attn::BwdParams p;
    p.q = q;
    p.k = k;
    p.v = v;
    p.dout = dout;
    p.q_row = q_row;
    p.q_b = q_b;
    p.q_h = q_h;
    p.d_row = d_row;
    p.d_b = d_b;
    p.d_h = d_h;
    p.lse = lse;
    p.dsum = dsum;
    p.dq = dq;
    p.dk = dk;
    p.dv = dv;
    p.g_row = g_row;
    p.g_b = g_b;
    p.g_h = g_h;
    p.split_lo = split_lo;
    p.heads = static_cast<int>(heads);
    p.seq = static_cast<int>(seq);
    p.scale = scale;
    p.n_blocks = static_cast<int>((seq + attn::BQ - 1) / attn::BQ);
    if (p.n_blocks > 65535) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "attention: sequence too long");
    dim3 grid(static_cast<unsigned>(bh), static_cast<unsigned>(p.n_blocks));
    {
        CUtensorMap mq[2], md[2], nq[2], nd[2];
        CHELIS_TRY(head_map(&mq[0], q_hi, bh, seq, d, attn::BQ2, false));
        CHELIS_TRY(head_map(&mq[1], q_lo, bh, seq, d, attn::BQ2, false));
        CHELIS_TRY(head_map(&md[0], do_hi, bh, seq, d, attn::BQ2, false));
        CHELIS_TRY(head_map(&md[1], do_lo, bh, seq, d, attn::BQ2, false));
        CHELIS_TRY(head_map(&nq[0], q_hi, bh, seq, d, 32, true));
        CHELIS_TRY(head_map(&nq[1], q_lo, bh, seq, d, 32, true));
        CHELIS_TRY(head_map(&nd[0], do_hi, bh, seq, d, 32, true));
        CHELIS_TRY(head_map(&nd[1], do_lo, bh, seq, d, 32, true));
        CUtensorMap mvv[2];
        CHELIS_TRY(head_map(&mvv[0], v_hi, bh, seq, d, attn::BQ, false));
        CHELIS_TRY(head_map(&mvv[1], v_lo, bh, seq, d, attn::BQ, false));
        auto launch = [&](auto kern, int smem) -> int {
            static uint64_t done[2] = {0, 0};
            CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(kern), smem,
                                        &done[d == 64 ? 1 : 0], "cudaFuncSetAttribute(attn dkv)"));
            kern<<<grid, attn::THREADS_BWD, smem, s>>>(mq[0], mq[1], md[0], md[1], nq[0], nq[1],
                                                       nd[0], nd[1], mvv[0], mvv[1], p);
            g_launches++;
            CHELIS_LAUNCH_CHECK("attn::dkv_kernel");
            return CHELIS_CUDA_OK;
        };
        if (d == 64) CHELIS_TRY(launch(attn::dkv_kernel<64>, attn::Dkv<64>::SMEM));
        else CHELIS_TRY(launch(attn::dkv_kernel<32>, attn::Dkv<32>::SMEM));
    }
    {
        CUtensorMap mk[2], mv[2], nk[2];
        CHELIS_TRY(head_map(&mk[0], k_hi, bh, seq, d, attn::BK2, false));
        CHELIS_TRY(head_map(&mk[1], k_lo, bh, seq, d, attn::BK2, false));
        CHELIS_TRY(head_map(&mv[0], v_hi, bh, seq, d, attn::BK2, false));
        CHELIS_TRY(head_map(&mv[1], v_lo, bh, seq, d, attn::BK2, false));
        CHELIS_TRY(head_map(&nk[0], k_hi, bh, seq, d, 32, true));
        CHELIS_TRY(head_map(&nk[1], k_lo, bh, seq, d, 32, true));
        auto launch = [&](auto kern, int smem) -> int {
            static uint64_t done[2] = {0, 0};
            CHELIS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(kern), smem,
                                        &done[d == 64 ? 1 : 0], "cudaFuncSetAttribute(attn dq)"));
            kern<<<grid, attn::THREADS_BWD, smem, s>>>(mk[0], mk[1], mv[0], mv[1], nk[0], nk[1], p);
            g_launches++;
            CHELIS_LAUNCH_CHECK("attn::dq_kernel");
            return CHELIS_CUDA_OK;
        };
        if (d == 64) CHELIS_TRY(launch(attn::dq_kernel<64>, attn::Dq<64>::SMEM));
        else CHELIS_TRY(launch(attn::dq_kernel<32>, attn::Dq<32>::SMEM));
    }
    return CHELIS_CUDA_OK;
}

}  // namespace chelis

using namespace chelis;

extern "C" int chelis_cuda_attention_causal_fwd(int64_t bh, int64_t seq, int64_t dh, float scale,
                                                const float *q, const float *k, const float *v,
                                                float *o, float *lse) {
    if (bh < 0 || seq < 0 || dh <= 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in attention at i64");
    if (bh == 0 || seq == 0) return CHELIS_CUDA_OK;
    if (!flash_attention_supported(dh))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "flash attention covers head dims 32, 64");
    cudaStream_t s = current_stream();
    const int64_t n = bh * seq * dh;
    void *buf = nullptr;
    CHELIS_TRY(scratch_alloc(&buf, 4 * n * sizeof(float), s));
    float *khi = static_cast<float *>(buf), *klo = khi + n, *vhi = klo + n, *vlo = vhi + n;
    int st = split_flat(k, khi, klo, n, s);
    if (st == CHELIS_CUDA_OK) st = split_flat(v, vhi, vlo, n, s);
    if (st == CHELIS_CUDA_OK)
        st = flash_fwd(bh, 1, seq, dh, scale, q, dh, seq * dh, 0, khi, klo, vhi, vlo, o, dh,
                       seq * dh, 0, lse, s);
    scratch_free(buf, s);
    return st;
}

extern "C" int chelis_cuda_attention_causal_bwd(int64_t bh, int64_t seq, int64_t dh, float scale,
                                                const float *q, const float *k, const float *v,
                                                const float *o, const float *lse,
                                                const float *dout, float *dq, float *dk,
                                                float *dv) {
    if (bh < 0 || seq < 0 || dh <= 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in attention at i64");
    if (bh == 0 || seq == 0) return CHELIS_CUDA_OK;
    if (!flash_attention_supported(dh))
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "flash attention covers head dims 32, 64");
    cudaStream_t s = current_stream();
    const int64_t n = bh * seq * dh;
    void *buf = nullptr;
    CHELIS_TRY(scratch_alloc(&buf, (8 * n + bh * seq) * sizeof(float), s));
    float *f = static_cast<float *>(buf);
    float *qh = f, *ql = f + n, *kh = f + 2 * n, *kl = f + 3 * n, *vh = f + 4 * n, *vl = f + 5 * n,
          *doh = f + 6 * n, *dol = f + 7 * n, *dsum = f + 8 * n;
    int st = split_flat(q, qh, ql, n, s);
    if (st == CHELIS_CUDA_OK) st = split_flat(k, kh, kl, n, s);
    if (st == CHELIS_CUDA_OK) st = split_flat(v, vh, vl, n, s);
    if (st == CHELIS_CUDA_OK) st = split_flat(dout, doh, dol, n, s);
    if (st == CHELIS_CUDA_OK)
        st = flash_bwd(bh, 1, seq, dh, scale, q, k, v, dh, seq * dh, 0, dout, dh, seq * dh, 0, o,
                       dh, seq * dh, 0, lse, qh, ql, kh, kl, vh, vl, doh, dol, dsum, dq, dk, dv,
                       dh, seq * dh, 0, s);
    scratch_free(buf, s);
    return st;
}
