// rows.cu -- fused elementwise / reduction groups over the last axis of a
// [rows, hidden] f32 tensor, and their adjoints:
//   layer_norm (tier2.rs:1248-1375), softmax (tier2.rs:1079-1180) and its
//   adjoint (grad.rs:2248-2280), keyed dropout / DropoutReplay
//   (dtype_semantics.rs:4256-4280), row sum / max, the fused chain
//   layer_norm -> softmax -> dropout -> row sum and its adjoint, column sums,
//   bool count and cumsum.
//
// Row layout in registers.  A CTA of T threads owns one row at a time.  The
// row is cut into "chunks" of 4*T elements; thread t holds elements
// [4t, 4t+4) of every chunk (one float4 per chunk: 128-bit coalesced loads).
// NC = ceil(hidden / 4T) chunks are held in registers (NC <= 8).
//
// Sums use the canonical adjacent-pair tree (spec/05-risc-primitives.md:
// 452-466, 515-531) bit for bit: every chunk is an aligned power-of-two
// block, so its sum is a subtree (thread-local pairs, then the warp and
// block xor butterflies); the chunk sums then combine pass by pass.  A
// ragged last chunk uses the same butterfly with absent operands passed
// through (the tree over a prefix of leaves).
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>

#include "common.cuh"
#include "crmath.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int rows_mode();

namespace rows {

// ---------------------------------------------------------------------------
// block-level canonical tree
// ---------------------------------------------------------------------------
// Reduce v[c][0..3] (thread t's 4 leaves of chunk c, valid when the element
// index is < n) to the canonical tree total over all n leaves.  `red` is
// shared scratch of at least NC * (T/32) floats.  Every thread returns the
// total.  Ends with a __syncthreads so `red` can be reused (TRAIL = false
// leaves it out: the caller alternates two scratch areas, so the next
// reduction's barrier already orders this one's reads before any rewrite).
template <int T, int NC, bool TRAIL = true>
__device__ __forceinline__ float block_tree(const float (&v)[NC][4], int n, float *red) {
    constexpr int W = T / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool full = (n == NC * 4 * T);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        float s;
        if (full) {
            s = __fadd_rn(__fadd_rn(v[c][0], v[c][1]), __fadd_rn(v[c][2], v[c][3]));
            s = warp_tree_full(s);
        } else {
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            const int cnt = n - e0;  // leaves of this thread still valid
            const float s01 = tree_pair(v[c][0], cnt > 0, v[c][1], cnt > 1);
            const float s23 = tree_pair(v[c][2], cnt > 2, v[c][3], cnt > 3);
            s = tree_pair(s01, cnt > 0, s23, cnt > 2);
            bool valid = cnt > 0;
            s = warp_tree(s, valid);
            if (!valid) s = __int_as_float(0x7fc00001);  // marker, never read as a leaf
        }
        if (lane == 0) red[c * W + warp] = s;
    }
    __syncthreads();
    // every thread: butterfly over the W warp sums of each chunk, then the
    // pass-by-pass tree over the chunk sums
    float chunk[NC];
    int nchunks = 0;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int c0 = c * 4 * T;
        if (c0 < n) {
            float w[W];
#pragma unroll
            for (int i = 0; i < W; ++i) w[i] = red[c * W + i];
            // number of warps with at least one valid leaf in this chunk
            const int per_warp = 4 * 32;
            int vw = (n - c0 + per_warp - 1) / per_warp;
            if (vw > W) vw = W;
#pragma unroll
            for (int width = 1; width < W; width <<= 1) {
#pragma unroll
                for (int i = 0; i + width < W; i += 2 * width) {
                    const bool lv = i < vw, rv = i + width < vw;
                    w[i] = tree_pair(w[i], lv, w[i + width], rv);
                }
            }
            chunk[c] = w[0];
            ++nchunks;
        }
    }
    // pass-by-pass over nchunks (<= NC) values
#pragma unroll
    for (int width = 1; width < NC; width <<= 1) {
#pragma unroll
        for (int i = 0; i + width < NC; i += 2 * width) {
            const bool lv = i < nchunks, rv = i + width < nchunks;
            chunk[i] = tree_pair(chunk[i], lv, chunk[i + width], rv);
        }
    }
    if (TRAIL) __syncthreads();
    return chunk[0];
}

// Row maximum (order-free except for NaN, which fmaxf would drop: a NaN
// anywhere makes the result NaN, as the first-NaN rule of [05-OP-12] does
// for softmax, where only NaN-ness matters downstream).
template <int T, int NC, bool TRAIL = true>
__device__ __forceinline__ float block_max(const float (&v)[NC][4], int n, float *red) {
    constexpr int W = T / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = -INFINITY;
    bool nan = false;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = c * 4 * T + 4 * threadIdx.x + i;
            if (e < n) {
                m = fmaxf(m, v[c][i]);
                nan |= isnan(v[c][i]);
            }
        }
    m = warp_max(m);
    nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) red[warp] = nan ? __int_as_float(0x7fc00000) : m;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < W; ++i) {
        const float o = red[i];
        r = (isnan(r) || isnan(o)) ? __int_as_float(0x7fc00000) : fmaxf(r, o);
    }
    if (TRAIL) __syncthreads();
    return r;
}

template <int NC, int T>
__device__ __forceinline__ void load_row(float (&v)[NC][4], const float *__restrict__ row, int n,
                                         bool vec) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int e0 = c * 4 * T + 4 * threadIdx.x;
        if (vec && e0 + 3 < n) {
            const float4 q = __ldg(reinterpret_cast<const float4 *>(row + e0));
            v[c][0] = q.x;
            v[c][1] = q.y;
            v[c][2] = q.z;
            v[c][3] = q.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = (e0 + i < n) ? row[e0 + i] : 0.0f;
        }
    }
}

template <int NC, int T>
__device__ __forceinline__ void store_row(const float (&v)[NC][4], float *__restrict__ row, int n,
                                          bool vec) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int e0 = c * 4 * T + 4 * threadIdx.x;
        if (vec && e0 + 3 < n) {
            *reinterpret_cast<float4 *>(row + e0) = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (e0 + i < n) row[e0 + i] = v[c][i];
        }
    }
}

__device__ __forceinline__ float canon(float x) {
    return isnan(x) ? __int_as_float(0x7fc00000) : x;
}

// ---------------------------------------------------------------------------
// standalone row ops
// ---------------------------------------------------------------------------
// FAST-mode block sum: each thread's partial, one warp butterfly, then the
// warp partials (every thread reads them back; the caller alternates two
// scratch areas, so one barrier suffices).  Butterfly order, not the
// canonical tree: within f32 rel 1e-5 of it.
template <int T>
__device__ __forceinline__ float block_sum_fast(float v, float *red) {
    constexpr int W = T / 32;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float w[W];
#pragma unroll
    for (int i = 0; i < W; ++i) w[i] = red[i];
#pragma unroll
    for (int width = 1; width < W; width <<= 1)
#pragma unroll
        for (int i = 0; i + width < W; i += 2 * width) w[i] += w[i + width];
    return w[0];
}

template <int T, int NC, bool EXACT>
__global__ void __launch_bounds__(T, NC <= 4 ? 3 : 1)
    layer_norm_kernel(const float *__restrict__ xin, const float *__restrict__ gamma,
                      const float *__restrict__ beta, float eps, float *__restrict__ yout,
                      int64_t rows, int n) {
    __shared__ float red[2][NC * (T / 32) + 8];
    const float hf = static_cast<float>(n), rh = __fdiv_rn(1.0f, hf);
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(xin) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(yout) & 15) == 0);
    // gamma / beta in shared memory in the row layout (thread t's float4 of
    // chunk c at [c * T + t]), read back as conflict-free float4; rows of
    // 8 chunks keep them in registers (static shared memory is 48 KiB)
    constexpr bool SMEM_GB = NC <= 4;
    __shared__ float4 sg[SMEM_GB ? NC * T : 1], sb[SMEM_GB ? NC * T : 1];
    float g[SMEM_GB ? 1 : NC][4], b[SMEM_GB ? 1 : NC][4];
    if constexpr (SMEM_GB) {
        for (int e = threadIdx.x; e < NC * 4 * T; e += T) {
            reinterpret_cast<float *>(sg)[e] = e < n ? gamma[e] : 0.0f;
            reinterpret_cast<float *>(sb)[e] = e < n ? beta[e] : 0.0f;
        }
        __syncthreads();
    } else {
        load_row<NC, T>(g, gamma, n, (reinterpret_cast<uintptr_t>(gamma) & 15) == 0 && n % 4 == 0);
        load_row<NC, T>(b, beta, n, (reinterpret_cast<uintptr_t>(beta) & 15) == 0 && n % 4 == 0);
    }
    // the next row's loads are issued before this row's reductions, so each
    // CTA keeps two rows in flight
    float nxt[NC][4];
    if (blockIdx.x < rows) load_row<NC, T>(nxt, xin + blockIdx.x * static_cast<int64_t>(n), n, vec);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float v[NC][4], c2[NC][4];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = nxt[c][i];
        if (r + gridDim.x < rows) load_row<NC, T>(nxt, xin + (r + gridDim.x) * n, n, vec);
        float s1, s2, mean;
        if constexpr (EXACT) {
            s1 = block_tree<T, NC, false>(v, n, red[0]);
            mean = __fdiv_rn(s1, hf);
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[c][i] = __fsub_rn(v[c][i], mean);
                    c2[c][i] = __fmul_rn(v[c][i], v[c][i]);
                }
            s2 = block_tree<T, NC, false>(c2, n, red[1]);
        } else {
            // zeros past the row end (load_row) add nothing to the sum; the
            // squared deviations are masked to the row
            float t = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; ++c) t += (v[c][0] + v[c][1]) + (v[c][2] + v[c][3]);
            s1 = block_sum_fast<T>(t, red[0]);
            mean = __fmul_rn(s1, rh);
            float q = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    v[c][i] = __fsub_rn(v[c][i], mean);
                    const bool valid = c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n;
                    q = valid ? fmaf(v[c][i], v[c][i], q) : q;
                }
            s2 = block_sum_fast<T>(q, red[1]);
        }
        const float var = EXACT ? __fdiv_rn(s2, hf) : __fmul_rn(s2, rh);
        const float d = __fsqrt_rn(__fadd_rn(var, eps));
        const float rd = __fdiv_rn(1.0f, d);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float gg[4], bb[4];
            if constexpr (SMEM_GB) {
                const float4 g4 = sg[c * T + threadIdx.x], b4 = sb[c * T + threadIdx.x];
                gg[0] = g4.x; gg[1] = g4.y; gg[2] = g4.z; gg[3] = g4.w;
                bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) { gg[i] = g[SMEM_GB ? 0 : c][i]; bb[i] = b[SMEM_GB ? 0 : c][i]; }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float nn = EXACT ? __fdiv_rn(v[c][i], d) : __fmul_rn(v[c][i], rd);
                v[c][i] = canon(__fadd_rn(__fmul_rn(nn, gg[i]), bb[i]));
            }
        }
        store_row<NC, T>(v, yout + r * n, n, vec);
    }
}

template <int T, int NC, bool EXACT>
__global__ void __launch_bounds__(T)
    softmax_kernel(const float *__restrict__ xin, float *__restrict__ yout, int64_t rows, int n) {
    __shared__ float red[2][NC * (T / 32) + 8];
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(xin) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(yout) & 15) == 0);
    float nxt[NC][4];
    if (blockIdx.x < rows) load_row<NC, T>(nxt, xin + blockIdx.x * static_cast<int64_t>(n), n, vec);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float v[NC][4];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = nxt[c][i];
        if (r + gridDim.x < rows) load_row<NC, T>(nxt, xin + (r + gridDim.x) * n, n, vec);
        const float mx = block_max<T, NC, false>(v, n, red[0]);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float d = __fsub_rn(v[c][i], mx);
                v[c][i] = EXACT ? crmath::expf_cr(d) : expf(d);  // EXACT: CORE-MATH's bits
            }
        float z;
        if constexpr (EXACT) {
            z = block_tree<T, NC, false>(v, n, red[1]);
        } else {
            float t = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n) t += v[c][i];
            z = block_sum_fast<T>(t, red[1]);
        }
        const float rz = __fdiv_rn(1.0f, z);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[c][i] = canon(EXACT ? __fdiv_rn(v[c][i], z) : __fmul_rn(v[c][i], rz));
        store_row<NC, T>(v, yout + r * n, n, vec);
    }
}

template <int T, int NC>
__global__ void __launch_bounds__(T)
    softmax_bwd_kernel(const float *__restrict__ yin, const float *__restrict__ gin,
                       float *__restrict__ dx, int64_t rows, int n) {
    __shared__ float red[NC * (T / 32) + 8];
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(yin) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(gin) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(dx) & 15) == 0);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float y[NC][4], g[NC][4], gy[NC][4];
        load_row<NC, T>(y, yin + r * n, n, vec);
        load_row<NC, T>(g, gin + r * n, n, vec);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) gy[c][i] = __fmul_rn(g[c][i], y[c][i]);
        const float q = block_tree<T, NC>(gy, n, red);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) gy[c][i] = canon(__fmul_rn(y[c][i], __fsub_rn(g[c][i], q)));
        store_row<NC, T>(gy, dx + r * n, n, vec);
    }
}

// Row sum of a row that fits one CTA's registers (width <= NC * 4T): the
// canonical tree of block_tree (the same value as the chunked carry form
// below), float4 loads, next row prefetched.
template <int T, int NC>
__global__ void __launch_bounds__(T)
    row_sum_nc_kernel(const float *__restrict__ x, int64_t rows, int n, float *__restrict__ out) {
    __shared__ float red[2][NC * (T / 32) + 8];
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    float nxt[NC][4];
    if (blockIdx.x < rows) load_row<NC, T>(nxt, x + blockIdx.x * static_cast<int64_t>(n), n, vec);
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float v[NC][4];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = nxt[c][i];
        if (r + gridDim.x < rows) load_row<NC, T>(nxt, x + (r + gridDim.x) * n, n, vec);
        const float s = block_tree<T, NC, false>(v, n, red[((r - blockIdx.x) / gridDim.x) & 1]);
        if (threadIdx.x == 0) out[r] = canon(s);
    }
}

// Row sum of arbitrary width: chunk subtrees of 4T leaves, chunk sums
// pushed by thread 0 into a carry tree (the C lane's streaming form).
template <int T>
__global__ void __launch_bounds__(T)
    row_sum_kernel(const float *__restrict__ x, int64_t rows, int64_t cols,
                   float *__restrict__ out) {
    __shared__ float red[T / 32 + 8];
    float level[40];
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *row = x + r * cols;
        int64_t count = 0;
        for (int64_t c0 = 0; c0 < cols; c0 += 4 * T) {
            float v[1][4];
            const int64_t rem = cols - c0;
            const int nvalid = rem < 4 * T ? static_cast<int>(rem) : 4 * T;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int e = 4 * threadIdx.x + i;
                v[0][i] = e < nvalid ? row[c0 + e] : 0.0f;
            }
            const float s = block_tree<T, 1>(v, nvalid, red);
            if (threadIdx.x == 0) {
                float carry = s;
                int depth = 0;
                for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)
                    carry = __fadd_rn(level[depth], carry);
                level[depth] = carry;
            }
        }
        if (threadIdx.x == 0) {
            float total = 0.0f;
            bool found = false;
            int depth = 0;
            for (int64_t remaining = count; remaining; remaining >>= 1, ++depth) {
                if (remaining & 1) {
                    total = found ? __fadd_rn(level[depth], total) : level[depth];
                    found = true;
                }
            }
            out[r] = canon(total);
        }
    }
}

// [05-OP-12]: first NaN (with its payload) wins, else the maximum with the
// first representation among equals.  One warp per row.
__global__ void row_max_kernel(const float *__restrict__ x, int64_t rows, int64_t cols,
                               float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows;
         r += warps) {
        const float *row = x + r * cols;
        float best = 0.0f;
        int64_t bi = INT64_MAX;  // index of the selected element
        for (int64_t j = lane; j < cols; j += 32) {
            const float v = row[j];
            bool take;
            if (bi == INT64_MAX) take = true;
            else if (isnan(best)) take = false;  // an earlier NaN stays
            else if (isnan(v)) take = true;
            else take = v > best;
            if (take) { best = v; bi = j; }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, off);
            bool take;
            if (oi == INT64_MAX) take = false;
            else if (bi == INT64_MAX) take = true;
            else if (isnan(best) || isnan(ob)) {
                take = isnan(ob) && (!isnan(best) || oi < bi);
            } else if (ob > best) take = true;
            else if (ob == best) take = oi < bi;
            else take = false;
            if (take) { best = ob; bi = oi; }
        }
        if (lane == 0) out[r] = best;
    }
}

// The same selection with float4 loads and 32-bit indices, for rows whose
// width is a multiple of 4 (< 2^31) in a 16-byte aligned matrix: lane l scans
// the quads l, l + 32, l + 64, ... of its row, so indices still increase
// along a lane, with four quads in flight.  Within a lane an element
// replaces the candidate iff the candidate is not NaN and the element is NaN
// or strictly greater (the first NaN, else the first of equal maxima, stays);
// lanes merge by the rule of row_max_kernel.
__device__ __forceinline__ void max_take(float v, int j, float &best, int &bi) {
    const bool take = !isnan(best) && (isnan(v) || v > best);
    best = take ? v : best;
    bi = take ? j : bi;
}
__global__ void row_max4_kernel(const float *__restrict__ x, int64_t rows, int cols,
                                float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int nq = cols >> 2;
    for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows;
         r += warps) {
        const float4 *row = reinterpret_cast<const float4 *>(x + r * cols);
        float best = 0.0f;
        int bi = INT_MAX;
        int k = lane;
        if (k < nq) {
            const float4 a = __ldcs(row + k);
            best = a.x;
            bi = 4 * k;
            max_take(a.y, 4 * k + 1, best, bi);
            max_take(a.z, 4 * k + 2, best, bi);
            max_take(a.w, 4 * k + 3, best, bi);
            k += 32;
        }
        for (; k + 96 < nq; k += 128) {
            float4 a[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) a[u] = __ldcs(row + k + 32 * u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = 4 * (k + 32 * u);
                max_take(a[u].x, j, best, bi);
                max_take(a[u].y, j + 1, best, bi);
                max_take(a[u].z, j + 2, best, bi);
                max_take(a[u].w, j + 3, best, bi);
            }
        }
        for (; k < nq; k += 32) {
            const float4 a = __ldcs(row + k);
            max_take(a.x, 4 * k, best, bi);
            max_take(a.y, 4 * k + 1, best, bi);
            max_take(a.z, 4 * k + 2, best, bi);
            max_take(a.w, 4 * k + 3, best, bi);
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            bool take;
            if (oi == INT_MAX) take = false;
            else if (bi == INT_MAX) take = true;
            else if (isnan(best) || isnan(ob)) {
                take = isnan(ob) && (!isnan(best) || oi < bi);
            } else if (ob > best) take = true;
            else if (ob == best) take = oi < bi;
            else take = false;
            if (take) { best = ob; bi = oi; }
        }
        if (lane == 0) out[r] = best;
    }
}

// Column sums (axis 0) of [rows, cols]: aligned row blocks of RB leaves
// (complete subtrees of the canonical tree over rows) reduced per column
// with a register carry tree, then the block sums reduced the same way by a
// second launch.  A partial last block is the tree over its prefix.
constexpr int COL_RB = 64;
__global__ void col_block_kernel(const float *__restrict__ x, int64_t rows, int64_t cols,
                                 int64_t rb, float *__restrict__ out) {
    const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t blk = blockIdx.y;
    if (col >= cols) return;
    const int64_t r0 = blk * rb;
    int64_t r1 = r0 + rb;
    if (r1 > rows) r1 = rows;
    float level[40];
    int64_t count = 0;
    for (int64_t r = r0; r < r1; ++r) {
        float carry = x[r * cols + col];
        int depth = 0;
        for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth)
            carry = __fadd_rn(level[depth], carry);
        level[depth] = carry;
    }
    float total = 0.0f;
    bool found = false;
    int depth = 0;
    for (int64_t remaining = count; remaining; remaining >>= 1, ++depth) {
        if (remaining & 1) {
            total = found ? __fadd_rn(level[depth], total) : level[depth];
            found = true;
        }
    }
    out[blk * cols + col] = total;
}

// Full aligned blocks of COL_RB = 64 rows, four columns per thread: the
// canonical tree over 64 leaves is the balanced binary tree, taken here as
// four 16-row subtrees reduced pairwise in registers ((s0 + s1) + (s2 + s3)),
// so the loads are float4 and independent.  Same values as col_block_kernel.
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                       __fadd_rn(a.w, b.w));
}
// RB = 32 takes two 16-row subtrees: twice the blocks for the same matrix,
// so the last wave of the grid leaves fewer SMs idle.
template <int RB>
__global__ void col_block4_kernel(const float *__restrict__ x, int64_t cols, float *__restrict__ out) {
    constexpr int Q = RB / 16;
    const int64_t c4 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // float4 column
    if (c4 * 4 >= cols) return;
    const int64_t blk = blockIdx.y;
    const float4 *src = reinterpret_cast<const float4 *>(x + blk * RB * cols) + c4;
    const int64_t stride = cols / 4;
    float4 sub[Q];
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __ldcs(src + (q * 16 + i) * stride);
#pragma unroll
        for (int width = 1; width < 16; width <<= 1)
#pragma unroll
            for (int i = 0; i + width < 16; i += 2 * width) v[i] = add4(v[i], v[i + width]);
        sub[q] = v[0];
    }
    if constexpr (Q == 4)
        reinterpret_cast<float4 *>(out + blk * cols)[c4] = add4(add4(sub[0], sub[1]), add4(sub[2], sub[3]));
    else
        reinterpret_cast<float4 *>(out + blk * cols)[c4] = add4(sub[0], sub[1]);
}

// ---------------------------------------------------------------------------
// dropout, count, cumsum
// ---------------------------------------------------------------------------
__global__ void dropout_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t n,
                               uint64_t key, uint64_t threshold, float den, int64_t index_base) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool keep = dropout_keep(key, static_cast<uint64_t>(index_base + i), threshold);
        y[i] = keep ? canon(__fdiv_rn(x[i], den)) : 0.0f;
    }
}

// Four consecutive elements per thread step (float4 in and out, four
// independent keyed-RNG chains in flight); elements past the last full
// quad go through dropout_kernel.
__global__ void dropout4_kernel(const float4 *__restrict__ x, float4 *__restrict__ y, int64_t n4,
                                uint64_t key, uint64_t threshold, float den, int64_t index_base) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 v = __ldcs(x + i);
        const uint64_t e = static_cast<uint64_t>(index_base + 4 * i);
        const bool k0 = dropout_keep(key, e, threshold), k1 = dropout_keep(key, e + 1, threshold);
        const bool k2 = dropout_keep(key, e + 2, threshold), k3 = dropout_keep(key, e + 3, threshold);
        __stcs(y + i, make_float4(k0 ? canon(__fdiv_rn(v.x, den)) : 0.0f,
                                  k1 ? canon(__fdiv_rn(v.y, den)) : 0.0f,
                                  k2 ? canon(__fdiv_rn(v.z, den)) : 0.0f,
                                  k3 ? canon(__fdiv_rn(v.w, den)) : 0.0f));
    }
}

__global__ void dropout_mask_kernel(uint8_t *__restrict__ keep, int64_t n, uint64_t key,
                                    uint64_t threshold, int64_t index_base) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        keep[i] = dropout_keep(key, static_cast<uint64_t>(index_base + i), threshold) ? 1 : 0;
}

__global__ void count_kernel(const uint8_t *__restrict__ x, int64_t n,
                             unsigned long long *__restrict__ out) {
    unsigned long long c = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        c += x[i] ? 1ull : 0ull;
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if ((threadIdx.x & 31) == 0) atomicAdd(out, c);
}

// Sequential scan per lane ([05-OP-53]): 4 warps per CTA, a warp owns 32
// lanes; each 32-step
// slab of the 32 lanes is staged through shared memory so the global reads
// and writes stay coalesced while each thread scans its own lane in order.
template <typename V>
__global__ void cumsum_kernel(const V *__restrict__ x, V *__restrict__ y, int64_t lanes,
                              int64_t len, int reverse) {
    __shared__ V tile[4][32][33];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t lane0 = (static_cast<int64_t>(blockIdx.x) * 4 + w) * 32;
    if (lane0 >= lanes) return;
    V acc = V(0);
    bool first = true;
    const int64_t nslab = (len + 31) / 32;
    for (int64_t sb = 0; sb < nslab; ++sb) {
        const int64_t slab = reverse ? (nslab - 1 - sb) : sb;
        const int64_t t0 = slab * 32;
        // stage: row i of the tile = lane (lane0 + i), columns t0..t0+31
        for (int i = 0; i < 32; ++i) {
            const int64_t l = lane0 + i, t = t0 + lane;
            tile[w][i][lane] = (l < lanes && t < len) ? x[l * len + t] : V(0);
        }
        __syncwarp();
        const int64_t my = lane0 + lane;
        const int cnt = static_cast<int>((len - t0) < 32 ? (len - t0) : 32);
        for (int jj = 0; jj < cnt; ++jj) {
            const int j = reverse ? (cnt - 1 - jj) : jj;
            const V v = tile[w][lane][j];
            acc = first ? v : acc + v;
            first = false;
            tile[w][lane][j] = isnan(acc) ? V(NAN) : acc;
        }
        __syncwarp();
        for (int i = 0; i < 32; ++i) {
            const int64_t l = lane0 + i, t = t0 + lane;
            if (l < lanes && t < len) y[l * len + t] = tile[w][i][lane];
        }
        __syncwarp();
        (void)my;
    }
}

}  // namespace rows

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

// Least 53-bit integer u whose f32 rounding reaches rate * 2^53, so that
// keep <=> (word >> 11) >= u reproduces round_f32(unit) >= rate exactly
// (PreparedDropout::apply, dtype_semantics.rs:4265-4277).
uint64_t dropout_threshold(float rate) {
    const double target = static_cast<double>(rate) * 9007199254740992.0;  // exact
    uint64_t lo = 0, hi = 1ull << 53;  // answer in [lo, hi]
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        const float f = static_cast<float>(mid);  // RN to f32 of an exact integer
        if (static_cast<double>(f) >= target) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

namespace {

int check_rate(float rate) {
    if (!(rate >= 0.0f && rate < 1.0f))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in dropout at f32");
    return CHELIS_CUDA_OK;
}

template <typename F>
int dispatch_nc(int hidden, int threads, F &&f) {
    const int per = 4 * threads;
    const int nc = (hidden + per - 1) / per;
    if (nc <= 1) return f(std::integral_constant<int, 1>());
    if (nc <= 2) return f(std::integral_constant<int, 2>());
    if (nc <= 4) return f(std::integral_constant<int, 4>());
    if (nc <= 8) return f(std::integral_constant<int, 8>());
    return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "row width %d beyond %d", hidden, 8 * per);
}

int rows_grid(int64_t rows, int per_sm) {
    int64_t g = static_cast<int64_t>(sm_count()) * per_sm;
    if (rows < g) g = rows;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

int col_sum_into(const float *x, int64_t rows, int64_t cols, float *out, cudaStream_t s);

}  // namespace chelis

using namespace chelis;
using namespace chelis::rows;

namespace chelis {

// Canonical column sums of a [rows, cols] matrix into out[cols] (aligned
// row blocks reduced level by level; one scratch buffer of ceil(rows/rb) *
// cols floats per level when rows > 64).
int col_sum_into(const float *x, int64_t rows, int64_t cols, float *out, cudaStream_t s) {
    if (cols == 0) return CHELIS_CUDA_OK;
    if (rows == 0)
        return check_cuda(cudaMemsetAsync(out, 0, cols * sizeof(float), s), "cudaMemsetAsync");
    const unsigned cb = static_cast<unsigned>((cols + 127) / 128);
    if (rows <= COL_RB) {
        col_block_kernel<<<dim3(cb, 1), 128, 0, s>>>(x, rows, cols, rows, out);
        g_launches++;
        CHELIS_LAUNCH_CHECK("col_block_kernel");
        return CHELIS_CUDA_OK;
    }
    // aligned row blocks of rb rows (any aligned power-of-two block is a
    // subtree of the canonical tree): 32 on the float4 path, 64 otherwise
    const bool v4 = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int64_t rb = v4 ? 32 : COL_RB;
    const int64_t nb = (rows + rb - 1) / rb;
    void *tmp = nullptr;
    CHELIS_TRY(scratch_alloc(&tmp, static_cast<size_t>(nb * cols) * sizeof(float), s));
    float *blk = static_cast<float *>(tmp);
    int st;
    const int64_t nfull = rows / rb;
    if (v4 && nfull > 0 && nfull <= 65535) {
        // full blocks with float4 columns, the ragged last block (if any) below
        const unsigned cb4 = static_cast<unsigned>((cols / 4 + 127) / 128);
        col_block4_kernel<32><<<dim3(cb4, static_cast<unsigned>(nfull)), 128, 0, s>>>(x, cols, blk);
        g_launches++;
        st = check_cuda(cudaGetLastError(), "col_block4_kernel");
        if (st == CHELIS_CUDA_OK && nb > nfull) {
            col_block_kernel<<<dim3(cb, 1), 128, 0, s>>>(x + nfull * rb * cols, rows - nfull * rb,
                                                         cols, rb, blk + nfull * cols);
            g_launches++;
            st = check_cuda(cudaGetLastError(), "col_block_kernel");
        }
    } else {
        col_block_kernel<<<dim3(cb, static_cast<unsigned>(nb)), 128, 0, s>>>(x, rows, cols, rb, blk);
        g_launches++;
        st = check_cuda(cudaGetLastError(), "col_block_kernel");
    }
    if (st == CHELIS_CUDA_OK) st = col_sum_into(static_cast<float *>(tmp), nb, cols, out, s);
    scratch_free(tmp, s);
    return st;
}

}  // namespace chelis

namespace {
constexpr int kRowThreads = 256;

// wide_ok: the op has a path for rows wider than the register-resident kernels
int check_rows_args(const void *x, int64_t rows, int64_t hidden, bool wide_ok = false) {
    if (rows < 0 || hidden < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in rows at i64");
    if ((!wide_ok && hidden > 8 * 4 * kRowThreads) || hidden > INT32_MAX)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "row width %lld beyond %d",
                         static_cast<long long>(hidden), 8 * 4 * kRowThreads);
    (void)x;
    return CHELIS_CUDA_OK;
}
}  // namespace

extern "C" {

int chelis_cuda_layer_norm_f32(const float *x, const float *gamma, const float *beta, float eps,
                               float *y, int64_t rows, int64_t hidden) {
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    if (hidden == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    if (rows == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    const int n = static_cast<int>(hidden);
    const unsigned grid = static_cast<unsigned>(rows_grid(rows, 8));
    return dispatch_nc(n, kRowThreads, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        if (exact) layer_norm_kernel<kRowThreads, NC, true><<<grid, kRowThreads, 0, s>>>(x, gamma, beta, eps, y, rows, n);
        else layer_norm_kernel<kRowThreads, NC, false><<<grid, kRowThreads, 0, s>>>(x, gamma, beta, eps, y, rows, n);
        g_launches++;
        CHELIS_LAUNCH_CHECK("layer_norm_kernel");
        return CHELIS_CUDA_OK;
    });
}

}  // extern "C"

namespace chelis {
namespace {

// Rows wider than the register-resident kernels take (8192): the softmax
// lowering (max -> sub -> exp -> sum -> div, tier2.rs:1079-1180) and its
// adjoint y * (g - sum(g * y)) as FusedElem groups over the row, with the
// per-row max / sums broadcast back (stride 0 along the row).
int softmax_rows_wide(const float *x, const float *g, float *out, int64_t rows, int64_t cols,
                      cudaStream_t s) {
    void *scratch = nullptr;
    CHELIS_TRY(scratch_alloc(&scratch, 2 * static_cast<size_t>(rows) * sizeof(float), s));
    float *r1 = static_cast<float *>(scratch), *r2 = r1 + rows;
    const int64_t shape[2] = {rows, cols};
    const int64_t dense[2] = {cols, 1};
    int rc;
    if (!g) {  // forward: out = softmax(x)
        const chelis_fused_step ident[1] = {{CHELIS_FUSED_MAX_ELEM, 0, 0}};
        const chelis_fused_step shift_exp[2] = {{CHELIS_FUSED_SUB, 0, 1}, {CHELIS_FUSED_EXP, -1, -1}};
        const chelis_fused_step divide[1] = {{CHELIS_FUSED_DIV, 0, 1}};
        const void *in_x[1] = {x};
        rc = chelis_cuda_fused_reduce(CHELIS_DTYPE_F32, ident, 1, in_x, dense, 1, shape, 2, 1,
                                      CHELIS_FUSED_REDUCE_MAX, r1);
        const void *in_xm[2] = {x, r1};
        const int64_t st_xm[4] = {cols, 1, 1, 0};
        if (rc == CHELIS_CUDA_OK)
            rc = chelis_cuda_fused_elementwise(CHELIS_DTYPE_F32, shift_exp, 2, in_xm, st_xm, 2, shape, 2, out);
        const void *in_e[1] = {out};
        if (rc == CHELIS_CUDA_OK)
            rc = chelis_cuda_fused_reduce(CHELIS_DTYPE_F32, ident, 1, in_e, dense, 1, shape, 2, 1,
                                          CHELIS_FUSED_REDUCE_SUM, r2);
        const void *in_ez[2] = {out, r2};
        if (rc == CHELIS_CUDA_OK)
            rc = chelis_cuda_fused_elementwise(CHELIS_DTYPE_F32, divide, 1, in_ez, st_xm, 2, shape, 2, out);
    } else {  // adjoint: out = x * (g - sum(g * x)), x the softmax output
        const chelis_fused_step prod[1] = {{CHELIS_FUSED_MUL, 0, 1}};
        const chelis_fused_step grad[2] = {{CHELIS_FUSED_SUB, 0, 2}, {CHELIS_FUSED_MUL, 1, -1}};
        const void *in_gy[2] = {g, x};
        const int64_t st_gy[4] = {cols, 1, cols, 1};
        rc = chelis_cuda_fused_reduce(CHELIS_DTYPE_F32, prod, 1, in_gy, st_gy, 2, shape, 2, 1,
                                      CHELIS_FUSED_REDUCE_SUM, r1);
        const void *in_gyq[3] = {g, x, r1};
        const int64_t st_gyq[6] = {cols, 1, cols, 1, 1, 0};
        if (rc == CHELIS_CUDA_OK)
            rc = chelis_cuda_fused_elementwise(CHELIS_DTYPE_F32, grad, 2, in_gyq, st_gyq, 3, shape, 2, out);
    }
    scratch_free(scratch, s);
    return rc;
}

}  // namespace
}  // namespace chelis

extern "C" {

int chelis_cuda_softmax_rows_f32(const float *x, float *y, int64_t rows, int64_t cols) {
    CHELIS_TRY(check_rows_args(x, rows, cols, true));
    if (rows == 0 || cols == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (cols > 8 * 4 * kRowThreads) return softmax_rows_wide(x, nullptr, y, rows, cols, s);
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    const int n = static_cast<int>(cols);
    const unsigned grid = static_cast<unsigned>(rows_grid(rows, 8));
    return dispatch_nc(n, kRowThreads, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        if (exact) softmax_kernel<kRowThreads, NC, true><<<grid, kRowThreads, 0, s>>>(x, y, rows, n);
        else softmax_kernel<kRowThreads, NC, false><<<grid, kRowThreads, 0, s>>>(x, y, rows, n);
        g_launches++;
        CHELIS_LAUNCH_CHECK("softmax_kernel");
        return CHELIS_CUDA_OK;
    });
}

int chelis_cuda_softmax_rows_bwd_f32(const float *y, const float *g, float *dx, int64_t rows,
                                     int64_t cols) {
    CHELIS_TRY(check_rows_args(y, rows, cols, true));
    if (rows == 0 || cols == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (cols > 8 * 4 * kRowThreads) return softmax_rows_wide(y, g, dx, rows, cols, s);
    const int n = static_cast<int>(cols);
    const unsigned grid = static_cast<unsigned>(rows_grid(rows, 8));
    return dispatch_nc(n, kRowThreads, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        softmax_bwd_kernel<kRowThreads, NC><<<grid, kRowThreads, 0, s>>>(y, g, dx, rows, n);
        g_launches++;
        CHELIS_LAUNCH_CHECK("softmax_bwd_kernel");
        return CHELIS_CUDA_OK;
    });
}

int chelis_cuda_row_sum_f32(const float *x, int64_t rows, int64_t cols, float *out) {
    if (rows < 0 || cols < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in sum at i64");
    if (rows == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    if (cols == 0) return check_cuda(cudaMemsetAsync(out, 0, rows * sizeof(float), s), "memset");
    const unsigned grid = static_cast<unsigned>(rows_grid(rows, 8));
    if (cols <= 8 * 4 * kRowThreads) {
        const int n = static_cast<int>(cols);
        return dispatch_nc(n, kRowThreads, [&](auto ncv) -> int {
            constexpr int NC = decltype(ncv)::value;
            row_sum_nc_kernel<kRowThreads, NC><<<grid, kRowThreads, 0, s>>>(x, rows, n, out);
            g_launches++;
            CHELIS_LAUNCH_CHECK("row_sum_nc_kernel");
            return CHELIS_CUDA_OK;
        });
    }
    row_sum_kernel<256><<<grid, 256, 0, s>>>(x, rows, cols, out);
    g_launches++;
    CHELIS_LAUNCH_CHECK("row_sum_kernel");
    return CHELIS_CUDA_OK;
}

int chelis_cuda_col_sum_f32(const float *x, int64_t rows, int64_t cols, float *out) {
    if (rows < 0 || cols < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in sum at i64");
    return col_sum_into(x, rows, cols, out, current_stream());
}

int chelis_cuda_row_max_f32(const float *x, int64_t rows, int64_t cols, float *out) {
    if (rows < 0 || cols < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in max_reduce at i64");
    if (rows == 0) return CHELIS_CUDA_OK;
    if (cols == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in max_reduce at f32");
    cudaStream_t s = current_stream();
    int64_t blocks = (rows * 32 + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (cols % 4 == 0 && cols < INT_MAX && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        row_max4_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, rows, static_cast<int>(cols), out);
        g_launches++;
        CHELIS_LAUNCH_CHECK("row_max4_kernel");
        return CHELIS_CUDA_OK;
    }
    row_max_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, rows, cols, out);
    g_launches++;
    CHELIS_LAUNCH_CHECK("row_max_kernel");
    return CHELIS_CUDA_OK;
}

int chelis_cuda_count_bool(const uint8_t *x, int64_t n, int64_t *out_device) {
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in count at i64");
    cudaStream_t s = current_stream();
    CHELIS_TRY(check_cuda(cudaMemsetAsync(out_device, 0, sizeof(int64_t), s), "memset"));
    if (n == 0) return CHELIS_CUDA_OK;
    int64_t blocks = (n + 1023) / 1024;
    if (blocks > 148 * 8) blocks = 148 * 8;
    count_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        x, n, reinterpret_cast<unsigned long long *>(out_device));
    g_launches++;
    CHELIS_LAUNCH_CHECK("count_kernel");
    return CHELIS_CUDA_OK;
}

int chelis_cuda_dropout_f32(const float *x, float *y, int64_t n, uint64_t key, float rate,
                            int64_t index_base) {
    CHELIS_TRY(check_rate(rate));
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in dropout at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    volatile float one = 1.0f;
    const float den = one - rate;
    const uint64_t thr = dropout_threshold(rate);
    const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
    int64_t done = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
        n >= 4) {
        const int64_t n4 = n / 4;
        int64_t blocks = (n4 + 255) / 256;
        if (blocks > cap) blocks = cap;
        dropout4_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
            reinterpret_cast<const float4 *>(x), reinterpret_cast<float4 *>(y), n4, key, thr, den,
            index_base);
        g_launches++;
        CHELIS_LAUNCH_CHECK("dropout4_kernel");
        done = 4 * n4;
    }
    if (done < n) {
        int64_t blocks = (n - done + 255) / 256;
        if (blocks > cap) blocks = cap;
        dropout_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x + done, y + done, n - done, key,
                                                                   thr, den, index_base + done);
        g_launches++;
        CHELIS_LAUNCH_CHECK("dropout_kernel");
    }
    return CHELIS_CUDA_OK;
}

int chelis_cuda_dropout_mask(uint8_t *keep, int64_t n, uint64_t key, float rate,
                             int64_t index_base) {
    CHELIS_TRY(check_rate(rate));
    if (n < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in dropout at i64");
    if (n == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    dropout_mask_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        keep, n, key, dropout_threshold(rate), index_base);
    g_launches++;
    CHELIS_LAUNCH_CHECK("dropout_mask_kernel");
    return CHELIS_CUDA_OK;
}

int chelis_cuda_cumsum_f64(const double *x, double *y, int64_t lanes, int64_t len, int reverse) {
    if (lanes < 0 || len < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in cumsum at i64");
    if (lanes == 0 || len == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    const unsigned grid = static_cast<unsigned>((lanes + 127) / 128);
    cumsum_kernel<double><<<grid, 128, 0, s>>>(x, y, lanes, len, reverse);
    g_launches++;
    CHELIS_LAUNCH_CHECK("cumsum_kernel<f64>");
    return CHELIS_CUDA_OK;
}

int chelis_cuda_cumsum_f32(const float *x, float *y, int64_t lanes, int64_t len, int reverse) {
    if (lanes < 0 || len < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in cumsum at i64");
    if (lanes == 0 || len == 0) return CHELIS_CUDA_OK;
    cudaStream_t s = current_stream();
    const unsigned grid = static_cast<unsigned>((lanes + 127) / 128);
    cumsum_kernel<float><<<grid, 128, 0, s>>>(x, y, lanes, len, reverse);
    g_launches++;
    CHELIS_LAUNCH_CHECK("cumsum_kernel<f32>");
    return CHELIS_CUDA_OK;
}

}  // extern "C"
