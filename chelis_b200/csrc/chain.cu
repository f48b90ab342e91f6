// chain.cu -- the fused chain layer_norm -> softmax -> keyed dropout -> row
// sum over a [rows, hidden] f32 tensor, and its reverse-mode adjoint for
// loss = sum(rowsum), following the adjoint graphs of
// crates/chelis-dag-core/src/grad.rs (Sum -> Expand :2586, Dropout ->
// DropoutReplay :2515-2525, Softmax :2248-2280, Mul :1934-1942, Div
// :1943-1961, Sqrt :2342-2355) with the fan-in order of
// balanced_adjoint_sum (:1713-1745).
//
// One CTA of T threads owns one row at a time (the rows.cu layout: chunks of
// 4T elements, thread t holds [4t, 4t+4) of each).  In EXACT mode every row
// sum is the canonical adjacent-pair tree, bit for bit.  The forward can save, per row,
// its statistics (mean, sqrt(var+eps), softmax max and denominator) and the
// keyed-dropout keep bits (one bit per element, warp-ballot packed), so the
// adjoint re-derives nothing that needs a reduction or the RNG.
//
// Shared memory holds gamma / beta in the same chunk layout, accessed as
// float4 so a warp's access is conflict-free; the adjoint keeps its dgamma /
// dbeta partials in registers (a thread owns the same columns in every row).  Block reductions alternate between two scratch areas,
// so each costs one barrier.
//
// Modes: EXACT divides where the C lane divides (IEEE __fdiv_rn) and uses
// CUDA's expf, following the adjoint graph step by step; FAST multiplies by
// per-row reciprocals, uses __expf (ex2.approx), reduces in butterfly order,
// folds the row sum into the softmax denominator's reduction (four block
// reductions per forward row instead of five) and runs the adjoint in its
// closed form (two reductions instead of three); both stay within f32 rel
// 1e-5 of the oracle.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "crmath.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int rows_mode();
uint64_t dropout_threshold(float rate);
int col_sum_into(const float *x, int64_t rows, int64_t cols, float *out, cudaStream_t s);

namespace chain {

// canonical tree of a thread's 4 leaves of one chunk; `cnt` of them valid
__device__ __forceinline__ float quad(float a, float b, float c, float d, int cnt) {
    if (cnt >= 4) return __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d));
    const float s01 = tree_pair(a, cnt > 0, b, cnt > 1);
    const float s23 = tree_pair(c, cnt > 2, d, cnt > 3);
    return tree_pair(s01, cnt > 0, s23, cnt > 2);
}

// Leaves of chunk c this thread holds (4 unless the row ends inside its
// quad); FULL rows (hidden == NC * 4 * T) need no bounds arithmetic.
template <bool FULL, int T>
__device__ __forceinline__ int lanes_left(int n, int c) {
    return FULL ? 4 : n - (c * 4 * T + 4 * static_cast<int>(threadIdx.x));
}

// Two reduction scratch areas used alternately: a reduction writes its warp
// partials into one area, synchronises once and reads them back; the next
// reduction uses the other area, so no thread can overwrite partials that a
// slower thread of the previous reduction is still reading.
template <int T, int NC>
struct Red {
    float *base;
    int flip = 0;
    __device__ float *next() {
        float *r = base + flip * (NC * (T / 32) + 8);
        flip ^= 1;
        return r;
    }
};

// Warp butterfly of NC values per lane that halves the values each lane
// carries at every level: at lane bit `off` a lane keeps the lower (bit
// clear) or upper (bit set) half of its values and adds its partner's copy
// of that half.  Every value still follows the xor butterfly (adjacent lane
// pairs first), so each chunk's warp sum is bit-identical to a butterfly of
// that chunk alone, with log2(NC) + ... fewer shuffles.  Returns the warp
// sum of chunk `chunk` (held by the lane; lanes 0..NC-1 hold distinct
// chunks).
template <int NC>
__device__ __forceinline__ float warp_tree_multi(float (&v)[NC], int lane, int &chunk) {
    chunk = 0;
    int off = 1;
#pragma unroll
    for (int cnt = NC; cnt > 1; cnt >>= 1, off <<= 1) {
        const bool bit = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < cnt / 2; ++j) {
            const float send = bit ? v[j] : v[j + cnt / 2];
            const float keep = bit ? v[j + cnt / 2] : v[j];
            v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
        }
        if (bit) chunk += cnt / 2;
    }
    float s = v[0];
#pragma unroll
    for (; off < 32; off <<= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    return s;
}

// Reduce per-chunk thread partials part[c] (the subtree of this thread's
// leaves of chunk c) to the canonical total over n leaves.  Every thread
// returns the total.
template <int T, int NC>
__device__ __forceinline__ float tree_parts(const float (&part)[NC], int n, Red<T, NC> &rs) {
    constexpr int W = T / 32;
    float *red = rs.next();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool full = (n == NC * 4 * T);
    if (full) {
        float v[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) v[c] = part[c];
        int chunk;
        const float s = warp_tree_multi<NC>(v, lane, chunk);
        if (lane < NC) red[chunk * W + warp] = s;
        __syncthreads();
        // lane c < NC of every warp: tree over the W warp sums of chunk c,
        // then the chunk sums pairwise across lanes (chunk c sits in lane c)
        float t = 0.0f;
        if (lane < NC) {
            float w[W];
#pragma unroll
            for (int i = 0; i < W; ++i) w[i] = red[lane * W + i];
#pragma unroll
            for (int width = 1; width < W; width <<= 1)
#pragma unroll
                for (int i = 0; i + width < W; i += 2 * width) w[i] = __fadd_rn(w[i], w[i + width]);
            t = w[0];
        }
#pragma unroll
        for (int off = 1; off < NC; off <<= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
        return __shfl_sync(0xffffffffu, t, 0);
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        float s = part[c];
        if (full) {
            s = warp_tree_full(s);
        } else {
            bool valid = (n - (c * 4 * T + 4 * static_cast<int>(threadIdx.x))) > 0;
            s = warp_tree(s, valid);
        }
        if (lane == 0) red[c * W + warp] = s;
    }
    __syncthreads();
    float chunk[NC];
    int nchunks = 0;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int c0 = c * 4 * T;
        if (c0 < n) {
            float w[W];
#pragma unroll
            for (int i = 0; i < W; ++i) w[i] = red[c * W + i];
            int vw = (n - c0 + 127) / 128;
            if (vw > W) vw = W;
#pragma unroll
            for (int width = 1; width < W; width <<= 1)
#pragma unroll
                for (int i = 0; i + width < W; i += 2 * width)
                    w[i] = tree_pair(w[i], i < vw, w[i + width], i + width < vw);
            chunk[c] = w[0];
            ++nchunks;
        }
    }
#pragma unroll
    for (int width = 1; width < NC; width <<= 1)
#pragma unroll
        for (int i = 0; i + width < NC; i += 2 * width)
            chunk[i] = tree_pair(chunk[i], i < nchunks, chunk[i + width], i + width < nchunks);
    return chunk[0];
}

template <int T, int NC, bool FULL = false>
__device__ __forceinline__ float tree4(const float (&v)[NC][4], int n, Red<T, NC> &rs) {
    float part[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c)
        part[c] = quad(v[c][0], v[c][1], v[c][2], v[c][3], lanes_left<FULL, T>(n, c));
    return tree_parts<T, NC>(part, FULL ? NC * 4 * T : n, rs);
}

template <int T, int NC, bool FULL = false>
__device__ __forceinline__ float row_max(const float (&v)[NC][4], int n, Red<T, NC> &rs) {
    constexpr int W = T / 32;
    float *red = rs.next();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = -INFINITY;
    bool nan = false;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (FULL || c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n) {
                m = fmaxf(m, v[c][i]);
                nan |= isnan(v[c][i]);
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
    return r;
}

// EXACT: the correctly rounded exp (CORE-MATH's results, as the C lane);
// FAST: the MUFU approximation
template <bool EXACT>
__device__ __forceinline__ float exp_(float x) {
    return EXACT ? crmath::expf_cr(x) : __expf(x);
}
template <bool EXACT>
__device__ __forceinline__ float div_(float a, float b, float rb) {
    return EXACT ? __fdiv_rn(a, b) : __fmul_rn(a, rb);
}
__device__ __forceinline__ float canon(float x) { return isnan(x) ? __int_as_float(0x7fc00000) : x; }

struct Params {
    const float *x, *gamma, *beta;
    float eps;
    uint64_t key, threshold;
    float den, rden, one_over_den;
    float hf, rh;
    int64_t rows;
    int hidden;
    int64_t index_base;
    int words_per_row;        // keep-bit words per row = NC * T / 8
    float *rowsum;            // fwd out
    float *stats;             // fwd out [rows][4] (optional)
    uint32_t *keep_out;       // fwd out [rows][words_per_row] (optional)
    const float *stats_in;    // bwd in (optional)
    const uint32_t *keep_in;  // bwd in (optional)
    float *dx;
    float *dgamma_part, *dbeta_part;  // [grid][hidden]
    int rows_per_cta;
};

template <int NC, int T>
__device__ __forceinline__ void load4(float (&v)[NC][4], const float *__restrict__ row, int n, bool vec) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int e0 = c * 4 * T + 4 * threadIdx.x;
        if (vec && e0 + 3 < n) {
            const float4 q = __ldcs(reinterpret_cast<const float4 *>(row + e0));
            v[c][0] = q.x; v[c][1] = q.y; v[c][2] = q.z; v[c][3] = q.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = (e0 + i < n) ? row[e0 + i] : 0.0f;
        }
    }
}

// stage a row-shaped vector (or zeros) into shared memory: sm[c*4T + 4t + i]
template <int NC, int T>
__device__ __forceinline__ void stage(float *sm, const float *__restrict__ src, int n) {
    for (int e = threadIdx.x; e < NC * 4 * T; e += T) sm[e] = (src && e < n) ? src[e] : 0.0f;
}
template <int T>
__device__ __forceinline__ float4 ld4(const float *sm, int c) {
    return reinterpret_cast<const float4 *>(sm)[c * T + threadIdx.x];
}
__device__ __forceinline__ float at(const float4 &q, int i) {
    return i == 0 ? q.x : i == 1 ? q.y : i == 2 ? q.z : q.w;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (addresses 16-byte aligned, size a multiple of 16; no multicast)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Ring of RING row slots in shared memory, each [x row: L floats][keep
// words][stats: 4 floats], filled by bulk copies that thread 0 issues RING
// rows ahead, so a CTA's next rows stream in while it works on this one.
template <int T, int NC>
struct RowRing {
    // rows in flight per CTA: one being read, three landing (two CTAs per SM
    // at hidden 4096 keep ~100 KB of rows in flight per SM)
    static constexpr int RING = 4;
    static constexpr int L = NC * 4 * T;
    static constexpr int WORDS = NC * T / 8;
    static constexpr int SLOT = L + WORDS + 4;  // floats
    static constexpr size_t bytes() { return RING * SLOT * sizeof(float) + 2 * RING * sizeof(uint64_t); }
    float *base;
    uint64_t *full;
    __device__ float *slot(int i) const { return base + i * SLOT; }
    __device__ void issue(int i, const Params &p, int64_t r) const {
        const int n = p.hidden;
        const uint32_t xb = static_cast<uint32_t>(n) * 4u;
        const uint32_t kb = static_cast<uint32_t>(p.words_per_row) * 4u;
        mbar_arrive_expect_tx(&full[i], xb + kb + 16u);
        float *d = slot(i);
        bulk_load(d, p.x + r * n, xb, &full[i]);
        bulk_load(d + L, p.keep_in + r * p.words_per_row, kb, &full[i]);
        bulk_load(d + L + WORDS, p.stats_in + 4 * r, 16u, &full[i]);
    }
};

// ---------------------------------------------------------------------------
// FAST-mode row statistics.  Four block reductions per row -- sum (mean), sum
// of squared deviations (variance), max, and one joint reduction of the
// softmax denominator z with its kept part ks = sum of exp(y - max) over the
// elements dropout keeps -- where the EXACT form needs five: the forward's
// row sum of dropout(softmax(y)) is ks / z / (1 - rate), so neither the
// per-element division by z nor a reduction of the dropped-out probabilities
// is needed.  Sums run in butterfly order with contraction allowed; every
// result stays within f32 rel 1e-5 of the C lane's canonical trees.  The
// forward and the adjoint's recomputing path both call fast_stats, so saved
// and recomputed statistics are bit-identical.
// ---------------------------------------------------------------------------
template <int T, int NV>
__device__ __forceinline__ void block_sums(float *a, float *red) {
    constexpr int W = T / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int j = 0; j < NV; ++j) a[j] += __shfl_xor_sync(0xffffffffu, a[j], off);
    if (lane == 0)
#pragma unroll
        for (int j = 0; j < NV; ++j) red[j * W + warp] = a[j];
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        float w[W];
#pragma unroll
        for (int i = 0; i < W; i += 4) {
            const float4 q = *reinterpret_cast<const float4 *>(red + j * W + i);
            w[i] = q.x; w[i + 1] = q.y; w[i + 2] = q.z; w[i + 3] = q.w;
        }
#pragma unroll
        for (int width = 1; width < W; width <<= 1)
#pragma unroll
            for (int i = 0; i + width < W; i += 2 * width) w[i] += w[i + width];
        a[j] = w[0];
    }
}

template <int T>
__device__ __forceinline__ float block_max_fast(float m, float *red) {
    constexpr int W = T / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int i = 1; i < W; ++i) r = fmaxf(r, red[i]);
    return r;
}

struct RowStats {
    float mean, d, mx, z, ks;
};

// x: the row in the chunk layout (zeros past the row end); keepm: bit
// (c*4+i) set where dropout keeps the element.  A NaN anywhere in the row
// makes mean, and with it every later statistic but mx, NaN.
template <int T, int NC, bool FULL>
__device__ __forceinline__ RowStats fast_stats(const float (&x)[NC][4], uint32_t keepm, int n,
                                               const float *sg, const float *sb, float eps,
                                               float rh, Red<T, NC> &rs) {
    RowStats st;
    float a[2];
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c) s += (x[c][0] + x[c][1]) + (x[c][2] + x[c][3]);
    a[0] = s;
    block_sums<T, 1>(a, rs.next());
    st.mean = a[0] * rh;
    float q = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float cc = x[c][i] - st.mean;
            const bool valid = FULL || c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n;
            q = valid ? fmaf(cc, cc, q) : q;
        }
    a[0] = q;
    block_sums<T, 1>(a, rs.next());
    st.d = __fsqrt_rn(a[0] * rh + eps);
    const float rd = __frcp_rn(st.d);
    float y[NC][4];
    float m = -INFINITY;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const bool valid = FULL || c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n;
            const float v = fmaf((x[c][i] - st.mean) * rd, at(g4, i), at(b4, i));
            y[c][i] = valid ? v : -INFINITY;
            m = fmaxf(m, y[c][i]);
        }
    }
    st.mx = block_max_fast<T>(m, rs.next());
    float z = 0.0f, ks = 0.0f;
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float e = __expf(y[c][i] - st.mx);
            z += e;
            ks += ((keepm >> (c * 4 + i)) & 1u) ? e : 0.0f;
        }
    a[0] = z;
    a[1] = ks;
    block_sums<T, 2>(a, rs.next());
    st.z = a[0];
    st.ks = a[1];
    return st;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <int T, int NC, bool EXACT, bool FULL>
__global__ void __launch_bounds__(T, NC >= 8 ? 1 : 3) fwd_kernel(Params p) {
    extern __shared__ __align__(16) float smem[];
    float *sg = smem;                 // gamma
    float *sb = sg + NC * 4 * T;      // beta
    Red<T, NC> rs{sb + NC * 4 * T};
    const int n = FULL ? NC * 4 * T : p.hidden;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
    stage<NC, T>(sg, p.gamma, n);
    stage<NC, T>(sb, p.beta, n);
    __syncthreads();
    for (int64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        float v[NC][4];
        load4<NC, T>(v, p.x + r * n, n, vec);
        // keep bits first: independent of x, they overlap the loads in flight
        const uint64_t base = static_cast<uint64_t>(p.index_base + r * n);
        uint32_t keepm = 0;
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int e = c * 4 * T + 4 * threadIdx.x + i;
                const bool keep = e < n && dropout_keep(p.key, base + e, p.threshold);
                keepm |= (keep ? 1u : 0u) << (c * 4 + i);
            }
        if (p.keep_out) {
            uint32_t *kw = p.keep_out + r * p.words_per_row;
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t bits = __ballot_sync(0xffffffffu, (keepm >> (c * 4 + i)) & 1u);
                    if (lane == 0) kw[(c * (T / 32) + warp) * 4 + i] = bits;
                }
        }
        if constexpr (!EXACT) {
            const RowStats st = fast_stats<T, NC, FULL>(v, keepm, n, sg, sb, p.eps, p.rh, rs);
            if (threadIdx.x == 0) {
                p.rowsum[r] = canon(__fmul_rn(__fdiv_rn(st.ks, st.z), p.rden));
                if (p.stats)
                    *reinterpret_cast<float4 *>(p.stats + 4 * r) = make_float4(st.mean, st.d, st.mx, st.z);
            }
            continue;
        }
        const float s1 = tree4<T, NC, FULL>(v, n, rs);
        const float mean = div_<EXACT>(s1, p.hf, p.rh);
        float part[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = __fsub_rn(v[c][i], mean);
            part[c] = quad(__fmul_rn(v[c][0], v[c][0]), __fmul_rn(v[c][1], v[c][1]),
                           __fmul_rn(v[c][2], v[c][2]), __fmul_rn(v[c][3], v[c][3]),
                           lanes_left<FULL, T>(n, c));
        }
        const float s2 = tree_parts<T, NC>(part, n, rs);
        const float var = div_<EXACT>(s2, p.hf, p.rh);
        const float d = __fsqrt_rn(__fadd_rn(var, p.eps));
        const float rd = __fdiv_rn(1.0f, d);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[c][i] = __fadd_rn(__fmul_rn(div_<EXACT>(v[c][i], d, rd), at(g4, i)), at(b4, i));
        }
        const float mx = row_max<T, NC, FULL>(v, n, rs);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = exp_<EXACT>(__fsub_rn(v[c][i], mx));
        const float z = tree4<T, NC, FULL>(v, n, rs);
        const float rz = __fdiv_rn(1.0f, z);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float s = div_<EXACT>(v[c][i], z, rz);
                v[c][i] = ((keepm >> (c * 4 + i)) & 1u) ? div_<EXACT>(s, p.den, p.rden) : 0.0f;
            }
        const float rsum = tree4<T, NC, FULL>(v, n, rs);
        if (threadIdx.x == 0) {
            p.rowsum[r] = canon(rsum);
            if (p.stats)
                *reinterpret_cast<float4 *>(p.stats + 4 * r) = make_float4(mean, d, mx, z);
        }
    }
}

// ---------------------------------------------------------------------------
// adjoint
// ---------------------------------------------------------------------------
template <int T, int NC, bool EXACT, bool FULL>
__global__ void __launch_bounds__(T, NC >= 8 ? 1 : 2) bwd_kernel(Params p) {
    extern __shared__ __align__(16) float smem[];
    constexpr int L = NC * 4 * T;
    float *sg = smem;          // gamma
    float *sb = sg + L;        // beta
    Red<T, NC> rs{sb + L};
    const int n = FULL ? NC * 4 * T : p.hidden;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(p.dx) & 15) == 0);
    // saved-state adjoint: stream x, keep bits and statistics through the ring
    const bool ring = vec && p.keep_in && p.stats_in &&
                      ((reinterpret_cast<uintptr_t>(p.keep_in) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(p.stats_in) & 15) == 0);
    RowRing<T, NC> rr;
    rr.base = sb + L + 2 * (NC * (T / 32) + 8);
    rr.full = reinterpret_cast<uint64_t *>(rr.base + RowRing<T, NC>::RING * RowRing<T, NC>::SLOT);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(rr.full + 2 * RowRing<T, NC>::RING);
    const int64_t r_begin = static_cast<int64_t>(blockIdx.x) * p.rows_per_cta;
    int64_t r_end = r_begin + p.rows_per_cta;
    if (r_end > p.rows) r_end = p.rows;
    if (ring && threadIdx.x == 0) {
        for (int i = 0; i < RowRing<T, NC>::RING; ++i) mbar_init(&rr.full[i], 1);
        *abort_flag = 0;
        fence_mbarrier_init();
        for (int i = 0; i < RowRing<T, NC>::RING && r_begin + i < r_end; ++i) rr.issue(i, p, r_begin + i);
    }
    stage<NC, T>(sg, p.gamma, n);
    stage<NC, T>(sb, p.beta, n);
    __syncthreads();
    int64_t issued = r_begin + RowRing<T, NC>::RING;  // next row to stream (thread 0)
    // this CTA's dgamma / dbeta partials for the columns this thread owns,
    // summed over its rows in row order (registers: the thread holds the
    // same columns for every row)
    float4 acc_g[NC], acc_b[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) acc_g[c] = acc_b[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int64_t r = r_begin; r < r_end; ++r) {
        float c_[NC][4];
        uint32_t keepm = 0;  // bit (c*4+i): element kept
        const int li = static_cast<int>(r - r_begin);
        const float *slot = nullptr;
        if (ring) {
            const int si = li % RowRing<T, NC>::RING;
            if (!mbar_wait_bounded(&rr.full[si], (li / RowRing<T, NC>::RING) & 1, DEVERR_TIMEOUT_PRODUCER))
                *abort_flag = 1;
            slot = rr.slot(si);
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int e0 = c * 4 * T + 4 * threadIdx.x;
                if (e0 + 3 < n) {
                    const float4 q = reinterpret_cast<const float4 *>(slot)[c * T + threadIdx.x];
                    c_[c][0] = q.x; c_[c][1] = q.y; c_[c][2] = q.z; c_[c][3] = q.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) c_[c][i] = (e0 + i < n) ? slot[e0 + i] : 0.0f;
                }
            }
        } else {
            load4<NC, T>(c_, p.x + r * n, n, vec);
        }
        if (p.keep_in) {
            const uint32_t *kw = ring ? reinterpret_cast<const uint32_t *>(slot + L)
                                      : p.keep_in + r * p.words_per_row;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const uint4 w = reinterpret_cast<const uint4 *>(kw)[c * (T / 32) + warp];
                keepm |= ((w.x >> lane) & 1u) << (c * 4 + 0);
                keepm |= ((w.y >> lane) & 1u) << (c * 4 + 1);
                keepm |= ((w.z >> lane) & 1u) << (c * 4 + 2);
                keepm |= ((w.w >> lane) & 1u) << (c * 4 + 3);
            }
        } else {
            const uint64_t base = static_cast<uint64_t>(p.index_base + r * n);
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int e = c * 4 * T + 4 * threadIdx.x + i;
                    const bool keep = e < n && dropout_keep(p.key, base + e, p.threshold);
                    keepm |= (keep ? 1u : 0u) << (c * 4 + i);
                }
        }
        float mean, d, mx, z;
        if (p.stats_in) {
            const float4 st = ring ? *reinterpret_cast<const float4 *>(slot + L + RowRing<T, NC>::WORDS)
                                   : *reinterpret_cast<const float4 *>(p.stats_in + 4 * r);
            mean = st.x; d = st.y; mx = st.z; z = st.w;
        } else if constexpr (!EXACT) {
            const RowStats st = fast_stats<T, NC, FULL>(c_, keepm, n, sg, sb, p.eps, p.rh, rs);
            mean = st.mean; d = st.d; mx = st.mx; z = st.z;
        } else {
            mean = div_<EXACT>(tree4<T, NC, FULL>(c_, n, rs), p.hf, p.rh);
            float part[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                float q[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float cc = __fsub_rn(c_[c][i], mean);
                    q[i] = __fmul_rn(cc, cc);
                }
                part[c] = quad(q[0], q[1], q[2], q[3], lanes_left<FULL, T>(n, c));
            }
            const float var = div_<EXACT>(tree_parts<T, NC>(part, n, rs), p.hf, p.rh);
            d = __fsqrt_rn(__fadd_rn(var, p.eps));
            const float rd0 = __fdiv_rn(1.0f, d);
            float y[NC][4];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    y[c][i] = __fadd_rn(__fmul_rn(div_<EXACT>(__fsub_rn(c_[c][i], mean), d, rd0), at(g4, i)), at(b4, i));
            }
            mx = row_max<T, NC, FULL>(y, n, rs);
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < 4; ++i) y[c][i] = exp_<EXACT>(__fsub_rn(y[c][i], mx));
            z = tree4<T, NC, FULL>(y, n, rs);
        }
        if constexpr (!EXACT) {
            // Closed form of the same adjoint: with s = softmax(y), g the
            // replayed dropout cotangent (1/(1-rate) where kept, else 0) and
            // q = sum(g s), dy = s (g - q); dgamma += dy nn, dbeta += dy;
            // dn = dy gamma and dx = (dn - mean(dn) - nn mean(dn nn)) / d.
            // Two block reductions (q, then mean(dn) with mean(dn nn)) where
            // the graph's literal form takes three.
            const float rd = __frcp_rn(d), rz = __frcp_rn(z);
            float s[NC][4], nn[NC][4];
            float red2[2];
            float qp = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const bool valid = FULL || c * 4 * T + 4 * static_cast<int>(threadIdx.x) + i < n;
                    nn[c][i] = (c_[c][i] - mean) * rd;
                    const float y = fmaf(nn[c][i], at(g4, i), at(b4, i));
                    s[c][i] = valid ? __expf(y - mx) * rz : 0.0f;
                    qp += ((keepm >> (c * 4 + i)) & 1u) ? s[c][i] : 0.0f;
                }
            }
            red2[0] = qp;
            block_sums<T, 1>(red2, rs.next());
            const float q = red2[0] * p.one_over_den;
            if (ring) {
                // every thread has read its slot (the reduction synchronised
                // the CTA): refill it with the row RING ahead
                if (*abort_flag) break;
                if (threadIdx.x == 0 && issued < r_end) {
                    rr.issue(li % RowRing<T, NC>::RING, p, issued);
                    ++issued;
                }
            }
            float sdn = 0.0f, sdnn = 0.0f;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const float4 g4 = ld4<T>(sg, c);
                float dy[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float ds = ((keepm >> (c * 4 + i)) & 1u) ? p.one_over_den : 0.0f;
                    dy[i] = s[c][i] * (ds - q);
                    const float dn = dy[i] * at(g4, i);
                    s[c][i] = dn;
                    sdn += dn;
                    sdnn = fmaf(dn, nn[c][i], sdnn);
                }
                acc_b[c].x += dy[0]; acc_b[c].y += dy[1]; acc_b[c].z += dy[2]; acc_b[c].w += dy[3];
                acc_g[c].x = fmaf(dy[0], nn[c][0], acc_g[c].x);
                acc_g[c].y = fmaf(dy[1], nn[c][1], acc_g[c].y);
                acc_g[c].z = fmaf(dy[2], nn[c][2], acc_g[c].z);
                acc_g[c].w = fmaf(dy[3], nn[c][3], acc_g[c].w);
            }
            red2[0] = sdn;
            red2[1] = sdnn;
            block_sums<T, 2>(red2, rs.next());
            const float m1 = red2[0] * p.rh, m2 = red2[1] * p.rh;
            float *dxr = p.dx + r * n;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int e0 = c * 4 * T + 4 * threadIdx.x;
                float o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = canon(rd * (fmaf(-nn[c][i], m2, s[c][i]) - m1));
                if (vec && e0 + 3 < n) {
                    __stcs(reinterpret_cast<float4 *>(dxr + e0), make_float4(o[0], o[1], o[2], o[3]));
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        if (e0 + i < n) dxr[e0 + i] = o[i];
                }
            }
            continue;
        }
        const float rd = __fdiv_rn(1.0f, d);
        const float rz = __fdiv_rn(1.0f, z);
        const float two_d = __fmul_rn(2.0f, d);
        const float r2d = __fdiv_rn(1.0f, two_d);
        // s (softmax output) and the replayed unit cotangent ds; c_ becomes c
        float s[NC][4];
        float part[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
            float gy[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float cc = __fsub_rn(c_[c][i], mean);
                c_[c][i] = cc;
                const float y = __fadd_rn(__fmul_rn(div_<EXACT>(cc, d, rd), at(g4, i)), at(b4, i));
                s[c][i] = div_<EXACT>(exp_<EXACT>(__fsub_rn(y, mx)), z, rz);
                gy[i] = ((keepm >> (c * 4 + i)) & 1u) ? __fmul_rn(p.one_over_den, s[c][i]) : 0.0f;
            }
            part[c] = quad(gy[0], gy[1], gy[2], gy[3], lanes_left<FULL, T>(n, c));
        }
        const float q = tree_parts<T, NC>(part, n, rs);
        if (ring) {
            // every thread has read its slot (the reduction above synchronised
            // the CTA): refill it with the row RING ahead
            if (*abort_flag) break;
            if (threadIdx.x == 0 && issued < r_end) {
                rr.issue(li % RowRing<T, NC>::RING, p, issued);
                ++issued;
            }
        }
        // dy = s*(ds - q); dgamma += dy*nn; dbeta += dy; dn = dy*gamma;
        // dt = -((dn*nn)/d)/(2d); s becomes dn
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4 g4 = ld4<T>(sg, c);
            float4 &pg4 = acc_g[c], &pb4 = acc_b[c];
            float dt[4], dys[4], dyn[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float ds = ((keepm >> (c * 4 + i)) & 1u) ? p.one_over_den : 0.0f;
                const float dy = __fmul_rn(s[c][i], __fsub_rn(ds, q));
                const float nn = div_<EXACT>(c_[c][i], d, rd);
                dys[i] = dy;
                dyn[i] = __fmul_rn(dy, nn);
                const float dn = __fmul_rn(dy, at(g4, i));
                const float qq = div_<EXACT>(__fmul_rn(dn, nn), d, rd);
                dt[i] = div_<EXACT>(-qq, two_d, r2d);
                s[c][i] = dn;
            }
            // elements past the row end hold exact zeros in every term
            pg4.x = __fadd_rn(pg4.x, dyn[0]); pg4.y = __fadd_rn(pg4.y, dyn[1]);
            pg4.z = __fadd_rn(pg4.z, dyn[2]); pg4.w = __fadd_rn(pg4.w, dyn[3]);
            pb4.x = __fadd_rn(pb4.x, dys[0]); pb4.y = __fadd_rn(pb4.y, dys[1]);
            pb4.z = __fadd_rn(pb4.z, dys[2]); pb4.w = __fadd_rn(pb4.w, dys[3]);
            part[c] = quad(dt[0], dt[1], dt[2], dt[3], lanes_left<FULL, T>(n, c));
        }
        const float dvar = tree_parts<T, NC>(part, n, rs);
        const float ds2 = div_<EXACT>(dvar, p.hf, p.rh);
        // dc = (ds2*c + ds2*c) + dn/d ; s becomes dc
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float m4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pr = __fmul_rn(ds2, c_[c][i]);
                const float dc = __fadd_rn(__fadd_rn(pr, pr), div_<EXACT>(s[c][i], d, rd));
                s[c][i] = dc;
                m4[i] = -dc;
            }
            part[c] = quad(m4[0], m4[1], m4[2], m4[3], lanes_left<FULL, T>(n, c));
        }
        const float dm = tree_parts<T, NC>(part, n, rs);
        const float ds1 = div_<EXACT>(dm, p.hf, p.rh);
        float *dxr = p.dx + r * n;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            float o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i] = canon(__fadd_rn(ds1, s[c][i]));
            if (vec && e0 + 3 < n) {
                __stcs(reinterpret_cast<float4 *>(dxr + e0), make_float4(o[0], o[1], o[2], o[3]));
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (e0 + i < n) dxr[e0 + i] = o[i];
            }
        }
    }
    if (ring && threadIdx.x == 0 && *abort_flag) {
        // bulk copies issued for rows this CTA no longer reads land before it retires
        for (int64_t r = r_begin; r < issued && r < r_end; ++r) {
            const int li = static_cast<int>(r - r_begin);
            mbar_wait_bounded(&rr.full[li % RowRing<T, NC>::RING], (li / RowRing<T, NC>::RING) & 1,
                              DEVERR_TIMEOUT_PRODUCER);
        }
    }
    // this CTA's partials: the thread's columns of chunk c are [e0, e0 + 4)
    float *og = p.dgamma_part + static_cast<int64_t>(blockIdx.x) * n;
    float *ob = p.dbeta_part + static_cast<int64_t>(blockIdx.x) * n;
    const bool vec_out = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.dgamma_part) & 15) == 0) &&
                         ((reinterpret_cast<uintptr_t>(p.dbeta_part) & 15) == 0);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int e0 = c * 4 * T + 4 * threadIdx.x;
        if (vec_out && e0 + 3 < n) {
            *reinterpret_cast<float4 *>(og + e0) = acc_g[c];
            *reinterpret_cast<float4 *>(ob + e0) = acc_b[c];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (e0 + i < n) {
                    og[e0 + i] = at(acc_g[c], i);
                    ob[e0 + i] = at(acc_b[c], i);
                }
        }
    }
}

}  // namespace chain

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

int chunks_for(int64_t hidden) {
    const int per = 4 * kRowThreads;
    const int nc = static_cast<int>((hidden + per - 1) / per);
    return nc <= 1 ? 1 : nc <= 2 ? 2 : nc <= 4 ? 4 : 8;
}

using ChainParams = chain::Params;

ChainParams make_chain_params(const float *x, const float *gamma, const float *beta, float eps,
                              uint64_t key, float rate, int64_t rows, int64_t hidden,
                              int64_t index_base) {
    ChainParams p{};
    p.x = x;
    p.gamma = gamma;
    p.beta = beta;
    p.eps = eps;
    p.key = key;
    p.threshold = dropout_threshold(rate);
    volatile float one = 1.0f;
    p.den = one - rate;
    p.rden = 1.0f / p.den;
    p.one_over_den = 1.0f / p.den;
    p.hf = static_cast<float>(hidden);
    p.rh = 1.0f / p.hf;
    p.rows = rows;
    p.hidden = static_cast<int>(hidden);
    p.index_base = index_base;
    p.words_per_row = chunks_for(hidden) * kRowThreads / 8;
    return p;
}

template <typename F>
int with_nc(int64_t hidden, F &&f) {
    switch (chunks_for(hidden)) {
        case 1: return f(std::integral_constant<int, 1>());
        case 2: return f(std::integral_constant<int, 2>());
        case 4: return f(std::integral_constant<int, 4>());
        default: return f(std::integral_constant<int, 8>());
    }
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
    return check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(bytes)),
                      "cudaFuncSetAttribute(chain)");
}

template <int T, int NC>
constexpr size_t red_bytes() {
    return 2 * (NC * (T / 32) + 8) * sizeof(float);
}

template <int T>
int launch_chain_fwd(const ChainParams &p, cudaStream_t s) {
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    return with_nc(p.hidden, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const size_t smem = 2 * NC * 4 * T * sizeof(float) + red_bytes<T, NC>();
        int64_t g = static_cast<int64_t>(sm_count()) * 3 * 8;
        if (g > p.rows) g = p.rows;
        const unsigned grid = static_cast<unsigned>(g);
        const bool full = p.hidden == NC * 4 * T;
        auto go = [&](auto kern) -> int {
            CHELIS_TRY(set_smem(kern, smem));
            kern<<<grid, T, smem, s>>>(p);
            return CHELIS_CUDA_OK;
        };
        if (exact) CHELIS_TRY(full ? go(chain::fwd_kernel<T, NC, true, true>) : go(chain::fwd_kernel<T, NC, true, false>));
        else CHELIS_TRY(full ? go(chain::fwd_kernel<T, NC, false, true>) : go(chain::fwd_kernel<T, NC, false, false>));
        g_launches++;
        CHELIS_LAUNCH_CHECK("chain::fwd_kernel");
        return CHELIS_CUDA_OK;
    });
}

template <int T>
int launch_chain_bwd(const ChainParams &p, int grid, cudaStream_t s) {
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    return with_nc(p.hidden, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const size_t smem = 2 * NC * 4 * T * sizeof(float) + red_bytes<T, NC>() +
                            chain::RowRing<T, NC>::bytes() + 16;
        const bool full = p.hidden == NC * 4 * T;
        auto go = [&](auto kern) -> int {
            CHELIS_TRY(set_smem(kern, smem));
            kern<<<grid, T, smem, s>>>(p);
            return CHELIS_CUDA_OK;
        };
        if (exact) CHELIS_TRY(full ? go(chain::bwd_kernel<T, NC, true, true>) : go(chain::bwd_kernel<T, NC, true, false>));
        else CHELIS_TRY(full ? go(chain::bwd_kernel<T, NC, false, true>) : go(chain::bwd_kernel<T, NC, false, false>));
        g_launches++;
        CHELIS_LAUNCH_CHECK("chain::bwd_kernel");
        return CHELIS_CUDA_OK;
    });
}

}  // namespace

int chain_bwd_grid(int64_t rows) {
    // two resident CTAs per SM at hidden <= 4096 (shared memory: gamma, beta
    // and the row ring), each owning a contiguous run of rows
    int64_t g = static_cast<int64_t>(sm_count()) * 2;
    return static_cast<int>(rows < g ? (rows < 1 ? 1 : rows) : g);
}

int chain_bwd_with_partials(const ChainParams &p0, float *dgamma, float *dbeta, float *part,
                            int grid, cudaStream_t s) {
    ChainParams p = p0;
    p.dgamma_part = part;
    p.dbeta_part = part + static_cast<int64_t>(grid) * p.hidden;
    p.rows_per_cta = static_cast<int>((p.rows + grid - 1) / grid);
    CHELIS_TRY(launch_chain_bwd<kRowThreads>(p, grid, s));
    CHELIS_TRY(col_sum_into(p.dgamma_part, grid, p.hidden, dgamma, s));
    CHELIS_TRY(col_sum_into(p.dbeta_part, grid, p.hidden, dbeta, s));
    return CHELIS_CUDA_OK;
}

}  // namespace chelis

using namespace chelis;

namespace {
int chain_bwd_common(ChainParams p, float *dgamma, float *dbeta) {
    cudaStream_t s = current_stream();
    if (p.rows == 0) {
        CHELIS_TRY(check_cuda(cudaMemsetAsync(dgamma, 0, p.hidden * sizeof(float), s), "memset"));
        return check_cuda(cudaMemsetAsync(dbeta, 0, p.hidden * sizeof(float), s), "memset");
    }
    const int grid = chain_bwd_grid(p.rows);
    void *part = nullptr;
    CHELIS_TRY(scratch_alloc(&part, static_cast<size_t>(2) * grid * p.hidden * sizeof(float), s));
    int st = chain_bwd_with_partials(p, dgamma, dbeta, static_cast<float *>(part), grid, s);
    scratch_free(part, s);
    return st;
}
}  // namespace

extern "C" {

int chelis_cuda_chain_fwd(const float *x, const float *gamma, const float *beta, float eps,
                          uint64_t key, float rate, int64_t rows, int64_t hidden,
                          int64_t index_base, float *rowsum, float *row_stats) {
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    CHELIS_TRY(check_rate(rate));
    if (hidden == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    if (rows == 0) return CHELIS_CUDA_OK;
    ChainParams p = make_chain_params(x, gamma, beta, eps, key, rate, rows, hidden, index_base);
    p.rowsum = rowsum;
    p.stats = row_stats;
    return launch_chain_fwd<kRowThreads>(p, current_stream());
}

int chelis_cuda_chain_bwd(const float *x, const float *gamma, const float *beta, float eps,
                          uint64_t key, float rate, int64_t rows, int64_t hidden,
                          int64_t index_base, const float *row_stats, float *dx, float *dgamma,
                          float *dbeta) {
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    CHELIS_TRY(check_rate(rate));
    if (hidden == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    ChainParams p = make_chain_params(x, gamma, beta, eps, key, rate, rows, hidden, index_base);
    p.stats_in = row_stats;
    p.dx = dx;
    return chain_bwd_common(p, dgamma, dbeta);
}

int64_t chelis_cuda_chain_saved_bytes(int64_t rows, int64_t hidden) {
    if (rows < 0 || hidden <= 0 || hidden > 8 * 4 * kRowThreads) return -1;
    return rows * (4 * static_cast<int64_t>(sizeof(float)) +
                   static_cast<int64_t>(chunks_for(hidden)) * kRowThreads / 8 * 4);
}

int chelis_cuda_chain_fwd_save(const float *x, const float *gamma, const float *beta, float eps,
                               uint64_t key, float rate, int64_t rows, int64_t hidden,
                               int64_t index_base, float *rowsum, void *saved) {
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    CHELIS_TRY(check_rate(rate));
    if (hidden == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    if (rows == 0) return CHELIS_CUDA_OK;
    if (!saved || (reinterpret_cast<uintptr_t>(saved) & 15))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "chain saved state must be 16-byte aligned");
    ChainParams p = make_chain_params(x, gamma, beta, eps, key, rate, rows, hidden, index_base);
    p.rowsum = rowsum;
    p.stats = static_cast<float *>(saved);
    p.keep_out = reinterpret_cast<uint32_t *>(static_cast<float *>(saved) + 4 * rows);
    return launch_chain_fwd<kRowThreads>(p, current_stream());
}

int chelis_cuda_chain_bwd_saved(const float *x, const float *gamma, const float *beta, float eps,
                                float rate, int64_t rows, int64_t hidden, const void *saved,
                                float *dx, float *dgamma, float *dbeta) {
    CHELIS_TRY(check_rows_args(x, rows, hidden));
    CHELIS_TRY(check_rate(rate));
    if (hidden == 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in layer_norm at f32");
    if (rows > 0 && (!saved || (reinterpret_cast<uintptr_t>(saved) & 15)))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "chain saved state must be 16-byte aligned");
    ChainParams p = make_chain_params(x, gamma, beta, eps, 0, rate, rows, hidden, 0);
    p.stats_in = static_cast<const float *>(saved);
    p.keep_in = reinterpret_cast<const uint32_t *>(static_cast<const float *>(saved) + 4 * rows);
    p.dx = dx;
    return chain_bwd_common(p, dgamma, dbeta);
}

}  // extern "C"
