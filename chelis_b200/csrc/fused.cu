// fused.cu -- the generic FusedElem group: a chain of elementwise steps over
// broadcast inputs evaluated in one pass, and the same chain reduced along
// one axis (Sum / Max): the groups chelis-dag-core's fusion pass emits
// (FusedElem dag.rs:1323-1325, steps FusedStepOp dag.rs:494-526, inputs
// FusedInput dag.rs:673-678).  The reference's GPU lane JIT-compiles one
// kernel string per chain (kernels.rs fused_elementwise :2391, reduce_fused
// :2175); here one ahead-of-time kernel interprets the step list.  Every
// thread walks the same steps in the same order, so the dispatch on the step
// opcode is uniform, and a thread's inputs and step values sit in a shared
// memory table laid out [row][element][thread]: a row is fetched by an index
// that is uniform across the warp, which a register array could not offer.
// Each thread carries E consecutive elements through the chain at once, so
// one opcode dispatch serves E elements and E loads per input are in flight
// together.
//
// Step semantics follow the C lane (crates/chelis-backend-c/src/emit.rs
// scalar_step_raw_expr :6744-6905 and fp_env.rs fused_step_nan_finalization
// :213-241): IEEE + - * / and sqrt; a NaN result is replaced by the canonical
// quiet NaN after every step except MaxElem / MinElem, which select an
// operand with its bits (the first operand when it is NaN, else a NaN second
// operand, else the first on ties); Round is rint (ties to even).
// Transcendental steps call CUDA's libm, which stands in for the reference's
// correctly rounded CORE-MATH within a few ulp: a chain with them matches to
// a tolerance, a chain without them bit for bit.  Pow keeps CORE-MATH's
// IEEE special cases that libm does not: a signaling NaN operand gives NaN
// even where a quiet one gives 1 (pow(sNaN, 0), pow(1, sNaN)).
//
// Reductions follow emit_fused_reduce (emit.rs:9580-9860): Sum is the
// canonical adjacent-pair tree over the axis ([05-OP-30]; the C lane's carry
// tree), finalized once; Max is chelis_fmax_propnan_f32 folded from -inf
// (any NaN gives the canonical NaN; among equal values the later one wins,
// which decides the sign of a zero maximum).  An empty Max axis is the
// Domain trap "max_reduce" ([05-OP-12]); an empty Sum axis gives zeros.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "crmath.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int scratch_alloc(void **ptr, size_t bytes, cudaStream_t stream);
void scratch_free(void *ptr, cudaStream_t stream);

namespace fused {

constexpr int MAX_STEPS = 32, MAX_INPUTS = 8, MAX_RANK = 6, THREADS = 128;
enum Mode { DENSE = 0, STRIDED32 = 1, STRIDED64 = 2 };
enum StepFlag { A_PREV = 1, B_PREV = 2, STORE = 4, HEAVY = 8 };

struct Program {
    uint8_t op[MAX_STEPS];
    uint8_t a[MAX_STEPS], b[MAX_STEPS];  // table rows: inputs 0..n_inputs-1, then the steps
    uint8_t flags[MAX_STEPS];            // A_PREV / B_PREV: operand is the step before; STORE: a later step reads the row
    uint8_t row[MAX_STEPS];              // table row of a STORE step
    int32_t n_steps, n_inputs, rank;
    int32_t n_rows;                       // inputs, then the STORE steps (a scratch row follows)
    int32_t vec_mask;                     // input k may be read E elements at a time (aligned, unit stride)
    const void *in[MAX_INPUTS];
    int64_t stride[MAX_INPUTS][MAX_RANK];  // element strides over the iteration shape
    int64_t shape[MAX_RANK];               // iteration shape (the output's, or the reduced input's)
    uint32_t div_mul[MAX_RANK];            // n / shape[d] = umulhi(n, mul) >> shr for n < 2^31
    uint32_t div_shr[MAX_RANK];            //   (mul 0: shape[d] is 1)
    int64_t total;
};

template <typename T> __device__ __forceinline__ T canon_nan(T x);
template <> __device__ __forceinline__ float canon_nan(float x) {
    return isnan(x) ? __int_as_float(0x7fc00000) : x;
}
template <> __device__ __forceinline__ double canon_nan(double x) {
    return isnan(x) ? __longlong_as_double(0x7ff8000000000000ll) : x;
}
__device__ __forceinline__ bool is_snan(float x) {
    return isnan(x) && !(__float_as_uint(x) & 0x00400000u);
}
__device__ __forceinline__ bool is_snan(double x) {
    return isnan(x) && !(static_cast<unsigned long long>(__double_as_longlong(x)) & 0x0008000000000000ull);
}

__device__ __forceinline__ float m_add(float x, float y) { return __fadd_rn(x, y); }
__device__ __forceinline__ double m_add(double x, double y) { return __dadd_rn(x, y); }
__device__ __forceinline__ float m_sub(float x, float y) { return __fsub_rn(x, y); }
__device__ __forceinline__ double m_sub(double x, double y) { return __dsub_rn(x, y); }
__device__ __forceinline__ float m_mul(float x, float y) { return __fmul_rn(x, y); }
__device__ __forceinline__ double m_mul(double x, double y) { return __dmul_rn(x, y); }
__device__ __forceinline__ float m_div(float x, float y) { return __fdiv_rn(x, y); }
__device__ __forceinline__ double m_div(double x, double y) { return __ddiv_rn(x, y); }
__device__ __forceinline__ float m_sqrt(float x) { return __fsqrt_rn(x); }
__device__ __forceinline__ double m_sqrt(double x) { return __dsqrt_rn(x); }
__device__ __forceinline__ float m_floor(float x) { return floorf(x); }
__device__ __forceinline__ double m_floor(double x) { return ::floor(x); }
__device__ __forceinline__ float m_ceil(float x) { return ceilf(x); }
__device__ __forceinline__ double m_ceil(double x) { return ::ceil(x); }
__device__ __forceinline__ float m_rint(float x) { return rintf(x); }
__device__ __forceinline__ double m_rint(double x) { return ::rint(x); }
__device__ __forceinline__ float m_abs(float x) { return fabsf(x); }
__device__ __forceinline__ double m_abs(double x) { return ::fabs(x); }
// Internal step codes past the public FusedStepOp range: f32 exp / log through
// the correctly rounded functions (crmath.cuh) in the EXACT rows mode.
constexpr int OP_EXP_CR = CHELIS_FUSED_ROUND + 1, OP_LOG_CR = CHELIS_FUSED_ROUND + 2;
__device__ __forceinline__ float m_exp_cr(float x) { return crmath::expf_cr(x); }
__device__ __forceinline__ double m_exp_cr(double x) { return ::exp(x); }
__device__ __forceinline__ float m_log_cr(float x) { return crmath::logf_cr(x); }
__device__ __forceinline__ double m_log_cr(double x) { return ::log(x); }
__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return ::exp(x); }
__device__ __forceinline__ float m_log(float x) { return logf(x); }
__device__ __forceinline__ double m_log(double x) { return ::log(x); }
__device__ __forceinline__ float m_sin(float x) { return sinf(x); }
__device__ __forceinline__ double m_sin(double x) { return ::sin(x); }
__device__ __forceinline__ float m_cos(float x) { return cosf(x); }
__device__ __forceinline__ double m_cos(double x) { return ::cos(x); }
__device__ __forceinline__ float m_tan(float x) { return tanf(x); }
__device__ __forceinline__ double m_tan(double x) { return ::tan(x); }
__device__ __forceinline__ float m_atan(float x) { return atanf(x); }
__device__ __forceinline__ double m_atan(double x) { return ::atan(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return ::tanh(x); }
__device__ __forceinline__ float m_erf(float x) { return erff(x); }
__device__ __forceinline__ double m_erf(double x) { return ::erf(x); }
__device__ __forceinline__ float m_erfc(float x) { return erfcf(x); }
__device__ __forceinline__ double m_erfc(double x) { return ::erfc(x); }
template <typename T>
__device__ __forceinline__ T m_pow(T x, T y) {
    if (is_snan(x) || is_snan(y)) return canon_nan(x + y);
    if constexpr (sizeof(T) == 4) return powf(x, y);
    else return ::pow(x, y);
}

// The light steps over E elements (all but pow, sin, cos, tan): x, y in, r out.  The opcode is uniform
// across the grid, so the switch is taken once per step for all E elements.
template <typename T, int E>
__device__ __forceinline__ void apply_light(int op, const T (&x)[E], const T (&y)[E], T (&r)[E]) {
#define CHELIS_FUSED_EACH(expr)                                          \
    {                                                                    \
        _Pragma("unroll") for (int e = 0; e < E; ++e) r[e] = (expr);     \
    }                                                                    \
    break;
    switch (op) {
        case CHELIS_FUSED_ADD: CHELIS_FUSED_EACH(canon_nan(m_add(x[e], y[e])))
        case CHELIS_FUSED_SUB: CHELIS_FUSED_EACH(canon_nan(m_sub(x[e], y[e])))
        case CHELIS_FUSED_MUL: CHELIS_FUSED_EACH(canon_nan(m_mul(x[e], y[e])))
        case CHELIS_FUSED_DIV: CHELIS_FUSED_EACH(canon_nan(m_div(x[e], y[e])))
        case CHELIS_FUSED_FLOOR_DIV: CHELIS_FUSED_EACH(canon_nan(m_floor(m_div(x[e], y[e]))))
        case CHELIS_FUSED_MAX_ELEM:
            CHELIS_FUSED_EACH((isnan(x[e]) || (!isnan(y[e]) && x[e] >= y[e])) ? x[e] : y[e])
        case CHELIS_FUSED_MIN_ELEM:
            CHELIS_FUSED_EACH((isnan(x[e]) || (!isnan(y[e]) && x[e] <= y[e])) ? x[e] : y[e])
        case CHELIS_FUSED_NEG: CHELIS_FUSED_EACH(canon_nan(-x[e]))
        case CHELIS_FUSED_RECIP: CHELIS_FUSED_EACH(canon_nan(m_div(T(1), x[e])))
        case CHELIS_FUSED_SQRT: CHELIS_FUSED_EACH(canon_nan(m_sqrt(x[e])))
        case CHELIS_FUSED_ABS: CHELIS_FUSED_EACH(canon_nan(m_abs(x[e])))
        case CHELIS_FUSED_FLOOR: CHELIS_FUSED_EACH(canon_nan(m_floor(x[e])))
        case CHELIS_FUSED_CEIL: CHELIS_FUSED_EACH(canon_nan(m_ceil(x[e])))
        case CHELIS_FUSED_ROUND: CHELIS_FUSED_EACH(canon_nan(m_rint(x[e])))
        case CHELIS_FUSED_EXP: CHELIS_FUSED_EACH(canon_nan(m_exp(x[e])))
        case CHELIS_FUSED_LOG: CHELIS_FUSED_EACH(canon_nan(m_log(x[e])))
        case CHELIS_FUSED_ATAN: CHELIS_FUSED_EACH(canon_nan(m_atan(x[e])))
        case CHELIS_FUSED_TANH: CHELIS_FUSED_EACH(canon_nan(m_tanh(x[e])))
        case CHELIS_FUSED_ERF: CHELIS_FUSED_EACH(canon_nan(m_erf(x[e])))
        case CHELIS_FUSED_ERFC: CHELIS_FUSED_EACH(canon_nan(m_erfc(x[e])))
        default: CHELIS_FUSED_EACH(x[e])  // heavy steps take run_steps' other path
    }
#undef CHELIS_FUSED_EACH
}

// The heavy steps (pow, sin, cos, tan: libm calls whose slow paths hold
// many registers or a local array), one element at a time.
template <typename T>
__device__ __forceinline__ T apply_heavy(int op, T x, T y) {
    switch (op) {
        case CHELIS_FUSED_POW: return canon_nan(m_pow(x, y));
        case CHELIS_FUSED_EXP: return canon_nan(m_exp(x));
        case CHELIS_FUSED_LOG: return canon_nan(m_log(x));
        case OP_EXP_CR: return canon_nan(m_exp_cr(x));
        case OP_LOG_CR: return canon_nan(m_log_cr(x));
        case CHELIS_FUSED_SIN: return canon_nan(m_sin(x));
        case CHELIS_FUSED_COS: return canon_nan(m_cos(x));
        case CHELIS_FUSED_TAN: return canon_nan(m_tan(x));
        case CHELIS_FUSED_ATAN: return canon_nan(m_atan(x));
        case CHELIS_FUSED_TANH: return canon_nan(m_tanh(x));
        case CHELIS_FUSED_ERF: return canon_nan(m_erf(x));
        case CHELIS_FUSED_ERFC: return canon_nan(m_erfc(x));
        default: return x;
    }
}

// Table cell of row `row`, element e: tab[(row * E + e) * THREADS].  The
// step before stays in registers (`last`): an operand that names it is not
// re-read, and a step's row is written only when a later step, not the next
// one, reads it.  A heavy step runs its E elements in a loop (one libm
// call's registers, not E of them) through the table's scratch row.
template <typename T, int E>
__device__ __forceinline__ void run_steps(const Program &p, T *tab, T (&last)[E]) {
    T *scratch = tab + p.n_rows * (E * THREADS);
    for (int s = 0; s < p.n_steps; ++s) {
        const int f = p.flags[s];
        if (f & HEAVY) {
            if (f & (A_PREV | B_PREV)) {
#pragma unroll
                for (int e = 0; e < E; ++e) scratch[e * THREADS] = last[e];
            }
            const T *ra = (f & A_PREV) ? scratch : tab + p.a[s] * (E * THREADS);
            const T *rb = (f & B_PREV) ? scratch : tab + p.b[s] * (E * THREADS);
            const int op = p.op[s];
#pragma unroll 1
            for (int e = 0; e < E; ++e)
                scratch[e * THREADS] = apply_heavy<T>(op, ra[e * THREADS], rb[e * THREADS]);
#pragma unroll
            for (int e = 0; e < E; ++e) last[e] = scratch[e * THREADS];
        } else {
            T x[E], y[E];
            if (f & A_PREV) {
#pragma unroll
                for (int e = 0; e < E; ++e) x[e] = last[e];
            } else {
                const T *ra = tab + p.a[s] * (E * THREADS);
#pragma unroll
                for (int e = 0; e < E; ++e) x[e] = ra[e * THREADS];
            }
            if (f & B_PREV) {
#pragma unroll
                for (int e = 0; e < E; ++e) y[e] = last[e];
            } else {
                const T *rb = tab + p.b[s] * (E * THREADS);
#pragma unroll
                for (int e = 0; e < E; ++e) y[e] = rb[e * THREADS];
            }
            apply_light<T, E>(p.op[s], x, y, last);
        }
        if (f & STORE) {
            T *rr = tab + p.row[s] * (E * THREADS);
#pragma unroll
            for (int e = 0; e < E; ++e) rr[e * THREADS] = last[e];
        }
    }
}

// Element offsets: 32-bit where every offset of every input fits.
template <int MODE> struct OffOf { using type = int64_t; };
template <> struct OffOf<STRIDED32> { using type = int32_t; };
template <int MODE> using Off = typename OffOf<MODE>::type;

// Element offsets of flat index i of the iteration shape in every input.
template <int MODE>
__device__ __forceinline__ void decode(const Program &p, int64_t i, Off<MODE> (&off)[MAX_INPUTS]) {
#pragma unroll
    for (int k = 0; k < MAX_INPUTS; ++k) off[k] = MODE == DENSE ? i : 0;
    if (MODE == DENSE) return;
    if (MODE == STRIDED32) {
        uint32_t rem = static_cast<uint32_t>(i);
        int32_t o[MAX_INPUTS] = {};
#pragma unroll
        for (int d = MAX_RANK - 1; d >= 0; --d) {
            if (d < p.rank) {
                uint32_t c = rem;
                if (d > 0) {
                    const uint32_t q = p.div_mul[d] ? (__umulhi(rem, p.div_mul[d]) >> p.div_shr[d]) : rem;
                    c = rem - q * static_cast<uint32_t>(p.shape[d]);
                    rem = q;
                }
#pragma unroll
                for (int k = 0; k < MAX_INPUTS; ++k)
                    if (k < p.n_inputs) o[k] += static_cast<int32_t>(c) * static_cast<int32_t>(p.stride[k][d]);
            }
        }
#pragma unroll
        for (int k = 0; k < MAX_INPUTS; ++k) off[k] = o[k];
    } else {
        int64_t rem = i;
#pragma unroll
        for (int d = MAX_RANK - 1; d >= 0; --d) {
            if (d < p.rank) {
                int64_t c = rem;
                if (d > 0) {
                    c = rem % p.shape[d];
                    rem /= p.shape[d];
                }
#pragma unroll
                for (int k = 0; k < MAX_INPUTS; ++k)
                    if (k < p.n_inputs) off[k] += c * p.stride[k][d];
            }
        }
    }
}

// Load G groups of W elements of every input, then run the chain; `last`
// receives the group's value at the G*W elements (group g's element e at
// g*W + e).  Input k's group g starts at off[g][k], its elements e *
// stride[k][axis] apart (e * dense_step when MODE is dense).  VEC: inputs in
// vec_mask read a group as one aligned 16-byte vector (W*sizeof(T) == 16).
template <typename T, int G, int W, bool VEC, int MODE>
__device__ __forceinline__ void load_run(const Program &p, const Off<MODE> (&off)[G][MAX_INPUTS],
                                         int axis, Off<MODE> dense_step, T *tab, T (&last)[G * W]) {
    constexpr int E = G * W;
#pragma unroll
    for (int k = 0; k < MAX_INPUTS; ++k) {
        if (k >= p.n_inputs) break;
        const Off<MODE> st = MODE == DENSE ? dense_step : static_cast<Off<MODE>>(p.stride[k][axis]);
        constexpr int Q = W * sizeof(T) / 16;  // 16-byte vectors per group
        const bool vec = VEC && Q > 0 && ((p.vec_mask >> k) & 1);
        T v[E];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const T *src = static_cast<const T *>(p.in[k]) + off[g][k];
            if constexpr (VEC && Q > 0 && W * sizeof(T) == Q * 16) {
                if (vec) {
#pragma unroll
                    for (int q = 0; q < Q; ++q) {
                        if constexpr (sizeof(T) == 4) {
                            const float4 w = __ldg(reinterpret_cast<const float4 *>(src) + q);
                            T *d = v + g * W + 4 * q;
                            d[0] = w.x, d[1] = w.y, d[2] = w.z, d[3] = w.w;
                        } else {
                            const double2 w = __ldg(reinterpret_cast<const double2 *>(src) + q);
                            T *d = v + g * W + 2 * q;
                            d[0] = w.x, d[1] = w.y;
                        }
                    }
                    continue;
                }
            }
#pragma unroll
            for (int e = 0; e < W; ++e) v[g * W + e] = __ldg(src + e * st);
        }
        T *row = tab + k * (E * THREADS);
#pragma unroll
        for (int e = 0; e < E; ++e) row[e * THREADS] = v[e];
    }
    run_steps<T, E>(p, tab, last);
}

template <typename T, int W>
__device__ __forceinline__ void store_group(T *dst, const T *r) {
    if constexpr (W * sizeof(T) % 16 == 0) {
#pragma unroll
        for (int q = 0; q < static_cast<int>(W * sizeof(T) / 16); ++q) {
            if constexpr (sizeof(T) == 4)
                reinterpret_cast<float4 *>(dst)[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
            else
                reinterpret_cast<double2 *>(dst)[q] = make_double2(r[2 * q], r[2 * q + 1]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < W; ++e) dst[e] = r[e];
    }
}

// Elementwise.  W = 16 bytes of elements (W = 1: one element at a time).
// A warp takes 32*G consecutive W-element vectors at once, lane l the
// vectors l, l+32, ...: each load instruction of the warp reads 512
// contiguous bytes, and G loads per input are in flight per thread.  When
// MODE is strided, W divides the innermost extent, so a vector never
// crosses a row.  Leftover vectors go one per thread, then (dense only) the
// ragged end element by element.
template <typename T, int MODE, int G, int W>
__global__ void __launch_bounds__(THREADS) elementwise_kernel(Program p, T *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char fused_smem[];
    T *tab = reinterpret_cast<T *>(fused_smem) + threadIdx.x;
    const int axis = p.rank > 0 ? p.rank - 1 : 0;  // a vector runs along the innermost axis
    const int lane = threadIdx.x & 31;
    const int64_t n_vec = p.total / W;
    const int64_t n_wc = n_vec / (32 * G);
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (THREADS / 32);
    const int64_t gwarp = static_cast<int64_t>(blockIdx.x) * (THREADS / 32) + (threadIdx.x >> 5);
    for (int64_t wc = gwarp; wc < n_wc; wc += warps) {
        Off<MODE> off[G][MAX_INPUTS];
#pragma unroll
        for (int g = 0; g < G; ++g) decode<MODE>(p, (wc * (32 * G) + g * 32 + lane) * W, off[g]);
        T r[G * W];
        load_run<T, G, W, true, MODE>(p, off, axis, 1, tab, r);
#pragma unroll
        for (int g = 0; g < G; ++g) store_group<T, W>(out + (wc * (32 * G) + g * 32 + lane) * W, r + g * W);
    }
    const int64_t gtid = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x;
    {
        const int64_t v = n_wc * (32 * G) + gtid;
        if (v < n_vec) {
            Off<MODE> off[1][MAX_INPUTS];
            decode<MODE>(p, v * W, off[0]);
            T r[W];
            load_run<T, 1, W, true, MODE>(p, off, axis, 1, tab, r);
            store_group<T, W>(out + v * W, r);
        }
    }
    if (W > 1) {
        const int64_t i = n_vec * W + gtid;
        if (i < p.total) {
            Off<MODE> off[1][MAX_INPUTS];
            decode<MODE>(p, i, off[0]);
            T r[1];
            load_run<T, 1, 1, false, MODE>(p, off, axis, 1, tab, r);
            out[i] = r[0];
        }
    }
}

struct Span {
    int64_t len, inner, seg, nseg;  // axis extent, inner extent, segment leaves, segments per output
};

// Carry-tree push of one leaf (emit.rs emit_carry_tree_push :8129): leaf
// `count` first combines with the completed subtrees its trailing one bits
// name, the earlier subtree on the left.
template <typename T, int N>
__device__ __forceinline__ void carry_push(T (&level)[N], int64_t &count, T leaf) {
    int depth = 0;
    for (int64_t pending = count++; pending & 1; pending >>= 1, ++depth) leaf = level[depth] + leaf;
    level[depth] = leaf;
}
// Carry-tree total (emit_carry_tree_total :8179) started from `total`
// (valid when `found`): the levels from the lowest up, each on the left.
template <typename T, int N>
__device__ __forceinline__ T carry_total(const T (&level)[N], int64_t count, T total, bool found) {
    int depth = 0;
    for (int64_t remaining = count; remaining; remaining >>= 1, ++depth)
        if (remaining & 1) {
            total = found ? level[depth] + total : level[depth];
            found = true;
        }
    return found ? total : T(0);
}
// chelis_fmax_propnan fold step: NaN is sticky (tracked apart), else the
// later of equal values wins.
template <typename T>
__device__ __forceinline__ void max_push(T &best, bool &nan, T v) {
    if (isnan(v)) nan = true;
    else if (!(best > v)) best = v;
}
// Pair tree over n aligned leaves held in registers (n a power of two).
template <typename T, int N>
__device__ __forceinline__ T reg_tree(T (&r)[N]) {
#pragma unroll
    for (int width = 1; width < N; width <<= 1)
#pragma unroll
        for (int i = 0; i + width < N; i += 2 * width) r[i] = r[i] + r[i + width];
    return r[0];
}

// Reduction over the last axis (inner extent 1, so the axis's leaves are
// consecutive flat indices): one warp per span.  A pass covers 32*W
// consecutive leaves, lane l the aligned group [l*W, l*W + W): its pair
// tree, then the warp's butterfly, give the aligned subtree of the pass.
// G passes are loaded together and their subtrees paired in registers into
// one aligned subtree of G*32*W leaves, a leaf of the span's carry tree.
// What remains after the last such block, fewer than G*32*W leaves, is the
// tree's lowest part: its own passes (a small carry tree, then a ragged
// pass) give the value the total starts from.  Max keeps, per lane, the
// maximum and the last index holding it.
template <typename T, int MODE, int G, int W>
__global__ void __launch_bounds__(THREADS)
    reduce_last_kernel(Program p, int axis, int kind, Span sp, int64_t spans, T *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char fused_smem[];
    T *tab = reinterpret_cast<T *>(fused_smem) + threadIdx.x;
    const int lane = threadIdx.x & 31;
    constexpr int PASS = 32 * W, BLOCK = G * PASS;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (THREADS / 32);
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (THREADS / 32) + (threadIdx.x >> 5); w < spans;
         w += warps) {
        const int64_t o = w / sp.nseg, g0 = w % sp.nseg;
        const int64_t j0 = g0 * sp.seg;
        const int64_t n = (sp.len - j0) < sp.seg ? (sp.len - j0) : sp.seg;
        Off<MODE> base[MAX_INPUTS];
        decode<MODE>(p, o * sp.len + j0, base);
        // the group of W leaves from leaf j of the span, for each input
        auto group_off = [&](int64_t j, Off<MODE> (&off)[MAX_INPUTS]) {
#pragma unroll
            for (int k = 0; k < MAX_INPUTS; ++k)
                off[k] = base[k] + static_cast<Off<MODE>>(j) *
                                       (MODE == DENSE ? 1 : static_cast<Off<MODE>>(p.stride[k][axis]));
        };
        T result;
        if (kind == CHELIS_FUSED_REDUCE_SUM) {
            T level[48];
            int64_t count = 0;
            int64_t c0 = 0;
            for (; c0 + BLOCK <= n; c0 += BLOCK) {
                Off<MODE> off[G][MAX_INPUTS];
#pragma unroll
                for (int g = 0; g < G; ++g) group_off(c0 + g * PASS + lane * W, off[g]);
                T r[G * W];
                load_run<T, G, W, true, MODE>(p, off, axis, 1, tab, r);
                T pass[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    T q[W];
#pragma unroll
                    for (int e = 0; e < W; ++e) q[e] = r[g * W + e];
                    pass[g] = warp_tree_full(reg_tree(q));
                }
                carry_push(level, count, reg_tree(pass));
            }
            // the lowest part: full passes into a small carry tree, then a ragged pass
            T low[8];
            int64_t low_count = 0;
            T tail = T(0);
            bool has_tail = false;
            for (; c0 < n; c0 += PASS) {
                const int64_t left = n - c0;
                const int64_t mine = left - lane * W;  // this lane's valid leaves
                T q[W];
                bool valid;
                if (left >= PASS) {
                    Off<MODE> off[1][MAX_INPUTS];
                    group_off(c0 + lane * W, off[0]);
                    load_run<T, 1, W, true, MODE>(p, off, axis, 1, tab, q);
                    reg_tree(q);
                    valid = true;
                } else {
#pragma unroll
                    for (int e = 0; e < W; ++e) {
                        q[e] = T(0);
                        if (e < mine) {
                            Off<MODE> off[1][MAX_INPUTS];
                            group_off(c0 + lane * W + e, off[0]);
                            T one[1];
                            load_run<T, 1, 1, false, MODE>(p, off, axis, 1, tab, one);
                            q[e] = one[0];
                        }
                    }
#pragma unroll
                    for (int width = 1; width < W; width <<= 1)
#pragma unroll
                        for (int i = 0; i + width < W; i += 2 * width)
                            q[i] = tree_pair(q[i], i < mine, q[i + width], i + width < mine);
                    valid = mine > 0;
                }
                T s = warp_tree(q[0], valid);
                s = __shfl_sync(0xffffffffu, s, 0);
                if (left >= PASS) {
                    carry_push(low, low_count, s);
                } else {
                    tail = s;
                    has_tail = true;
                }
            }
            const bool has_low = low_count > 0 || has_tail;
            const T low_total = carry_total(low, low_count, tail, has_tail);
            result = carry_total(level, count, low_total, has_low);
            if (sp.nseg == 1) result = canon_nan(result);
        } else {
            T best = -INFINITY;
            int64_t at = -1;
            bool nan = false;
            auto take = [&](T v, int64_t j) {
                if (isnan(v)) nan = true;
                else if (!(best > v)) { best = v; at = j; }
            };
            int64_t c0 = 0;
            for (; c0 + BLOCK <= n; c0 += BLOCK) {
                Off<MODE> off[G][MAX_INPUTS];
#pragma unroll
                for (int g = 0; g < G; ++g) group_off(c0 + g * PASS + lane * W, off[g]);
                T r[G * W];
                load_run<T, G, W, true, MODE>(p, off, axis, 1, tab, r);
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int e = 0; e < W; ++e) take(r[g * W + e], c0 + g * PASS + lane * W + e);
            }
            for (; c0 < n; c0 += PASS) {
                const int64_t mine = n - c0 - lane * W;
                for (int e = 0; e < W && e < mine; ++e) {
                    Off<MODE> off[1][MAX_INPUTS];
                    group_off(c0 + lane * W + e, off[0]);
                    T one[1];
                    load_run<T, 1, 1, false, MODE>(p, off, axis, 1, tab, one);
                    take(one[0], c0 + lane * W + e);
                }
            }
            nan = __any_sync(0xffffffffu, nan);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const T ob = __shfl_xor_sync(0xffffffffu, best, off);
                const long long oa = __shfl_xor_sync(0xffffffffu, static_cast<long long>(at), off);
                if (ob > best || (ob == best && oa > at)) { best = ob; at = oa; }
            }
            result = nan ? canon_nan(T(NAN)) : best;
        }
        if (lane == 0) out[w] = result;
    }
}

// Reduction over a leading axis (inner extent > 1): one thread per span,
// walking its leaves in order, E at a time (E loads in flight); neighbouring
// threads take neighbouring inner indices, so each load is a coalesced row.
// A span starts at an aligned leaf, so each E leaves form an aligned
// subtree, paired in registers and pushed as one carry-tree leaf; the last
// n mod E leaves are the tree's lowest part.
template <typename T, int MODE, int E>
__global__ void __launch_bounds__(THREADS)
    reduce_inner_kernel(Program p, int axis, int kind, Span sp, int64_t spans, T *__restrict__ out) {
    extern __shared__ __align__(16) unsigned char fused_smem[];
    T *tab = reinterpret_cast<T *>(fused_smem) + threadIdx.x;
    const Off<MODE> dense_step = static_cast<Off<MODE>>(sp.inner);
    const int64_t outputs = spans / sp.nseg;
    for (int64_t t = static_cast<int64_t>(blockIdx.x) * THREADS + threadIdx.x; t < spans;
         t += static_cast<int64_t>(gridDim.x) * THREADS) {
        // spans ordered (segment, output) so a warp shares its segment
        const int64_t g = t / outputs, o = t % outputs;
        const int64_t hi = o / sp.inner, lo = o % sp.inner;
        const int64_t j0 = g * sp.seg;
        const int64_t n = (sp.len - j0) < sp.seg ? (sp.len - j0) : sp.seg;
        Off<MODE> base[MAX_INPUTS];
        decode<MODE>(p, (hi * sp.len + j0) * sp.inner + lo, base);
        auto at = [&](int64_t j, Off<MODE> (&off)[MAX_INPUTS]) {
#pragma unroll
            for (int k = 0; k < MAX_INPUTS; ++k)
                off[k] = base[k] + static_cast<Off<MODE>>(j) *
                                       (MODE == DENSE ? dense_step : static_cast<Off<MODE>>(p.stride[k][axis]));
        };
        T level[48];
        int64_t count = 0;
        T best = -INFINITY;
        bool nan = false;
        int64_t j = 0;
        for (; j + E <= n; j += E) {
            Off<MODE> off[1][MAX_INPUTS];
            at(j, off[0]);
            T r[E];
            load_run<T, 1, E, false, MODE>(p, off, axis, dense_step, tab, r);
            if (kind == CHELIS_FUSED_REDUCE_SUM) {
                carry_push(level, count, reg_tree(r));
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) max_push(best, nan, r[e]);
            }
        }
        T r[E];
        const int rest = static_cast<int>(n - j);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            r[e] = T(0);
            if (e < rest) {
                Off<MODE> off[1][MAX_INPUTS];
                at(j + e, off[0]);
                T one[1];
                load_run<T, 1, 1, false, MODE>(p, off, axis, dense_step, tab, one);
                r[e] = one[0];
                if (kind != CHELIS_FUSED_REDUCE_SUM) max_push(best, nan, one[0]);
            }
        }
        T result;
        if (kind == CHELIS_FUSED_REDUCE_SUM) {
#pragma unroll
            for (int width = 1; width < E; width <<= 1)
#pragma unroll
                for (int i = 0; i + width < E; i += 2 * width)
                    r[i] = tree_pair(r[i], i < rest, r[i + width], i + width < rest);
            result = carry_total(level, count, r[0], rest > 0);
            if (sp.nseg == 1) result = canon_nan(result);
        } else {
            result = nan ? canon_nan(T(NAN)) : best;
        }
        out[sp.nseg == 1 ? o : o * sp.nseg + g] = result;
    }
}

// Combine the segment results of each output: one CTA per output.  The
// segments are aligned subtrees of the output's tree (a ragged last one is
// its lowest part), so Sum is the canonical pair tree over the segment
// values: thread t folds the aligned run of c segments from t*c through a
// carry tree, then the runs pair up across lanes and warps.  Max folds
// chelis_fmax_propnan in segment order (the later of equal values wins).
constexpr int FINISH_THREADS = 256;
template <typename T>
__global__ void __launch_bounds__(FINISH_THREADS)
    finish_kernel(const T *__restrict__ part, int kind, Span sp, int64_t outputs, T *__restrict__ out) {
    __shared__ T red_v[FINISH_THREADS / 32];
    __shared__ long long red_i[FINISH_THREADS / 32];
    __shared__ int red_f[FINISH_THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t n = sp.nseg;
    int64_t c = 1;
    while (c * FINISH_THREADS < n) c <<= 1;
    for (int64_t o = blockIdx.x; o < outputs; o += gridDim.x) {
        const T *seg = part + o * n;
        const int64_t lo = threadIdx.x * c, hi = lo + c < n ? lo + c : n;
        if (kind == CHELIS_FUSED_REDUCE_SUM) {
            T level[48];
            int64_t count = 0;
            for (int64_t g = lo; g < hi; ++g) carry_push(level, count, seg[g]);
            bool valid = lo < n;
            T v = warp_tree(carry_total(level, count, T(0), false), valid);
            if (lane == 0) {
                red_v[warp] = v;
                red_f[warp] = valid;
            }
            __syncthreads();
            if (warp == 0) {
                bool wv = lane < FINISH_THREADS / 32 && red_f[lane];
                T w = wv ? red_v[lane] : T(0);
                w = warp_tree(w, wv);
                if (lane == 0) out[o] = canon_nan(w);
            }
        } else {
            T best = -INFINITY;
            long long at = -1;
            bool nan = false;
            for (int64_t g = lo; g < hi; ++g) {
                const T v = seg[g];
                if (isnan(v)) nan = true;
                else if (!(best > v)) { best = v; at = g; }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const T ob = __shfl_xor_sync(0xffffffffu, best, off);
                const long long oa = __shfl_xor_sync(0xffffffffu, at, off);
                if (ob > best || (ob == best && oa > at)) { best = ob; at = oa; }
            }
            nan = __any_sync(0xffffffffu, nan);
            if (lane == 0) {
                red_v[warp] = best;
                red_i[warp] = at;
                red_f[warp] = nan;
            }
            __syncthreads();
            if (warp == 0) {
                const bool in = lane < FINISH_THREADS / 32;
                T b = in ? red_v[lane] : T(-INFINITY);
                long long i = in ? red_i[lane] : -1;
                const bool any_nan = __any_sync(0xffffffffu, in && red_f[lane]);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    const T ob = __shfl_xor_sync(0xffffffffu, b, off);
                    const long long oi = __shfl_xor_sync(0xffffffffu, i, off);
                    if (ob > b || (ob == b && oi > i)) { b = ob; i = oi; }
                }
                if (lane == 0) out[o] = any_nan ? canon_nan(T(NAN)) : b;
            }
        }
        __syncthreads();
    }
}

}  // namespace fused

namespace {

// n / d = umulhi(n, mul) >> shr for every n < 2^31 (division by an
// invariant integer, Granlund & Montgomery 1994): with c = ceil(log2 d),
// mul = ceil(2^(31+c) / d) < 2^32 and shr = c - 1; d = 1 has mul 0.
void fast_divisor(uint32_t d, uint32_t &mul, uint32_t &shr) {
    if (d <= 1) {
        mul = 0;
        shr = 0;
        return;
    }
    int c = 0;
    while ((uint64_t(1) << c) < d) ++c;
    mul = static_cast<uint32_t>(((uint64_t(1) << (31 + c)) + d - 1) / d);
    shr = static_cast<uint32_t>(c - 1);
}

int build_program(fused::Program &p, int &mode, const chelis_fused_step *steps, int32_t n_steps,
                  const void *const *inputs, const int64_t *strides, int32_t n_inputs,
                  const int64_t *shape, int32_t rank, size_t elem) {
    using namespace fused;
    if (n_steps < 1 || n_steps > MAX_STEPS || n_inputs < 0 || n_inputs > MAX_INPUTS || rank < 0 ||
        rank > MAX_RANK)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                         "fused group admits 1..%d steps, <= %d inputs and rank <= %d", MAX_STEPS,
                         MAX_INPUTS, MAX_RANK);
    if (!steps || (n_inputs > 0 && (!inputs || (rank > 0 && !strides))) || (rank > 0 && !shape))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused group: null program, input or shape array");
    p = Program{};
    p.n_steps = n_steps;
    p.n_inputs = n_inputs;
    p.rank = rank;
    p.total = 1;
    for (int d = 0; d < rank; ++d) {
        if (shape[d] < 0) return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused group: negative extent");
        p.shape[d] = shape[d];
        p.total *= shape[d];
    }
    for (int s = 0; s < n_steps; ++s) {
        const int op = steps[s].op;
        if (op < 0 || op > CHELIS_FUSED_ROUND)
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused step %d: unknown op %d", s, op);
        if (op == CHELIS_FUSED_TRUNC_DIV)  // emit.rs:6806: integer-only, never on a float chain
            return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                             "fused step %d: trunc_div is integer-only", s);
        const bool binary = op <= CHELIS_FUSED_MIN_ELEM;
        auto valid = [&](int32_t v) { return (v >= 0 && v < n_inputs) || (v < 0 && -1 - v < s); };
        if (!valid(steps[s].a) || (binary && !valid(steps[s].b)))
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused step %d: operand out of range", s);
        p.op[s] = static_cast<uint8_t>(op);
        if (elem == 4 && rows_mode() == CHELIS_CUDA_ROWS_EXACT) {  // correctly rounded exp / log
            if (op == CHELIS_FUSED_EXP) p.op[s] = OP_EXP_CR;
            if (op == CHELIS_FUSED_LOG) p.op[s] = OP_LOG_CR;
        }
        switch (p.op[s]) {  // calls with a large register or local-memory footprint
            case CHELIS_FUSED_POW: case CHELIS_FUSED_SIN: case CHELIS_FUSED_COS: case CHELIS_FUSED_TAN:
            case OP_EXP_CR: case OP_LOG_CR:
                p.flags[s] |= HEAVY;
                break;
            default: break;
        }
    }
    // Operands: an input's row is its index; the step just before is
    // forwarded in registers; any other step is read from its row, which only
    // the steps read that way own (rows after the inputs, in step order).
    int32_t ref[MAX_STEPS][2];
    for (int s = 0; s < n_steps; ++s) {
        ref[s][0] = steps[s].a;
        ref[s][1] = steps[s].op <= CHELIS_FUSED_MIN_ELEM ? steps[s].b : steps[s].a;
        for (int i = 0; i < 2; ++i)
            if (s > 0 && ref[s][i] == -1 - (s - 1)) p.flags[s] |= i == 0 ? A_PREV : B_PREV;
    }
    int rows = n_inputs;
    for (int j = 0; j < n_steps; ++j) {
        for (int t = j + 2; t < n_steps; ++t)
            if (ref[t][0] == -1 - j || ref[t][1] == -1 - j) p.flags[j] |= STORE;
        if (p.flags[j] & STORE) p.row[j] = static_cast<uint8_t>(rows++);
    }
    p.n_rows = rows;
    for (int s = 0; s < n_steps; ++s) {
        auto row_of = [&](int32_t v) { return static_cast<uint8_t>(v >= 0 ? v : p.row[-1 - v]); };
        p.a[s] = row_of(ref[s][0]);
        p.b[s] = row_of(ref[s][1]);
    }
    bool dense = true;
    int64_t reach = 0;  // largest |offset| any input reaches
    for (int k = 0; k < n_inputs; ++k) {
        if (!inputs[k] && p.total > 0)
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused input %d is null", k);
        if ((reinterpret_cast<uintptr_t>(inputs[k]) % elem) != 0)
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused input %d is misaligned", k);
        p.in[k] = inputs[k];
        int64_t expect = 1, span = 0;
        for (int d = rank - 1; d >= 0; --d) {
            const int64_t st = strides[k * rank + d];
            p.stride[k][d] = st;
            if (shape[d] > 1 && st != expect) dense = false;
            if (shape[d] > 0) span += (st < 0 ? -st : st) * (shape[d] - 1);
            expect *= shape[d];
        }
        if (span > reach) reach = span;
    }
    const int64_t lim = int64_t(1) << 31;
    mode = dense ? DENSE : (p.total < lim && reach < lim ? STRIDED32 : STRIDED64);
    for (int d = 0; d < rank; ++d)
        fast_divisor(static_cast<uint32_t>(mode == STRIDED32 ? shape[d] : 1), p.div_mul[d], p.div_shr[d]);
    return CHELIS_CUDA_OK;
}

unsigned grid_of(int64_t units, int per_block) {
    const int64_t g = (units + per_block - 1) / per_block;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    return static_cast<unsigned>(g > cap ? cap : (g < 1 ? 1 : g));
}

// Shared-memory table for E elements per thread; E = 4 when it fits the
// default 48 KiB, else 1.
size_t table_bytes(const fused::Program &p, size_t elem, int e) {
    return static_cast<size_t>(p.n_rows + 1) * e * fused::THREADS * elem;  // + the scratch row
}
bool table_fits(const fused::Program &p, size_t elem, int e) { return table_bytes(p, elem, e) <= 48 * 1024; }

// Inputs that may be read as aligned 16-byte vectors of W elements running
// along `axis` (unit stride there, every other stride a multiple of W, base
// aligned): a vector then never straddles a row of another axis.
int32_t vector_inputs(const fused::Program &p, int mode, int axis, int w) {
    int32_t mask = 0;
    for (int k = 0; k < p.n_inputs; ++k) {
        bool ok = reinterpret_cast<uintptr_t>(p.in[k]) % 16 == 0 && p.rank > 0;
        if (mode == fused::DENSE) {
            int64_t inner = 1;  // elements from one axis step to the next
            for (int d = axis + 1; d < p.rank; ++d) inner *= p.shape[d];
            ok = ok && inner == 1;
        } else {
            ok = ok && p.stride[k][axis] == 1;
            for (int d = 0; d < p.rank; ++d)
                if (d != axis && p.shape[d] > 1 && p.stride[k][d] % w != 0) ok = false;
        }
        if (ok) mask |= 1 << k;
    }
    return mask;
}

template <typename T, int MODE, int G, int W>
void launch_ew(const fused::Program &p, T *out, cudaStream_t s) {
    const size_t smem = table_bytes(p, sizeof(T), G * W);
    const int64_t units = p.total / W / (32 * G) * 32 + 128;  // threads of the main loop + leftovers
    fused::elementwise_kernel<T, MODE, G, W>
        <<<grid_of(units, fused::THREADS), fused::THREADS, smem, s>>>(p, out);
}

template <typename T, int G, int W>
void launch_ew_mode(const fused::Program &p, int mode, T *out, cudaStream_t s) {
    using namespace fused;
    if (mode == DENSE) launch_ew<T, DENSE, G, W>(p, out, s);
    else if (mode == STRIDED32) launch_ew<T, STRIDED32, G, W>(p, out, s);
    else launch_ew<T, STRIDED64, G, W>(p, out, s);
}

template <typename T>
int launch_elementwise(fused::Program &p, int mode, T *out, cudaStream_t s) {
    using namespace fused;
    // 16-byte vectors of W elements along the innermost axis (a strided
    // vector must not cross a row), two per thread when the table fits
    constexpr int W = 16 / sizeof(T);
    const bool vec_ok = reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                        (mode == DENSE || (p.rank > 0 && p.shape[p.rank - 1] % W == 0));
    p.vec_mask = vec_ok ? vector_inputs(p, mode, p.rank > 0 ? p.rank - 1 : 0, W) : 0;
    if (vec_ok && table_fits(p, sizeof(T), 2 * W)) launch_ew_mode<T, 2, W>(p, mode, out, s);
    else if (vec_ok && table_fits(p, sizeof(T), W)) launch_ew_mode<T, 1, W>(p, mode, out, s);
    else launch_ew_mode<T, 1, 1>(p, mode, out, s);
    g_launches++;
    CHELIS_LAUNCH_CHECK("fused::elementwise_kernel");
    return CHELIS_CUDA_OK;
}

template <typename T, int MODE, int G, int W>
void launch_last(const fused::Program &p, int axis, int kind, fused::Span sp, int64_t spans, T *dst,
                 cudaStream_t s) {
    using namespace fused;
    reduce_last_kernel<T, MODE, G, W><<<grid_of(spans, THREADS / 32), THREADS,
                                        table_bytes(p, sizeof(T), G * W), s>>>(p, axis, kind, sp, spans,
                                                                               dst);
}

template <typename T, int MODE, int E>
void launch_inner(const fused::Program &p, int axis, int kind, fused::Span sp, int64_t spans, T *dst,
                  cudaStream_t s) {
    using namespace fused;
    reduce_inner_kernel<T, MODE, E><<<grid_of(spans, THREADS), THREADS, table_bytes(p, sizeof(T), E),
                                      s>>>(p, axis, kind, sp, spans, dst);
}

template <typename T, int MODE>
void launch_red(fused::Program &p, int axis, int kind, fused::Span sp, int64_t spans, T *dst,
                cudaStream_t s) {
    constexpr int W = 16 / sizeof(T);
    if (sp.inner == 1) {
        // groups of W leaves along the axis; vectors where the axis has unit
        // stride and the rows start aligned
        const bool rows_aligned = MODE != fused::DENSE || sp.len % W == 0;
        p.vec_mask = rows_aligned ? vector_inputs(p, MODE, axis, W) : 0;
        if (table_fits(p, sizeof(T), 4 * W)) launch_last<T, MODE, 4, W>(p, axis, kind, sp, spans, dst, s);
        else if (table_fits(p, sizeof(T), W)) launch_last<T, MODE, 1, W>(p, axis, kind, sp, spans, dst, s);
        else launch_last<T, MODE, 1, 1>(p, axis, kind, sp, spans, dst, s);
    } else {
        p.vec_mask = 0;
        constexpr int E = 32 / sizeof(T);  // leaves in flight per thread
        if (table_fits(p, sizeof(T), E)) launch_inner<T, MODE, E>(p, axis, kind, sp, spans, dst, s);
        else launch_inner<T, MODE, 1>(p, axis, kind, sp, spans, dst, s);
    }
}

template <typename T>
int launch_reduce(fused::Program p, int mode, int axis, int kind, fused::Span sp, int64_t outputs,
                  T *dst, cudaStream_t s) {
    using namespace fused;
    const int64_t spans = outputs * sp.nseg;
    if (mode == DENSE) launch_red<T, DENSE>(p, axis, kind, sp, spans, dst, s);
    else if (mode == STRIDED32) launch_red<T, STRIDED32>(p, axis, kind, sp, spans, dst, s);
    else launch_red<T, STRIDED64>(p, axis, kind, sp, spans, dst, s);
    g_launches++;
    CHELIS_LAUNCH_CHECK(sp.inner == 1 ? "fused::reduce_last_kernel" : "fused::reduce_inner_kernel");
    return CHELIS_CUDA_OK;
}

template <typename T>
int fused_reduce_t(const fused::Program &p, int mode, int kind, int axis, int64_t outputs, T *out,
                   cudaStream_t s) {
    using namespace fused;
    Span sp{};
    sp.len = p.shape[axis];
    sp.inner = 1;
    for (int d = axis + 1; d < p.rank; ++d) sp.inner *= p.shape[d];
    // Split the axis into aligned power-of-two segments when the outputs
    // alone cannot fill the GPU: a warp (last axis) or a thread (leading
    // axis) per segment, then finish_kernel combines each output's segments.
    const int64_t want = static_cast<int64_t>(sm_count()) * (sp.inner == 1 ? 64 : 2048);
    const int64_t min_seg = sp.inner == 1 ? 1024 : 64;
    sp.seg = sp.len;
    sp.nseg = 1;
    if (outputs < want && sp.len > 2 * min_seg) {
        const int64_t per = (sp.len * outputs + want - 1) / want;  // leaves per unit to fill the GPU
        int64_t seg = min_seg;
        while (seg < per) seg <<= 1;
        if (seg < sp.len) {
            sp.seg = seg;
            sp.nseg = (sp.len + seg - 1) / seg;
        }
    }
    if (sp.nseg == 1) return launch_reduce<T>(p, mode, axis, kind, sp, outputs, out, s);
    void *part = nullptr;
    CHELIS_TRY(scratch_alloc(&part, static_cast<size_t>(outputs * sp.nseg) * sizeof(T), s));
    int rc = launch_reduce<T>(p, mode, axis, kind, sp, outputs, static_cast<T *>(part), s);
    if (rc == CHELIS_CUDA_OK) {
        const int64_t blocks = outputs < 65535 ? outputs : 65535;
        finish_kernel<T><<<static_cast<unsigned>(blocks), FINISH_THREADS, 0, s>>>(
            static_cast<const T *>(part), kind, sp, outputs, out);
        g_launches++;
        rc = check_cuda(cudaGetLastError(), "fused::finish_kernel");
    }
    scratch_free(part, s);
    return rc;
}

}  // namespace
}  // namespace chelis

using namespace chelis;

namespace chelis {
namespace fusedjit {
int try_elementwise(bool f32, const chelis_fused_step *steps, int n_steps, const fused::Program &p,
                    int mode, void *out, cudaStream_t s);
int try_reduce(bool f32, const chelis_fused_step *steps, int n_steps, const fused::Program &p,
               int mode, int axis, int kind, int64_t outputs, void *out, cudaStream_t s);
}  // namespace fusedjit
}  // namespace chelis

extern "C" int chelis_cuda_fused_elementwise(int32_t dtype, const chelis_fused_step *steps,
                                             int32_t n_steps, const void *const *inputs,
                                             const int64_t *strides, int32_t n_inputs,
                                             const int64_t *shape, int32_t rank, void *out) {
    if (dtype != CHELIS_DTYPE_F32 && dtype != CHELIS_DTYPE_F64)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "fused group admits f32 and f64");
    const size_t elem = dtype == CHELIS_DTYPE_F32 ? 4 : 8;
    fused::Program p;
    int mode = 0;
    CHELIS_TRY(build_program(p, mode, steps, n_steps, inputs, strides, n_inputs, shape, rank, elem));
    if (p.total == 0) return CHELIS_CUDA_OK;
    if (!out) return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused output is null");
    if (reinterpret_cast<uintptr_t>(out) % elem != 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused output is misaligned");
    cudaStream_t s = current_stream();
    // the chain compiled for itself (fused_jit.cu) where it fits that form
    const int jit = fusedjit::try_elementwise(dtype == CHELIS_DTYPE_F32, steps, n_steps, p, mode, out, s);
    if (jit >= 0) return jit;
    return dtype == CHELIS_DTYPE_F32 ? launch_elementwise<float>(p, mode, static_cast<float *>(out), s)
                                     : launch_elementwise<double>(p, mode, static_cast<double *>(out), s);
}

extern "C" int chelis_cuda_fused_reduce(int32_t dtype, const chelis_fused_step *steps,
                                        int32_t n_steps, const void *const *inputs,
                                        const int64_t *strides, int32_t n_inputs,
                                        const int64_t *shape, int32_t rank, int32_t axis,
                                        int32_t kind, void *out) {
    if (dtype != CHELIS_DTYPE_F32 && dtype != CHELIS_DTYPE_F64)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "fused group admits f32 and f64");
    if (kind != CHELIS_FUSED_REDUCE_SUM && kind != CHELIS_FUSED_REDUCE_MAX)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused reduce: unknown kind %d", kind);
    if (rank < 1 || axis < 0 || axis >= rank)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused reduce: axis %d out of range for rank %d",
                         axis, rank);
    const size_t elem = dtype == CHELIS_DTYPE_F32 ? 4 : 8;
    fused::Program p;
    int mode = 0;
    CHELIS_TRY(build_program(p, mode, steps, n_steps, inputs, strides, n_inputs, shape, rank, elem));
    const char *prim = dtype == CHELIS_DTYPE_F32 ? "f32" : "f64";
    if (kind == CHELIS_FUSED_REDUCE_MAX && p.shape[axis] == 0)  // emit.rs:9652-9665
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in max_reduce at %s", prim);
    int64_t outputs = 1;
    for (int d = 0; d < rank; ++d)
        if (d != axis) outputs *= p.shape[d];
    if (outputs == 0) return CHELIS_CUDA_OK;
    if (!out) return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused output is null");
    if (reinterpret_cast<uintptr_t>(out) % elem != 0)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "fused output is misaligned");
    cudaStream_t s = current_stream();
    if (p.shape[axis] == 0)  // an empty Sum is zero (the C lane's zero fill)
        return check_cuda(cudaMemsetAsync(out, 0, static_cast<size_t>(outputs) * elem, s),
                          "cudaMemsetAsync(fused_reduce)");
    const int jit = fusedjit::try_reduce(dtype == CHELIS_DTYPE_F32, steps, n_steps, p, mode, axis, kind,
                                         outputs, out, s);
    if (jit >= 0) return jit;
    return dtype == CHELIS_DTYPE_F32
               ? fused_reduce_t<float>(p, mode, kind, axis, outputs, static_cast<float *>(out), s)
               : fused_reduce_t<double>(p, mode, kind, axis, outputs, static_cast<double *>(out), s);
}
