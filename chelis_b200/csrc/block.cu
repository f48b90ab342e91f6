// block.cu -- the pre-LN transformer block, forward and reverse mode, f32.
//
//   h1 = layer_norm(x; g1, b1)                      (tier2.rs:1248-1375)
//   [q k v] = h1 . Wqkv                              (three matmuls, fused)
//   per head: p = softmax(where(causal, (q.k^T)*scale, -inf)); o = p.v
//                                                   (spec 05 section 4.7)
//   x2 = x + o . Wo
//   h2 = layer_norm(x2; g2, b2)
//   y  = x2 + gelu(h2 . W1) . W2                    (gelu = m(x)*Phi(x),
//                                                    spec 05 section 3.3)
// and the vector-Jacobian product for an upstream cotangent dy: dx and the
// gradients of Wqkv, Wo, W1, W2, g1, b1, g2, b2 (grad.rs adjoint graphs;
// the matmul adjoint is a matmul with a transposed operand, [05-OP-51]).
//
// Every matmul runs on the tcgen05 3xTF32 kernel (chelis_cuda_sgemm); the
// row work runs on the kernels below.  Attention runs on the fused kernels
// of attention.cu (scores kept in tensor memory, reverse mode recomputed
// from the saved log-sum-exp) for head dims 32 and 64 in the FAST rows
// mode; otherwise (EXACT rows mode, other head dims) it is materialised per
// head ([B*H, S, S] scores), the unfused form of the reference graph.
#include <cuda_runtime.h>

#include <atomic>

#include "common.cuh"
#include "gelu.cuh"

namespace chelis {

extern std::atomic<uint64_t> g_launches;
int rows_mode();

namespace block {

using chain::Red;
using chain::at;
using chain::canon;
using chain::div_;
using chain::exp_;
using chain::ld4;
using chain::load4;
using chain::quad;
using chain::stage;
using chain::tree4;
using chain::tree_parts;

// hi = RN_tf32(v), lo = RN_tf32(v - hi) (lo = 0 for non-finite v) of four
// results, stored as element group i of the split: the transformer step's
// producers write the split of a tensor that the matmuls only read split.
__device__ __forceinline__ void split_store(float4 *__restrict__ hi, float4 *__restrict__ lo, int64_t i,
                                            const float (&v)[4]) {
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        h[j] = tf32x3::rna_tf32(v[j]);
        l[j] = isfinite(v[j]) ? tf32x3::rna_tf32(__fsub_rn(v[j], h[j])) : 0.0f;
    }
    hi[i] = make_float4(h[0], h[1], h[2], h[3]);
    lo[i] = make_float4(l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------------------
// layer_norm forward, saving (mean, sqrt(var + eps)) per row
// ---------------------------------------------------------------------------
template <int T, int NC, bool EXACT>
__global__ void __launch_bounds__(T) ln_fwd_kernel(const float *__restrict__ x,
                                                   const float *__restrict__ gamma,
                                                   const float *__restrict__ beta, float eps,
                                                   float *__restrict__ y, float2 *__restrict__ stats,
                                                   int64_t rows, int n, float *__restrict__ yhi,
                                                   float *__restrict__ ylo) {
    extern __shared__ __align__(16) float smem[];
    float *sg = smem, *sb = sg + NC * 4 * T;
    Red<T, NC> rs{sb + NC * 4 * T};
    const float hf = static_cast<float>(n), rh = __fdiv_rn(1.0f, hf);
    const bool vec = (n % 4 == 0);
    stage<NC, T>(sg, gamma, n);
    stage<NC, T>(sb, beta, n);
    __syncthreads();
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float v[NC][4];
        load4<NC, T>(v, x + r * n, n, vec);
        const float mean = div_<EXACT>(tree4<T, NC>(v, n, rs), hf, rh);
        float part[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = __fsub_rn(v[c][i], mean);
            part[c] = quad(__fmul_rn(v[c][0], v[c][0]), __fmul_rn(v[c][1], v[c][1]),
                           __fmul_rn(v[c][2], v[c][2]), __fmul_rn(v[c][3], v[c][3]),
                           n - (c * 4 * T + 4 * static_cast<int>(threadIdx.x)));
        }
        const float var = div_<EXACT>(tree_parts<T, NC>(part, n, rs), hf, rh);
        const float d = __fsqrt_rn(__fadd_rn(var, eps));
        const float rd = __fdiv_rn(1.0f, d);
        if (threadIdx.x == 0) stats[r] = make_float2(mean, d);
        if (y == nullptr && yhi == nullptr) continue;  // statistics only (the standalone layer_norm adjoint)
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4 g4 = ld4<T>(sg, c), b4 = ld4<T>(sb, c);
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            float o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                o[i] = canon(__fadd_rn(__fmul_rn(div_<EXACT>(v[c][i], d, rd), at(g4, i)), at(b4, i)));
            if (yhi != nullptr) {
                // the tf32 split of y only (n % 32 == 0: the split cache's
                // [rows][n] layout), y itself is read through it alone
                if (e0 + 3 < n) split_store(reinterpret_cast<float4 *>(yhi + r * n),
                                            reinterpret_cast<float4 *>(ylo + r * n), e0 / 4, o);
                continue;
            }
            float *yr = y + r * n;
            if (vec && e0 + 3 < n) *reinterpret_cast<float4 *>(yr + e0) = make_float4(o[0], o[1], o[2], o[3]);
            else
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (e0 + i < n) yr[e0 + i] = o[i];
        }
    }
}

// ---------------------------------------------------------------------------
// layer_norm adjoint (the LN part of the chain adjoint): dx = resid + dLN,
// per-CTA dgamma / dbeta partials
// ---------------------------------------------------------------------------
template <int T, int NC, bool EXACT>
__global__ void __launch_bounds__(T) ln_bwd_kernel(const float *__restrict__ x,
                                                   const float *__restrict__ dy,
                                                   const float2 *__restrict__ stats,
                                                   const float *__restrict__ gamma,
                                                   const float *__restrict__ resid,
                                                   float *__restrict__ dx, float *__restrict__ pg_out,
                                                   float *__restrict__ pb_out, int64_t rows, int n,
                                                   int rows_per_cta) {
    extern __shared__ __align__(16) float smem[];
    constexpr int L = NC * 4 * T;
    float *sg = smem, *pg = sg + L, *pb = pg + L;
    Red<T, NC> rs{pb + L};
    const float hf = static_cast<float>(n), rh = __fdiv_rn(1.0f, hf);
    const bool vec = (n % 4 == 0);
    stage<NC, T>(sg, gamma, n);
    stage<NC, T>(pg, nullptr, n);
    stage<NC, T>(pb, nullptr, n);
    __syncthreads();
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
    int64_t r1 = r0 + rows_per_cta;
    if (r1 > rows) r1 = rows;
    for (int64_t r = r0; r < r1; ++r) {
        float c_[NC][4], g_[NC][4];
        load4<NC, T>(c_, x + r * n, n, vec);
        load4<NC, T>(g_, dy + r * n, n, vec);
        const float2 st = stats[r];
        const float mean = st.x, d = st.y;
        const float rd = __fdiv_rn(1.0f, d);
        const float two_d = __fmul_rn(2.0f, d);
        const float r2d = __fdiv_rn(1.0f, two_d);
        float part[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const float4 gm = ld4<T>(sg, c);
            float4 pg4 = ld4<T>(pg, c), pb4 = ld4<T>(pb, c);
            float dt[4], dyn[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float cc = __fsub_rn(c_[c][i], mean);
                c_[c][i] = cc;
                const float nn = div_<EXACT>(cc, d, rd);
                const float g = g_[c][i];
                dyn[i] = __fmul_rn(g, nn);
                const float dn = __fmul_rn(g, at(gm, i));
                dt[i] = div_<EXACT>(-div_<EXACT>(__fmul_rn(dn, nn), d, rd), two_d, r2d);
                g_[c][i] = div_<EXACT>(dn, d, rd);  // dc1
            }
            pg4.x = __fadd_rn(pg4.x, dyn[0]); pg4.y = __fadd_rn(pg4.y, dyn[1]);
            pg4.z = __fadd_rn(pg4.z, dyn[2]); pg4.w = __fadd_rn(pg4.w, dyn[3]);
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            float dyv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) dyv[i] = (e0 + i < n) ? dy[r * n + e0 + i] : 0.0f;
            pb4.x = __fadd_rn(pb4.x, dyv[0]); pb4.y = __fadd_rn(pb4.y, dyv[1]);
            pb4.z = __fadd_rn(pb4.z, dyv[2]); pb4.w = __fadd_rn(pb4.w, dyv[3]);
            reinterpret_cast<float4 *>(pg)[c * T + threadIdx.x] = pg4;
            reinterpret_cast<float4 *>(pb)[c * T + threadIdx.x] = pb4;
            part[c] = quad(dt[0], dt[1], dt[2], dt[3], n - e0);
        }
        const float ds2 = div_<EXACT>(tree_parts<T, NC>(part, n, rs), hf, rh);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            float m4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pr = __fmul_rn(ds2, c_[c][i]);
                const float dc = __fadd_rn(__fadd_rn(pr, pr), g_[c][i]);
                g_[c][i] = dc;
                m4[i] = -dc;
            }
            part[c] = quad(m4[0], m4[1], m4[2], m4[3], n - (c * 4 * T + 4 * static_cast<int>(threadIdx.x)));
        }
        const float ds1 = div_<EXACT>(tree_parts<T, NC>(part, n, rs), hf, rh);
        float *dxr = dx + r * n;
        const float *rr = resid ? resid + r * n : nullptr;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int e0 = c * 4 * T + 4 * threadIdx.x;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (e0 + i < n) {
                    float v = __fadd_rn(ds1, g_[c][i]);
                    if (rr) v = __fadd_rn(rr[e0 + i], v);
                    dxr[e0 + i] = canon(v);
                }
            }
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n; e += T) {
        pg_out[static_cast<int64_t>(blockIdx.x) * n + e] = pg[e];
        pb_out[static_cast<int64_t>(blockIdx.x) * n + e] = pb[e];
    }
}

// ---------------------------------------------------------------------------
// causal softmax over [rows = BH*S, S] in place: p = softmax(where(j <= i,
// s*scale, -inf)), i = row % S.  Masked entries become exact +0.
// ---------------------------------------------------------------------------
template <int T, int NC, bool EXACT>
__global__ void __launch_bounds__(T) causal_softmax_kernel(float *__restrict__ s, int64_t rows,
                                                           int n, float scale) {
    __shared__ float redbuf[2 * (NC * (T / 32) + 8)];
    Red<T, NC> rs{redbuf};
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const int qi = static_cast<int>(r % n);
        float v[NC][4];
        load4<NC, T>(v, s + r * n, n, true);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int e = c * 4 * T + 4 * threadIdx.x + i;
                v[c][i] = (e <= qi) ? __fmul_rn(v[c][i], scale) : -INFINITY;
            }
        const float mx = chain::row_max<T, NC>(v, n, rs);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = exp_<EXACT>(__fsub_rn(v[c][i], mx));
        const float z = tree4<T, NC>(v, n, rs);
        const float rz = __fdiv_rn(1.0f, z);
        float *o = s + r * n;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            float w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = canon(div_<EXACT>(v[c][i], z, rz));
            if (e0 < n) *reinterpret_cast<float4 *>(o + e0) = make_float4(w[0], w[1], w[2], w[3]);
        }
    }
}

// dS = (P * (dP - sum(dP * P))) * scale, in place over dP
template <int T, int NC>
__global__ void __launch_bounds__(T) softmax_scaled_bwd_kernel(const float *__restrict__ p,
                                                               float *__restrict__ dp,
                                                               int64_t rows, int n, float scale) {
    __shared__ float redbuf[2 * (NC * (T / 32) + 8)];
    Red<T, NC> rs{redbuf};
    for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
        float y[NC][4], g[NC][4], gy[NC][4];
        load4<NC, T>(y, p + r * n, n, true);
        load4<NC, T>(g, dp + r * n, n, true);
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < 4; ++i) gy[c][i] = __fmul_rn(g[c][i], y[c][i]);
        const float q = tree4<T, NC>(gy, n, rs);
        float *o = dp + r * n;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int e0 = c * 4 * T + 4 * threadIdx.x;
            float w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                w[i] = canon(__fmul_rn(__fmul_rn(y[c][i], __fsub_rn(g[c][i], q)), scale));
            if (e0 < n) *reinterpret_cast<float4 *>(o + e0) = make_float4(w[0], w[1], w[2], w[3]);
        }
    }
}

// gelu and its adjoint (gelu.cuh, shared with the GEMM epilogues)
__global__ void gelu_fwd_kernel(const float *__restrict__ u, float *__restrict__ g, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        g[i] = gelu::value(u[i]);
}

__global__ void gelu_bwd_kernel(const float *__restrict__ u, float *__restrict__ dg, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dg[i] = canon(__fmul_rn(dg[i], gelu::derivative(u[i])));
}

// The same two maps written straight into the tf32 split of their result
// (hi = RN_tf32(v), lo = RN_tf32(v - hi), lo = 0 for non-finite v: the split
// cache's layout for a row-major [rows][F] tensor when F % 32 == 0), four
// elements per thread: the result itself is only ever read through its
// split, so it is never stored, and the matmuls that consume it skip their
// split pre-pass.
__global__ void gelu_fwd_split_kernel(const float4 *__restrict__ u, float4 *__restrict__ hi,
                                      float4 *__restrict__ lo, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 x = u[i];
        const float v[4] = {gelu::value(x.x), gelu::value(x.y), gelu::value(x.z), gelu::value(x.w)};
        split_store(hi, lo, i, v);
    }
}

__global__ void gelu_bwd_split_kernel(const float4 *__restrict__ u, const float4 *__restrict__ dg,
                                      float4 *__restrict__ hi, float4 *__restrict__ lo, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 x = u[i], d = __ldcs(dg + i);
        const float v[4] = {canon(__fmul_rn(d.x, gelu::derivative(x.x))),
                            canon(__fmul_rn(d.y, gelu::derivative(x.y))),
                            canon(__fmul_rn(d.z, gelu::derivative(x.z))),
                            canon(__fmul_rn(d.w, gelu::derivative(x.w)))};
        split_store(hi, lo, i, v);
    }
}

// y = a + b
__global__ void add_kernel(const float *__restrict__ a, const float *__restrict__ b,
                           float *__restrict__ y, int64_t n4) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 p = reinterpret_cast<const float4 *>(a)[i];
        const float4 q = reinterpret_cast<const float4 *>(b)[i];
        reinterpret_cast<float4 *>(y)[i] = make_float4(__fadd_rn(p.x, q.x), __fadd_rn(p.y, q.y),
                                                       __fadd_rn(p.z, q.z), __fadd_rn(p.w, q.w));
    }
}

// [B, S, 3, H, D] <-> three [B, H, S, D]; dir 0: split, 1: merge
__global__ void qkv_permute_kernel(float *__restrict__ qkv, float *__restrict__ q,
                                   float *__restrict__ k, float *__restrict__ v, int b_, int s_,
                                   int h_, int d4, int dir) {
    const int64_t total = static_cast<int64_t>(b_) * s_ * 3 * h_ * d4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i;
        const int dd = static_cast<int>(t % d4); t /= d4;
        const int hh = static_cast<int>(t % h_); t /= h_;
        const int w = static_cast<int>(t % 3); t /= 3;
        const int ss = static_cast<int>(t % s_); t /= s_;
        const int bb = static_cast<int>(t);
        float *dst = (w == 0 ? q : w == 1 ? k : v);
        const int64_t o = ((static_cast<int64_t>(bb) * h_ + hh) * s_ + ss) * d4 + dd;
        float4 *pa = reinterpret_cast<float4 *>(qkv) + i;
        float4 *pb = reinterpret_cast<float4 *>(dst) + o;
        if (dir == 0) *pb = *pa;
        else *pa = *pb;
    }
}

// [B, S, 3, H, D] -> q, k, v [B, H, S, D] f32 plus hi / lo (tf32 split) of
// each, the operand copies the fused attention kernels stream with TMA
__global__ void qkv_heads_split_kernel(const float *__restrict__ qkv, float *__restrict__ q,
                                       float *__restrict__ k, float *__restrict__ v,
                                       float *__restrict__ hl, int64_t act, int b_, int s_, int h_,
                                       int d4) {
    const int64_t total = static_cast<int64_t>(b_) * s_ * 3 * h_ * d4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i;
        const int dd = static_cast<int>(t % d4); t /= d4;
        const int hh = static_cast<int>(t % h_); t /= h_;
        const int w = static_cast<int>(t % 3); t /= 3;
        const int ss = static_cast<int>(t % s_); t /= s_;
        const int bb = static_cast<int>(t);
        const int64_t o = ((static_cast<int64_t>(bb) * h_ + hh) * s_ + ss) * d4 + dd;
        const float4 x = reinterpret_cast<const float4 *>(qkv)[i];
        reinterpret_cast<float4 *>(w == 0 ? q : w == 1 ? k : v)[o] = x;
        uint32_t hi[4], lo[4];
        attn::split_tf32(x.x, hi[0], lo[0]);
        attn::split_tf32(x.y, hi[1], lo[1]);
        attn::split_tf32(x.z, hi[2], lo[2]);
        attn::split_tf32(x.w, hi[3], lo[3]);
        // hl: [q_hi, q_lo, k_hi, k_lo, v_hi, v_lo], act floats each
        float *base = hl + 2 * w * act;
        reinterpret_cast<uint4 *>(base)[o] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        reinterpret_cast<uint4 *>(base + act)[o] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// [B, S, H, D] -> hi / lo in [B, H, S, D]
__global__ void rows_heads_split_kernel(const float *__restrict__ x, float *__restrict__ hi,
                                        float *__restrict__ lo, int b_, int s_, int h_, int d4) {
    const int64_t total = static_cast<int64_t>(b_) * s_ * h_ * d4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i;
        const int dd = static_cast<int>(t % d4); t /= d4;
        const int hh = static_cast<int>(t % h_); t /= h_;
        const int ss = static_cast<int>(t % s_); t /= s_;
        const int bb = static_cast<int>(t);
        const int64_t o = ((static_cast<int64_t>(bb) * h_ + hh) * s_ + ss) * d4 + dd;
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        uint32_t h4[4], l4[4];
        attn::split_tf32(v.x, h4[0], l4[0]);
        attn::split_tf32(v.y, h4[1], l4[1]);
        attn::split_tf32(v.z, h4[2], l4[2]);
        attn::split_tf32(v.w, h4[3], l4[3]);
        reinterpret_cast<uint4 *>(hi)[o] = make_uint4(h4[0], h4[1], h4[2], h4[3]);
        reinterpret_cast<uint4 *>(lo)[o] = make_uint4(l4[0], l4[1], l4[2], l4[3]);
    }
}

// [B, H, S, D] <-> [B, S, H, D]; dir 0: heads -> rows, 1: rows -> heads
__global__ void heads_permute_kernel(float *__restrict__ hsd, float *__restrict__ shd, int b_,
                                     int s_, int h_, int d4, int dir) {
    const int64_t total = static_cast<int64_t>(b_) * s_ * h_ * d4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t t = i;
        const int dd = static_cast<int>(t % d4); t /= d4;
        const int hh = static_cast<int>(t % h_); t /= h_;
        const int ss = static_cast<int>(t % s_); t /= s_;
        const int bb = static_cast<int>(t);
        const int64_t o = ((static_cast<int64_t>(bb) * h_ + hh) * s_ + ss) * d4 + dd;
        float4 *ps = reinterpret_cast<float4 *>(shd) + i;
        float4 *ph = reinterpret_cast<float4 *>(hsd) + o;
        if (dir == 0) *ps = *ph;
        else *ph = *ps;
    }
}

}  // namespace block
}  // namespace chelis

// ---------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------
using namespace chelis;

namespace {

struct BlockDims {
    int64_t B, S, D, H, Dh, F, BS, BH;
};

int block_dims(const chelis_block_params *p, BlockDims &d) {
    if (!p || p->batch <= 0 || p->seq <= 0 || p->d_model <= 0 || p->heads <= 0 || p->d_ff <= 0 ||
        p->d_model % p->heads)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in transformer_block at i64");
    d.B = p->batch; d.S = p->seq; d.D = p->d_model; d.H = p->heads; d.F = p->d_ff;
    d.Dh = d.D / d.H; d.BS = d.B * d.S; d.BH = d.B * d.H;
    if (d.D > 8192 || d.S > 8192 || d.D % 4 || d.Dh % 4 || d.S % 4 || d.F % 4)
        return set_error(CHELIS_CUDA_ERR_UNSUPPORTED,
                         "transformer block admits d_model, seq <= 8192 and d_model, seq, d_ff "
                         "and the head dim multiples of 4");
    return CHELIS_CUDA_OK;
}

// workspace layout in floats
// (P, dP: [B*H, S, S] of the materialised attention path, taken from the
// pool by chelis_cuda_block_step only when that path runs; hl: hi / lo
// copies of q, k, v, dO for the fused path; lse, dsum: [B*H, S].)
// The 3xTF32 hi / lo copies of every matmul operand, made once per step
// (each tensor feeds two matmuls, forward and reverse, and its row-major
// split serves both orientations when its row length is a multiple of 32).
enum SplitTensor { S_H1, S_WQKV, S_O, S_WO, S_H2, S_W1, S_G, S_W2, S_DY, S_DG, S_DX2, S_DQKV, S_COUNT };

struct Ws {
    float *h1, *qkv, *q, *k, *v, *P, *oh, *o, *x2, *h2, *u, *g, *dg, *dh2, *dx2, *dO, *doh, *dP,
        *dq, *dk, *dv, *dqkv, *dh1, *part, *hl, *lse, *dsum;
    float2 *st1, *st2;
    float *shi[S_COUNT], *slo[S_COUNT];  // null when the dims do not admit cached splits
    int64_t total;
};

bool split_cache_dims(const BlockDims &d) { return d.D % 32 == 0 && d.F % 32 == 0; }

int ln_grid() { return sm_count() * 2; }

Ws carve(const BlockDims &d, float *base) {
    Ws w{};
    int64_t off = 0;
    auto take = [&](int64_t n) {
        float *p = base ? base + off : nullptr;
        off += (n + 63) / 64 * 64;
        return p;
    };
    const int64_t act = d.BS * d.D, ff = d.BS * d.F;
    w.h1 = take(act); w.qkv = take(3 * act); w.q = take(act); w.k = take(act); w.v = take(act);
    w.oh = take(act); w.o = take(act); w.x2 = take(act); w.h2 = take(act);
    w.u = take(ff); w.g = take(ff); w.dg = take(ff); w.dh2 = take(act); w.dx2 = take(act);
    w.dO = take(act); w.doh = take(act); w.dq = take(act); w.dk = take(act);
    w.dv = take(act); w.dqkv = take(3 * act); w.dh1 = take(act);
    w.hl = take(8 * act); w.lse = take(d.BH * d.S); w.dsum = take(d.BH * d.S);
    w.part = take(2 * static_cast<int64_t>(ln_grid()) * d.D);
    w.st1 = reinterpret_cast<float2 *>(take(2 * d.BS));
    w.st2 = reinterpret_cast<float2 *>(take(2 * d.BS));
    if (split_cache_dims(d)) {
        const int64_t n[S_COUNT] = {act, 3 * d.D * d.D, act, d.D * d.D, act, d.D * d.F, ff,
                                    d.F * d.D, act, ff, act, 3 * act};
        for (int i = 0; i < S_COUNT; ++i) {
            w.shi[i] = take(n[i]);
            w.slo[i] = take(n[i]);
        }
    }
    w.total = off;
    return w;
}

unsigned grid_for(int64_t n, int per = 256) {
    int64_t g = (n + per - 1) / per;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    return static_cast<unsigned>(g > cap ? cap : (g < 1 ? 1 : g));
}

template <typename F>
int with_rows_nc(int64_t n, F &&f) {
    const int64_t c = (n + 1023) / 1024;
    if (c <= 1) return f(std::integral_constant<int, 1>());
    if (c <= 2) return f(std::integral_constant<int, 2>());
    if (c <= 4) return f(std::integral_constant<int, 4>());
    return f(std::integral_constant<int, 8>());
}

template <typename K>
int smem_attr(K k, size_t bytes) {
    return check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(bytes)),
                      "cudaFuncSetAttribute(block)");
}

int ln_fwd(const float *x, const float *g, const float *b, float eps, float *y, float2 *st,
           int64_t rows, int64_t n, cudaStream_t s, float *yhi = nullptr, float *ylo = nullptr) {
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    return with_rows_nc(n, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const size_t smem = 2 * NC * 1024 * sizeof(float) + 2 * (NC * 8 + 8) * sizeof(float);
        const unsigned grid = static_cast<unsigned>(rows < sm_count() * 8 ? rows : sm_count() * 8);
        if (exact) {
            CHELIS_TRY(smem_attr(block::ln_fwd_kernel<256, NC, true>, smem));
            block::ln_fwd_kernel<256, NC, true><<<grid, 256, smem, s>>>(x, g, b, eps, y, st, rows, static_cast<int>(n), yhi, ylo);
        } else {
            CHELIS_TRY(smem_attr(block::ln_fwd_kernel<256, NC, false>, smem));
            block::ln_fwd_kernel<256, NC, false><<<grid, 256, smem, s>>>(x, g, b, eps, y, st, rows, static_cast<int>(n), yhi, ylo);
        }
        g_launches++;
        CHELIS_LAUNCH_CHECK("ln_fwd_kernel");
        return CHELIS_CUDA_OK;
    });
}

int ln_bwd(const float *x, const float *dy, const float2 *st, const float *g, const float *resid,
           float *dx, float *part, float *dgamma, float *dbeta, int64_t rows, int64_t n,
           cudaStream_t s) {
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    int grid = ln_grid();
    if (grid > rows) grid = static_cast<int>(rows);
    const int rpc = static_cast<int>((rows + grid - 1) / grid);
    float *pg = part, *pb = part + static_cast<int64_t>(grid) * n;
    CHELIS_TRY(with_rows_nc(n, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const size_t smem = 3 * NC * 1024 * sizeof(float) + 2 * (NC * 8 + 8) * sizeof(float);
        if (exact) {
            CHELIS_TRY(smem_attr(block::ln_bwd_kernel<256, NC, true>, smem));
            block::ln_bwd_kernel<256, NC, true><<<grid, 256, smem, s>>>(x, dy, st, g, resid, dx, pg, pb, rows, static_cast<int>(n), rpc);
        } else {
            CHELIS_TRY(smem_attr(block::ln_bwd_kernel<256, NC, false>, smem));
            block::ln_bwd_kernel<256, NC, false><<<grid, 256, smem, s>>>(x, dy, st, g, resid, dx, pg, pb, rows, static_cast<int>(n), rpc);
        }
        g_launches++;
        CHELIS_LAUNCH_CHECK("ln_bwd_kernel");
        return CHELIS_CUDA_OK;
    }));
    CHELIS_TRY(col_sum_into(pg, grid, n, dgamma, s));
    return col_sum_into(pb, grid, n, dbeta, s);
}

int softmax_causal(float *P, int64_t rows, int64_t n, float scale, cudaStream_t s) {
    const bool exact = rows_mode() == CHELIS_CUDA_ROWS_EXACT;
    return with_rows_nc(n, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const unsigned grid = static_cast<unsigned>(rows < sm_count() * 16 ? rows : sm_count() * 16);
        if (exact) block::causal_softmax_kernel<256, NC, true><<<grid, 256, 0, s>>>(P, rows, static_cast<int>(n), scale);
        else block::causal_softmax_kernel<256, NC, false><<<grid, 256, 0, s>>>(P, rows, static_cast<int>(n), scale);
        g_launches++;
        CHELIS_LAUNCH_CHECK("causal_softmax_kernel");
        return CHELIS_CUDA_OK;
    });
}

int softmax_bwd_scaled(const float *P, float *dP, int64_t rows, int64_t n, float scale, cudaStream_t s) {
    return with_rows_nc(n, [&](auto ncv) -> int {
        constexpr int NC = decltype(ncv)::value;
        const unsigned grid = static_cast<unsigned>(rows < sm_count() * 16 ? rows : sm_count() * 16);
        block::softmax_scaled_bwd_kernel<256, NC><<<grid, 256, 0, s>>>(P, dP, rows, static_cast<int>(n), scale);
        g_launches++;
        CHELIS_LAUNCH_CHECK("softmax_scaled_bwd_kernel");
        return CHELIS_CUDA_OK;
    });
}

int add(const float *a, const float *b, float *y, int64_t n, cudaStream_t s) {
    block::add_kernel<<<grid_for(n / 4), 256, 0, s>>>(a, b, y, n / 4);
    g_launches++;
    CHELIS_LAUNCH_CHECK("add_kernel");
    return CHELIS_CUDA_OK;
}

// row-major C = op(A) . op(B) on the calling thread's stream
int mm(int ta, int tb, int64_t m, int64_t n, int64_t k, const float *a, int64_t lda,
       const float *b, int64_t ldb, float *c, int64_t ldc, int64_t batch = 1, int64_t sa = 0,
       int64_t sb = 0, int64_t sc = 0) {
    return chelis_cuda_sgemm(ta, tb, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc, batch);
}

// Matmuls of the step.  With cached splits (3xTF32 mode, row lengths that
// are multiples of 32) each operand tensor is split once, at its first use,
// and the products run on the split copies; otherwise every product goes
// through chelis_cuda_sgemm (its own split, or the exact tree mode).
struct Matmuls {
    const Ws &w;
    bool cached = false;
    bool done[S_COUNT] = {};
    // the split of tensor t ([rows][cols] row-major at x), once per step
    int split(int t, const float *x, int64_t rows, int64_t cols) {
        if (!cached || done[t]) return CHELIS_CUDA_OK;
        done[t] = true;
        return chelis_cuda_tf32x3_split(0, 0, rows, cols, x, cols, 0, 1, w.shi[t], w.slo[t]);
    }
    // C[m][n] = op(A) . op(B); A is tensor ta_id stored [k][m] (ta) or
    // [m][k], B is tb_id stored [n][k] (tb) or [k][n]
    int run(int ta, int tb, int64_t m, int64_t n, int64_t k, const float *a, int a_id,
            const float *b, int b_id, float *c) {
        if (!cached) return mm(ta, tb, m, n, k, a, ta ? m : k, b, tb ? k : n, c, n);
        CHELIS_TRY(split(a_id, a, ta ? k : m, ta ? m : k));
        CHELIS_TRY(split(b_id, b, tb ? n : k, tb ? k : n));
        return chelis_cuda_sgemm_tf32x3_presplit(m, n, k, 1, ta ? 1 : 0, w.shi[a_id],
                                                 w.slo[a_id], tb ? 0 : 1, w.shi[b_id],
                                                 w.slo[b_id], c, n, 0);
    }
    // The product with a residual added as C is stored (tf32x3::EPI_ADD):
    // C = A.B + in.  Without cached splits, the product then an add kernel.
    int run_add(int ta, int tb, int64_t m, int64_t n, int64_t k, const float *a, int a_id,
                const float *b, int b_id, float *c, const float *in, cudaStream_t s) {
        if (!cached) {
            CHELIS_TRY(run(ta, tb, m, n, k, a, a_id, b, b_id, c));
            block::add_kernel<<<grid_for(m * n / 4), 256, 0, s>>>(in, c, c, m * n / 4);
            g_launches++;
            return check_cuda(cudaGetLastError(), "add_kernel");
        }
        CHELIS_TRY(split(a_id, a, ta ? k : m, ta ? m : k));
        CHELIS_TRY(split(b_id, b, tb ? n : k, tb ? k : n));
        tf32x3::EpiArgs e;
        e.op = tf32x3::EPI_ADD;
        e.in = in;
        return sgemm_presplit_epi(m, n, k, ta ? 1 : 0, w.shi[a_id], w.slo[a_id], tb ? 0 : 1,
                                  w.shi[b_id], w.slo[b_id], c, e);
    }
};

}  // namespace

// ---------------------------------------------------------------------------
// Optional phase timing of chelis_cuda_block_step: CUDA events recorded on
// the call's stream at the boundaries of its phases, read back after the
// step.  A diagnostic for one host thread at a time (the events are
// process-wide); off by default, and then no event is recorded.
// ---------------------------------------------------------------------------
namespace block_timing {
constexpr int kPhases = 16;
const char *const kNames[kPhases] = {
    "ln1",          "gemm_qkv",     "attention_fwd", "gemm_o_residual", "ln2",
    "gemm_mlp_up",  "gelu",         "gemm_mlp_down_residual", "gemm_dw2_da", "gelu_bwd",
    "gemm_dw1_dh2", "ln2_bwd",      "gemm_dwo_do",   "attention_bwd",   "gemm_dwqkv_dh1",
    "ln1_bwd"};
bool g_on = false;
int g_dev = -1;
cudaEvent_t g_ev[kPhases + 1] = {};
bool g_rec[kPhases + 1] = {};

inline void mark(int i, cudaStream_t s) {
    if (!g_on) return;
    g_rec[i] = cudaEventRecord(g_ev[i], s) == cudaSuccess;
}
inline void reset() {
    for (bool &r : g_rec) r = false;
}
// Destroy the phase events (on the device that created them) and turn timing off.
void release() {
    if (g_dev >= 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(g_dev);
        for (cudaEvent_t &e : g_ev) {
            if (e) cudaEventDestroy(e);
            e = nullptr;
        }
        cudaSetDevice(prev);
    }
    g_dev = -1;
    g_on = false;
    reset();
}
}  // namespace block_timing

extern "C" int64_t chelis_cuda_block_workspace_bytes(const chelis_block_params *p) {
    BlockDims d;
    if (block_dims(p, d) != CHELIS_CUDA_OK) return -1;
    return carve(d, nullptr).total * static_cast<int64_t>(sizeof(float));
}

// ---------------------------------------------------------------------------
// Gradient reduction overlapped with the reverse pass: each parameter
// gradient is summed across the data-parallel ranks as soon as the reverse
// pass has written it, on the library's communication stream, while the
// reverse pass goes on; the caller's stream waits for all of them at the
// end of the step.  Events are created once per device (one host thread per
// device at a time drives a communicator).
// ---------------------------------------------------------------------------
namespace grad_reduce {
constexpr int kMax = 8;
cudaEvent_t g_ev[64][kMax + 1] = {};

struct Overlap {
    bool on = false;
    int dev = 0, n = 0;
    cudaStream_t comm = nullptr;
    int begin(cudaStream_t) {
        if (dp_nranks() <= 1) return CHELIS_CUDA_OK;
        CHELIS_TRY(current_device_checked(&dev));
        if (dev >= 64) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "device index %d", dev);
        CHELIS_TRY(dp_comm_stream(&comm));
        for (cudaEvent_t &e : g_ev[dev])
            if (!e)
                CHELIS_TRY(check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming),
                                      "cudaEventCreate(grad reduce)"));
        on = true;
        return CHELIS_CUDA_OK;
    }
    // sum `count` floats at `buf` across ranks once the work queued on `s`
    // so far (which wrote them) is done
    int reduce(float *buf, int64_t count, cudaStream_t s) {
        if (!on) return CHELIS_CUDA_OK;
        if (n >= kMax) return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "too many gradient buckets");
        cudaEvent_t e = g_ev[dev][n++];
        CHELIS_TRY(check_cuda(cudaEventRecord(e, s), "cudaEventRecord(grad ready)"));
        CHELIS_TRY(check_cuda(cudaStreamWaitEvent(comm, e, 0), "cudaStreamWaitEvent(comm)"));
        return dp_allreduce_f32_on(buf, count, comm);
    }
    // two gradients in one reduction when the caller laid them out back to back
    int reduce_pair(float *a, float *b, int64_t count, cudaStream_t s) {
        if (b == a + count) return reduce(a, 2 * count, s);
        CHELIS_TRY(reduce(a, count, s));
        return reduce(b, count, s);
    }
    // the caller's stream waits for every reduction issued
    int join(cudaStream_t s) {
        if (!on) return CHELIS_CUDA_OK;
        cudaEvent_t e = g_ev[dev][kMax];
        CHELIS_TRY(check_cuda(cudaEventRecord(e, comm), "cudaEventRecord(grads reduced)"));
        return check_cuda(cudaStreamWaitEvent(s, e, 0), "cudaStreamWaitEvent(grads reduced)");
    }
};

// Destroy the reduction events of every device.
void release_events() {
    int prev = 0;
    cudaGetDevice(&prev);
    for (int d = 0; d < 64; ++d)
        for (cudaEvent_t &e : g_ev[d])
            if (e) {
                cudaSetDevice(d);
                cudaEventDestroy(e);
                e = nullptr;
            }
    cudaSetDevice(prev);
}
}  // namespace grad_reduce

namespace {
int block_step_impl(const chelis_block_params *p, void *workspace, bool reduce_grads) {
    BlockDims d;
    CHELIS_TRY(block_dims(p, d));
    cudaStream_t s = current_stream();
    const bool fused = rows_mode() == CHELIS_CUDA_ROWS_FAST && flash_attention_supported(d.Dh);
    const int64_t big = d.BH * d.S * d.S;
    void *owned = nullptr, *owned_big = nullptr;
    float *base = static_cast<float *>(workspace);
    if (!base) {
        CHELIS_TRY(scratch_alloc(&owned, carve(d, nullptr).total * sizeof(float), s));
        base = static_cast<float *>(owned);
    }
    Ws w = carve(d, base);
    if (!fused) {
        int st0 = scratch_alloc(&owned_big, 2 * big * sizeof(float), s);
        if (st0 != CHELIS_CUDA_OK) {
            if (owned) scratch_free(owned, s);
            return st0;
        }
        w.P = static_cast<float *>(owned_big);
        w.dP = w.P + big;
    }
    const float scale = 1.0f / sqrtf(static_cast<float>(d.Dh));
    const int64_t D = d.D, S = d.S, Dh = d.Dh, F = d.F, BS = d.BS, BH = d.BH, H = d.H;
    const int64_t act = BS * D;
    const int d4 = static_cast<int>(Dh / 4);
    // split copies for the fused path: [q_hi, q_lo, k_hi, k_lo, v_hi, v_lo, dO_hi, dO_lo]
    float *hl = w.hl;
    int st = CHELIS_CUDA_OK;
    Matmuls mx{w};
    mx.cached = gemm_mode() == CHELIS_CUDA_GEMM_3XTF32 && w.shi[0] != nullptr;
    grad_reduce::Overlap gr;
    if (reduce_grads && p->dy && (st = gr.begin(s))) {
        if (owned_big) scratch_free(owned_big, s);
        if (owned) scratch_free(owned, s);
        return st;
    }
    using block_timing::mark;
    block_timing::reset();
    do {
        // ---------------- forward ----------------
        mark(0, s);
        if (mx.cached) {
            if ((st = ln_fwd(p->x, p->ln1_gamma, p->ln1_beta, p->eps, nullptr, w.st1, BS, D, s,
                             w.shi[S_H1], w.slo[S_H1])))
                break;
            mx.done[S_H1] = true;
        } else if ((st = ln_fwd(p->x, p->ln1_gamma, p->ln1_beta, p->eps, w.h1, w.st1, BS, D, s))) {
            break;
        }
        mark(1, s);
        if ((st = mx.run(0, 0, BS, 3 * D, D, w.h1, S_H1, p->w_qkv, S_WQKV, w.qkv))) break;
        mark(2, s);
        if (fused) {
            block::qkv_heads_split_kernel<<<grid_for(BS * 3 * D / 4), 256, 0, s>>>(
                w.qkv, w.q, w.k, w.v, hl, act, static_cast<int>(d.B), static_cast<int>(S),
                static_cast<int>(H), d4);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "qkv_heads_split_kernel"))) break;
            // o straight into the [B, S, H, Dh] rows layout the projection reads
            if ((st = flash_fwd(BH, H, S, Dh, scale, w.q, Dh, H * S * Dh, S * Dh, hl + 2 * act,
                                hl + 3 * act, hl + 4 * act, hl + 5 * act, w.o, D, S * D, Dh, w.lse,
                                s)))
                break;
        } else {
            block::qkv_permute_kernel<<<grid_for(BS * 3 * D / 4), 256, 0, s>>>(
                w.qkv, w.q, w.k, w.v, static_cast<int>(d.B), static_cast<int>(S), static_cast<int>(H), d4, 0);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "qkv_permute_kernel"))) break;
            if ((st = mm(0, 1, S, S, Dh, w.q, Dh, w.k, Dh, w.P, S, BH, S * Dh, S * Dh, S * S))) break;
            if ((st = softmax_causal(w.P, BH * S, S, scale, s))) break;
            if ((st = mm(0, 0, S, Dh, S, w.P, S, w.v, Dh, w.oh, Dh, BH, S * S, S * Dh, S * Dh))) break;
            block::heads_permute_kernel<<<grid_for(BS * D / 4), 256, 0, s>>>(
                w.oh, w.o, static_cast<int>(d.B), static_cast<int>(S), static_cast<int>(H), d4, 0);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "heads_permute_kernel"))) break;
        }
        mark(3, s);
        if ((st = mx.run_add(0, 0, BS, D, D, w.o, S_O, p->w_o, S_WO, w.x2, p->x, s))) break;
        mark(4, s);
        if (mx.cached) {
            if ((st = ln_fwd(w.x2, p->ln2_gamma, p->ln2_beta, p->eps, nullptr, w.st2, BS, D, s,
                             w.shi[S_H2], w.slo[S_H2])))
                break;
            mx.done[S_H2] = true;
        } else if ((st = ln_fwd(w.x2, p->ln2_gamma, p->ln2_beta, p->eps, w.h2, w.st2, BS, D, s))) {
            break;
        }
        mark(5, s);
        if ((st = mx.run(0, 0, BS, F, D, w.h2, S_H2, p->w_1, S_W1, w.u))) break;
        mark(6, s);
        if (mx.cached) {
            block::gelu_fwd_split_kernel<<<grid_for(BS * F / 4), 256, 0, s>>>(
                reinterpret_cast<const float4 *>(w.u), reinterpret_cast<float4 *>(w.shi[S_G]),
                reinterpret_cast<float4 *>(w.slo[S_G]), BS * F / 4);
            mx.done[S_G] = true;
        } else {
            block::gelu_fwd_kernel<<<grid_for(BS * F), 256, 0, s>>>(w.u, w.g, BS * F);
        }
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "gelu_fwd_kernel"))) break;
        mark(7, s);
        if ((st = mx.run_add(0, 0, BS, D, F, w.g, S_G, p->w_2, S_W2, p->y, w.x2, s))) break;
        mark(8, s);
        if (!p->dy) break;
        // ---------------- reverse mode ----------------
        const float *dy = p->dy;
        if ((st = mx.run(1, 0, F, D, BS, w.g, S_G, dy, S_DY, p->dw_2))) break;
        if ((st = gr.reduce(p->dw_2, F * D, s))) break;
        if ((st = mx.run(0, 1, BS, F, D, dy, S_DY, p->w_2, S_W2, w.dg))) break;
        mark(9, s);
        if (mx.cached) {
            block::gelu_bwd_split_kernel<<<grid_for(BS * F / 4), 256, 0, s>>>(
                reinterpret_cast<const float4 *>(w.u), reinterpret_cast<const float4 *>(w.dg),
                reinterpret_cast<float4 *>(w.shi[S_DG]), reinterpret_cast<float4 *>(w.slo[S_DG]),
                BS * F / 4);
            mx.done[S_DG] = true;
        } else {
            block::gelu_bwd_kernel<<<grid_for(BS * F), 256, 0, s>>>(w.u, w.dg, BS * F);
        }
        g_launches++;
        if ((st = check_cuda(cudaGetLastError(), "gelu_bwd_kernel"))) break;
        mark(10, s);
        if ((st = mx.run(1, 0, D, F, BS, w.h2, S_H2, w.dg, S_DG, p->dw_1))) break;
        if ((st = gr.reduce(p->dw_1, D * F, s))) break;
        if ((st = mx.run(0, 1, BS, D, F, w.dg, S_DG, p->w_1, S_W1, w.dh2))) break;
        mark(11, s);
        if ((st = ln_bwd(w.x2, w.dh2, w.st2, p->ln2_gamma, dy, w.dx2, w.part, p->dln2_gamma,
                         p->dln2_beta, BS, D, s))) break;
        if ((st = gr.reduce_pair(p->dln2_gamma, p->dln2_beta, D, s))) break;
        mark(12, s);
        if ((st = mx.run(1, 0, D, D, BS, w.o, S_O, w.dx2, S_DX2, p->dw_o))) break;
        if ((st = gr.reduce(p->dw_o, D * D, s))) break;
        if ((st = mx.run(0, 1, BS, D, D, w.dx2, S_DX2, p->w_o, S_WO, w.dO))) break;
        mark(13, s);
        if (fused) {
            block::rows_heads_split_kernel<<<grid_for(BS * D / 4), 256, 0, s>>>(
                w.dO, hl + 6 * act, hl + 7 * act, static_cast<int>(d.B), static_cast<int>(S),
                static_cast<int>(H), d4);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "rows_heads_split_kernel"))) break;
            // dq, dk, dv straight into the [B, S, 3, H, Dh] layout of dqkv, or
            // of its tf32 split when the matmuls read dqkv through the split
            float *gq = mx.cached ? w.shi[S_DQKV] : w.dqkv;
            const int64_t split_lo = mx.cached ? w.slo[S_DQKV] - w.shi[S_DQKV] : 0;
            if ((st = flash_bwd(BH, H, S, Dh, scale, w.q, w.k, w.v, Dh, H * S * Dh, S * Dh, w.dO, D,
                                S * D, Dh, w.o, D, S * D, Dh, w.lse, hl, hl + act, hl + 2 * act,
                                hl + 3 * act, hl + 4 * act, hl + 5 * act, hl + 6 * act, hl + 7 * act,
                                w.dsum, gq, gq + D, gq + 2 * D, 3 * D, S * 3 * D, Dh, s, split_lo)))
                break;
            if (mx.cached) mx.done[S_DQKV] = true;
        } else {
            block::heads_permute_kernel<<<grid_for(BS * D / 4), 256, 0, s>>>(
                w.doh, w.dO, static_cast<int>(d.B), static_cast<int>(S), static_cast<int>(H), d4, 1);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "heads_permute_kernel"))) break;
            if ((st = mm(0, 1, S, S, Dh, w.doh, Dh, w.v, Dh, w.dP, S, BH, S * Dh, S * Dh, S * S))) break;
            if ((st = mm(1, 0, S, Dh, S, w.P, S, w.doh, Dh, w.dv, Dh, BH, S * S, S * Dh, S * Dh))) break;
            if ((st = softmax_bwd_scaled(w.P, w.dP, BH * S, S, scale, s))) break;
            if ((st = mm(0, 0, S, Dh, S, w.dP, S, w.k, Dh, w.dq, Dh, BH, S * S, S * Dh, S * Dh))) break;
            if ((st = mm(1, 0, S, Dh, S, w.dP, S, w.q, Dh, w.dk, Dh, BH, S * S, S * Dh, S * Dh))) break;
            block::qkv_permute_kernel<<<grid_for(BS * 3 * D / 4), 256, 0, s>>>(
                w.dqkv, w.dq, w.dk, w.dv, static_cast<int>(d.B), static_cast<int>(S), static_cast<int>(H), d4, 1);
            g_launches++;
            if ((st = check_cuda(cudaGetLastError(), "qkv_permute_kernel"))) break;
        }
        mark(14, s);
        if ((st = mx.run(1, 0, D, 3 * D, BS, w.h1, S_H1, w.dqkv, S_DQKV, p->dw_qkv))) break;
        if ((st = gr.reduce(p->dw_qkv, D * 3 * D, s))) break;
        if ((st = mx.run(0, 1, BS, D, 3 * D, w.dqkv, S_DQKV, p->w_qkv, S_WQKV, w.dh1))) break;
        mark(15, s);
        if ((st = ln_bwd(p->x, w.dh1, w.st1, p->ln1_gamma, w.dx2, p->dx, w.part, p->dln1_gamma,
                         p->dln1_beta, BS, D, s))) break;
        mark(16, s);
        if ((st = gr.reduce_pair(p->dln1_gamma, p->dln1_beta, D, s))) break;
    } while (0);
    // the caller's stream waits for the reductions issued, also after an error
    if (gr.on) {
        const int js = gr.join(s);
        if (st == CHELIS_CUDA_OK) st = js;
    }
    if (owned_big) scratch_free(owned_big, s);
    if (owned) scratch_free(owned, s);
    return st;
}
}  // namespace

extern "C" int chelis_cuda_block_step(const chelis_block_params *p, void *workspace) {
    return block_step_impl(p, workspace, false);
}

extern "C" int chelis_cuda_block_step_dp(const chelis_block_params *p, void *workspace) {
    return block_step_impl(p, workspace, true);
}

extern "C" int chelis_cuda_block_timing(int enable) {
    using namespace block_timing;
    int dev = 0;
    CHELIS_TRY(current_device_checked(&dev));
    if (g_dev >= 0 && (!enable || g_dev != dev)) {
        for (cudaEvent_t &e : g_ev) {
            if (e) cudaEventDestroy(e);
            e = nullptr;
        }
        g_dev = -1;
    }
    g_on = false;
    reset();
    if (!enable) return CHELIS_CUDA_OK;
    for (cudaEvent_t &e : g_ev)
        CHELIS_TRY(check_cuda(cudaEventCreate(&e), "cudaEventCreate(block timing)"));
    g_dev = dev;
    g_on = true;
    return CHELIS_CUDA_OK;
}

extern "C" int chelis_cuda_block_phase_ms(float *ms, int32_t n) {
    using namespace block_timing;
    if (!ms || n < kPhases)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "block_phase_ms needs room for %d phases", kPhases);
    if (!g_on) return set_error(CHELIS_CUDA_ERR_DOMAIN, "block timing is off");
    for (int i = 0; i < kPhases; ++i) ms[i] = 0.0f;
    for (int i = kPhases; i >= 0; --i)
        if (g_rec[i]) {
            CHELIS_TRY(check_cuda(cudaEventSynchronize(g_ev[i]), "cudaEventSynchronize"));
            break;
        }
    for (int i = 0; i < kPhases; ++i)
        if (g_rec[i] && g_rec[i + 1])
            CHELIS_TRY(check_cuda(cudaEventElapsedTime(&ms[i], g_ev[i], g_ev[i + 1]),
                                  "cudaEventElapsedTime"));
    return CHELIS_CUDA_OK;
}

extern "C" const char *chelis_cuda_block_phase_name(int32_t i) {
    return (i >= 0 && i < block_timing::kPhases) ? block_timing::kNames[i] : nullptr;
}
