// gelu.cuh -- gelu = m(x) * Phi(x) with the compensated Phi graph of spec 05
// section 3.3 (crates/chelis-dag-core/src/tier2.rs lower_gelu), and its
// derivative Phi(x) + x * phi(x).  One definition for every kernel that
// evaluates them (the block step's row kernels and the GEMM epilogues that
// fold them into the matmul producing their input), so all give the same bits.
#pragma once

#include <cuda_runtime.h>

namespace chelis {
namespace gelu {

__device__ __forceinline__ float canon(float x) { return isnan(x) ? __int_as_float(0x7fc00000) : x; }

__device__ __forceinline__ float phi_graph(float x) {
    const float c = 0x1.6a09e6p-1f;       // RN_f32(1/sqrt(2))
    const float cl = 0x1.9fcef4p-27f;     // RN_f32(1/sqrt(2) - c)
    const float k = 0x1.20dd76p+0f;       // RN_f32(2/sqrt(pi))
    const float sp = 4097.0f;             // Veltkamp splitter for f32
    const float e = erfcf(__fmul_rn(-x, c));
    const float z = (fabsf(x) < 64.0f) ? x : 0.0f;
    const float a = -z;
    const float th = __fmul_rn(a, c);
    const float ta = __fmul_rn(sp, a);
    const float ah = __fsub_rn(ta, __fsub_rn(ta, a));
    const float al = __fsub_rn(a, ah);
    const float tc = __fmul_rn(sp, c);
    const float ch = __fsub_rn(tc, __fsub_rn(tc, c));
    const float cr = __fsub_rn(c, ch);
    float tl = __fsub_rn(__fmul_rn(ah, ch), th);
    tl = __fadd_rn(tl, __fmul_rn(ah, cr));
    tl = __fadd_rn(tl, __fmul_rn(al, ch));
    tl = __fadd_rn(tl, __fmul_rn(al, cr));
    tl = __fadd_rn(tl, __fmul_rn(a, cl));
    const float corr = __fmul_rn(__fmul_rn(k, expf(-__fmul_rn(th, th))), tl);
    return __fmul_rn(0.5f, __fsub_rn(e, corr));
}

// gelu(x), NaN canonical
__device__ __forceinline__ float value(float x) {
    const float m = (x < -3.40282347e+38f) ? -0.0f : x;
    return canon(__fmul_rn(m, phi_graph(x)));
}

// d gelu / dx at x: Phi(x) + x * phi(x), phi the standard normal density
__device__ __forceinline__ float derivative(float x) {
    const float pdf = __fmul_rn(0.3989422804f, expf(__fmul_rn(-0.5f, __fmul_rn(x, x))));
    return isinf(x) ? (x > 0.0f ? 1.0f : 0.0f) : __fadd_rn(phi_graph(x), __fmul_rn(x, pdf));
}

}  // namespace gelu
}  // namespace chelis
