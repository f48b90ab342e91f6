// crmath.cuh -- correctly rounded binary32 exp and log on the device.
//
// The C lane evaluates exp / log through CORE-MATH, correctly rounded
// (crates/chelis-crmath; the binary32 entry points chelis_crmath_ffi_expf /
// _logf, crmath_ffi.c:15-45), so a kernel that must match it bit for bit
// needs correctly rounded results too; CUDA's expf / logf are within a few
// ulp only.  These functions are written from the mathematics, with Ziv's
// rounding test (a cheap approximation with a proven error bound decides the
// rounding unless the bound straddles a rounding boundary; then a far more
// accurate one does):
//
//  fast path  (double precision, relative error below 2^-51):
//   exp: x = k ln2/64 + r, |r| <= ln2/128 (Cody-Waite reduction with a
//        38-bit leading part of ln2/64, so k * hi is exact);
//        e^x = 2^(k/64) e^r, 2^(j/64) from a double-double table, e^r by
//        its Taylor series to r^6 (truncation below 2^-64).
//   log: x = 2^E m, m c = 1 + u with c a 9-bit approximation of 1/m from a
//        128-entry table (u exact in double, |u| < 2^-7.7; buckets near 1
//        have c = 1, and m is halved from sqrt 2 on so that x near 1 never
//        cancels); log x = E ln2 - log c + log1p(u), log1p by its series to
//        u^9.
//  The result y is accepted when y(1 - 2^-49) and y(1 + 2^-49) round to the
//  same float.
//  slow path  (double-double, relative error near 2^-100): the same
//   reductions carried in double-double (error-free transformations: Knuth's
//   TwoSum, the FMA TwoProduct, Dekker's products), e^r to r^11 and log1p to
//   u^14, then the double-double rounded to float, ties by the low part.
//
// exp and log of binary32 never fall exactly on a rounding boundary except at
// the exact cases (e^0 = 1, log 1 = 0), so a slow path this accurate rounds
// correctly; the tests compare every one of the 2^32 inputs with CORE-MATH.
// NaN inputs give a quiet NaN, as x + x does.
#pragma once

#ifndef __CUDACC_RTC__  // also compiled by NVRTC into the per-chain FusedElem kernels
#include <cuda_runtime.h>
#endif

#include "crmath_tables.cuh"

namespace chelis {
namespace crmath {

struct DD {
    double hi, lo;
};

__device__ __forceinline__ DD two_sum(double a, double b) {
    const double s = __dadd_rn(a, b);
    const double bb = __dsub_rn(s, a);
    const double e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
    return {s, e};
}
__device__ __forceinline__ DD quick_two_sum(double a, double b) {  // |a| >= |b|
    const double s = __dadd_rn(a, b);
    return {s, __dsub_rn(b, __dsub_rn(s, a))};
}
__device__ __forceinline__ DD two_prod(double a, double b) {
    const double p = __dmul_rn(a, b);
    return {p, __fma_rn(a, b, -p)};
}
__device__ __forceinline__ DD dd_add(DD a, DD b) {
    DD s = two_sum(a.hi, b.hi);
    const DD t = two_sum(a.lo, b.lo);
    s.lo = __dadd_rn(s.lo, t.hi);
    s = quick_two_sum(s.hi, s.lo);
    s.lo = __dadd_rn(s.lo, t.lo);
    return quick_two_sum(s.hi, s.lo);
}
__device__ __forceinline__ DD dd_mul(DD a, DD b) {
    DD p = two_prod(a.hi, b.hi);
    p.lo = __fma_rn(a.hi, b.lo, __fma_rn(a.lo, b.hi, p.lo));
    return quick_two_sum(p.hi, p.lo);
}
__device__ __forceinline__ DD dd_mul_d(DD a, double b) {
    DD p = two_prod(a.hi, b);
    p.lo = __fma_rn(a.lo, b, p.lo);
    return quick_two_sum(p.hi, p.lo);
}

// The float nearest to hi + lo (ties to even): hi's own rounding unless hi
// lies exactly on the midpoint between two floats, where lo decides.
__device__ __forceinline__ float round_dd(DD v) {
    const float f = __double2float_rn(v.hi);
    const double fd = static_cast<double>(f);
    if (fd == v.hi || isinf(f)) return f;
    const float inf = __int_as_float(0x7f800000);
    const float g = fd < v.hi ? nextafterf(f, inf) : nextafterf(f, -inf);
    const double mid = __dmul_rn(__dadd_rn(fd, static_cast<double>(g)), 0.5);
    if (v.hi != mid || v.lo == 0.0) return f;  // not a tie, or an exact tie (already even)
    return (v.lo > 0.0) == (static_cast<double>(g) > fd) ? g : f;
}

// y accepted if it lies at least 2^-49 |y| away from every rounding boundary
// (the fast paths' error stays below 2^-51)
__device__ __forceinline__ bool ziv(double y, float *out) {
    const double e = __dmul_rn(fabs(y), 0x1p-49);
    const float a = __double2float_rn(__dsub_rn(y, e));
    const float b = __double2float_rn(__dadd_rn(y, e));
    *out = a;
    return __float_as_uint(a) == __float_as_uint(b);
}

__device__ __noinline__ float expf_slow(double x, double kd, int k) {
    // r = x - k ln2/64 as a double-double: x - k*H exactly (TwoSum of the
    // exact product), minus k*L (TwoProduct) and k*L2
    DD r = two_sum(x, -kd * kLn2Over64Hi);
    r = dd_add(r, two_prod(-kd, kLn2Over64Lo));
    r = dd_add(r, DD{-kd * kLn2Over64Lo2, 0.0});
    DD q{kInvFact[11][0], kInvFact[11][1]};
    for (int n = 10; n >= 0; --n) q = dd_add(DD{kInvFact[n][0], kInvFact[n][1]}, dd_mul(r, q));
    const int j = k & 63;
    DD y = dd_mul(q, DD{kExp2Table[j][0], kExp2Table[j][1]});
    const int e = (k - j) / 64;
    y.hi = scalbn(y.hi, e);
    y.lo = scalbn(y.lo, e);
    return round_dd(y);
}

__device__ __forceinline__ float expf_cr(float xf) {
    if (isnan(xf)) return xf + xf;
    if (xf > 89.0f) return __int_as_float(0x7f800000);  // e^89 > FLT_MAX + half an ulp
    if (xf < -104.0f) return 0.0f;       // e^-104 < 2^-150: rounds to +0
    const double x = xf;
    const double kd = rint(x * k64OverLn2);
    const int k = static_cast<int>(kd);
    const double r = __fma_rn(-kd, kLn2Over64Lo, __fma_rn(-kd, kLn2Over64Hi, x));
    // p = e^r - 1 = r + r^2/2 + ... + r^6/720
    double p = __fma_rn(r, 0x1.6c16c16c16c17p-10, 0x1.1111111111111p-7);
    p = __fma_rn(r, p, 0x1.5555555555555p-5);
    p = __fma_rn(r, p, 0x1.5555555555555p-3);
    p = __fma_rn(r, p, 0.5);
    p = __fma_rn(r, p, 1.0);
    p = __dmul_rn(p, r);
    const int j = k & 63;
    const double th = kExp2Table[j][0], tl = kExp2Table[j][1];
    double y = __dadd_rn(th, __fma_rn(th, p, tl));
    y = scalbn(y, (k - j) / 64);
    float out;
    if (ziv(y, &out)) return out;
    return expf_slow(x, kd, k);
}

__device__ __noinline__ float logf_slow(double E, double m, int i) {
    const double c = kLogTable[i][0];
    const double u = __fma_rn(m, c, -1.0);  // exact
    // log1p(u) = u (1 - u (1/2 - u (1/3 - ...))) to u^14
    DD q{kInv[14][0], kInv[14][1]};
    for (int n = 13; n >= 1; --n) {
        DD uq = dd_mul_d(q, u);
        uq.hi = -uq.hi;
        uq.lo = -uq.lo;
        q = dd_add(DD{kInv[n][0], kInv[n][1]}, uq);
    }
    DD l = dd_mul_d(q, u);
    // + E ln2 (E * kLn2Hi exact) - log c
    DD t = dd_add(DD{E * kLn2Hi, 0.0}, two_prod(E, kLn2Lo));
    t = dd_add(t, DD{E * kLn2Lo2, 0.0});
    t = dd_add(t, DD{kLogTable[i][1], kLogTable[i][2]});
    return round_dd(dd_add(t, l));
}

__device__ __forceinline__ float logf_cr(float xf) {
    unsigned int bits = __float_as_uint(xf);
    if (isnan(xf)) return xf + xf;
    if (bits == 0u || bits == 0x80000000u) return __int_as_float(0xff800000);  // log(+-0) = -inf
    if (bits >> 31) return __uint_as_float(0x7fc00000u);      // log(x < 0) = NaN
    if (isinf(xf)) return xf;
    int E = 0;
    if (bits < 0x00800000u) {  // subnormal: scale by 2^24
        xf *= 16777216.0f;
        bits = __float_as_uint(xf);
        E = -24;
    }
    E += static_cast<int>(bits >> 23) - 127;
    const int i = static_cast<int>((bits >> 16) & 0x7f);
    double m = static_cast<double>(__uint_as_float((bits & 0x007fffffu) | 0x3f800000u));
    if (kLogTable[i][3] != 0.0) {
        m *= 0.5;
        E += 1;
    }
    const double Ed = static_cast<double>(E);
    const double c = kLogTable[i][0];
    const double u = __fma_rn(m, c, -1.0);
    // log1p(u) to u^9, Horner from u^9 down
    double q = 0x1.c71c71c71c71cp-4;             // 1/9
    q = __fma_rn(u, q, -0x1.0000000000000p-3);   // -1/8
    q = __fma_rn(u, q, 0x1.2492492492492p-3);    // 1/7
    q = __fma_rn(u, q, -0x1.5555555555555p-3);   // -1/6
    q = __fma_rn(u, q, 0x1.999999999999ap-3);    // 1/5
    q = __fma_rn(u, q, -0.25);                   // -1/4
    q = __fma_rn(u, q, 0x1.5555555555555p-2);    // 1/3
    q = __fma_rn(u, q, -0.5);                    // -1/2
    q = __fma_rn(u, q, 1.0);
    const double l = __dmul_rn(q, u);
    const double t1 = Ed * kLn2Hi;  // exact (45-bit kLn2Hi, |E| < 2^8)
    const double a = __dadd_rn(t1, kLogTable[i][1]);
    const double y = __dadd_rn(a, __fma_rn(Ed, kLn2Lo, __dadd_rn(l, kLogTable[i][2])));
    float out;
    if (ziv(y, &out)) return out;
    return logf_slow(Ed, m, i);
}

}  // namespace crmath
}  // namespace chelis
