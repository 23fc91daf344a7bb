// Float elementary functions bit-identical to the system libm (GNU C Library
// 2.39) that the reference's CPU code calls: expf (the decoder's softmax and
// SiLU, the graph node's Silu), expm1f and tanhf (the graph node's Gelu).
// Scalar code only (no shared memory, no warp intrinsics), so the same
// source also compiles as host code with plain float operations standing in
// for the __f*_rn intrinsics.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

namespace leafq {

// expf: Arm's optimized-routines algorithm, as glibc 2.39 carries it.  With
// N = 32, z = x * N / ln 2 is split as k + r (k the nearest integer, taken
// with the 0x1.8p52 shift trick), 2^(k/N) is assembled from a table of
// 2^(i/N) and k's high bits, and 2^(r/N) is a cubic in r; all in double with
// fused multiply-adds, one rounding to float at the end.  The constants below
// are the algorithm's published ones; the table is 2^(i/32) rounded to
// double, computed on the host.  Checked against libm expf on all 2^32 float
// inputs.

struct ExpTable {
    unsigned long long bits[32];  // bits of 2^(i/32) as double, minus i << 47
};

// expf(x) as libm computes it.
__device__ __forceinline__ float expf_libm(float x, const ExpTable& tab) {
    const uint32_t ux = __float_as_uint(x);
    const uint32_t abstop = (ux >> 20) & 0x7ffu;
    if (abstop >= 0x42bu) {  // |x| >= 88 (top 12 bits of 88.0f), inf, nan
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8u) return __fadd_rn(x, x);
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
    const double shift = 0x1.8p+52;
    const double xd = static_cast<double>(x);
    double kd = __fma_rn(inv_ln2_n, xd, shift);
    const unsigned long long ki = static_cast<unsigned long long>(__double_as_longlong(kd));
    kd = __dsub_rn(kd, shift);
    const double r = __fma_rn(inv_ln2_n, xd, -kd);
    unsigned long long t = tab.bits[ki % 32];
    t += ki << 47;
    const double sc = __longlong_as_double(static_cast<long long>(t));
    const double c0 = 0x1.c6af84b912394p-5 / 32.0 / 32.0 / 32.0;
    const double c1 = 0x1.ebfce50fac4f3p-3 / 32.0 / 32.0;
    const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double z = __fma_rn(c0, r, c1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(c2, r, 1.0);
    y = __fma_rn(z, r2, y);
    y = __dmul_rn(y, sc);
    return __double2float_rn(y);
}

// 2^(i/32) rounded to double, minus i << 47 (the table of expf_libm).
inline const ExpTable& exp_table() {
    static const ExpTable table = [] {
        ExpTable t;
        for (int i = 0; i < 32; ++i) {
            const double v = static_cast<double>(std::exp2(static_cast<long double>(i) / 32.0L));
            unsigned long long bits;
            std::memcpy(&bits, &v, sizeof(bits));
            t.bits[i] = bits - (static_cast<unsigned long long>(i) << 47);
        }
        return t;
    }();
    return table;
}

// expm1f and tanhf as the system libm computes them (GNU C Library 2.39,
// whose float expm1 and tanh are the Sun fdlibm algorithms of 1993).
// expm1: reduce x = k ln2 + r with ln2 split in a high and a low part (the
// rounding error of the reduction carried as c), approximate expm1(r) with
// fdlibm's rational form R(r^2) = 1 + r^2 (Q1 + ... + Q5 r^8), then rebuild
// 2^k (expm1(r) + 1) - 1 by exponent arithmetic in the branch for k.
// tanh: |x| >= 1 uses 1 - 2 / (expm1(2|x|) + 2), smaller |x| uses
// -t / (t + 2) with t = expm1(-2|x|), |x| >= 22 gives 1 - tiny, tiny |x|
// gives x (1 + x).  Every step is one float rounding (no contraction), as
// the baseline x86-64 build does.  The constants are the algorithm's
// published ones.  Checked against libm tanhf on all 2^32 float inputs.
__device__ __forceinline__ float expm1f_libm(float x) {
    const float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
    const float q1 = -3.3333335072e-02f, q2 = 1.5873016091e-03f, q3 = -7.9365076090e-05f,
                q4 = 4.0082177293e-06f, q5 = -2.0109921195e-07f;
    uint32_t hx = __float_as_uint(x);
    const uint32_t negative = hx & 0x80000000u;
    hx &= 0x7fffffffu;
    if (hx >= 0x4195b844u) {  // |x| >= 56 ln2
        if (hx >= 0x42b17218u) {  // |x| >= 88.72
            if (hx > 0x7f800000u) return __fadd_rn(x, x);  // NaN
            if (hx == 0x7f800000u) return negative ? -1.0f : x;
            if (x > 8.8721679688e+01f) return __int_as_float(0x7f800000);  // overflow
        }
        if (negative) return -1.0f;  // tiny - 1 rounds to -1
    }
    float c = 0.0f;
    int k = 0;
    if (hx > 0x3eb17218u) {  // |x| > ln2 / 2
        float hi, lo;
        if (hx < 0x3F851592u) {  // and |x| < 3 ln2 / 2
            if (!negative) { hi = __fsub_rn(x, ln2_hi); lo = ln2_lo; k = 1; }
            else { hi = __fadd_rn(x, ln2_hi); lo = -ln2_lo; k = -1; }
        } else {
            k = __float2int_rz(__fadd_rn(__fmul_rn(invln2, x), negative ? -0.5f : 0.5f));
            const float t = __int2float_rn(k);
            hi = __fsub_rn(x, __fmul_rn(t, ln2_hi));
            lo = __fmul_rn(t, ln2_lo);
        }
        x = __fsub_rn(hi, lo);
        c = __fsub_rn(__fsub_rn(hi, x), lo);
    } else if (hx < 0x33000000u) {  // |x| < 2^-25
        return x;
    }
    const float hfx = __fmul_rn(0.5f, x);
    const float hxs = __fmul_rn(x, hfx);
    float r1 = __fadd_rn(q4, __fmul_rn(hxs, q5));
    r1 = __fadd_rn(q3, __fmul_rn(hxs, r1));
    r1 = __fadd_rn(q2, __fmul_rn(hxs, r1));
    r1 = __fadd_rn(q1, __fmul_rn(hxs, r1));
    r1 = __fadd_rn(1.0f, __fmul_rn(hxs, r1));
    float t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
    float e = __fmul_rn(hxs, __fdiv_rn(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(x, t))));
    if (k == 0) return __fsub_rn(x, __fsub_rn(__fmul_rn(x, e), hxs));
    e = __fsub_rn(__fmul_rn(x, __fsub_rn(e, c)), c);
    e = __fsub_rn(e, hxs);
    if (k == -1) return __fsub_rn(__fmul_rn(0.5f, __fsub_rn(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return __fmul_rn(-2.0f, __fsub_rn(e, __fadd_rn(x, 0.5f)));
        return __fadd_rn(1.0f, __fmul_rn(2.0f, __fsub_rn(x, e)));
    }
    float y;
    if (k <= -2 || k > 56) {  // 2^k (1 + expm1(r)) - 1 with the exponent added last
        y = __fsub_rn(1.0f, __fsub_rn(e, x));
        y = __uint_as_float(__float_as_uint(y) + (static_cast<uint32_t>(k) << 23));
        return __fsub_rn(y, 1.0f);
    }
    if (k < 23) {
        t = __uint_as_float(0x3f800000u - (0x1000000u >> k));  // 1 - 2^-k
        y = __fsub_rn(t, __fsub_rn(e, x));
    } else {
        t = __uint_as_float(static_cast<uint32_t>(0x7f - k) << 23);  // 2^-k
        y = __fadd_rn(__fsub_rn(x, __fadd_rn(e, t)), 1.0f);
    }
    return __uint_as_float(__float_as_uint(y) + (static_cast<uint32_t>(k) << 23));
}

__device__ __forceinline__ float tanhf_libm(float x) {
    const uint32_t jx = __float_as_uint(x);
    const uint32_t ix = jx & 0x7fffffffu;
    if (ix >= 0x7f800000u) {  // inf or NaN: 1 / x -+ 1
        const float inv = __fdiv_rn(1.0f, x);
        return (jx & 0x80000000u) ? __fsub_rn(inv, 1.0f) : __fadd_rn(inv, 1.0f);
    }
    float z;
    if (ix < 0x41b00000u) {  // |x| < 22
        if (ix == 0) return x;
        if (ix < 0x24000000u) return __fmul_rn(x, __fadd_rn(1.0f, x));  // |x| < 2^-55
        const float ax = __uint_as_float(ix);
        if (ix >= 0x3f800000u) {  // |x| >= 1
            const float t = expm1f_libm(__fmul_rn(2.0f, ax));
            z = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(t, 2.0f)));
        } else {
            const float t = expm1f_libm(__fmul_rn(-2.0f, ax));
            z = __fdiv_rn(-t, __fadd_rn(t, 2.0f));
        }
    } else {
        z = 1.0f;  // 1 - tiny rounds to 1
    }
    return (jx & 0x80000000u) ? -z : z;
}

// The graph executor's fused Gelu, tanh form (executor.cpp:236-240), in
// C++'s left-to-right order with one float rounding per step:
// (0.5f * v) * (1 + tanhf(c * (v + ((0.044715f * v) * v) * v))).
__device__ __forceinline__ float gelu_tanh_libm(float v) {
    const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
    const float th = tanhf_libm(__fmul_rn(0.7978845608028654f, __fadd_rn(v, cube)));
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, th));
}

}  // namespace leafq
