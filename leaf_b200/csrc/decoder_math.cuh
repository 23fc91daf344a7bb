// Exponential of the decoder's softmax and SiLU, bit-identical to the system
// libm's expf (GNU C Library 2.39, whose expf is Arm's optimized-routines
// algorithm): with N = 32, z = x * N / ln 2 is split as k + r (k the nearest
// integer, taken with the 0x1.8p52 shift trick), 2^(k/N) is assembled from a
// table of 2^(i/N) and k's high bits, and 2^(r/N) is a cubic in r; all in
// double with fused multiply-adds, one rounding to float at the end.  The
// constants below are the algorithm's published ones; the table is
// 2^(i/32) rounded to double, computed on the host.  Checked against libm
// expf on all 2^32 float inputs.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

namespace leafq {

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


}  // namespace leafq

namespace leafq {

// Left-to-right float sum of v[0..n) (n a multiple of 4, v 16-byte aligned,
// shared memory), as `for (i) s += v[i]` computes it -- the reference's order
// for RMSNorm's sum of squares (norm(), decoder.cpp:714-719).  One thread;
// loads run 16 values ahead of the dependent additions, which are the whole
// cost (2048 values: about 4 us).  A block-parallel exact alternative (per
// binade of the running sum, additions as two-state parity transducers and
// a scan) was built and checked bit for bit, and measured slower on B200.
__device__ __forceinline__ float sum_in_order(const float* v, int n) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    const int vecs = n / 4;
    float s = 0.0f;
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) a[u] = u < vecs ? v4[u] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < vecs; c += 4) {
        float4 b[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) b[u] = c + 4 + u < vecs ? v4[c + 4 + u] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (c + u < vecs) {
                s = __fadd_rn(s, a[u].x);
                s = __fadd_rn(s, a[u].y);
                s = __fadd_rn(s, a[u].z);
                s = __fadd_rn(s, a[u].w);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = b[u];
    }
    return s;
}

}  // namespace leafq
