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

// ---------------------------------------------------------------------------
// Left-to-right float sum of squares, computed by a whole thread block and
// bit-identical to `for (i) s += x[i] * x[i]` (norm(), decoder.cpp:714-719).
//
// Every addend p = x*x is non-negative, so the running sum s only grows.
// While s stays inside one binade [2^e, 2^(e+1)) every partial sum is an
// integer multiple m of u = 2^(e-23), and fl(s + p) = (m + n) u where n is p/u
// rounded to nearest -- ties to the even result, which depends only on the
// parity of m.  An addend is therefore a two-state transducer (input parity
// -> increment, output parity); transducers compose associatively, so a
// block-wide scan gives every partial sum of the binade at once.  The first
// addition that leaves the binade (m + n >= 2^24) is redone as a plain float
// addition, and the scan restarts from there with the next binade.  A
// 2048-element sum of similar magnitudes takes the first 64 additions
// sequentially and then about five scans instead of 2048 dependent additions.
struct SumStep {
    int inc0, inc1;  // increment (units of u, saturated at 2^25) for input parity 0 / 1
    int out0, out1;  // output parity for input parity 0 / 1
};

__device__ __forceinline__ SumStep sum_step_identity() { return {0, 0, 0, 1}; }

__device__ __forceinline__ int sat_add(int a, int b) {
    const int r = a + b;  // a, b <= 2^25: no overflow
    return r > (1 << 25) ? (1 << 25) : r;
}

// a, then b.
__device__ __forceinline__ SumStep sum_step_then(const SumStep& a, const SumStep& b) {
    SumStep r;
    r.inc0 = sat_add(a.inc0, a.out0 ? b.inc1 : b.inc0);
    r.out0 = a.out0 ? b.out1 : b.out0;
    r.inc1 = sat_add(a.inc1, a.out1 ? b.inc1 : b.inc0);
    r.out1 = a.out1 ? b.out1 : b.out0;
    return r;
}

// Adding p (>= 0) to a multiple of u = 2^(e-23) that stays below 2^(e+1).
__device__ __forceinline__ SumStep sum_step_of(float p, int e) {
    const uint32_t bits = __float_as_uint(p);
    const int field = static_cast<int>((bits >> 23) & 0xffu);
    SumStep t;
    if (field == 0xff) {  // inf / nan: force the plain addition
        t.inc0 = t.inc1 = 1 << 25;
        t.out0 = 0;
        t.out1 = 1;
        return t;
    }
    const int ep = field ? field - 127 : -126;
    const uint32_t mp = field ? ((bits & 0x7fffffu) | 0x800000u) : (bits & 0x7fffffu);
    const int shift = e - ep;  // p / u = mp * 2^-shift
    int q;
    int cls;  // -1 below half, 0 tie, +1 above half
    if (shift < 0) {
        q = 1 << 25;  // p >= 2^(e+1): leaves the binade
        cls = -1;
    } else if (shift == 0) {
        q = static_cast<int>(mp);
        cls = -1;
    } else if (shift > 25) {
        q = 0;
        cls = -1;
    } else {
        q = static_cast<int>(mp >> shift);
        const uint32_t rem = mp & ((1u << shift) - 1u), half = 1u << (shift - 1);
        cls = rem < half ? -1 : (rem > half ? 1 : 0);
    }
    if (cls < 0) {
        t.inc0 = t.inc1 = q;
        t.out0 = q & 1;
        t.out1 = (q + 1) & 1;
    } else if (cls > 0) {
        t.inc0 = t.inc1 = q + 1;
        t.out0 = (q + 1) & 1;
        t.out1 = q & 1;
    } else {
        t.inc0 = q + (q & 1);
        t.inc1 = q + ((q + 1) & 1);
        t.out0 = t.out1 = 0;
    }
    return t;
}

__device__ __forceinline__ float pow2f(int k) {  // 2^k, k in [-149, 127]
    return k >= -126 ? __int_as_float((k + 127) << 23) : __int_as_float(1 << (k + 149));
}

struct SumScratch {
    SumStep warp_total[32];
    int crossing;
    float s;
    int i0;
};

// NT threads (a multiple of 32, at most 1024) call this together; `sync`
// is their barrier.  x: shared memory, n <= 8 * NT elements.
template <int NT, typename Sync>
__device__ float sum_squares_sequential_order(const float* x, int n, SumScratch* sc, int tid, Sync sync) {
    constexpr int kPer = 8;
    const int per = (n + NT - 1) / NT;  // <= kPer
    const int lane = tid & 31, warp = tid >> 5;
    float p[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int i = tid * per + j;
        p[j] = (j < per && i < n) ? __fmul_rn(x[i], x[i]) : 0.0f;
    }
    const int head = n < 64 ? n : 64;
    if (tid == 0) {
        float s = 0.0f;
        for (int i = 0; i < head; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        sc->s = s;
        sc->i0 = head;
    }
    sync();
    for (;;) {
        const float s = sc->s;
        const int i0 = sc->i0;
        if (i0 >= n) break;
        const uint32_t sb = __float_as_uint(s);
        const int sfield = static_cast<int>((sb >> 23) & 0xffu);
        if (s == 0.0f || sfield == 0xff) {  // no binade yet / not finite: one plain step
            sync();
            if (tid == 0) {
                sc->s = __fadd_rn(s, __fmul_rn(x[i0], x[i0]));
                sc->i0 = i0 + 1;
            }
            sync();
            continue;
        }
        const int e = sfield ? sfield - 127 : -126;
        const int m = static_cast<int>(sfield ? ((sb & 0x7fffffu) | 0x800000u) : (sb & 0x7fffffu));
        const int par0 = m & 1;
        // This thread's elements at or after i0, composed in order.
        SumStep own = sum_step_identity();
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int i = tid * per + j;
            if (j < per && i >= i0 && i < n) own = sum_step_then(own, sum_step_of(p[j], e));
        }
        // Exclusive scan over threads (thread order = element order).
        SumStep incl = own;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            SumStep prev;
            prev.inc0 = __shfl_up_sync(0xffffffffu, incl.inc0, o);
            prev.inc1 = __shfl_up_sync(0xffffffffu, incl.inc1, o);
            prev.out0 = __shfl_up_sync(0xffffffffu, incl.out0, o);
            prev.out1 = __shfl_up_sync(0xffffffffu, incl.out1, o);
            if (lane >= o) incl = sum_step_then(prev, incl);
        }
        SumStep lane_excl;
        lane_excl.inc0 = __shfl_up_sync(0xffffffffu, incl.inc0, 1);
        lane_excl.inc1 = __shfl_up_sync(0xffffffffu, incl.inc1, 1);
        lane_excl.out0 = __shfl_up_sync(0xffffffffu, incl.out0, 1);
        lane_excl.out1 = __shfl_up_sync(0xffffffffu, incl.out1, 1);
        if (lane == 0) lane_excl = sum_step_identity();
        if (lane == 31) sc->warp_total[warp] = incl;
        if (tid == 0) sc->crossing = n;
        sync();
        SumStep prefix = sum_step_identity();
        for (int w = 0; w < warp; ++w) prefix = sum_step_then(prefix, sc->warp_total[w]);
        prefix = sum_step_then(prefix, lane_excl);
        // Partial sums of this thread's elements; the first that leaves the
        // binade.  Partial sums only grow, so exactly one thread -- the one
        // whose own prefix is still inside the binade -- finds it.
        int mb = sat_add(m, par0 ? prefix.inc1 : prefix.inc0);
        int par = par0 ? prefix.out1 : prefix.out0;
        int my_c = n, my_m = 0;
        if (mb < (1 << 24)) {
#pragma unroll
            for (int j = 0; j < kPer; ++j) {
                const int i = tid * per + j;
                if (j < per && i >= i0 && i < n && my_c == n) {
                    const SumStep t = sum_step_of(p[j], e);
                    const int inc = par ? t.inc1 : t.inc0;
                    if (mb + inc >= (1 << 24)) {
                        my_c = i;
                        my_m = mb;
                    } else {
                        mb += inc;
                        par = par ? t.out1 : t.out0;
                    }
                }
            }
        }
        if (my_c < n) sc->crossing = my_c;
        const bool last_owner = (n - 1) / per == tid;
        sync();
        const int c = sc->crossing;
        if (c == n) {
            if (last_owner) {  // the whole rest stays in the binade
                sc->s = __fmul_rn(__int2float_rn(mb), pow2f(e - 23));
                sc->i0 = n;
            }
        } else if (my_c == c) {
            const float before = __fmul_rn(__int2float_rn(my_m), pow2f(e - 23));
            sc->s = __fadd_rn(before, __fmul_rn(x[c], x[c]));
            sc->i0 = c + 1;
        }
        sync();
    }
    const float result = sc->s;
    sync();  // the scratch may be reused after return
    return result;
}

}  // namespace leafq
