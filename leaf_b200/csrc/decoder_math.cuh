// Scalar and warp-level arithmetic of the decoder kernels.
#pragma once

#include "libm_math.cuh"

namespace leafq {

// Left-to-right float sum of v[0..n) (n a multiple of 4, v 16-byte aligned,
// shared memory), as `for (i) s += v[i]` computes it -- the reference's order
// for RMSNorm's sum of squares (norm(), decoder.cpp:714-719).  One thread;
// loads run 16 values ahead of the dependent additions, which are the whole
// cost (2048 values: about 4 us).  sum_in_order_par below gives the same
// bits for non-negative values with a whole block in a fraction of the time.
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

// ----------------------------------------------------------------------------
// The same left-to-right sum for NON-NEGATIVE values (sums of squares), by a
// block of NT threads, each holding four consecutive values, bit for bit.
//
// While the running sum s stays inside one binade [2^e, 2^(e+1)), it is an
// integer multiple m of that binade's ulp u, and s + v rounds to the multiple
// nearest to m + v/u: when the remainder of v/u is not exactly one half, m
// grows by round(v/u) whatever m is.  So a run of such additions inside one
// binade adds the integer sum of their increments to m -- to the float's
// bits -- and integer sums are order-free.
//
// The binade of every partial sum is predicted from an approximate prefix sum
// (any order).  An element whose addition is predicted to change the binade,
// or whose v/u has a remainder of exactly one half (a tie, decided by the
// parity of m), is a "head": it is added as a plain float addition.  The
// others add their increment, in the binade of the head before them.  Thread 0
// then walks the heads in order: s += head; if s lies in the head's binade,
// s's bits advance by the increments up to the next head, and the result must
// still lie in that binade -- which proves that no partial sum left it, so
// every step was exact.  A run that fails either check is added element by
// element, so a wrong prediction costs time only.  Non-finite sums, and rows
// with more heads than the scratch holds, take the plain loop.
//
// Threads t = 0 .. NT-1 (whole warps, all of them) call it with the same v, n
// and scratch; sync() is their barrier.  Thread t passes x = v[4t .. 4t+3]
// (zeros past n).  v is the whole row in shared memory (read only where the
// plain loop runs), n a multiple of 4 and at most 4 * NT.  Typical rows of
// 2048 squares have about 15 heads.
template <int NT>
struct OrderedSumScratch {
    static constexpr int kWarps = NT / 32;
    static constexpr int kPieces = 64;
    // Heads in order: {C lo, C hi, position << 12 | binade, head value bits}
    // with C the sum of the increments before the head, then {C total, n << 12};
    // the walk rewrites them as {increment, position << 12 | binade, head value
    // bits, next position} followed by three zero slots.
    int4 piece[kPieces + 4];
    float warp_total[kWarps];
    int warp_heads[kWarps];
    long long warp_inc[kWarps];
    float result;
};

namespace ordered_sum {

constexpr int kElemSat = 1 << 23;  // an increment this large always fails the walk's check

__device__ __forceinline__ uint32_t binade(float x) { return __float_as_uint(x) >> 23; }

// Adding v >= 0 to a sum in binade E (exponent field): the increment of m,
// round(v / u) (saturated), and whether v / u has a remainder of exactly one
// half.  v / u is v scaled by a power of two, exact in two float
// multiplications (a product that underflows is far below one half).
__device__ __forceinline__ int step_increment(float v, uint32_t E, int& tie) {
    const int k = 150 - max(static_cast<int>(E), 1);  // u = 2^-k
    const int k1 = k >> 1, k2 = k - k1;                 // each in [-52, 75]
    const float f = __fmul_rn(__fmul_rn(v, __int_as_float((k1 + 127) << 23)), __int_as_float((k2 + 127) << 23));
    tie = __fsub_rn(f, floorf(f)) == 0.5f;
    return f < static_cast<float>(kElemSat) ? __float2int_rn(f) : kElemSat;
}

}  // namespace ordered_sum

template <int NT, class Sync>
__device__ __forceinline__ float sum_in_order_par(float4 x, const float* v, int n, int t,
                                                  OrderedSumScratch<NT>& ws, Sync sync) {
    using namespace ordered_sum;
    constexpr int W = NT / 32;
    const unsigned full = 0xffffffffu;
    const int lane = t & 31, warp = t >> 5;

    // 1. Approximate prefix sums: a lane scan, then the warp totals.
    const float a = __fadd_rn(__fadd_rn(x.x, x.y), __fadd_rn(x.z, x.w));
    float inc = a;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(full, inc, o);
        if (lane >= o) inc = __fadd_rn(inc, y);
    }
    if (lane == 31) ws.warp_total[warp] = inc;
    sync();
    // Warp totals scanned across lanes (every warp computes the same values).
    float wscan = lane < W ? ws.warp_total[lane] : 0.0f;
#pragma unroll
    for (int o = 1; o < W; o <<= 1) {
        const float y = __shfl_up_sync(full, wscan, o);
        if (lane >= o) wscan = __fadd_rn(wscan, y);
    }
    const float before = warp > 0 ? __shfl_sync(full, wscan, warp > 0 ? warp - 1 : 0) : 0.0f;
    const float next_warp = __shfl_sync(full, wscan, warp);
    const float total = __shfl_sync(full, wscan, W - 1);
    const float base = __fadd_rn(before, __fsub_rn(inc, a));  // approximate sum before x
    // The approximate sum after x is the next thread's base, so a run that
    // crosses threads keeps one predicted binade.
    float next_base = __shfl_down_sync(full, base, 1);
    if (lane == 31) next_base = next_warp;
    const bool fast = fabsf(total) <= 3.4e38f && n <= 4 * NT;  // the same in every thread

    // 2. Heads and increments of this thread's four elements.
    const float P1 = __fadd_rn(base, x.x), P2 = __fadd_rn(P1, x.y), P3 = __fadd_rn(P2, x.z);
    const uint32_t E0 = binade(base), E1 = binade(P1), E2 = binade(P2), E3 = binade(P3), E4 = binade(next_base);
    int tie0, tie1, tie2, tie3;
    const int d0 = step_increment(x.x, E0, tie0), d1 = step_increment(x.y, E1, tie1);
    const int d2 = step_increment(x.z, E2, tie2), d3 = step_increment(x.w, E3, tie3);
    const bool mine = 4 * t < n;
    const int h0 = mine & ((t == 0) | tie0 | (E1 != E0)), h1 = mine & (tie1 | (E2 != E1));
    const int h2 = mine & (tie2 | (E3 != E2)), h3 = mine & (tie3 | (E4 != E3));
    const int i0 = mine & !h0 ? d0 : 0, i1 = mine & !h1 ? d1 : 0;
    const int i2 = mine & !h2 ? d2 : 0, i3 = mine & !h3 ? d3 : 0;
    const int nh = h0 + h1 + h2 + h3;
    const int incsum = i0 + i1 + i2 + i3;
    // Within a warp the increments add up to at most 32 x 4 x kElemSat = 2^30: the
    // warp scan runs in 32 bits, the sums across warps in 64.
    int hinc = nh;
    int cinc32 = incsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(full, hinc, o);
        const int z = __shfl_up_sync(full, cinc32, o);
        if (lane >= o) {
            hinc += y;
            cinc32 += z;
        }
    }
    const long long cinc = cinc32;
    if (lane == 31) {
        ws.warp_heads[warp] = hinc;
        ws.warp_inc[warp] = cinc;
    }
    sync();
    // Lane w (< W) holds warp w's heads and increments (at most 2^30, split
    // into 16-bit limbs so that no 32-bit sum over the block's warps can
    // wrap); independent warp reductions over the lanes of earlier warps and
    // over all of them give this warp's offsets and the totals.
    static_assert(NT / 32 <= 32, "one lane per warp");
    const bool mine_w = lane < W, earlier = lane < warp;
    const unsigned hw = mine_w ? static_cast<unsigned>(ws.warp_heads[lane]) : 0u;
    const unsigned cw = mine_w ? static_cast<unsigned>(ws.warp_inc[lane]) : 0u;
    const unsigned clo = cw & 0xffffu, chi = cw >> 16;
    const int heads_before = static_cast<int>(__reduce_add_sync(full, earlier ? hw : 0u));
    const long long c_before = (static_cast<long long>(__reduce_add_sync(full, earlier ? chi : 0u)) << 16) +
                               __reduce_add_sync(full, earlier ? clo : 0u);
    const int heads = static_cast<int>(__reduce_add_sync(full, hw));
    const long long c_total =
        (static_cast<long long>(__reduce_add_sync(full, chi)) << 16) + __reduce_add_sync(full, clo);
    if (!fast || heads > OrderedSumScratch<NT>::kPieces) {  // the plain loop
        if (t == 0) {
            float s = 0.0f;
            for (int i = 0; i < n; ++i) s = __fadd_rn(s, v[i]);
            ws.result = s;
        }
        sync();
        return ws.result;
    }

    // 3. The heads in order, each with the sum of the increments before it.
    {
        int k = heads_before + hinc - nh;
        long long c = c_before + cinc - incsum;
        const int i = 4 * t;
        if (h0) ws.piece[k++] = make_int4(static_cast<int>(c), static_cast<int>(c >> 32), (i << 12) | static_cast<int>(E1), __float_as_int(x.x));
        c += i0;
        if (h1) ws.piece[k++] = make_int4(static_cast<int>(c), static_cast<int>(c >> 32), ((i + 1) << 12) | static_cast<int>(E2), __float_as_int(x.y));
        c += i1;
        if (h2) ws.piece[k++] = make_int4(static_cast<int>(c), static_cast<int>(c >> 32), ((i + 2) << 12) | static_cast<int>(E3), __float_as_int(x.z));
        c += i2;
        if (h3) ws.piece[k] = make_int4(static_cast<int>(c), static_cast<int>(c >> 32), ((i + 3) << 12) | static_cast<int>(E4), __float_as_int(x.w));
        if (t == NT - 1)
            ws.piece[heads] = make_int4(static_cast<int>(c_total), static_cast<int>(c_total >> 32), n << 12, 0);
    }
    sync();

    // 4. The walk.  Warp 0 turns each head into {increment to the next head,
    // position << 12 | binade, head value bits, next position} (three zero
    // slots follow the last head: they add nothing).  Thread 0 then follows
    // the chain four heads at a time, the checks off the chain: a batch with
    // a failed check is redone from its start, checking each head.
    if (warp == 0) {
        int4 d[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
            const int j = lane + 32 * r;
            d[r] = make_int4(0, 0, 0, 0);
            if (j < heads) {
                const int4 p = ws.piece[j], pn = ws.piece[j + 1];
                const long long c0 = (static_cast<long long>(p.y) << 32) | static_cast<uint32_t>(p.x);
                const long long c1 = (static_cast<long long>(pn.y) << 32) | static_cast<uint32_t>(pn.x);
                d[r] = make_int4(static_cast<int>(min(c1 - c0, static_cast<long long>(kElemSat))), p.z, p.w,
                                 pn.z >> 12);
            }
        }
        __syncwarp();
#pragma unroll
        for (int r = 0; r < 3; ++r)
            if (lane + 32 * r < heads + 3) ws.piece[lane + 32 * r] = d[r];
        __syncwarp();
        if (lane == 0) {
            float s = 0.0f;
            for (int j = 0; j < heads; j += 4) {
                int4 p[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) p[u] = ws.piece[j + u];
                const float s0 = s;
                bool ok = true;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t Ej = static_cast<uint32_t>(p[u].y) & 0xfffu;
                    s = __fadd_rn(s, __int_as_float(p[u].z));
                    const uint32_t b = __float_as_uint(s);
                    const uint32_t nb = b + static_cast<uint32_t>(p[u].x);
                    ok &= (j + u >= heads) | (((b >> 23) == Ej) & ((nb >> 23) == Ej));
                    s = __uint_as_float(nb);
                }
                if (!ok) {
                    s = s0;
                    for (int u = 0; u < 4 && j + u < heads; ++u) {
                        const uint32_t Ej = static_cast<uint32_t>(p[u].y) & 0xfffu;
                        s = __fadd_rn(s, __int_as_float(p[u].z));
                        const uint32_t b = __float_as_uint(s);
                        const uint32_t nb = b + static_cast<uint32_t>(p[u].x);
                        if (((b >> 23) == Ej) & ((nb >> 23) == Ej)) {
                            s = __uint_as_float(nb);
                        } else {
                            for (int e = (p[u].y >> 12) + 1; e < p[u].w; ++e) s = __fadd_rn(s, v[e]);
                        }
                    }
                }
            }
            ws.result = s;
        }
    }
    sync();
    return ws.result;
}

}  // namespace leafq
