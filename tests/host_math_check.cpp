// Host build of leaf_b200/csrc/libm_math.cuh, the device restatements of
// libm's expf, expm1f / tanhf and the graph node's Gelu: the __f*_rn / __d*_rn
// intrinsics become plain IEEE float and double operations (compiled with
// -ffp-contract=off, so each is one rounding, as on the device), and the
// functions are compared bit for bit with the system libm over every
// stride-th float bit pattern.  Prints the mismatch count of each function.
// Test infrastructure (tests/test_libm_math_host.py); not part of the library.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#define __device__
#define __forceinline__ inline
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fsub_rn(float a, float b) { return a - b; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __fdiv_rn(float a, float b) { return a / b; }
static inline double __dmul_rn(double a, double b) { return a * b; }
static inline double __dsub_rn(double a, double b) { return a - b; }
static inline double __fma_rn(double a, double b, double c) { return std::fma(a, b, c); }
static inline float __double2float_rn(double d) { return static_cast<float>(d); }
static inline long long __double_as_longlong(double d) { long long v; std::memcpy(&v, &d, 8); return v; }
static inline double __longlong_as_double(long long v) { double d; std::memcpy(&d, &v, 8); return d; }
static inline uint32_t __float_as_uint(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float __uint_as_float(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline float __int_as_float(int v) { float f; std::memcpy(&f, &v, 4); return f; }
static inline int __float2int_rz(float f) { return static_cast<int>(f); }
static inline float __int2float_rn(int v) { return static_cast<float>(v); }

#include "../leaf_b200/csrc/libm_math.cuh"

static bool same(float a, float b) {
    return __float_as_uint(a) == __float_as_uint(b) || (std::isnan(a) && std::isnan(b));
}

int main(int argc, char** argv) {
    const uint64_t stride = argc > 1 ? std::strtoull(argv[1], nullptr, 10) : 257;
    const leafq::ExpTable& tab = leafq::exp_table();
    const float root_two_over_pi = 0.7978845608028654f;
    unsigned long long bad_exp = 0, bad_tanh = 0, bad_gelu = 0, count = 0;
    for (uint64_t u = 0; u < (1ull << 32); u += stride, ++count) {
        const float x = __uint_as_float(static_cast<uint32_t>(u));
        if (!same(leafq::expf_libm(x, tab), expf(x))) ++bad_exp;
        if (!same(leafq::tanhf_libm(x), tanhf(x))) ++bad_tanh;
        const float g = 0.5f * x * (1.0f + tanhf(root_two_over_pi * (x + 0.044715f * x * x * x)));
        if (!same(leafq::gelu_tanh_libm(x), g)) ++bad_gelu;
    }
    std::printf("%llu %llu %llu %llu\n", count, bad_exp, bad_tanh, bad_gelu);
    return 0;
}
