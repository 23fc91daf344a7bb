// Graph executor INT8 GEMM with per-output-channel weight scales,
// leaf::kernels::gemm_i8_per_channel (kernels/gemm.cpp:99-166): a [m, k]
// int8, b [k, n] int8 (n contiguous, the ONNX MatMul layout), out [m, n].
//
// 64x64 output tile per 256-thread block, 64-byte K steps staged in shared
// memory; b is transposed into shared memory on the way in so that four
// consecutive k of one column form one dp4a operand.  Each thread owns a
// 4x4 patch of int32 accumulators (exact), then the reference epilogue:
// value = (float(acc) * input_scale) * weight_scales[n]; value += bias[n]
// when given; ReLU as std::max(value, 0.0f) (keeps -0.0f and NaN).
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int TM = 64, TN = 64, TK = 64;
constexpr int kPad = 4;

__global__ void __launch_bounds__(256) gemm_i8_per_channel_kernel(
    const int8_t* __restrict__ a, const int8_t* __restrict__ b, const float* __restrict__ bias,
    float input_scale, const float* __restrict__ ws, float* __restrict__ out, int64_t m, int64_t k,
    int64_t n, int relu) {
    __shared__ __align__(16) int8_t As[TM][TK + kPad];
    __shared__ __align__(16) int8_t Bt[TN][TK + kPad];
    grid_dependency_wait();
    grid_launch_dependents();
    const int tid = threadIdx.x;
    const int tx = tid % 16, ty = tid / 16;
    const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.x * TN;
    int acc[4][4] = {};
    for (int64_t k0 = 0; k0 < k; k0 += TK) {
        // A tile: 64 rows x 64 bytes, 16 bytes per thread.
        {
            const int r = tid / 4, c = (tid % 4) * 16;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int64_t gm = m0 + r, gk = k0 + c + i;
                As[r][c + i] = (gm < m && gk < k) ? a[gm * k + gk] : int8_t(0);
            }
        }
        // B tile: 64 k-rows x 64 columns, stored transposed.
        {
            const int r = tid / 4, c = (tid % 4) * 16;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int64_t gk = k0 + r, gn = n0 + c + i;
                Bt[c + i][r] = (gk < k && gn < n) ? b[gk * n + gn] : int8_t(0);
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < TK; kk += 4) {
            int av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = *reinterpret_cast<const int*>(&As[ty * 4 + i][kk]);
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = *reinterpret_cast<const int*>(&Bt[tx * 4 + j][kk]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = dp4a(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t gm = m0 + ty * 4 + i;
        if (gm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx * 4 + j;
            if (gn >= n) continue;
            float value = __fmul_rn(__fmul_rn(__int2float_rn(acc[i][j]), input_scale), __ldg(ws + gn));
            if (bias) value = __fadd_rn(value, __ldg(bias + gn));
            if (relu) value = value < 0.0f ? 0.0f : value;
            out[gm * n + gn] = value;
        }
    }
}

}  // namespace

int launch_gemm_i8_per_channel(cudaStream_t s, const int8_t* a, const int8_t* b,
                               const float* bias, float input_scale, const float* wscales,
                               float* out, int64_t m, int64_t k, int64_t n, int activation) {
    if (m == 0 || n == 0) return LEAFQ_OK;
    const dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
    return launch(gemm_i8_per_channel_kernel, grid, dim3(256), 0, s, false, "gemm_i8_per_channel", a, b,
                  bias, input_scale, wscales, out, m, k, n, activation == 1 ? 1 : 0);
}

}  // namespace leafq
