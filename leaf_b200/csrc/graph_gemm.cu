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
#include <algorithm>

#include "decoder_math.cuh"
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int TM = 64, TN = 64, TK = 64;
constexpr int kPad = 4;

// The Gemm / MatMul node epilogue of execute_quant_linear
// (executor.cpp:593-613) applied after the per-channel scale:
// value = alpha * value; value += beta * C[index] (C a scalar, a row [n] or
// the full [m, n]); then the node's fused activation.
struct GraphGlue {
    int on;           // 0: plain gemm_i8_per_channel epilogue
    float alpha, beta;
    const float* c;   // NULL: no C input
    int c_kind;       // 1 scalar, 2 row [n], 3 full [m, n]
    int activation;   // 0 none, 1 Relu, 2 Silu
};

__device__ __forceinline__ float graph_glue(float value, const GraphGlue& g, int64_t row, int64_t col,
                                            int64_t n, const ExpTable& tab) {
    value = __fmul_rn(g.alpha, value);
    if (g.c) {
        const int64_t idx = g.c_kind == 1 ? 0 : g.c_kind == 2 ? col : row * n + col;
        value = __fadd_rn(value, __fmul_rn(g.beta, __ldg(g.c + idx)));
    }
    if (g.activation == 1) value = value < 0.0f ? 0.0f : value;  // std::max(value, 0.0f)
    if (g.activation == 2) value = __fdiv_rn(value, __fadd_rn(1.0f, expf_libm(-value, tab)));
    return value;
}

// b is [k, n] (n contiguous; ONNX MatMul / Gemm without transB) or, with
// b_kmajor, [n, k] (k contiguous; Gemm with transB = 1).
__global__ void __launch_bounds__(256) gemm_i8_per_channel_kernel(
    const int8_t* __restrict__ a, const int8_t* __restrict__ b, const float* __restrict__ bias,
    float input_scale, const float* __restrict__ ws, float* __restrict__ out, int64_t m, int64_t k,
    int64_t n, int relu, int b_kmajor, const GraphGlue glue, const __grid_constant__ ExpTable tab_g) {
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
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
                Bt[c + i][r] = (gk < k && gn < n) ? b[b_kmajor ? gn * k + gk : gk * n + gn] : int8_t(0);
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
            if (glue.on) value = graph_glue(value, glue, gm, gn, n, tab);
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
    const GraphGlue none{0, 1.0f, 0.0f, nullptr, 0, 0};
    return launch(gemm_i8_per_channel_kernel, grid, dim3(256), 0, s, false, "gemm_i8_per_channel", a, b,
                  bias, input_scale, wscales, out, m, k, n, activation == 1 ? 1 : 0, 0, none, exp_table());
}

namespace {
// Static quantiser of a [k, m] input read transposed into [m, k] codes
// (execute_quant_linear with transA, executor.cpp:549-556: the transpose is
// taken before quantize_input, which is elementwise).
__global__ void graph_quantize_transposed_kernel(const float* __restrict__ x, int64_t m, int64_t k,
                                                 float scale, int8_t* __restrict__ q, int32_t* error_flag) {
    const int64_t count = m * k;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / k, col = i - row * k;
        const float v = x[col * m + row];
        if (!isfinite(v)) {
            if (error_flag) atomicExch(error_flag, 1);
            q[i] = 0;
            continue;
        }
        float scaled = __fdiv_rn(v, scale);
        scaled = fmaxf(-127.0f, fminf(127.0f, scaled));
        q[i] = static_cast<int8_t>(__float2int_rn(scaled));
    }
}
}  // namespace

int launch_graph_linear(cudaStream_t s, const float* a, int64_t m, int64_t k, int trans_a,
                        const int8_t* weight, int64_t n, int trans_b, float input_scale,
                        const float* wscales, float alpha, float beta, const float* c, int c_kind,
                        int activation, float* out, int8_t* codes, int32_t* error_flag) {
    if (m == 0 || n == 0) return LEAFQ_OK;
    int st;
    if (trans_a) {
        const int64_t blocks = std::min<int64_t>((m * k + 255) / 256, static_cast<int64_t>(sm_count()) * 8);
        st = launch(graph_quantize_transposed_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s,
                    false, "graph_quantize", a, m, k, input_scale, codes, error_flag);
    } else {
        st = launch_graph_quantize(s, a, m * k, input_scale, codes, error_flag);
    }
    if (st) return st;
    const GraphGlue glue{1, alpha, beta, c, c ? c_kind : 0, activation};
    const dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
    return launch(gemm_i8_per_channel_kernel, grid, dim3(256), 0, s, false, "gemm_i8_per_channel", codes,
                  weight, static_cast<const float*>(nullptr), input_scale, wscales, out, m, k, n, 0,
                  trans_b ? 1 : 0, glue, exp_table());
}

}  // namespace leafq
