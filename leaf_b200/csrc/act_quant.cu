// Activation quantisers.
//
// quantize_act_kernel: per-token dynamic INT8 (decoder.cpp:1028-1038 with
//   quantize_input_avx, :618-627).  One 256-thread block per token row: a
//   block-wide absmax (fmaxf is exact and order-free), then
//   scale = max(absmax / 127, 1e-12) with IEEE division, multiplier =
//   1 / scale (IEEE), code = round-half-even(x * multiplier).  __fmul_rn and
//   __fdiv_rn keep the compiler from fusing or approximating any step.
// quantize_act_warp_kernel: the same arithmetic with one warp per token row
//   and the row held in registers (rows of at most 2048 aligned floats): one
//   read of x, a shuffle-only absmax, and up to 16 float4 loads in flight per
//   lane, where the block kernel reads each row twice across two block
//   barriers with 2 loads in flight per thread (4096 x 2048: about 2 TB/s).
// graph_quantize_kernel: the graph executor's static quantiser
//   (executor.cpp:220-230): division by the calibrated scale, clamp to
//   [-127, 127], nearbyint.
#include <algorithm>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kQuantThreads = 256;

__device__ __forceinline__ int8_t code_of(float value, float multiplier) { return act_code(value, multiplier); }

__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max_f32(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (blockDim.x >> 5) ? scratch[lane] : 0.0f;
        v = warp_max_f32(v);
        if (lane == 0) scratch[32] = v;
    }
    __syncthreads();
    return scratch[32];
}

__device__ __forceinline__ float4 scale4(float4 v, const float* __restrict__ col_scale, int64_t i) {
    if (!col_scale) return v;
    const float4 f = __ldg(reinterpret_cast<const float4*>(col_scale) + i);
    return make_float4(__fmul_rn(v.x, f.x), __fmul_rn(v.y, f.y), __fmul_rn(v.z, f.z), __fmul_rn(v.w, f.w));
}

// col_scale (may be NULL): the calibrated SmoothQuant factors of the
// weight's input_scale tensor, x[t][col] * col_scale[col] taken before the
// quantisation (decoder.cpp:1008-1019; one float rounding, as there).
__global__ void __launch_bounds__(kQuantThreads) quantize_act_kernel(const float* __restrict__ x,
                                                                      int64_t cols,
                                                                      int8_t* __restrict__ q,
                                                                      float* __restrict__ scales,
                                                                      const float* __restrict__ col_scale) {
    __shared__ float scratch[33];
    grid_dependency_wait();
    grid_launch_dependents();
    const int64_t row = blockIdx.x;
    const float* in = x + row * cols;
    int8_t* out = q + row * cols;
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(in) & 15u) == 0) &&
                     ((reinterpret_cast<uintptr_t>(col_scale) & 15u) == 0);
    auto scalar = [&](int64_t i) {
        const float v = __ldg(in + i);
        return col_scale ? __fmul_rn(v, __ldg(col_scale + i)) : v;
    };
    float m = 0.0f;
    if (vec) {
        const float4* in4 = reinterpret_cast<const float4*>(in);
        for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
            const float4 v = scale4(__ldg(in4 + i), col_scale, i);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, fabsf(scalar(i)));
    }
    const float absmax = block_max(m, scratch);
    const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
    const float multiplier = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) scales[row] = scale;
    if (vec && ((reinterpret_cast<uintptr_t>(out) & 3u) == 0)) {
        const float4* in4 = reinterpret_cast<const float4*>(in);
        char4* out4 = reinterpret_cast<char4*>(out);
        for (int64_t i = threadIdx.x; i < cols / 4; i += blockDim.x) {
            const float4 v = scale4(__ldg(in4 + i), col_scale, i);
            out4[i] = make_char4(code_of(v.x, multiplier), code_of(v.y, multiplier),
                                 code_of(v.z, multiplier), code_of(v.w, multiplier));
        }
    } else {
        for (int64_t i = threadIdx.x; i < cols; i += blockDim.x)
            out[i] = code_of(scalar(i), multiplier);
    }
}

constexpr int kWarpQuantWarps = 1;  // warps (token rows) per block: small blocks fit beside an early-launched GEMM CTA
constexpr int kWarpQuantMaxCols = 32 * 4 * 16;

// Token row blockIdx.x * kWarpQuantWarps + warp; lane holds float4 columns lane + 32 j.
// Requires cols % 4 == 0, x, q and col_scale 16- / 4- / 16-byte aligned (every
// row too: cols % 4 == 0 keeps x rows 16-byte and code rows 4-byte aligned).
template <int kVec>
__global__ void __launch_bounds__(kWarpQuantWarps * 32) quantize_act_warp_kernel(
    const float* __restrict__ x, int64_t tokens, int64_t cols, int8_t* __restrict__ q, float* __restrict__ scales,
    const float* __restrict__ col_scale) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarpQuantWarps + (threadIdx.x >> 5);
    if (row >= tokens) return;
    const int64_t vecs = cols / 4;
    const float4* in4 = reinterpret_cast<const float4*>(x + row * cols);
    float4 v[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        const int64_t i = lane + 32 * j;
        v[j] = i < vecs ? __ldg(in4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        const int64_t i = lane + 32 * j;
        if (col_scale && i < vecs) v[j] = scale4(v[j], col_scale, i);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    }
    m = warp_max_f32(m);
    const float scale = fmaxf(__fdiv_rn(m, 127.0f), 1e-12f);
    const float multiplier = __fdiv_rn(1.0f, scale);
    if (lane == 0) scales[row] = scale;
    char4* out4 = reinterpret_cast<char4*>(q + row * cols);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        const int64_t i = lane + 32 * j;
        if (i < vecs)
            out4[i] = make_char4(code_of(v[j].x, multiplier), code_of(v[j].y, multiplier),
                                 code_of(v[j].z, multiplier), code_of(v[j].w, multiplier));
    }
}

template <int kVec>
int launch_warp_quant(cudaStream_t s, const float* x, int64_t tokens, int64_t cols, int8_t* q, float* scales,
                      bool pdl, const float* col_scale) {
    const int64_t blocks = (tokens + kWarpQuantWarps - 1) / kWarpQuantWarps;
    return launch(quantize_act_warp_kernel<kVec>, dim3(static_cast<unsigned>(blocks)), dim3(kWarpQuantWarps * 32),
                  0, s, pdl, "quantize_act_warp", x, tokens, cols, q, scales, col_scale);
}

__global__ void graph_quantize_kernel(const float* __restrict__ x, int64_t count, float scale,
                                      int8_t* __restrict__ q, int32_t* error_flag) {
    grid_dependency_wait();
    grid_launch_dependents();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
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

int launch_quantize_act(cudaStream_t s, const float* x, int64_t tokens, int64_t cols, int8_t* q,
                        float* scales, bool pdl, const float* col_scale) {
    if (tokens == 0) return LEAFQ_OK;
    // Fewer rows than SMs (decode batches): a 256-thread block per row, so the
    // row's loads and codes are spread over eight warps instead of one.
    const bool warp_rows = tokens >= sm_count() && cols % 4 == 0 && cols <= kWarpQuantMaxCols && aligned16(x) &&
                           (reinterpret_cast<uintptr_t>(q) & 3u) == 0 && (!col_scale || aligned16(col_scale));
    if (warp_rows) {
        const int64_t vecs = cols / 4;
        if (vecs <= 32) return launch_warp_quant<1>(s, x, tokens, cols, q, scales, pdl, col_scale);
        if (vecs <= 64) return launch_warp_quant<2>(s, x, tokens, cols, q, scales, pdl, col_scale);
        if (vecs <= 128) return launch_warp_quant<4>(s, x, tokens, cols, q, scales, pdl, col_scale);
        if (vecs <= 256) return launch_warp_quant<8>(s, x, tokens, cols, q, scales, pdl, col_scale);
        return launch_warp_quant<16>(s, x, tokens, cols, q, scales, pdl, col_scale);
    }
    return launch(quantize_act_kernel, dim3(static_cast<unsigned>(tokens)), dim3(kQuantThreads), 0,
                  s, pdl, "quantize_act", x, cols, q, scales, col_scale);
}

namespace {
__global__ void scale_columns_kernel(const float* __restrict__ x, int64_t tokens, int64_t cols,
                                     const float* __restrict__ col_scale, float* __restrict__ y) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int64_t n = tokens * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        y[i] = __fmul_rn(x[i], __ldg(col_scale + i % cols));
}
}  // namespace

int launch_scale_columns(cudaStream_t s, const float* x, int64_t tokens, int64_t cols, const float* col_scale,
                         float* y, bool pdl) {
    if (tokens == 0) return LEAFQ_OK;
    const int64_t blocks = std::min<int64_t>((tokens * cols + 255) / 256, static_cast<int64_t>(sm_count()) * 8);
    return launch(scale_columns_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, pdl, "scale_columns",
                  x, tokens, cols, col_scale, y);
}

int launch_graph_quantize(cudaStream_t s, const float* x, int64_t count, float scale, int8_t* q,
                          int32_t* error_flag) {
    if (count == 0) return LEAFQ_OK;
    const int64_t blocks64 = (count + 255) / 256;
    const unsigned blocks = static_cast<unsigned>(blocks64 < 4 * 148 * 8 ? blocks64 : 4 * 148 * 8);
    return launch(graph_quantize_kernel, dim3(blocks), dim3(256), 0, s, false, "graph_quantize", x,
                  count, scale, q, error_flag);
}

}  // namespace leafq
