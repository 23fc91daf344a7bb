// Integer linear from codes for any group size (W8A8 grouped, W4A8), and
// the exact-order generic weight-only kernel (W4A32 / W8A32 / FP32 with any
// token count or group).
//
// linear_int_q_kernel: one warp per (token, row) -- few tokens, INT4, groups
//   that are not multiples of 32, or when the int32 group sums are wanted
//   (grouped INT8 with more tokens runs on the tensor cores instead,
//   gemm_grouped_tc.cu).  Groups are walked in
//   order; each group's int32 sum is exact (dp4a when the group is a
//   multiple of 4 codes), then result = fma(float(acc) * sx, sw, result)
//   (decoder.cpp:566-568, GCC-fused), or the two-rounding form of the VNNI
//   tile (:695-700) when `fused` is false; finally + bias (:1229).
// linear_f32act_kernel: one warp per (row, block of four tokens), lanes laid
//   out as the eight AVX lanes of the four accumulators of dot_avx
//   (decoder.cpp:355-391), so every rounding happens in the same order:
//   four 8-lane FMA chains over 32-column blocks when the block has one
//   token, one chain per token over 8-column steps otherwise, the lane tree
//   of reduce() (:294-298), the scalar tail, and result = fma(partial,
//   scale, result) per group.
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

__device__ __forceinline__ int weight_code(const uint8_t* w, int64_t index, int bits) {
    if (bits == 8) return static_cast<int8_t>(w[index]);
    const int code = (w[index >> 1] >> ((index & 1) * 4)) & 15;
    return code >= 8 ? code - 16 : code;
}

__device__ __forceinline__ float weight_value(const void* w, int64_t index, int bits) {
    if (bits == 32) return static_cast<const float*>(w)[index];
    return static_cast<float>(weight_code(static_cast<const uint8_t*>(w), index, bits));
}

// Eight signed nibbles of one 32-bit word as two words of four int8 each:
// lo = nibbles 0,1,2,3 (columns c..c+3), hi = nibbles 4..7.
__device__ __forceinline__ void unpack_nibbles(uint32_t packed, int& lo, int& hi) {
    // Spread nibbles into bytes: byte j of lo = nibble j, byte j of hi = nibble j + 4.
    const uint32_t even = packed & 0x0f0f0f0fu;         // nibbles 0,2,4,6 in bytes 0..3
    const uint32_t odd = (packed >> 4) & 0x0f0f0f0fu;   // nibbles 1,3,5,7 in bytes 0..3
    uint32_t a = __byte_perm(even, odd, 0x5140);        // n0 n1 n2 n3
    uint32_t b = __byte_perm(even, odd, 0x7362);        // n4 n5 n6 n7
    // Sign-extend each 4-bit value held in a byte: (v ^ 8) - 8 per byte.
    a ^= 0x08080808u;
    b ^= 0x08080808u;
    lo = static_cast<int>(__vsub4(a, 0x08080808u));
    hi = static_cast<int>(__vsub4(b, 0x08080808u));
}

__global__ void linear_int_q_kernel(const int8_t* __restrict__ q, const float* __restrict__ sx,
                                    int64_t tokens, int64_t cols, const uint8_t* __restrict__ w,
                                    const float* __restrict__ ws, int64_t rows, int bits,
                                    int64_t group, const float* __restrict__ bias,
                                    float* __restrict__ y, int32_t* __restrict__ acc, int fused) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t groups = cols / group;
    // Word-wise path: 4 codes per step for int8 (group % 4 == 0), 8 for int4
    // (group % 8 == 0); rows stay 4-byte aligned when cols allows it.
    const bool words8 = bits == 8 && group % 4 == 0 && cols % 4 == 0 &&
                        (reinterpret_cast<uintptr_t>(w) & 3u) == 0 &&
                        (reinterpret_cast<uintptr_t>(q) & 3u) == 0;
    const bool words4 = bits == 4 && group % 8 == 0 && cols % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(w) & 3u) == 0 &&
                        (reinterpret_cast<uintptr_t>(q) & 3u) == 0;
    for (int64_t item = warp0; item < rows * tokens; item += nwarps) {
        const int64_t row = item % rows, t = item / rows;
        const int8_t* qt = q + t * cols;
        const float token_scale = sx[t];
        float result = 0.0f;
        for (int64_t g = 0; g < groups; ++g) {
            const int64_t c0 = g * group, c1 = c0 + group;
            int sum = 0;
            if (words8) {
                const int* wr = reinterpret_cast<const int*>(w + row * cols);
                const int* qr = reinterpret_cast<const int*>(qt);
                for (int64_t c = c0 / 4 + lane; c < c1 / 4; c += 32) sum = dp4a(wr[c], qr[c], sum);
            } else if (words4) {
                const uint32_t* wr = reinterpret_cast<const uint32_t*>(w + row * (cols / 2));
                const int* qr = reinterpret_cast<const int*>(qt);
                for (int64_t c = c0 / 8 + lane; c < c1 / 8; c += 32) {
                    int lo, hi;
                    unpack_nibbles(wr[c], lo, hi);
                    sum = dp4a(lo, qr[2 * c], sum);
                    sum = dp4a(hi, qr[2 * c + 1], sum);
                }
            } else {
                for (int64_t c = c0 + lane; c < c1; c += 32)
                    sum += weight_code(w, row * cols + c, bits) * static_cast<int>(qt[c]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (acc && lane == 0) acc[(t * rows + row) * groups + g] = sum;
            const float product = __fmul_rn(__int2float_rn(sum), token_scale);
            const float scale = __ldg(ws + row * groups + g);
            result = fused ? __fmaf_rn(product, scale, result)
                           : __fadd_rn(result, __fmul_rn(product, scale));
        }
        if (lane == 0) y[t * rows + row] = __fadd_rn(result, bias ? __ldg(bias + row) : 0.0f);
    }
}

// dot_avx's reduce(): lanes (i, i+4), then (h0 + h2) + (h1 + h3).  `v` is
// lane l's value for l in [base, base + 8); the result is valid in lane base.
__device__ __forceinline__ float lane_tree8(float v) {
    const float h = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
    const float p = __fadd_rn(h, __shfl_down_sync(0xffffffffu, h, 2, 8));
    return __fadd_rn(p, __shfl_down_sync(0xffffffffu, p, 1, 8));
}

__global__ void linear_f32act_kernel(const float* __restrict__ x, int64_t tokens, int64_t cols,
                                     const void* __restrict__ w, const float* __restrict__ ws,
                                     int64_t rows, int bits, int64_t group,
                                     const float* __restrict__ bias, float* __restrict__ y) {
    grid_dependency_wait();
    grid_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int seg = lane >> 3, sub = lane & 7;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t gsize = bits == 32 ? cols : group;
    const int64_t groups = cols / gsize;
    const int64_t blocks = (tokens + 3) / 4;
    for (int64_t item = warp0; item < rows * blocks; item += nwarps) {
        const int64_t row = item % rows, blk = item / rows;
        const int64_t token0 = blk * 4;
        const int count = static_cast<int>(min64(4, tokens - token0));
        const float* xb = x + token0 * cols;
        const int64_t base = row * cols;
        float result = 0.0f;  // lane 8*t holds token t's result
        for (int64_t g = 0; g < groups; ++g) {
            int64_t col = g * gsize;
            const int64_t end = col + gsize;
            float chain = 0.0f;  // lane 8*t + l: chain of token t, AVX lane l
            if (count == 1) {
                // Four accumulators a,b,c,d = lanes 0-7, 8-15, 16-23, 24-31.
                for (; col + 32 <= end; col += 32)
                    chain = __fmaf_rn(weight_value(w, base + col + lane, bits), xb[col + lane], chain);
                const float b = __shfl_down_sync(0xffffffffu, chain, 8);
                const float c = __shfl_down_sync(0xffffffffu, chain, 16);
                const float d = __shfl_down_sync(0xffffffffu, chain, 24);
                if (lane < 8) chain = __fadd_rn(__fadd_rn(chain, b), __fadd_rn(c, d));
                else chain = 0.0f;
            }
            for (; col + 8 <= end; col += 8) {
                if (seg < count)
                    chain = __fmaf_rn(weight_value(w, base + col + sub, bits),
                                      xb[seg * cols + col + sub], chain);
            }
            float partial = lane_tree8(chain);
            const float scale = bits == 32 ? 1.0f : __ldg(ws + row * groups + g);
            if (sub == 0 && seg < count) {
                for (; col < end; ++col) {
                    const float stored = bits == 32 ? weight_value(w, base + col, bits)
                        : __fmul_rn(weight_value(w, base + col, bits), scale);
                    const float value = __fdiv_rn(stored, scale);
                    partial = __fmaf_rn(value, xb[seg * cols + col], partial);
                }
                result = __fmaf_rn(partial, scale, result);
            }
        }
        if (sub == 0 && seg < count)
            y[(token0 + seg) * rows + row] = __fadd_rn(result, bias ? __ldg(bias + row) : 0.0f);
    }
}

unsigned warp_grid(int64_t items, int threads) {
    const int64_t warps_per_block = threads / 32;
    int64_t blocks = (items + warps_per_block - 1) / warps_per_block;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return static_cast<unsigned>(blocks);
}

}  // namespace

int launch_linear_int_q(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens,
                        int64_t cols, const void* weight, const float* wscales, int64_t rows,
                        int bits, int64_t group, const float* bias, float* y, int32_t* acc,
                        bool fused, bool pdl) {
    if (rows == 0 || tokens == 0) return LEAFQ_OK;
    // Grouped INT8 with many tokens: the tensor cores (same bits; no int32
    // group sums are written there, so a caller asking for them stays here).
    if (!acc && gemm_grouped_tc_supported(tokens, cols, rows, bits, group, weight, q))
        return launch_gemm_grouped_tc(s, q, sx, tokens, cols, static_cast<const int8_t*>(weight), wscales, rows,
                                      group, bias, y, fused, pdl);
    return launch(linear_int_q_kernel, dim3(warp_grid(rows * tokens, 256)), dim3(256), 0, s, pdl,
                  "linear_int_q", q, sx, tokens, cols, static_cast<const uint8_t*>(weight),
                  wscales, rows, bits, group, bias, y, acc, fused ? 1 : 0);
}

int launch_linear_f32act(cudaStream_t s, const float* x, int64_t tokens, int64_t cols,
                         const void* weight, const float* wscales, int64_t rows, int bits,
                         int64_t group, const float* bias, float* y, bool pdl) {
    if (rows == 0 || tokens == 0) return LEAFQ_OK;
    const int64_t items = rows * ((tokens + 3) / 4);
    return launch(linear_f32act_kernel, dim3(warp_grid(items, 256)), dim3(256), 0, s, pdl,
                  "linear_f32act", x, tokens, cols, weight, wscales, rows, bits, group, bias, y);
}

}  // namespace leafq
