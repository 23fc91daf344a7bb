// W4A32 decode GEMV (INT4 weight-only, fp32 activations, one token) in the
// exact rounding order of the reference's dot_avx (decoder.cpp:355-391).
//
// For one token and a group of G = 32k columns, dot_avx keeps four 8-lane
// accumulators a,b,c,d fed by FMAs over 32-column blocks (a: columns 0-7 of
// each block, b: 8-15, c: 16-23, d: 24-31), combines them as
// (a + b) + (c + d), reduces the 8 lanes as (l, l+4) then (h0 + h2) +
// (h1 + h3) (reduce(), :294-298) and adds partial * scale to the row sum
// with one FMA, group after group (GCC fuses :386).
//
// Groups of 32 columns run gemv_w4a32_g32_kernel below (16 compute warps,
// packed f32x2 arithmetic, a walker warp overlapping the ordered group
// chains with the next stage).  Other group sizes run gemv_w4a32_kernel:
// one block per SM, a producer warp streams stages of 16
// rows -- the packed weights (cols / 2 bytes per row) and their group
// scales -- with 1-D bulk copies.  Each of the 256 consumer threads owns one
// group index g (and a row slot when a row has fewer than 256 groups) and
// keeps that group's x values in registers for the whole kernel, so x is
// read once per block.  Per stage, threads compute their group's partial
// for their rows into shared memory; then one thread per row walks the
// groups in order with the fused multiply-add.  All arithmetic uses the
// explicit _rn intrinsics, so nothing is re-associated or contracted.
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumers = 256;
constexpr int kThreads = kConsumers + 32;
constexpr int kRowsPerStage = 16;
constexpr int kSmemBudget = 200 * 1024;

struct W4Args {
    const float* x;
    const uint8_t* w;
    const float* ws;
    const float* bias;
    float* y;
    int64_t cols;
    int64_t rows;
    int groups;  // groups per row
    int stages;
};

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

// Signed value of nibble `i` of a 32-bit word, as an exact float: the
// nibble (xor 8) is placed in the mantissa of 2^23 and the bias removed.
__device__ __forceinline__ float nibble_value(uint32_t biased_bytes, int byte_index) {
    // biased_bytes holds four nibbles (already xor 8) in its bytes.
    const uint32_t bits = __byte_perm(biased_bytes, 0x4B000000u, 0x7540u | (byte_index & 3));
    return __fsub_rn(__uint_as_float(bits), 8388616.0f);  // 2^23 + 8
}

template <int GS>
__global__ void __launch_bounds__(kThreads, 1) gemv_w4a32_kernel(const W4Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int S = a.stages;
    const int G = a.groups;
    const int row_bytes = static_cast<int>(a.cols / 2);
    const int w_bytes = kRowsPerStage * row_bytes;
    const int s_bytes = kRowsPerStage * G * 4;
    const int stage_bytes = w_bytes + s_bytes;
    uint8_t* stages = smem;
    float* P = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes);  // [RS][G+1]
    float* SC = P + kRowsPerStage * (G + 1);
    uint64_t* full = reinterpret_cast<uint64_t*>(SC + kRowsPerStage * (G + 1));
    uint64_t* empty = full + S;
    // Raised when a wait gives up; consumers keep arriving at every block
    // barrier and return together after it.
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.x * a.rows / gridDim.x;
    const int64_t row1 = (int64_t)(blockIdx.x + 1) * a.rows / gridDim.x;
    const int nblocks = static_cast<int>((row1 - row0 + kRowsPerStage - 1) / kRowsPerStage);

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers / 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    grid_launch_dependents();

    if (warp == kConsumers / 32) {
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            for (int s = 0; s < nblocks; ++s) {
                const int buf = s % S;
                if (s >= S && !mbar_wait(&empty[buf], ((s / S) - 1) & 1, kSiteW4Empty)) break;
                const int64_t r = row0 + (int64_t)s * kRowsPerStage;
                const int live = static_cast<int>(min64(kRowsPerStage, row1 - r));
                uint8_t* dst = stages + (size_t)buf * stage_bytes;
                mbar_arrive_expect_tx(&full[buf], static_cast<uint32_t>(live * (row_bytes + G * 4)));
                bulk_copy_g2s(dst, a.w + r * row_bytes, static_cast<uint32_t>(live * row_bytes),
                              &full[buf], policy);
                bulk_copy_g2s(dst + w_bytes, a.ws + r * G, static_cast<uint32_t>(live * G * 4),
                              &full[buf], policy);
            }
        }
        return;
    }

    grid_dependency_wait();
    const int tid = threadIdx.x;
    const int slots = kConsumers / G;  // >= 1
    const int g = tid % G;
    const int slot = tid / G;
    const bool active = slot < slots;
    float xr[GS];
#pragma unroll
    for (int i = 0; i < GS; i += 4) {
        const float4 v = active ? __ldg(reinterpret_cast<const float4*>(a.x + (int64_t)g * GS + i))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        xr[i] = v.x;
        xr[i + 1] = v.y;
        xr[i + 2] = v.z;
        xr[i + 3] = v.w;
    }

    for (int s = 0; s < nblocks; ++s) {
        const int buf = s % S;
        const int64_t r0 = row0 + (int64_t)s * kRowsPerStage;
        const int live = static_cast<int>(min64(kRowsPerStage, row1 - r0));
        const bool landed = mbar_wait(&full[buf], (s / S) & 1, kSiteW4Full);
        if (!landed) *abort_flag = 1;
        const uint8_t* sw = stages + (size_t)buf * stage_bytes;
        const float* sscale = reinterpret_cast<const float*>(sw + w_bytes);
        if (landed && active) {
            for (int r = slot; r < live; r += slots) {
                const uint4* packed =
                    reinterpret_cast<const uint4*>(sw + (size_t)r * row_bytes + (size_t)g * (GS / 2));
                float acc[4][8];
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int l = 0; l < 8; ++l) acc[j][l] = 0.0f;
#pragma unroll
                for (int blk = 0; blk < GS / 32; ++blk) {
                    const uint4 v = packed[blk];
                    const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // word j = columns 8j..8j+7 of this 32-column block.
                        const uint32_t even = (words[j] & 0x0f0f0f0fu) ^ 0x08080808u;
                        const uint32_t odd = ((words[j] >> 4) & 0x0f0f0f0fu) ^ 0x08080808u;
#pragma unroll
                        for (int l = 0; l < 8; ++l) {
                            const float wv = nibble_value((l & 1) ? odd : even, l >> 1);
                            acc[j][l] = __fmaf_rn(wv, xr[blk * 32 + 8 * j + l], acc[j][l]);
                        }
                    }
                }
                float lanes[8];
#pragma unroll
                for (int l = 0; l < 8; ++l)
                    lanes[l] = __fadd_rn(__fadd_rn(acc[0][l], acc[1][l]), __fadd_rn(acc[2][l], acc[3][l]));
                const float h0 = __fadd_rn(lanes[0], lanes[4]), h1 = __fadd_rn(lanes[1], lanes[5]);
                const float h2 = __fadd_rn(lanes[2], lanes[6]), h3 = __fadd_rn(lanes[3], lanes[7]);
                P[r * (G + 1) + g] = __fadd_rn(__fadd_rn(h0, h2), __fadd_rn(h1, h3));
                SC[r * (G + 1) + g] = sscale[r * G + g];
            }
        }
        consumer_sync();
        if (*abort_flag) return;
        if (lane == 0) mbar_arrive(&empty[buf]);
        if (tid < live) {
            float result = 0.0f;
            const float* pr = P + tid * (G + 1);
            const float* sr = SC + tid * (G + 1);
#pragma unroll 16
            for (int k = 0; k < G; ++k) result = __fmaf_rn(pr[k], sr[k], result);
            const int64_t row = r0 + tid;
            a.y[row] = __fadd_rn(result, a.bias ? __ldg(a.bias + row) : 0.0f);
        }
        consumer_sync();
    }
}

// ------------------------------------------------------------------------
// Groups of 32 columns (the reference's default INT4 export, config 1): one
// 32-column block per group, so every accumulator lane is one product
// fma(w, x, 0).  18 warps: 16 compute warps, a walker warp and the producer.
// Compute thread (g, slot) keeps group g's 32 x values in registers as 16
// packed pairs and computes the group partial of rows slot, slot + slots, ...
// of each stage with packed f32x2 arithmetic -- element-wise .rn operations
// on independent lanes, so each value's rounding sequence is dot_avx's:
//   a..d (pairs of lanes) = fma(w, x, 0); lanes = (a + b) + (c + d);
//   (h0, h1) = lanes[0:2] + lanes[4:6], (h2, h3) = lanes[2:4] + lanes[6:8];
//   partial = (h0 + h2) + (h1 + h3).
// The walker warp then runs each row's ordered chain
// result = fma(partial_g, scale_g, result) over the groups of stage s while
// the compute warps work on stage s + 1 (partials double-buffered; named
// barriers: kReady + b when buffer b is written, kFree + b when it is read).
constexpr int kCompute32 = 512;
constexpr int kThreads32 = kCompute32 + 64;
constexpr int kBarReady = 1, kBarFree = 3;

__global__ void __launch_bounds__(kThreads32, 1) gemv_w4a32_g32_kernel(const W4Args a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int S = a.stages;
    const int G = a.groups;
    const int row_bytes = static_cast<int>(a.cols / 2);
    const int w_bytes = kRowsPerStage * row_bytes;
    const int s_bytes = kRowsPerStage * G * 4;
    const int stage_bytes = w_bytes + s_bytes;
    const int pstride = G + 1;
    uint8_t* stages = smem;
    float* P = reinterpret_cast<float*>(smem + (size_t)S * stage_bytes);  // [2][RS][G+1]
    float* SC = P + 2 * kRowsPerStage * pstride;                          // [2][RS][G+1]
    uint64_t* full = reinterpret_cast<uint64_t*>(SC + 2 * kRowsPerStage * pstride);
    uint64_t* empty = full + S;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.x * a.rows / gridDim.x;
    const int64_t row1 = (int64_t)(blockIdx.x + 1) * a.rows / gridDim.x;
    const int nblocks = static_cast<int>((row1 - row0 + kRowsPerStage - 1) / kRowsPerStage);
    constexpr int kWalker = kCompute32 / 32, kProducer = kWalker + 1;
    constexpr int kParties = kCompute32 + 32;  // compute warps + walker

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCompute32 / 32);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    grid_launch_dependents();

    if (warp == kProducer) {
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            for (int s = 0; s < nblocks; ++s) {
                const int buf = s % S;
                if (s >= S && !mbar_wait(&empty[buf], ((s / S) - 1) & 1, kSiteW4Empty)) break;
                const int64_t r = row0 + (int64_t)s * kRowsPerStage;
                const int live = static_cast<int>(min64(kRowsPerStage, row1 - r));
                uint8_t* dst = stages + (size_t)buf * stage_bytes;
                mbar_arrive_expect_tx(&full[buf], static_cast<uint32_t>(live * (row_bytes + G * 4)));
                bulk_copy_g2s(dst, a.w + r * row_bytes, static_cast<uint32_t>(live * row_bytes), &full[buf],
                              policy);
                bulk_copy_g2s(dst + w_bytes, a.ws + r * G, static_cast<uint32_t>(live * G * 4), &full[buf],
                              policy);
            }
        }
        return;
    }

    if (warp == kWalker) {
        // Each row's groups in order: result = fma(partial, scale, result).
        float bias_r = 0.0f;
        for (int s = 0; s < nblocks; ++s) {
            const int pb = s & 1;
            const int64_t r0 = row0 + (int64_t)s * kRowsPerStage;
            const int live = static_cast<int>(min64(kRowsPerStage, row1 - r0));
            if (lane < live) bias_r = a.bias ? __ldg(a.bias + r0 + lane) : 0.0f;
            bar_sync(kBarReady + pb, kParties);
            if (!*abort_flag && lane < live) {
                const float* pr = P + (pb * kRowsPerStage + lane) * pstride;
                const float* sr = SC + (pb * kRowsPerStage + lane) * pstride;
                // Loads run 16 groups ahead of the dependent FMAs.
                float result = 0.0f;
#pragma unroll 16
                for (int k = 0; k < G; ++k) result = __fmaf_rn(pr[k], sr[k], result);
                a.y[r0 + lane] = __fadd_rn(result, bias_r);
            }
            bar_arrive(kBarFree + pb, kParties);
        }
        return;
    }

    // ---------------------------------------------------------- compute warps
    grid_dependency_wait();
    const int tid = threadIdx.x;
    const int slots = kCompute32 / G;  // >= 1
    const int g = tid % G;
    const int slot = tid / G;
    const bool active = slot < slots;
    unsigned long long x2[16];  // x[32 g + 2i], x[32 g + 2i + 1]
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = active ? __ldg(reinterpret_cast<const float4*>(a.x + (int64_t)g * 32) + i)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        x2[2 * i] = pack2(v.x, v.y);
        x2[2 * i + 1] = pack2(v.z, v.w);
    }
    const unsigned long long bias2 = pack2(8388616.0f, 8388616.0f);  // 2^23 + 8
    const unsigned long long zero2 = pack2(0.0f, 0.0f);
    for (int s = 0; s < nblocks; ++s) {
        const int buf = s % S;
        const int pb = s & 1;
        const int64_t r0 = row0 + (int64_t)s * kRowsPerStage;
        const int live = static_cast<int>(min64(kRowsPerStage, row1 - r0));
        const bool landed = mbar_wait(&full[buf], (s / S) & 1, kSiteW4Full);
        if (!landed) *abort_flag = 1;
        if (s >= 2) bar_sync(kBarFree + pb, kParties);  // the walker is done with buffer pb
        const uint8_t* sw = stages + (size_t)buf * stage_bytes;
        const float* sscale = reinterpret_cast<const float*>(sw + w_bytes);
        if (landed && active) {
            for (int r = slot; r < live; r += slots) {
                const uint4 v = *reinterpret_cast<const uint4*>(sw + (size_t)r * row_bytes + (size_t)g * 16);
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
                unsigned long long L[4];  // (lanes[2i], lanes[2i+1])
                unsigned long long acc[4][4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    // word j = columns 8j..8j+7: column 8j+2i is the low nibble of
                    // byte i, column 8j+2i+1 its high nibble.
                    const uint32_t even = (words[j] & 0x0f0f0f0fu) ^ 0x08080808u;
                    const uint32_t odd = ((words[j] >> 4) & 0x0f0f0f0fu) ^ 0x08080808u;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t lo = __byte_perm(even, 0x4B000000u, 0x7540u | i);
                        const uint32_t hi = __byte_perm(odd, 0x4B000000u, 0x7540u | i);
                        const unsigned long long w = sub2(pack2(__uint_as_float(lo), __uint_as_float(hi)), bias2);
                        acc[j][i] = fma2(w, x2[4 * j + i], zero2);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) L[i] = add2(add2(acc[0][i], acc[1][i]), add2(acc[2][i], acc[3][i]));
                const unsigned long long h01 = add2(L[0], L[2]);  // (h0, h1)
                const unsigned long long h23 = add2(L[1], L[3]);  // (h2, h3)
                const unsigned long long q = add2(h01, h23);      // (h0 + h2, h1 + h3)
                const float2 qq = unpack2(q);
                P[(pb * kRowsPerStage + r) * pstride + g] = __fadd_rn(qq.x, qq.y);
                SC[(pb * kRowsPerStage + r) * pstride + g] = sscale[r * G + g];
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
        bar_arrive(kBarReady + pb, kParties);
    }
}

template <int GS>
int launch_gs(cudaStream_t s, const W4Args& args, int grid, size_t smem, bool pdl) {
    const void* fn = reinterpret_cast<const void*>(gemv_w4a32_kernel<GS>);
    int st = allow_smem(fn, smem, "gemv_w4a32");
    if (st) return st;
    return launch(gemv_w4a32_kernel<GS>, dim3(grid), dim3(kThreads), smem, s, pdl, "gemv_w4a32",
                  args);
}

}  // namespace

bool gemv_w4a32_fast_supported(int64_t tokens, int64_t cols, int bits, int64_t group,
                               const void* weight, const float* wscales) {
    if (tokens != 1 || bits != 4) return false;
    if (group != 32 && group != 64 && group != 128) return false;
    if (cols % group != 0 || cols % 32 != 0) return false;
    const int64_t groups = cols / group;
    if (groups > kConsumers || groups % 4 != 0) return false;  // also covers the 32-column kernel (512 threads)
    return aligned16(weight) && aligned16(wscales);
}

int launch_gemv_w4a32_fast(cudaStream_t s, const float* x, int64_t cols, const uint8_t* weight,
                           const float* wscales, int64_t rows, int64_t group, const float* bias,
                           float* y, bool pdl) {
    if (rows == 0) return LEAFQ_OK;
    if (!aligned16(x)) return LEAFQ_ERR_UNSUPPORTED;
    W4Args a;
    a.x = x;
    a.w = weight;
    a.ws = wscales;
    a.bias = bias;
    a.y = y;
    a.cols = cols;
    a.rows = rows;
    a.groups = static_cast<int>(cols / group);
    const int64_t blocks_needed = (rows + kRowsPerStage - 1) / kRowsPerStage;
    const int grid = static_cast<int>(std::min<int64_t>(sm_count(), blocks_needed));
    const size_t stage_bytes = (size_t)kRowsPerStage * (cols / 2 + a.groups * 4);
    const size_t fixed = (size_t)2 * kRowsPerStage * (a.groups + 1) * 4;
    const int64_t max_rows = (rows + grid - 1) / grid;
    const int64_t max_stages = (max_rows + kRowsPerStage - 1) / kRowsPerStage;
    const int budget = std::min(max_smem_per_block(), kSmemBudget);
    const int64_t fit = (static_cast<int64_t>(budget) - static_cast<int64_t>(fixed)) /
                        static_cast<int64_t>(stage_bytes + 16);
    if (fit < 1) return LEAFQ_ERR_UNSUPPORTED;
    a.stages = static_cast<int>(std::min<int64_t>(fit, max_stages));
    if (group == 32) {
        // Two partial buffers for the walker.
        const size_t fixed32 = 2 * fixed;
        const int64_t fit32 = (static_cast<int64_t>(budget) - static_cast<int64_t>(fixed32)) /
                              static_cast<int64_t>(stage_bytes + 16);
        if (fit32 >= 2) {
            W4Args b = a;
            b.stages = static_cast<int>(std::min<int64_t>(fit32, max_stages));
            const size_t smem32 = stage_bytes * b.stages + fixed32 + 16 * b.stages + 16;
            const void* fn = reinterpret_cast<const void*>(gemv_w4a32_g32_kernel);
            int st = allow_smem(fn, smem32, "gemv_w4a32_g32");
            if (st) return st;
            return launch(gemv_w4a32_g32_kernel, dim3(grid), dim3(kThreads32), smem32, s, pdl, "gemv_w4a32_g32", b);
        }
    }
    const size_t smem = stage_bytes * a.stages + fixed + 16 * a.stages + 16;  // + abort flag
    switch (group) {
        case 32: return launch_gs<32>(s, a, grid, smem, pdl);
        case 64: return launch_gs<64>(s, a, grid, smem, pdl);
        default: return launch_gs<128>(s, a, grid, smem, pdl);
    }
}

}  // namespace leafq
