// W8A8 decode GEMV with fused per-token activation quantisation.
//
// Replaces the decode branch of Decoder::Impl::linear (decoder.cpp:1020-1044
// quantisation, :1221-1231 with quant_dot_avx :536-570) for per-row INT8
// weights (group == cols, the default export) and 1..8 tokens.
//
// Layout of one block (one per SM, ~200 KB of shared memory):
//   warp 8 (producer): streams this block's contiguous slice of weight rows
//     into a ring of stages with 1-D bulk copies (cp.async.bulk, TMA engine,
//     evict-first L2 policy).  A stage holds one chunk (<= 4 KB) of 8 rows.
//     Weight loads are issued before the kernel waits on the previous grid
//     (programmatic dependent launch), so the stream starts while the
//     producer of x is still finishing.
//   warps 0-7 (consumers): wait for x, compute each token's absmax and
//     scale redundantly per block (x is a few KB, L2-resident), write int8
//     codes to shared memory, then each warp takes one row of every stage:
//     lanes read 16 weight bytes and 16 code bytes per step and accumulate
//     with dp4a.  int32 sums are exact in any order; a warp reduction gives
//     the row sum and lane t finishes token t:
//       y = fma(float(acc) * sx, sw, 0.0f) + (bias or 0.0f)
//     which is the reference's result[t] += float(acc) * sx * sw (fused by
//     GCC into one FMA, decoder.cpp:567) followed by + bias (:1229).
// Bytes per call: rows * cols (weights) + 4 * rows (scales) [+ 4 * rows bias]
//   + 4 * tokens * (cols + rows): HBM-bound.
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kRowsPerStage = kConsumerWarps;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kChunkMax = 4096;
// About half an SM's shared memory, so that under programmatic dependent
// launch the next GEMV's block fits beside this one and starts its weight
// stream before this one ends.  96 KB in flight per SM is still well above
// what the HBM latency-bandwidth product needs (~40 KB per SM).
constexpr int kSmemBudget = 100 * 1024;
constexpr int kCodeBytesMax = 64 * 1024;

struct GemvArgs {
    const float* x;
    const int8_t* w;
    const float* ws;
    const float* bias;
    float* y;
    int64_t cols;
    int64_t rows;
    int tokens;
    int chunk;    // bytes of a row per stage (multiple of 16)
    int nchunks;  // ceil(cols / chunk)
    int stages;   // ring depth
    int qstride;  // bytes between token rows of the code buffer
    PeerStore peer;  // fused all-gather epilogue when peer.world > 0
};

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ int8_t to_code(float v, float multiplier) {
    int r = __float2int_rn(__fmul_rn(v, multiplier));
    r = r > 127 ? 127 : (r < -128 ? -128 : r);
    return static_cast<int8_t>(r);
}

template <int MAXT>
__global__ void __launch_bounds__(kThreads, 1) gemv_w8a8_kernel(const GemvArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int S = a.stages;
    const int chunk = a.chunk;
    uint8_t* stage_base = smem;
    int8_t* codes = reinterpret_cast<int8_t*>(smem + (size_t)S * kRowsPerStage * chunk);
    float* token_scale = reinterpret_cast<float*>(codes + MAXT * a.qstride);
    uint64_t* full = reinterpret_cast<uint64_t*>(token_scale + 8);
    uint64_t* empty = full + S;
    float* partial_max = reinterpret_cast<float*>(empty + S);  // [kConsumerWarps][MAXT]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row0 = (int64_t)blockIdx.x * a.rows / gridDim.x;
    const int64_t row1 = (int64_t)(blockIdx.x + 1) * a.rows / gridDim.x;
    const int nblocks = static_cast<int>((row1 - row0 + kRowsPerStage - 1) / kRowsPerStage);
    const int total = nblocks * a.nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    grid_launch_dependents();

    if (warp == kConsumerWarps) {
        // ---------------------------------------------------- producer
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            for (int s = 0; s < total; ++s) {
                const int buf = s % S;
                if (s >= S && !mbar_wait(&empty[buf], ((s / S) - 1) & 1, kSiteGemvEmpty)) break;
                const int rb = s / a.nchunks, c = s % a.nchunks;
                const int64_t r = row0 + (int64_t)rb * kRowsPerStage;
                const int live = static_cast<int>(min64(kRowsPerStage, row1 - r));
                const int64_t cbeg = (int64_t)c * chunk;
                const int cb = static_cast<int>(min64(chunk, a.cols - cbeg));
                mbar_arrive_expect_tx(&full[buf], static_cast<uint32_t>(live * cb));
                uint8_t* dst = stage_base + (size_t)buf * kRowsPerStage * chunk;
                for (int i = 0; i < live; ++i)
                    bulk_copy_g2s(dst + (size_t)i * chunk, a.w + (r + i) * a.cols + cbeg,
                                  static_cast<uint32_t>(cb), &full[buf], policy);
            }
        }
        return;
    }

    // -------------------------------------------------------- consumers
    const int tid = threadIdx.x;
    const int nthreads = kConsumerWarps * 32;
    // Weight scales and bias are read-only: fetch this warp's rows (row
    // row0 + 8 * rb + warp sits in lane rb) before waiting for x.
    float row_scale = 0.0f, row_bias = 0.0f;
    const bool rows_in_regs = nblocks <= 32;
    if (rows_in_regs && lane < nblocks) {
        const int64_t r = row0 + (int64_t)lane * kRowsPerStage + warp;
        if (r < row1) {
            row_scale = __ldg(a.ws + r);
            row_bias = a.bias ? __ldg(a.bias + r) : 0.0f;
        }
    }
    grid_dependency_wait();
    // The run tag of a fused all-gather (written by the previous collect).
    const uint32_t tag = a.peer.world ? *reinterpret_cast<const volatile uint32_t*>(a.peer.epoch) : 0u;
    // Per-token absmax (exact, order-free), scale and multiplier.  With one
    // or two tokens and cols <= 8192, x stays in registers between the
    // absmax pass and the coding pass (one read of x instead of two).
    constexpr int kXRegs = MAXT <= 2 ? 8 : 1;
    const int64_t vecs = a.cols / 4;
    const bool x_in_regs = MAXT <= 2 && vecs <= (int64_t)kXRegs * nthreads;
    float4 xr[MAXT][kXRegs];
    float m[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        m[t] = 0.0f;
        if (t < a.tokens) {
            const float4* in4 = reinterpret_cast<const float4*>(a.x + t * a.cols);
            if (x_in_regs) {
#pragma unroll
                for (int j = 0; j < kXRegs; ++j) {
                    const int64_t i = tid + (int64_t)j * nthreads;
                    xr[t][j] = i < vecs ? __ldg(in4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < kXRegs; ++j) {
                    const float4 v = xr[t][j];
                    m[t] = fmaxf(m[t], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
            } else {
                for (int64_t i = tid; i < vecs; i += nthreads) {
                    const float4 v = __ldg(in4 + i);
                    m[t] = fmaxf(m[t], fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m[t] = fmaxf(m[t], __shfl_xor_sync(0xffffffffu, m[t], o));
        if (lane == 0) partial_max[warp * MAXT + t] = m[t];
    }
    consumer_sync();
    float multiplier[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        float absmax = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) absmax = fmaxf(absmax, partial_max[w * MAXT + t]);
        const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
        multiplier[t] = __fdiv_rn(1.0f, scale);
        if (tid == 0) token_scale[t] = scale;
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        if (t < a.tokens) {
            char4* out4 = reinterpret_cast<char4*>(codes + t * a.qstride);
            const float mul = multiplier[t];
            if (x_in_regs) {
#pragma unroll
                for (int j = 0; j < kXRegs; ++j) {
                    const int64_t i = tid + (int64_t)j * nthreads;
                    const float4 v = xr[t][j];
                    if (i < vecs)
                        out4[i] = make_char4(to_code(v.x, mul), to_code(v.y, mul), to_code(v.z, mul),
                                             to_code(v.w, mul));
                }
            } else {
                const float4* in4 = reinterpret_cast<const float4*>(a.x + t * a.cols);
                for (int64_t i = tid; i < vecs; i += nthreads) {
                    const float4 v = __ldg(in4 + i);
                    out4[i] = make_char4(to_code(v.x, mul), to_code(v.y, mul), to_code(v.z, mul),
                                         to_code(v.w, mul));
                }
            }
        }
    }
    consumer_sync();

    // Main loop: warp `warp` owns row (row0 + 8 * rb + warp) of every stage.
    for (int rb = 0; rb < nblocks; ++rb) {
        const int64_t row = row0 + (int64_t)rb * kRowsPerStage + warp;
        const bool live = row < row1;
        int acc[MAXT];
#pragma unroll
        for (int t = 0; t < MAXT; ++t) acc[t] = 0;
        for (int c = 0; c < a.nchunks; ++c) {
            const int s = rb * a.nchunks + c;
            const int buf = s % S;
            if (!mbar_wait(&full[buf], (s / S) & 1, kSiteGemvFull)) return;
            if (live) {
                const uint8_t* wrow = stage_base + ((size_t)buf * kRowsPerStage + warp) * chunk;
                const int64_t cbeg = (int64_t)c * chunk;
                const int cb = static_cast<int>(min64(chunk, a.cols - cbeg));
                const int8_t* crow = codes + cbeg;
#pragma unroll 4
                for (int off = lane * 16; off < cb; off += 512) {
                    const int4 wv = *reinterpret_cast<const int4*>(wrow + off);
#pragma unroll
                    for (int t = 0; t < MAXT; ++t) {
                        const int4 qv = *reinterpret_cast<const int4*>(crow + t * a.qstride + off);
                        acc[t] = dp4a(wv.x, qv.x, acc[t]);
                        acc[t] = dp4a(wv.y, qv.y, acc[t]);
                        acc[t] = dp4a(wv.z, qv.z, acc[t]);
                        acc[t] = dp4a(wv.w, qv.w, acc[t]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        }
        const float sw_rb = __shfl_sync(0xffffffffu, row_scale, rb & 31);
        const float bias_rb = __shfl_sync(0xffffffffu, row_bias, rb & 31);
        if (live) {
            int mine = 0;
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
                if (lane == t) mine = acc[t];
            }
            if (lane < a.tokens) {
                const float sw = rows_in_regs ? sw_rb : __ldg(a.ws + row);
                const float bias = rows_in_regs ? bias_rb : (a.bias ? __ldg(a.bias + row) : 0.0f);
                const float product = __fmul_rn(__int2float_rn(mine), token_scale[lane]);
                const float result = __fmaf_rn(product, sw, 0.0f);
                const float y = __fadd_rn(result, bias);
                if (a.peer.world)
                    peer_store(a.peer, tag, lane, row, y);
                else
                    a.y[(int64_t)lane * a.rows + row] = y;
            }
        }
    }
}

template <int MAXT>
int launch_t(cudaStream_t s, const GemvArgs& args, int grid, size_t smem, bool pdl) {
    const void* fn = reinterpret_cast<const void*>(gemv_w8a8_kernel<MAXT>);
    int st = allow_smem(fn, smem, "gemv_w8a8");
    if (st) return st;
    return launch(gemv_w8a8_kernel<MAXT>, dim3(grid), dim3(kThreads), smem, s, pdl,
                  "gemv_w8a8", args);
}

}  // namespace

bool gemv_w8a8_supported(int64_t tokens, int64_t cols, int bits, int64_t group,
                         const void* weight, const float* x) {
    if (bits != 8 || group != cols || tokens < 1 || tokens > 8) return false;
    if (cols % 16 != 0 || !aligned16(weight) || !aligned16(x)) return false;
    const int maxt = tokens <= 1 ? 1 : tokens <= 2 ? 2 : tokens <= 4 ? 4 : 8;
    return maxt * cols <= kCodeBytesMax;
}

int launch_gemv_w8a8(cudaStream_t s, const float* x, int64_t tokens, int64_t cols,
                     const int8_t* weight, const float* wscales, int64_t rows, const float* bias,
                     float* y, bool pdl, const PeerStore* peer) {
    if (rows == 0 || tokens == 0) return LEAFQ_OK;
    GemvArgs a;
    a.peer = {};
    if (peer) a.peer = *peer;
    a.x = x;
    a.w = weight;
    a.ws = wscales;
    a.bias = bias;
    a.y = y;
    a.cols = cols;
    a.rows = rows;
    a.tokens = static_cast<int>(tokens);
    a.nchunks = static_cast<int>((cols + kChunkMax - 1) / kChunkMax);
    a.chunk = static_cast<int>(((cols + a.nchunks - 1) / a.nchunks + 15) / 16 * 16);
    const int maxt = tokens <= 1 ? 1 : tokens <= 2 ? 2 : tokens <= 4 ? 4 : 8;
    a.qstride = static_cast<int>((cols + 15) / 16 * 16);
    const int64_t blocks_needed = (rows + kRowsPerStage - 1) / kRowsPerStage;
    const int grid = static_cast<int>(std::min<int64_t>(sm_count(), blocks_needed));
    // Stages needed by the largest block, and what fits next to the codes.
    const int64_t max_rows = (rows + grid - 1) / grid;
    const int64_t max_stages = ((max_rows + kRowsPerStage - 1) / kRowsPerStage) * a.nchunks;
    const size_t fixed = (size_t)maxt * a.qstride + 8 * sizeof(float) + kConsumerWarps * 8 * 4 + 64;
    const size_t stage_bytes = (size_t)kRowsPerStage * a.chunk;
    int budget = std::min(max_smem_per_block(), kSmemBudget);
    int64_t fit = (static_cast<int64_t>(budget) - static_cast<int64_t>(fixed)) /
                  static_cast<int64_t>(stage_bytes + 16);
    if (fit < 1) return LEAFQ_ERR_UNSUPPORTED;
    a.stages = static_cast<int>(std::min<int64_t>(fit, max_stages));
    const size_t smem = stage_bytes * a.stages + fixed + 16 * a.stages;
    switch (maxt) {
        case 1: return launch_t<1>(s, a, grid, smem, pdl);
        case 2: return launch_t<2>(s, a, grid, smem, pdl);
        case 4: return launch_t<4>(s, a, grid, smem, pdl);
        default: return launch_t<8>(s, a, grid, smem, pdl);
    }
}

}  // namespace leafq
