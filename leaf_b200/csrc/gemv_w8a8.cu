// W8A8 decode GEMV with fused per-token activation quantisation.
//
// Replaces the decode branch of Decoder::Impl::linear (decoder.cpp:1020-1044
// quantisation, :1221-1231 with quant_dot_avx :536-570) for per-row INT8
// weights (group == cols, the default export) and 1..8 tokens.
//
// Layout of one block (two per SM for a call, up to 100 KB of shared memory
// each; small slices are sized by their rows so that the next call's blocks
// fit beside them):
//   warp 8 (producer): streams this block's contiguous slice of weight rows
//     into a ring of stages with 1-D bulk copies (cp.async.bulk, TMA engine,
//     evict-first L2 policy).  A stage holds one chunk (<= 2 KB) of 16 rows.
//     Weight loads are issued before the kernel waits on the previous grid
//     (programmatic dependent launch), so the stream starts while the
//     producer of x is still finishing.
//   warps 0-7 (consumers): wait for x, compute each token's absmax and
//     scale redundantly per block (x is a few KB, L2-resident), write int8
//     codes to shared memory, then each warp takes two rows of every stage
//     side by side: lanes read 16 bytes of each row and 16 code bytes per
//     step and accumulate with dp4a.  int32 sums are exact in any order; one
//     warp reduction gives both rows' sums and lanes t / 16 + t finish token
//     t of the two rows:
//       y = fma(float(acc) * sx, sw, 0.0f) + (bias or 0.0f)
//     which is the reference's result[t] += float(acc) * sx * sw (fused by
//     GCC into one FMA, decoder.cpp:567) followed by + bias (:1229).
//   Two blocks per SM (grid 2 x SMs), so twice the warps hide the per-row
//   latency of the dot, reduction and epilogue; registers are capped so that
//   four blocks fit, two of this call and two of the next.
// Bytes per call: rows * cols (weights) + 4 * rows (scales) [+ 4 * rows bias]
//   + 4 * tokens * (cols + rows): HBM-bound.
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kRowsPerStage = 2 * kConsumerWarps;  // warp w owns rows 2w and 2w + 1 of a stage
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kChunkMax = 2048;
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
    int stage_area;  // bytes of shared memory holding the stages (the codes follow)
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

// Four blocks per SM (56 registers): under programmatic dependent launch the
// next GEMV's two blocks per SM become resident beside this one's and
// stream their weights while this one computes.
template <int MAXT>
__global__ void __launch_bounds__(kThreads, 4) gemv_w8a8_kernel(const GemvArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int S = a.stages;
    const int chunk = a.chunk;
    uint8_t* stage_base = smem;
    int8_t* codes = reinterpret_cast<int8_t*>(smem + a.stage_area);
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
    float2 row_scale = make_float2(0.0f, 0.0f), row_bias = make_float2(0.0f, 0.0f);
    const bool rows_in_regs = nblocks <= 32;
    if (rows_in_regs && lane < nblocks) {
        const int64_t r = row0 + (int64_t)lane * kRowsPerStage + 2 * warp;
        if (r < row1) {
            row_scale.x = __ldg(a.ws + r);
            row_bias.x = a.bias ? __ldg(a.bias + r) : 0.0f;
        }
        if (r + 1 < row1) {
            row_scale.y = __ldg(a.ws + r + 1);
            row_bias.y = a.bias ? __ldg(a.bias + r + 1) : 0.0f;
        }
    }
    grid_dependency_wait();
    // The run tag of a fused all-gather (written by the previous collect).
    const uint32_t tag = a.peer.world ? *reinterpret_cast<const volatile uint32_t*>(a.peer.epoch) : 0u;
    // Per-token absmax (exact, order-free), scale and multiplier.  With one
    // or two tokens and cols <= 2048, x stays in registers between the
    // absmax pass and the coding pass (one read of x instead of two).
    constexpr int kXRegs = MAXT <= 2 ? 2 : 1;
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
        m[t] = warp_max_f32(m[t]);
        if (lane == 0) partial_max[warp * MAXT + t] = m[t];
    }
    consumer_sync();
    float multiplier[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        static_assert(kConsumerWarps <= 32 && (kConsumerWarps & (kConsumerWarps - 1)) == 0, "");
        const float absmax = warp_max_f32(partial_max[(lane & (kConsumerWarps - 1)) * MAXT + t]);
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

    // Main loop: warp `warp` owns rows row0 + 16 rb + 2 warp and the next of
    // every stage, side by side (two independent chains per lane).
    for (int rb = 0; rb < nblocks; ++rb) {
        const int64_t rowa = row0 + (int64_t)rb * kRowsPerStage + 2 * warp;
        const bool live0 = rowa < row1, live1 = rowa + 1 < row1;
        int acc0[MAXT], acc1[MAXT];
#pragma unroll
        for (int t = 0; t < MAXT; ++t) acc0[t] = acc1[t] = 0;
        for (int c = 0; c < a.nchunks; ++c) {
            const int s = rb * a.nchunks + c;
            const int buf = s % S;
            if (!mbar_wait(&full[buf], (s / S) & 1, kSiteGemvFull)) return;
            if (live0) {
                const uint8_t* w0 = stage_base + ((size_t)buf * kRowsPerStage + 2 * warp) * chunk;
                const uint8_t* w1 = w0 + chunk;
                const int64_t cbeg = (int64_t)c * chunk;
                const int cb = static_cast<int>(min64(chunk, a.cols - cbeg));
                const int8_t* crow = codes + cbeg;
#pragma unroll 4
                for (int off = lane * 16; off < cb; off += 512) {
                    const int4 u = *reinterpret_cast<const int4*>(w0 + off);
                    const int4 v = live1 ? *reinterpret_cast<const int4*>(w1 + off) : make_int4(0, 0, 0, 0);
#pragma unroll
                    for (int t = 0; t < MAXT; ++t) {
                        const int4 qv = *reinterpret_cast<const int4*>(crow + t * a.qstride + off);
                        acc0[t] = dp4a(u.x, qv.x, acc0[t]);
                        acc1[t] = dp4a(v.x, qv.x, acc1[t]);
                        acc0[t] = dp4a(u.y, qv.y, acc0[t]);
                        acc1[t] = dp4a(v.y, qv.y, acc1[t]);
                        acc0[t] = dp4a(u.z, qv.z, acc0[t]);
                        acc1[t] = dp4a(v.z, qv.z, acc1[t]);
                        acc0[t] = dp4a(u.w, qv.w, acc0[t]);
                        acc1[t] = dp4a(v.w, qv.w, acc1[t]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
        }
        const float2 sw_rb = make_float2(__shfl_sync(0xffffffffu, row_scale.x, rb & 31),
                                         __shfl_sync(0xffffffffu, row_scale.y, rb & 31));
        const float2 bias_rb = make_float2(__shfl_sync(0xffffffffu, row_bias.x, rb & 31),
                                           __shfl_sync(0xffffffffu, row_bias.y, rb & 31));
        if (live0) {
            // Both rows at once (integer sums: any order): lanes 0-15 finish
            // with row 2 warp, lanes 16-31 with the next; lane t and lane
            // 16 + t then hold token t's sums.
            const bool hi = lane >= 16;
            int mine = 0;
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                int v = (hi ? acc1[t] : acc0[t]) + __shfl_xor_sync(0xffffffffu, hi ? acc0[t] : acc1[t], 16);
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if ((lane & 15) == t) mine = v;
            }
            const int tok = lane & 15;
            const int64_t row = rowa + (hi ? 1 : 0);
            if (tok < a.tokens && (hi ? live1 : true)) {
                const float sw = rows_in_regs ? (hi ? sw_rb.y : sw_rb.x) : __ldg(a.ws + row);
                const float bias = rows_in_regs ? (hi ? bias_rb.y : bias_rb.x) : (a.bias ? __ldg(a.bias + row) : 0.0f);
                const float product = __fmul_rn(__int2float_rn(mine), token_scale[tok]);
                const float result = __fmaf_rn(product, sw, 0.0f);
                const float y = __fadd_rn(result, bias);
                if (a.peer.world)
                    peer_store(a.peer, tag, tok, row, y);
                else
                    a.y[(int64_t)tok * a.rows + row] = y;
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
    // Two blocks per SM: twice the consumer warps to hide the per-row
    // latency of the dot, reduction and epilogue.
    const int grid = static_cast<int>(std::min<int64_t>(2 * sm_count(), blocks_needed));
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
    // When the whole row slice is resident (every stage its own buffer) and
    // rows are one chunk wide, the last buffer only holds the slice's last
    // rows: size the shared memory by the rows, so that four blocks fit on
    // an SM (a config-0 slice of 20 rows x 2 KB: 42 KB instead of 66 KB).
    a.stage_area = static_cast<int>(stage_bytes * a.stages);
    if (a.stages == max_stages && a.nchunks == 1) {
        const int64_t last_rows = max_rows - (int64_t)kRowsPerStage * (a.stages - 1);
        a.stage_area = static_cast<int>(stage_bytes * (a.stages - 1) + (size_t)last_rows * a.chunk);
    }
    const size_t smem = (size_t)a.stage_area + fixed + 16 * a.stages;
    switch (maxt) {
        case 1: return launch_t<1>(s, a, grid, smem, pdl);
        case 2: return launch_t<2>(s, a, grid, smem, pdl);
        case 4: return launch_t<4>(s, a, grid, smem, pdl);
        default: return launch_t<8>(s, a, grid, smem, pdl);
    }
}

}  // namespace leafq
