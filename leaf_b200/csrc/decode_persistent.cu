// Persistent W8A8 decode kernel: every per-row INT8 linear of one decode
// step in a single cooperative launch.
//
// A decode step is a chain of linears (q|k|v -> o -> gate|up -> down -> ...
// -> lm_head, decoder.cpp:1321-1441), each reading the previous one's full
// output.  Launching one kernel per linear pays a launch, a ramp and a tail
// per linear; this kernel pays them once per step.
//
// One block per SM (cooperative launch: all blocks are co-resident).  Block b
// owns rows [b*N/G, (b+1)*N/G) of every linear.
//   warp 8 (producer): walks the linears of the plan in order and streams the
//     block's rows of each into a 12 x 16 KB ring with 1-D bulk copies (one
//     copy per stage when rows are contiguous).  It never waits on
//     activations, only on ring slots, so the weight stream runs continuously
//     across linear boundaries at the HBM rate.
//   warps 0-7 (consumers), per linear: fetch this linear's row scales / bias,
//     wait until every block has published the input (a per-linear counter in
//     global memory reaching G; bounded spin), read x, quantise it exactly as
//     decoder.cpp:1028-1038 (each block derives the identical scale), consume
//     the stages with dp4a, write y with the reference epilogue
//       y = fma(float(acc) * sx, sw, 0.0f) + (bias or 0.0f)
//     and publish: block barrier, then one release add on the counter.
// Every spin is bounded (2 s); on a timeout the device error word is set and
// the block returns.
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kRowsPerStage = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kSlotBytes = 16384;
constexpr int kSlots = 12;
constexpr int kChunk = 2048;            // bytes of a row per stage when cols > 2048
constexpr int kMaxCols = 8192;          // codes buffer (one token)
constexpr size_t kSmemBytes = (size_t)kSlots * kSlotBytes + kMaxCols + 2 * kSlots * 8 + 256;

struct Op {
    const float* x;
    float* y;
    const int8_t* w;
    const float* ws;
    const float* bias;
    int64_t rows;
    int64_t cols;
    int32_t wait;
    int32_t pad;
};

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until counter >= target.  Returns false on timeout/error.
__device__ __forceinline__ bool wait_counter(const uint32_t* counter, uint32_t target) {
    if (ld_acquire(counter) >= target) return true;
    const unsigned long long start = global_timer_ns();
    for (uint32_t spins = 1;; ++spins) {
        if (ld_acquire(counter) >= target) return true;
        if ((spins & 63u) == 0u) {
            if (device_error_raised()) return false;
            if (global_timer_ns() - start > kWaitLimitNs) {
                record_device_error(kSiteDecodeDependency);
                return false;
            }
        }
    }
}

__device__ __forceinline__ int8_t to_code(float v, float multiplier) {
    int r = __float2int_rn(__fmul_rn(v, multiplier));
    r = r > 127 ? 127 : (r < -128 ? -128 : r);
    return static_cast<int8_t>(r);
}

struct OpGeometry {
    int64_t row0, row1;
    int nblocks, nchunks, stride;
};

__device__ __forceinline__ OpGeometry geometry(const Op& op) {
    OpGeometry g;
    g.row0 = (int64_t)blockIdx.x * op.rows / gridDim.x;
    g.row1 = (int64_t)(blockIdx.x + 1) * op.rows / gridDim.x;
    g.nblocks = static_cast<int>((g.row1 - g.row0 + kRowsPerStage - 1) / kRowsPerStage);
    g.nchunks = static_cast<int>((op.cols + kChunk - 1) / kChunk);
    g.stride = static_cast<int>(op.cols <= kChunk ? op.cols : kChunk);
    return g;
}

__global__ void __launch_bounds__(kThreads, 1)
decode_persistent_kernel(const Op* __restrict__ ops, int nops, uint32_t* __restrict__ counters) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    int8_t* codes = reinterpret_cast<int8_t*>(smem + (size_t)kSlots * kSlotBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(codes + kMaxCols);
    uint64_t* empty = full + kSlots;
    float* partial_max = reinterpret_cast<float*>(empty + kSlots);  // [kConsumerWarps]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(partial_max + kConsumerWarps);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t G = gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            int s = 0;
            for (int j = 0; j < nops; ++j) {
                const Op op = ops[j];
                const OpGeometry g = geometry(op);
                for (int rb = 0; rb < g.nblocks; ++rb) {
                    const int64_t r = g.row0 + (int64_t)rb * kRowsPerStage;
                    const int live = static_cast<int>(min64(kRowsPerStage, g.row1 - r));
                    for (int c = 0; c < g.nchunks; ++c, ++s) {
                        const int slot = s % kSlots;
                        if (s >= kSlots &&
                            !mbar_wait(&empty[slot], ((s / kSlots) - 1) & 1, kSiteDecodeEmpty))
                            return;
                        const int64_t cbeg = (int64_t)c * kChunk;
                        const int cb = static_cast<int>(min64(g.stride, op.cols - cbeg));
                        uint8_t* dst = ring + (size_t)slot * kSlotBytes;
                        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(live * cb));
                        if (g.nchunks == 1) {
                            // Rows of one block are contiguous: one copy.
                            bulk_copy_g2s(dst, op.w + r * op.cols, static_cast<uint32_t>(live * cb),
                                          &full[slot], policy);
                        } else {
                            for (int i = 0; i < live; ++i)
                                bulk_copy_g2s(dst + (size_t)i * g.stride, op.w + (r + i) * op.cols + cbeg,
                                              static_cast<uint32_t>(cb), &full[slot], policy);
                        }
                    }
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    const int tid = threadIdx.x;
    const int nthreads = kConsumerWarps * 32;
    int s = 0;
    for (int j = 0; j < nops; ++j) {
        const Op op = ops[j];
        const OpGeometry g = geometry(op);
        // Row scale / bias of row (row0 + 8 * rb + warp) held in lane rb.
        const bool rows_in_regs = g.nblocks <= 32;
        float row_scale = 0.0f, row_bias = 0.0f;
        if (rows_in_regs && lane < g.nblocks) {
            const int64_t r = g.row0 + (int64_t)lane * kRowsPerStage + warp;
            if (r < g.row1) {
                row_scale = __ldg(op.ws + r);
                row_bias = op.bias ? __ldg(op.bias + r) : 0.0f;
            }
        }
        if (g.nblocks > 0) {
            // Wait for the input.
            if (op.wait >= 0) {
                if (tid == 0 && !wait_counter(counters + op.wait, G)) *abort_flag = 1;
                consumer_sync();
                if (*abort_flag) return;
            }
            // Quantise x (one token): absmax, scale, codes in shared memory.
            const int64_t vecs = op.cols / 4;
            const float4* in4 = reinterpret_cast<const float4*>(op.x);
            float4 xr[kMaxCols / 4 / (kConsumerWarps * 32)];
            float m = 0.0f;
#pragma unroll
            for (int k = 0; k < kMaxCols / 4 / (kConsumerWarps * 32); ++k) {
                const int64_t i = tid + (int64_t)k * nthreads;
                xr[k] = i < vecs ? __ldcg(in4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                m = fmaxf(m, fmaxf(fmaxf(fabsf(xr[k].x), fabsf(xr[k].y)), fmaxf(fabsf(xr[k].z), fabsf(xr[k].w))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) partial_max[warp] = m;
            consumer_sync();
            float absmax = 0.0f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) absmax = fmaxf(absmax, partial_max[w]);
            const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
            const float mul = __fdiv_rn(1.0f, scale);
            char4* out4 = reinterpret_cast<char4*>(codes);
#pragma unroll
            for (int k = 0; k < kMaxCols / 4 / (kConsumerWarps * 32); ++k) {
                const int64_t i = tid + (int64_t)k * nthreads;
                if (i < vecs)
                    out4[i] = make_char4(to_code(xr[k].x, mul), to_code(xr[k].y, mul),
                                         to_code(xr[k].z, mul), to_code(xr[k].w, mul));
            }
            consumer_sync();
            // Consume this linear's stages.
            for (int rb = 0; rb < g.nblocks; ++rb) {
                const int64_t row = g.row0 + (int64_t)rb * kRowsPerStage + warp;
                const bool live = row < g.row1;
                int acc = 0;
                for (int c = 0; c < g.nchunks; ++c, ++s) {
                    const int slot = s % kSlots;
                    if (!mbar_wait(&full[slot], (s / kSlots) & 1, kSiteDecodeFull)) return;
                    if (live) {
                        const uint8_t* wrow = ring + (size_t)slot * kSlotBytes + (size_t)warp * g.stride;
                        const int64_t cbeg = (int64_t)c * kChunk;
                        const int cb = static_cast<int>(min64(g.stride, op.cols - cbeg));
                        const int8_t* crow = codes + cbeg;
#pragma unroll 4
                        for (int off = lane * 16; off < cb; off += 512) {
                            const int4 wv = *reinterpret_cast<const int4*>(wrow + off);
                            const int4 qv = *reinterpret_cast<const int4*>(crow + off);
                            acc = dp4a(wv.x, qv.x, acc);
                            acc = dp4a(wv.y, qv.y, acc);
                            acc = dp4a(wv.z, qv.z, acc);
                            acc = dp4a(wv.w, qv.w, acc);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[slot]);
                }
                const float sw_rb = __shfl_sync(0xffffffffu, row_scale, rb & 31);
                const float bias_rb = __shfl_sync(0xffffffffu, row_bias, rb & 31);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (live && lane == 0) {
                    const float sw = rows_in_regs ? sw_rb : __ldg(op.ws + row);
                    const float bias = rows_in_regs ? bias_rb : (op.bias ? __ldg(op.bias + row) : 0.0f);
                    const float product = __fmul_rn(__int2float_rn(acc), scale);
                    op.y[row] = __fadd_rn(__fmaf_rn(product, sw, 0.0f), bias);
                }
            }
        }
        // Publish this block's slice of linear j.
        consumer_sync();
        if (tid == 0) {
            __threadfence();
            red_release_add(counters + j, 1u);
        }
    }
}

struct Plan {
    Op* ops_device = nullptr;
    uint32_t* counters = nullptr;
    int nops = 0;
    int device = 0;
};

}  // namespace
}  // namespace leafq

using namespace leafq;

extern "C" {

struct leafq_decode_plan_t {
    Plan plan;
};

int leafq_decode_plan_create(const leafq_decode_op* ops, int nops, int tokens,
                             leafq_decode_plan_t** out) {
    clear_error();
    if (!out || !ops || nops <= 0) {
        set_error("leafq_decode_plan_create: need at least one op and an output handle");
        return LEAFQ_ERR_INVALID;
    }
    *out = nullptr;
    if (tokens != 1) {
        set_error("leafq_decode_plan_create: the persistent decode kernel handles one token per step");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    std::vector<Op> host(nops);
    for (int j = 0; j < nops; ++j) {
        const leafq_decode_op& o = ops[j];
        const std::string at = " (op " + std::to_string(j) + ")";
        if (!o.x || !o.y || !o.weight || !o.weight_scales || o.rows <= 0 || o.cols <= 0) {
            set_error("leafq_decode_plan_create: null pointer or empty shape" + at);
            return LEAFQ_ERR_INVALID;
        }
        if (o.cols % 16 != 0 || o.cols > kMaxCols || !aligned16(o.x) || !aligned16(o.weight)) {
            set_error("leafq_decode_plan_create: cols must be a multiple of 16 and <= 8192, x and the "
                      "weight 16-byte aligned" + at);
            return LEAFQ_ERR_UNSUPPORTED;
        }
        if (o.wait >= j || o.wait < -1) {
            set_error("leafq_decode_plan_create: an op may only wait on an earlier op" + at);
            return LEAFQ_ERR_INVALID;
        }
        host[j] = Op{o.x, o.y, static_cast<const int8_t*>(o.weight), o.weight_scales, o.bias,
                     o.rows, o.cols, o.wait, 0};
    }
    auto* handle = new leafq_decode_plan_t();
    cudaGetDevice(&handle->plan.device);
    handle->plan.nops = nops;
    cudaError_t err = cudaMalloc(&handle->plan.ops_device, sizeof(Op) * nops);
    if (err == cudaSuccess) err = cudaMalloc(&handle->plan.counters, sizeof(uint32_t) * nops);
    if (err == cudaSuccess)
        err = cudaMemcpy(handle->plan.ops_device, host.data(), sizeof(Op) * nops, cudaMemcpyHostToDevice);
    if (err != cudaSuccess) {
        cudaFree(handle->plan.ops_device);
        cudaFree(handle->plan.counters);
        delete handle;
        return cuda_status(err, "leafq_decode_plan_create");
    }
    *out = handle;
    return LEAFQ_OK;
}

int leafq_decode_plan_run(void* stream, leafq_decode_plan_t* plan) {
    clear_error();
    if (!plan) {
        set_error("leafq_decode_plan_run: null plan");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaMemsetAsync(plan->plan.counters, 0, sizeof(uint32_t) * plan->plan.nops, s);
    if (err != cudaSuccess) return cuda_status(err, "leafq_decode_plan_run: counter reset");
    int st = allow_smem(reinterpret_cast<const void*>(decode_persistent_kernel), kSmemBytes,
                        "decode_persistent");
    if (st) return st;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(sm_count());
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = kSmemBytes;
    config.stream = s;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeCooperative;
    attribute[0].val.cooperative = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    err = cudaLaunchKernelEx(&config, decode_persistent_kernel, static_cast<const Op*>(plan->plan.ops_device),
                             plan->plan.nops, plan->plan.counters);
    return cuda_status(err, "leafq_decode_plan_run");
}

int leafq_decode_plan_destroy(leafq_decode_plan_t* plan) {
    clear_error();
    if (!plan) return LEAFQ_OK;
    cudaFree(plan->plan.ops_device);
    cudaFree(plan->plan.counters);
    delete plan;
    return LEAFQ_OK;
}

}  // extern "C"
