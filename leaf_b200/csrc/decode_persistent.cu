// Persistent W8A8 decode kernel: every per-row INT8 linear of one decode
// step in a single cooperative launch.
//
// A decode step is a chain of linears (q|k|v -> o -> gate|up -> down -> ...
// -> lm_head, decoder.cpp:1321-1441), each reading the previous one's full
// output.  One kernel per linear pays a launch, a ramp, a tail and a
// grid-completion flush per linear (>= 1.75 us each on B200 even for an empty
// kernel); this kernel pays them once per step.
//
// One block per SM (cooperative launch: all blocks co-resident).  Block b owns
// rows [b*N/G, (b+1)*N/G) of every linear.
//   warp 16 (producer): walks the linears in order and streams the block's
//     rows into a 192 KB shared-memory byte ring.  A stage is a row block of
//     up to 8 full rows -- contiguous in the weight, so one bulk copy of up to
//     64 KB (large copies matter: a 16 KB-copy ring streams at 97 % of the
//     measured HBM bandwidth, 2 KB copies at 59 %).  Stages are placed back to
//     back and wrap at the end of the ring; the producer reuses bytes once it
//     has seen the stages holding them released, in order.  It never waits on
//     activations, so the HBM stream continues across linears.
//   warps 0-15 (consumers, two groups of eight taking alternate row blocks,
//     one row per warp), per linear: fetch the rows' scales / bias, read x,
//     quantise it exactly as decoder.cpp:1028-1038 (every block derives the
//     identical scale), consume the stages with dp4a and write each row with
//     the reference epilogue y = fma(float(acc) * sx, sw, 0.0f) + (bias or 0).
//     Consumers recompute the same stage placement as the producer.
//
// Hand-off between linears is flag-in-data: a linear whose output feeds a
// later one writes each value as one 64-bit word {fp32 bits, launch tag}
// (single-copy atomic), and readers spin on the words themselves until every
// tag matches.  No fence, counter or grid barrier sits on the chain: the
// first reader sees a row one L2 round trip after its writer stored it.  The
// tag is a per-plan launch epoch; the last block to finish advances it.
// A linear's buffer is written once per launch, and a block can only write
// linear j+1 after reading all of linear j, so no buffer is overwritten while
// a reader still needs it.
//
// Every wait is bounded (2 s).  A wait that gives up records the site in the
// device error word and raises a block-wide abort flag; threads keep
// arriving at every block barrier and the block returns together after it
// (a thread that left early would strand the others at the barrier).
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumerWarps = 16;
constexpr int kRowsPerStage = 8;  // = warps per consumer group
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kRingBytes = 192 * 1024;
constexpr int kStageBarriers = 16;  // stages in flight at most
constexpr int kMaxCols = 8192;      // codes buffer (one token); a stage is <= 64 KB
constexpr int kMaxOps = 160;        // op table kept in shared memory
constexpr int kXVec = kMaxCols / 4 / (kConsumerWarps * 32);  // float4 of x per thread

struct Op {
    const float* x_plain;  // input ready at launch (wait < 0)
    const uint64_t* x_ll;  // input as tagged words (wait >= 0)
    uint64_t* y_ll;        // tagged output for later linears, or null
    float* y_plain;        // plain fp32 output for the caller, or null
    const int8_t* w;
    const float* ws;
    const float* bias;
    int64_t rows;
    int64_t cols;
    int32_t wait;
    int32_t pad;
};
static_assert(sizeof(Op) == 80, "op layout");

constexpr size_t kSmemBytes = (size_t)kRingBytes + kMaxCols + kMaxOps * sizeof(Op) +
                              2 * kStageBarriers * 8 + 256;

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ void load_tagged2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ void store_tagged(uint64_t* p, float v, uint32_t tag) {
    const uint64_t word = (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(word) : "memory");
}

__device__ __forceinline__ int8_t to_code(float v, float multiplier) {
    int r = __float2int_rn(__fmul_rn(v, multiplier));
    r = r > 127 ? 127 : (r < -128 ? -128 : r);
    return static_cast<int8_t>(r);
}

struct OpGeometry {
    int64_t row0, row1;
    int nblocks;
};

__device__ __forceinline__ OpGeometry geometry(const Op& op) {
    OpGeometry g;
    g.row0 = (int64_t)blockIdx.x * op.rows / gridDim.x;
    g.row1 = (int64_t)(blockIdx.x + 1) * op.rows / gridDim.x;
    g.nblocks = static_cast<int>((g.row1 - g.row0 + kRowsPerStage - 1) / kRowsPerStage);
    return g;
}

// Scale and bias of row block (group + 2 * lane), row wi, of `op` for this
// warp (zero when the lane has no such row or the op has over 64 blocks, in
// which case the epilogue reads them directly).
__device__ __forceinline__ void load_row_params(const Op& op, const OpGeometry& g, int group, int wi,
                                                int lane, float& scale, float& bias) {
    scale = 0.0f;
    bias = 0.0f;
    if (g.nblocks <= 2 * 32 && group + 2 * lane < g.nblocks) {
        const int64_t r = g.row0 + (int64_t)(group + 2 * lane) * kRowsPerStage + wi;
        if (r < g.row1) {
            scale = __ldg(op.ws + r);
            bias = op.bias ? __ldg(op.bias + r) : 0.0f;
        }
    }
}

__device__ __forceinline__ int block_rows(const OpGeometry& g, int rb) {
    return static_cast<int>(min64(kRowsPerStage, g.row1 - g.row0 - (int64_t)rb * kRowsPerStage));
}

// Stage placement in the byte ring.  `head` counts bytes ever placed
// (including wrap padding), `off` is head modulo the ring size, kept
// separately so no division is needed.  place() puts a stage of `bytes` at
// `off`, first moving to the start of the next lap when it would straddle
// the end, and returns its offset.  Producer and consumers call it on the
// same sequence of stages and so agree on every offset.
struct RingCursor {
    uint64_t head = 0;
    uint32_t off = 0;
    __device__ __forceinline__ uint32_t place(uint32_t bytes) {
        if (off + bytes > kRingBytes) {
            head += kRingBytes - off;
            off = 0;
        }
        const uint32_t start = off;
        head += bytes;
        off += bytes;
        return start;
    }
};

__global__ void __launch_bounds__(kThreads, 1)
decode_persistent_kernel(const Op* __restrict__ ops_global, int nops, uint32_t* __restrict__ sync) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    int8_t* codes = reinterpret_cast<int8_t*>(smem + kRingBytes);
    Op* ops = reinterpret_cast<Op*>(codes + kMaxCols);
    uint64_t* full = reinterpret_cast<uint64_t*>(ops + kMaxOps);
    uint64_t* empty = full + kStageBarriers;
    uint64_t* stage_end = empty + kStageBarriers;  // producer: ring head after each in-flight stage
    float* partial_max = reinterpret_cast<float*>(stage_end + kStageBarriers);  // [kConsumerWarps]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(partial_max + kConsumerWarps);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tid = threadIdx.x;

    // Op table into shared memory (all threads), barriers (thread 0).
    {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(ops_global);
        uint32_t* dst = reinterpret_cast<uint32_t*>(ops);
        const int words = nops * static_cast<int>(sizeof(Op) / 4);
        for (int i = tid; i < words; i += kThreads) dst[i] = __ldg(src + i);
    }
    if (tid == 0) {
        for (int b = 0; b < kStageBarriers; ++b) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], kRowsPerStage);  // the eight warps of one group
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    const uint32_t tag = *reinterpret_cast<volatile uint32_t*>(sync);  // this launch's epoch
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            RingCursor cursor;
            uint64_t released = 0;  // ring head after the last released stage
            int s = 0, rel = 0;
            bool go = true;
            for (int j = 0; j < nops && go; ++j) {
                const Op& op = ops[j];
                const OpGeometry g = geometry(op);
                for (int rb = 0; rb < g.nblocks; ++rb, ++s) {
                    const uint32_t bytes = static_cast<uint32_t>(block_rows(g, rb) * op.cols);
                    const uint32_t start = cursor.place(bytes);
                    // Wait until the bytes and the stage's barrier pair are free.
                    while (cursor.head - released > kRingBytes || s - rel >= kStageBarriers) {
                        const int b = rel % kStageBarriers;
                        if (!mbar_wait(&empty[b], (rel / kStageBarriers) & 1, kSiteDecodeEmpty)) {
                            go = false;
                            break;
                        }
                        released = stage_end[b];
                        ++rel;
                    }
                    if (!go) break;
                    const int b = s % kStageBarriers;
                    stage_end[b] = cursor.head;
                    mbar_arrive_expect_tx(&full[b], bytes);
                    bulk_copy_g2s(ring + start, op.w + (g.row0 + (int64_t)rb * kRowsPerStage) * op.cols,
                                  bytes, &full[b], policy);
                }
            }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    // Two groups of eight warps take alternate row blocks, so two stages
    // are consumed at once; warp wi of a group owns row wi of its stages.
    const int nthreads = kConsumerWarps * 32;
    const int group = warp / kRowsPerStage;
    const int wi = warp % kRowsPerStage;
    int s = 0;
    RingCursor cursor;
    bool ok = true;
    int prefetched_j = -1;
    float next_scale = 0.0f, next_bias = 0.0f;
    for (int j = 0; j < nops; ++j) {
        const Op& op = ops[j];
        const OpGeometry g = geometry(op);
        if (g.nblocks == 0) continue;  // no rows here: nothing to read or write
        // Row scale / bias of this warp's k-th row block (group + 2k) in lane
        // k, loaded one linear ahead so the epilogue never waits for them.
        const bool rows_in_regs = g.nblocks <= 2 * 32;
        float row_scale, row_bias;
        if (prefetched_j == j) {
            row_scale = next_scale;
            row_bias = next_bias;
        } else {
            load_row_params(op, g, group, wi, lane, row_scale, row_bias);
        }
        for (int j2 = j + 1; j2 < nops; ++j2) {
            const OpGeometry g2 = geometry(ops[j2]);
            if (g2.nblocks == 0) continue;
            load_row_params(ops[j2], g2, group, wi, lane, next_scale, next_bias);
            prefetched_j = j2;
            break;
        }
        // x into registers: plain fp32, or tagged words (spin until tagged).
        const int64_t vecs = op.cols / 4;
        float4 xr[kXVec];
        float m = 0.0f;
#pragma unroll
        for (int k = 0; k < kXVec; ++k) {
            const int64_t i = tid + (int64_t)k * nthreads;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < vecs) {
                if (op.wait < 0) {
                    v = __ldcg(reinterpret_cast<const float4*>(op.x_plain) + i);
                } else if (ok) {
                    const uint64_t* p = op.x_ll + 4 * i;
                    uint64_t a, b, c, d;
                    load_tagged2(p, a, b);
                    load_tagged2(p + 2, c, d);
                    if ((uint32_t)(a >> 32) != tag || (uint32_t)(b >> 32) != tag ||
                        (uint32_t)(c >> 32) != tag || (uint32_t)(d >> 32) != tag) {
                        const unsigned long long start = global_timer_ns();
                        for (uint32_t spins = 1;; ++spins) {
                            load_tagged2(p, a, b);
                            load_tagged2(p + 2, c, d);
                            if ((uint32_t)(a >> 32) == tag && (uint32_t)(b >> 32) == tag &&
                                (uint32_t)(c >> 32) == tag && (uint32_t)(d >> 32) == tag)
                                break;
                            if ((spins & 31u) == 0u &&
                                (device_error_raised() || global_timer_ns() - start > wait_limit_ns())) {
                                record_device_error(kSiteDecodeDependency);
                                ok = false;
                                *abort_flag = 1;
                                break;
                            }
                        }
                    }
                    v = make_float4(__uint_as_float((uint32_t)a), __uint_as_float((uint32_t)b),
                                    __uint_as_float((uint32_t)c), __uint_as_float((uint32_t)d));
                }
            }
            xr[k] = v;
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) partial_max[warp] = m;
        consumer_sync();  // also: every warp has finished the previous linear
        if (*abort_flag) return;
        float absmax = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) absmax = fmaxf(absmax, partial_max[w]);
        const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
        const float mul = __fdiv_rn(1.0f, scale);
        char4* out4 = reinterpret_cast<char4*>(codes);
#pragma unroll
        for (int k = 0; k < kXVec; ++k) {
            const int64_t i = tid + (int64_t)k * nthreads;
            if (i < vecs)
                out4[i] = make_char4(to_code(xr[k].x, mul), to_code(xr[k].y, mul), to_code(xr[k].z, mul),
                                     to_code(xr[k].w, mul));
        }
        consumer_sync();
        // Consume this linear's stages.  Every warp walks all row blocks to
        // keep the ring placement in step and takes its group's (alternate)
        // row blocks, one row per warp.
        const int cols = static_cast<int>(op.cols);
        for (int rb = 0; rb < g.nblocks; ++rb) {
            const int live_rows = block_rows(g, rb);
            const uint32_t start = cursor.place(static_cast<uint32_t>(live_rows * cols));
            if ((rb & 1) != group) continue;
            const int st = s + rb;
            const int b = st % kStageBarriers;
            if (ok && !mbar_wait(&full[b], (st / kStageBarriers) & 1, kSiteDecodeFull)) {
                ok = false;
                *abort_flag = 1;
            }
            const bool live = wi < live_rows;
            int acc = 0, acc2 = 0;  // two chains; int32 sums are exact in any order
            if (ok && live) {
                const uint8_t* wrow = ring + start + (size_t)wi * cols;
#pragma unroll 4
                for (int off = lane * 16; off < cols; off += 512) {
                    const int4 wv = *reinterpret_cast<const int4*>(wrow + off);
                    const int4 qv = *reinterpret_cast<const int4*>(codes + off);
                    acc = dp4a(wv.x, qv.x, acc);
                    acc2 = dp4a(wv.y, qv.y, acc2);
                    acc = dp4a(wv.z, qv.z, acc);
                    acc2 = dp4a(wv.w, qv.w, acc2);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[b]);
            acc += acc2;
            const float sw_rb = __shfl_sync(0xffffffffu, row_scale, (rb >> 1) & 31);
            const float bias_rb = __shfl_sync(0xffffffffu, row_bias, (rb >> 1) & 31);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (ok && live && lane == 0) {
                const int64_t row = g.row0 + (int64_t)rb * kRowsPerStage + wi;
                const float sw = rows_in_regs ? sw_rb : __ldg(op.ws + row);
                const float bias = rows_in_regs ? bias_rb : (op.bias ? __ldg(op.bias + row) : 0.0f);
                const float product = __fmul_rn(__int2float_rn(acc), scale);
                const float y = __fadd_rn(__fmaf_rn(product, sw, 0.0f), bias);
                if (op.y_ll) store_tagged(op.y_ll + row, y, tag);
                if (op.y_plain) op.y_plain[row] = y;
            }
        }
        s += g.nblocks;
    }
    // Last block out advances the epoch for the next launch.
    consumer_sync();
    if (tid == 0 && ok && !*abort_flag) {
        __threadfence();
        const uint32_t done = atomicAdd(sync + 1, 1u);
        if (done == gridDim.x - 1) {
            sync[1] = 0;
            sync[0] = tag + 1 == 0 ? 1 : tag + 1;
        }
    }
}

struct Plan {
    Op* ops_device = nullptr;
    uint32_t* sync = nullptr;        // [0] epoch (tag of the next launch), [1] blocks done
    uint64_t* buffers = nullptr;     // tagged outputs of linears that feed later ones
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
    if (nops > kMaxOps) {
        set_error("leafq_decode_plan_create: at most " + std::to_string(kMaxOps) + " ops per plan");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    std::vector<char> feeds(nops, 0);
    for (int j = 0; j < nops; ++j) {
        const leafq_decode_op& o = ops[j];
        const std::string at = " (op " + std::to_string(j) + ")";
        if (!o.weight || !o.weight_scales || o.rows <= 0 || o.cols <= 0) {
            set_error("leafq_decode_plan_create: null weight or empty shape" + at);
            return LEAFQ_ERR_INVALID;
        }
        if (o.cols % 16 != 0 || o.cols > kMaxCols || !aligned16(o.weight)) {
            set_error("leafq_decode_plan_create: cols must be a multiple of 16 and <= 8192 and the "
                      "weight 16-byte aligned" + at);
            return LEAFQ_ERR_UNSUPPORTED;
        }
        if (o.wait >= j || o.wait < -1) {
            set_error("leafq_decode_plan_create: an op may only read an earlier op's output" + at);
            return LEAFQ_ERR_INVALID;
        }
        if (o.wait < 0) {
            if (!o.x || !aligned16(o.x)) {
                set_error("leafq_decode_plan_create: an op without `wait` needs a 16-byte aligned x" + at);
                return LEAFQ_ERR_INVALID;
            }
        } else {
            if (o.x_offset < 0 || o.x_offset % 4 != 0 || o.x_offset + o.cols > ops[o.wait].rows) {
                set_error("leafq_decode_plan_create: x_offset must be a multiple of 4 and x must lie "
                          "inside the producing op's output" + at);
                return LEAFQ_ERR_INVALID;
            }
            feeds[o.wait] = 1;
        }
    }
    // Tagged buffers for every output another op reads.
    std::vector<size_t> offset(nops, 0);
    size_t words = 0;
    for (int j = 0; j < nops; ++j)
        if (feeds[j]) {
            offset[j] = words;
            words += static_cast<size_t>((ops[j].rows + 1) / 2 * 2);
        }
    auto* handle = new leafq_decode_plan_t();
    Plan& p = handle->plan;
    cudaGetDevice(&p.device);
    p.nops = nops;
    cudaError_t err = cudaMalloc(&p.ops_device, sizeof(Op) * nops);
    if (err == cudaSuccess) err = cudaMalloc(&p.sync, 2 * sizeof(uint32_t));
    if (err == cudaSuccess && words) err = cudaMalloc(&p.buffers, words * sizeof(uint64_t));
    if (err == cudaSuccess && words) err = cudaMemset(p.buffers, 0, words * sizeof(uint64_t));
    const uint32_t sync_init[2] = {1u, 0u};  // tags start at 1; zeroed words never match
    if (err == cudaSuccess) err = cudaMemcpy(p.sync, sync_init, sizeof(sync_init), cudaMemcpyHostToDevice);
    if (err == cudaSuccess) {
        std::vector<Op> host(nops);
        for (int j = 0; j < nops; ++j) {
            const leafq_decode_op& o = ops[j];
            Op& d = host[j];
            d.x_plain = o.wait < 0 ? o.x : nullptr;
            d.x_ll = o.wait >= 0 ? p.buffers + offset[o.wait] + o.x_offset : nullptr;
            d.y_ll = feeds[j] ? p.buffers + offset[j] : nullptr;
            d.y_plain = o.y;
            d.w = static_cast<const int8_t*>(o.weight);
            d.ws = o.weight_scales;
            d.bias = o.bias;
            d.rows = o.rows;
            d.cols = o.cols;
            d.wait = o.wait;
            d.pad = 0;
        }
        err = cudaMemcpy(p.ops_device, host.data(), sizeof(Op) * nops, cudaMemcpyHostToDevice);
    }
    if (err != cudaSuccess) {
        cudaFree(p.ops_device);
        cudaFree(p.sync);
        cudaFree(p.buffers);
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
    int st = allow_smem(reinterpret_cast<const void*>(decode_persistent_kernel), kSmemBytes,
                        "decode_persistent");
    if (st) return st;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(sm_count());
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = kSmemBytes;
    config.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeCooperative;
    attribute[0].val.cooperative = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, decode_persistent_kernel,
                                               static_cast<const Op*>(plan->plan.ops_device),
                                               plan->plan.nops, plan->plan.sync);
    return cuda_status(err, "leafq_decode_plan_run");
}

int leafq_decode_plan_destroy(leafq_decode_plan_t* plan) {
    clear_error();
    if (!plan) return LEAFQ_OK;
    cudaFree(plan->plan.ops_device);
    cudaFree(plan->plan.sync);
    cudaFree(plan->plan.buffers);
    delete plan;
    return LEAFQ_OK;
}

}  // extern "C"
