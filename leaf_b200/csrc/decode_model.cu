// One decode step of a whole Llama-family W8A8 decoder in a single
// cooperative launch: embedding, per layer RMSNorm -> q|k|v -> RoPE, KV
// append and attention -> o + residual -> RMSNorm -> gate|up -> SiLU gate ->
// down + residual, final RMSNorm, lm_head and the greedy argmax
// (Decoder::Impl::forward_into, decoder.cpp:1282-1452, for one token, and
// the argmax of main_decoder.cpp:101).  Results are bit-identical to the
// reference: the linears are the exact integer path of decode_persistent.cu,
// the other operators keep the reference's order of every floating-point
// operation (sequential sums, libm's expf via decoder_math.cuh).
//
// Structure (one block per SM, 16 consumer warps + 1 producer warp):
// * The producer lane streams, linear after linear, the block's rows of
//   every weight into a 192 KB shared-memory byte ring with one bulk copy
//   per block of up to 8 rows; it never waits on activations, so HBM keeps
//   streaming through the non-linear operators.
// * Consumers walk the op list.  A linear's input is either a tagged vector
//   (flag-in-data words {fp32, launch tag} written by the op that produced
//   it) or RMSNorm of a tagged hidden vector (or of the embedding row, layer
//   0), which every block computes for itself -- identical in every block --
//   before quantising it.  Epilogues write tagged outputs: plain, residual
//   (h + y, the residual read from the tagged hidden vector), the SiLU gate
//   (gate and up rows are interleaved, and each consumer warp takes two
//   rows of a stage, so a row pair meets in one warp), or logits plus a
//   block-local argmax folded into one 64-bit atomicMax key.  The 16
//   consumer warps form four groups of four; group q takes the stages
//   rb % 4 == q.  RMSNorm's sum of squares runs on all consumer threads
//   (sum_in_order_par), bit-identical to the reference's sequential sum.
// * Attention for query head h runs in block h * G / heads: it reads the
//   tagged q, k, v of this token, applies RoPE from the host tables, appends
//   k, v to the layer's cache (one block per KV head), and attends over the
//   cached keys and the current one.
// * The last block to finish publishes the argmax as the next token id,
//   advances the position and the launch tag.
//
// Every wait is bounded (2 s) and reports through the device error word;
// after a wait gives up, threads keep arriving at every barrier and the
// block returns together.
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "decoder_math.cuh"
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kConsumerWarps = 16;
constexpr int kRowsPerStage = 8;  // rows per ring stage (one bulk copy)
constexpr int kGroups = 4;        // consumer warp groups: group q takes the stages rb % kGroups == q
constexpr int kGroupWarps = 4;    // warps per group, two rows of a stage each
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kNC = kConsumerWarps * 32;  // consumer threads
constexpr uint32_t kRingBytes = 192 * 1024;
// Blocks that run attention give the last 64 KB of their ring to it: with the
// codes buffer and the scratch behind it, 88 KB of keys / values / scores.
constexpr uint32_t kAttnRingBytes = 128 * 1024;
constexpr int kStageBarriers = 16;
constexpr int kMaxCols = 6144;  // widest linear input (TinyLlama's 5632); x stays in registers
constexpr int kXVec = kMaxCols / 4 / kNC;
constexpr int kScratchFloats = 4096;  // hidden row for RMSNorm; attention scores + V chunk
constexpr int kNormXVec = kScratchFloats / 4 / kNC;  // float4s of a normalised (hidden) row per thread
constexpr int kMaxCapacity = 2048;    // attention scores (first half of the scratch)
constexpr int kMaxDim = 256;
constexpr int kAttFloats = static_cast<int>((kRingBytes - kAttnRingBytes) / 4) + kMaxCols / 4 + kScratchFloats;
constexpr int kMaxOps = 1024;

enum : int32_t { kOpLinear = 0, kOpAttention = 1 };
enum : int32_t { kXTagged = 0, kXNormEmbed = 1, kXNormTagged = 2 };
enum : int32_t { kEpiTagged = 0, kEpiResidEmbed = 1, kEpiResidTagged = 2, kEpiSiluPair = 3, kEpiLogits = 4 };

struct MOp {
    int32_t kind, xsrc, epi, add_zero;
    const uint64_t* x_ll;      // kXTagged: x; kXNormTagged: the hidden vector
    const float* norm_w;       // RMSNorm weight
    uint64_t* y_ll;            // tagged output
    const uint64_t* resid_ll;  // kEpiResidTagged: the hidden vector added to y
    const int8_t* w;
    const float* ws;
    int64_t rows, cols;
    float* k_cache;            // attention: [kv][capacity][dim]
    float* v_cache;
};

struct Model {
    const int8_t* embed;
    const float* embed_scales;
    const float* cos_table;
    const float* sin_table;
    int32_t* ids;
    int32_t* position;
    int32_t* history;
    float* logits;
    uint32_t* sync;  // [0] launch tag, [1] blocks done, [2..3] argmax key
    int64_t capacity;
    float embedding_scale, epsilon, attn_scale;
    int32_t hidden, heads, kv_heads, dim, vocab;
    ExpTable tab;
};

constexpr size_t kSmemBytes = (size_t)kRingBytes + kMaxCols + kScratchFloats * 4 + 3 * kMaxDim * 4 +
                              2 * (kStageBarriers + 2) * 8 + kStageBarriers * 8 + 2 * 2 * 8 * 4 +
                              kConsumerWarps * 12 + 64 + sizeof(ExpTable) + 8 +
                              sizeof(OrderedSumScratch<kNC>) + 16;

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kNC) : "memory");
}

__device__ __forceinline__ uint64_t load_tagged(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_tagged(uint64_t* p, float v, uint32_t tag) {
    const uint64_t word = (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(word) : "memory");
}

// Spin until the word carries `tag`; false (and the error word set) after
// the wait limit or once another wait has given up.
__device__ __forceinline__ bool wait_tagged(const uint64_t* p, uint32_t tag, float& value) {
    uint64_t w = load_tagged(p);
    if (static_cast<uint32_t>(w >> 32) != tag) {
        const unsigned long long start = global_timer_ns();
        for (uint32_t spins = 1;; ++spins) {
            w = load_tagged(p);
            if (static_cast<uint32_t>(w >> 32) == tag) break;
            if ((spins & 31u) == 0u && (device_error_raised() || global_timer_ns() - start > wait_limit_ns())) {
                record_device_error(kSiteDecodeDependency);
                value = 0.0f;
                return false;
            }
        }
    }
    value = __uint_as_float(static_cast<uint32_t>(w));
    return true;
}

__device__ __forceinline__ void load_tagged2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// x[4i .. 4i+3] for this thread's kXVec float4s, as tagged words: the
// loads of two float4s are issued together, then their tags are checked (a
// float4 with a word not yet written is polled as a whole, bounded).
// Returns false if a wait gave up.
__device__ __forceinline__ bool load_tagged_x(const uint64_t* x, int64_t vecs, uint32_t tag, int tid,
                                              float4 (&xr)[kXVec]) {
    bool good = true;
#pragma unroll
    for (int k0 = 0; k0 < kXVec; k0 += 2) {
        uint64_t w[2][4];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int64_t i = tid + (int64_t)(k0 + k) * kNC;
            if (k0 + k < kXVec && i < vecs) {
                load_tagged2(x + 4 * i, w[k][0], w[k][1]);
                load_tagged2(x + 4 * i + 2, w[k][2], w[k][3]);
            } else {
                w[k][0] = w[k][1] = w[k][2] = w[k][3] = static_cast<uint64_t>(tag) << 32;
            }
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if (k0 + k >= kXVec) break;
            const int64_t i = tid + (int64_t)(k0 + k) * kNC;
            auto all_tagged = [&]() {
                return static_cast<uint32_t>(w[k][0] >> 32) == tag && static_cast<uint32_t>(w[k][1] >> 32) == tag &&
                       static_cast<uint32_t>(w[k][2] >> 32) == tag && static_cast<uint32_t>(w[k][3] >> 32) == tag;
            };
            if (i < vecs && good && !all_tagged()) {
                // Not all four written yet: poll the four words together (one
                // round trip per poll; they come from neighbouring rows, so
                // they land together), bounded.
                const unsigned long long start = global_timer_ns();
                for (uint32_t spins = 1;; ++spins) {
                    load_tagged2(x + 4 * i, w[k][0], w[k][1]);
                    load_tagged2(x + 4 * i + 2, w[k][2], w[k][3]);
                    if (all_tagged()) break;
                    if ((spins & 31u) == 0u &&
                        (device_error_raised() || global_timer_ns() - start > wait_limit_ns())) {
                        record_device_error(kSiteDecodeDependency);
                        good = false;
                        break;
                    }
                }
            }
            xr[k0 + k] = i < vecs && good
                             ? make_float4(__uint_as_float(static_cast<uint32_t>(w[k][0])),
                                           __uint_as_float(static_cast<uint32_t>(w[k][1])),
                                           __uint_as_float(static_cast<uint32_t>(w[k][2])),
                                           __uint_as_float(static_cast<uint32_t>(w[k][3])))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    return good;
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

// Rows [row0, row1) of `op` for this block; paired (SiLU) ops split whole
// row pairs so a pair never straddles blocks or stages.
__device__ __forceinline__ OpGeometry geometry(const MOp& op) {
    OpGeometry g;
    if (op.epi == kEpiSiluPair) {
        const int64_t pairs = op.rows / 2;
        g.row0 = 2 * ((int64_t)blockIdx.x * pairs / gridDim.x);
        g.row1 = 2 * ((int64_t)(blockIdx.x + 1) * pairs / gridDim.x);
    } else {
        g.row0 = (int64_t)blockIdx.x * op.rows / gridDim.x;
        g.row1 = (int64_t)(blockIdx.x + 1) * op.rows / gridDim.x;
    }
    g.nblocks = static_cast<int>((g.row1 - g.row0 + kRowsPerStage - 1) / kRowsPerStage);
    return g;
}

__device__ __forceinline__ int block_rows(const OpGeometry& g, int rb) {
    return static_cast<int>(min64(kRowsPerStage, g.row1 - g.row0 - (int64_t)rb * kRowsPerStage));
}

// Row scales (and the residual inputs, for residual epilogues) of rows
// 2 wi and 2 wi + 1 of row block (group + kGroups * lane) of `op`, in lane
// `lane` of the warp: lane k holds the values the warp needs for its k-th
// row block, so the epilogue never waits on a load.  Zero beyond
// 32 * kGroups row blocks (the epilogue then loads directly).
__device__ __forceinline__ float2 load_row_scales(const MOp& op, const OpGeometry& g, int group, int wi,
                                                  int lane) {
    float2 r = make_float2(0.0f, 0.0f);
    if (g.nblocks <= kGroups * 32 && group + kGroups * lane < g.nblocks) {
        const int64_t r0 = g.row0 + (int64_t)(group + kGroups * lane) * kRowsPerStage + 2 * wi;
        if (r0 < g.row1) r.x = __ldg(op.ws + r0);
        if (r0 + 1 < g.row1) r.y = __ldg(op.ws + r0 + 1);
    }
    return r;
}

struct RingCursor {
    uint64_t head = 0;
    uint32_t off = 0;
    uint32_t size = kRingBytes;
    __device__ __forceinline__ uint32_t place(uint32_t bytes) {
        if (off + bytes > size) {
            head += size - off;
            off = 0;
        }
        const uint32_t start = off;
        head += bytes;
        off += bytes;
        return start;
    }
};

// The query head this block attends for (-1: none).
__device__ __forceinline__ int my_head(int heads) {
    for (int h = 0; h < heads; ++h)
        if ((int64_t)h * gridDim.x / heads == blockIdx.x) return h;
    return -1;
}

// Embedding value Weight::value(id, c) * embedding_scale (per-row INT8).
__device__ __forceinline__ float embed_value(const Model& m, int32_t id, int64_t c) {
    const float q = static_cast<float>(m.embed[(int64_t)id * m.hidden + c]);
    return __fmul_rn(__fmul_rn(q, m.embed_scales[id]), m.embedding_scale);
}

__global__ void __launch_bounds__(kThreads, 1)
decode_model_kernel(const MOp* __restrict__ ops, int nops, const __grid_constant__ Model m) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    int8_t* codes = reinterpret_cast<int8_t*>(smem + kRingBytes);
    float* scratch = reinterpret_cast<float*>(codes + kMaxCols);      // [kScratchFloats]
    float* qkv_s = scratch + kScratchFloats;                           // q, k, v [3][kMaxDim]
    uint64_t* full = reinterpret_cast<uint64_t*>(qkv_s + 3 * kMaxDim);
    uint64_t* att_bar = full + kStageBarriers;  // [2] attention K / V staging
    uint64_t* empty = att_bar + 2;
    uint64_t* stage_end = empty + kStageBarriers;
    float* partial_max = reinterpret_cast<float*>(stage_end + kStageBarriers) + 32;  // [kConsumerWarps]
    float* best_v = partial_max + kConsumerWarps;                       // [kConsumerWarps]
    int32_t* best_row = reinterpret_cast<int32_t*>(best_v + kConsumerWarps);
    float* total_s = reinterpret_cast<float*>(best_row + kConsumerWarps);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(total_s + 1);
    // expf's table in shared memory (lanes index it with different k, which
    // the constant bank would serialise).
    ExpTable* tab_s = reinterpret_cast<ExpTable*>((reinterpret_cast<uintptr_t>(total_s + 2) + 7) & ~uintptr_t(7));
    OrderedSumScratch<kNC>* sum_ws =
        reinterpret_cast<OrderedSumScratch<kNC>*>((reinterpret_cast<uintptr_t>(tab_s + 1) + 15) & ~uintptr_t(15));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int b = 0; b < kStageBarriers; ++b) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], kGroupWarps);
        }
        mbar_init(&att_bar[0], 1);
        mbar_init(&att_bar[1], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (tid < 32) tab_s->bits[tid] = m.tab.bits[tid];
    const uint32_t tag = *reinterpret_cast<volatile uint32_t*>(m.sync);
    const int32_t id = *reinterpret_cast<volatile int32_t*>(m.ids);
    const int64_t pos = *reinterpret_cast<volatile int32_t*>(m.position);
    __syncthreads();
    // A step past the cache or an id outside the vocabulary does nothing
    // (every thread sees the same values, so the whole grid returns here).
    if (pos < 0 || pos >= m.capacity || id < 0 || id >= m.vocab) {
        if (tid == 0 && blockIdx.x == 0) record_device_error(kSiteDecodeDependency);
        return;
    }

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t policy = l2_policy_evict_first();
            RingCursor cursor;
            cursor.size = my_head(m.heads) >= 0 ? kAttnRingBytes : kRingBytes;
            uint64_t released = 0;
            int s = 0, rel = 0;
            bool go = true;
            for (int j = 0; j < nops && go; ++j) {
                const MOp op = ops[j];
                if (op.kind != kOpLinear) continue;
                const OpGeometry g = geometry(op);
                for (int rb = 0; rb < g.nblocks; ++rb, ++s) {
                    const uint32_t bytes = static_cast<uint32_t>(block_rows(g, rb) * op.cols);
                    const uint32_t start = cursor.place(bytes);
                    while (cursor.head - released > cursor.size || s - rel >= kStageBarriers) {
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
    const int group = warp / kGroupWarps;
    const int wi = warp % kGroupWarps;
    const int head = my_head(m.heads);
    int s = 0;
    RingCursor cursor;
    cursor.size = head >= 0 ? kAttnRingBytes : kRingBytes;
    bool ok = true;
    int prefetched_j = -1;
    float2 next_scale = make_float2(0.0f, 0.0f);
    uint32_t att_uses[2] = {0u, 0u};  // completed phases of att_bar[0 / 1]
    for (int j = 0; j < nops; ++j) {
        const MOp op = ops[j];
        if (op.kind == kOpAttention) {
            if (head < 0) continue;
            // ---------------------------------------------- attention
            // Cached keys / values of rows [0, pos) are staged through the
            // attention region (the ring's last 64 KB, the codes buffer and
            // the scratch: free in this block now).  When all keys and values
            // fit side by side, both are requested before the wait for this
            // token's q, k, v.  Otherwise the whole region holds keys for the
            // scores (one chunk up to ~320 keys of 64 floats), and then values
            // for the weighted sums, requested as soon as the scores are done
            // so that they land during the softmax (instead of a second key
            // and a second value chunk each waited for after the first).
            // Values come in one bulk copy per chunk.  Keys come as 16-byte
            // asynchronous copies by all consumer threads into rows padded by
            // 4 floats, so the 8 lanes of a quarter warp, each reading a float4
            // of its own key, hit 8 different bank groups.
            const int dim = m.dim, half = dim / 2;
            const int kvh = head / (m.heads / m.kv_heads);
            float* qs = qkv_s;
            float* ks = qkv_s + kMaxDim;
            float* vs = qkv_s + 2 * kMaxDim;
            float* kc = op.k_cache + (int64_t)kvh * m.capacity * dim;
            float* vc = op.v_cache + (int64_t)kvh * m.capacity * dim;
            const int64_t keys = pos + 1;
            float* att = reinterpret_cast<float*>(ring + kAttnRingBytes);
            const int keys_r = static_cast<int>((keys + 3) & ~3);
            float* scores = att;
            const int kst = dim + 4;  // padded key row (floats)
            const int avail = kAttFloats - keys_r;
            const int64_t least = pos > 0 ? pos : 1;
            const bool side_by_side = avail / (kst + dim) >= least;
            const int kchunk = static_cast<int>(side_by_side ? least : min64(avail / kst, least));
            const int vchunk = static_cast<int>(side_by_side ? least : min64(avail / dim, least));
            float* kbuf = att + keys_r;
            float* vbuf = side_by_side ? kbuf + kchunk * kst : kbuf;
            const uint64_t keep = l2_policy_evict_last();
            const int nchunks = static_cast<int>((pos + kchunk - 1) / kchunk);    // key chunks
            const int nvchunks = static_cast<int>((pos + vchunk - 1) / vchunk);  // value chunks
            auto issue = [&](const float* base, float* dst, uint64_t* bar, int c) {
                const int64_t k0 = (int64_t)c * vchunk;
                const uint32_t bytes = static_cast<uint32_t>(min64(vchunk, pos - k0) * dim * sizeof(float));
                mbar_arrive_expect_tx(bar, bytes);
                bulk_copy_g2s(dst, base + k0 * dim, bytes, bar, keep);
            };
            auto load_keys = [&](int c) {  // every consumer thread; completed by wait_async_copies()
                const int64_t k0 = (int64_t)c * kchunk;
                const int rows = static_cast<int>(min64(kchunk, pos - k0));
                const int vpr = dim / 4;
                for (int i = tid; i < rows * vpr; i += kNC) {
                    const int r = i / vpr, q = i - r * vpr;
                    async_copy16(kbuf + (size_t)r * kst + 4 * q, kc + (k0 + r) * dim + 4 * q);
                }
                commit_async_copies();
            };
            consumer_sync();  // every warp is done with the previous linear's codes
            if (nchunks > 0) load_keys(0);
            if (tid == 0 && nvchunks > 0 && side_by_side) issue(vc, vbuf, &att_bar[1], 0);
            // This position's rotation (independent of q and k), before the wait.
            float rope_c = 0.0f, rope_s = 0.0f;
            if (tid < half) {
                rope_c = m.cos_table[pos * half + tid];
                rope_s = m.sin_table[pos * half + tid];
            }
            for (int i = tid; i < 3 * dim; i += kNC) {
                const int part = i / dim, d = i % dim;
                const int64_t src = part == 0 ? (int64_t)head * dim + d
                                  : part == 1 ? (int64_t)m.heads * dim + (int64_t)kvh * dim + d
                                              : (int64_t)(m.heads + m.kv_heads) * dim + (int64_t)kvh * dim + d;
                float v = 0.0f;
                if (ok && !wait_tagged(op.x_ll + src, tag, v)) {
                    ok = false;
                    *abort_flag = 1;
                }
                qkv_s[part * kMaxDim + d] = v;
            }
            consumer_sync();
            // RoPE on q and k (decoder.cpp:1271-1279), in place.
            if (tid < half) {
                const float c = rope_c, sn = rope_s;
                const float a = qs[tid], b = qs[tid + half];
                const float ka = ks[tid], kb = ks[tid + half];
                qs[tid] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
                qs[tid + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sn));
                ks[tid] = __fsub_rn(__fmul_rn(ka, c), __fmul_rn(kb, sn));
                ks[tid + half] = __fadd_rn(__fmul_rn(kb, c), __fmul_rn(ka, sn));
            }
            consumer_sync();
            if (head % (m.heads / m.kv_heads) == 0)
                for (int d = tid; d < dim; d += kNC) {
                    kc[pos * dim + d] = ks[d];
                    vc[pos * dim + d] = vs[d];
                }
            // scores[k] = (q.k * scale) * scale with q.k summed left to right.
            float local_max = -INFINITY;
            if (tid == kNC - 1) {  // the current token's key (from shared memory), alongside
                float dot = 0.0f;
                for (int d = 0; d < dim; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], ks[d]));
                const float sc = __fmul_rn(__fmul_rn(dot, m.attn_scale), m.attn_scale);
                scores[pos] = sc;
                local_max = sc;
            }
            for (int c = 0; c < nchunks; ++c) {
                const int64_t k0 = (int64_t)c * kchunk;
                const int nk = static_cast<int>(min64(kchunk, pos - k0));
                if (c > 0) load_keys(c);
                wait_async_copies();
                consumer_sync();
                for (int k = tid; k < nk; k += kNC) {
                    if (!ok) break;
                    const float* krow = kbuf + k * kst;
                    float dot = 0.0f;
                    for (int d = 0; d < dim; d += 4) {
                        const float4 kv = *reinterpret_cast<const float4*>(krow + d);
                        dot = __fadd_rn(dot, __fmul_rn(qs[d], kv.x));
                        dot = __fadd_rn(dot, __fmul_rn(qs[d + 1], kv.y));
                        dot = __fadd_rn(dot, __fmul_rn(qs[d + 2], kv.z));
                        dot = __fadd_rn(dot, __fmul_rn(qs[d + 3], kv.w));
                    }
                    const float sc = __fmul_rn(__fmul_rn(dot, m.attn_scale), m.attn_scale);
                    scores[k0 + k] = sc;
                    local_max = fmaxf(local_max, sc);
                }
                consumer_sync();  // chunk consumed
            }
            // The keys are consumed: values into the same region now, while
            // the softmax runs.
            if (tid == 0 && nvchunks > 0 && !side_by_side) issue(vc, vbuf, &att_bar[1], 0);
            local_max = warp_max_f32(local_max);
            if (lane == 0) partial_max[warp] = local_max;
            consumer_sync();
            static_assert(kConsumerWarps <= 32 && (kConsumerWarps & (kConsumerWarps - 1)) == 0, "");
            const float maximum = warp_max_f32(partial_max[lane & (kConsumerWarps - 1)]);
            for (int64_t k = tid; k < keys; k += kNC) scores[k] = expf_libm(__fsub_rn(scores[k], maximum), *tab_s);
            consumer_sync();
            if (tid == 0) {
                float den = 0.0f;
                int64_t k = 0;
                for (; k + 4 <= keys; k += 4) {
                    const float4 e = *reinterpret_cast<const float4*>(scores + k);
                    den = __fadd_rn(den, e.x);
                    den = __fadd_rn(den, e.y);
                    den = __fadd_rn(den, e.z);
                    den = __fadd_rn(den, e.w);
                }
                for (; k < keys; ++k) den = __fadd_rn(den, scores[k]);
                *total_s = den;
            }
            consumer_sync();
            const float den = *total_s;
            for (int64_t k = tid; k < keys; k += kNC) scores[k] = __fdiv_rn(scores[k], den);
            consumer_sync();
            // out[d] = sum over keys, in order, of probability * v[k][d].
            float acc = 0.0f;
            for (int c = 0; c < nvchunks; ++c) {
                const int64_t k0 = (int64_t)c * vchunk;
                const int nk = static_cast<int>(min64(vchunk, pos - k0));
                if (c > 0 && tid == 0) issue(vc, vbuf, &att_bar[1], c);
                if (ok && !mbar_wait(&att_bar[1], att_uses[1] & 1, kSiteDecodeFull)) {
                    ok = false;
                    *abort_flag = 1;
                }
                ++att_uses[1];
                if (ok && tid < dim) {
                    const float* vb = vbuf + tid;
                    const float* pk = scores + k0;
#pragma unroll 8
                    for (int k = 0; k < nk; ++k) acc = __fadd_rn(acc, __fmul_rn(pk[k], vb[k * dim]));
                }
                consumer_sync();  // chunk consumed
            }
            if (tid < dim) {
                acc = __fadd_rn(acc, __fmul_rn(scores[pos], vs[tid]));
                store_tagged(op.y_ll + (int64_t)head * dim + tid, acc, tag);
            }
            consumer_sync();  // scratch and q/k/v are reused by the next op
            continue;
        }
        // ---------------------------------------------------- linear
        // The next attention's cached keys and values (written by earlier
        // launches, likely evicted by the weight stream) are pulled into L2
        // while this linear runs.
        if (head >= 0 && tid == 0 && j + 1 < nops && pos > 0) {
            const MOp nx = ops[j + 1];
            if (nx.kind == kOpAttention) {
                const int kvh = head / (m.heads / m.kv_heads);
                const uint32_t bytes = static_cast<uint32_t>(pos * m.dim * sizeof(float));
                const int64_t base = (int64_t)kvh * m.capacity * m.dim;
                for (uint32_t off = 0; off < bytes; off += 65536u) {
                    const uint32_t len = min(65536u, bytes - off);
                    bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(nx.k_cache + base) + off, len);
                    bulk_prefetch_l2(reinterpret_cast<const uint8_t*>(nx.v_cache + base) + off, len);
                }
            }
        }
        const OpGeometry g = geometry(op);
        if (g.nblocks == 0) continue;
        // Row scales of this warp's row blocks, one lane per block, loaded
        // one linear ahead.
        const bool rows_in_regs = g.nblocks <= kGroups * 32;
        const float2 row_scale = prefetched_j == j ? next_scale : load_row_scales(op, g, group, wi, lane);
        for (int j2 = j + 1; j2 < nops; ++j2) {
            const MOp op2 = ops[j2];
            if (op2.kind != kOpLinear) continue;
            const OpGeometry g2 = geometry(op2);
            if (g2.nblocks == 0) continue;
            next_scale = load_row_scales(op2, g2, group, wi, lane);
            prefetched_j = j2;
            break;
        }
        const int64_t vecs = op.cols / 4;
        float4 xr[kXVec];
        // The norm's weights do not depend on x: requested before waiting for
        // it, so the normalisation after the in-order sum finds them loaded.
        float4 nw[kNormXVec];
        if (op.xsrc != kXTagged) {
#pragma unroll
            for (int k = 0; k < kNormXVec; ++k) {
                const int64_t i = tid + (int64_t)k * kNC;
                nw[k] = i < vecs ? __ldg(reinterpret_cast<const float4*>(op.norm_w) + i)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        if (op.xsrc == kXTagged) {
            if (ok && !load_tagged_x(op.x_ll, vecs, tag, tid, xr)) {
                ok = false;
                *abort_flag = 1;
            }
        } else {
            // RMSNorm of the hidden vector (norm(), decoder.cpp:706-727).
            if (op.xsrc == kXNormEmbed) {
#pragma unroll
                for (int k = 0; k < kXVec; ++k) {
                    const int64_t i = tid + (int64_t)k * kNC;
                    xr[k] = i < vecs ? make_float4(embed_value(m, id, 4 * i), embed_value(m, id, 4 * i + 1),
                                                   embed_value(m, id, 4 * i + 2), embed_value(m, id, 4 * i + 3))
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            } else if (ok && !load_tagged_x(op.x_ll, vecs, tag, tid, xr)) {
                ok = false;
                *abort_flag = 1;
            }
            // Squares in parallel; then their left-to-right sum, bit for bit:
            // by all consumer threads (sum_in_order_par) for rows of up to
            // 4 * kNC values, else by one thread.
            float* sq4 = scratch;
            float4 sq0 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < kNormXVec; ++k) {
                const int64_t i = tid + (int64_t)k * kNC;
                if (i < vecs) {
                    const float4 q = make_float4(__fmul_rn(xr[k].x, xr[k].x), __fmul_rn(xr[k].y, xr[k].y),
                                                 __fmul_rn(xr[k].z, xr[k].z), __fmul_rn(xr[k].w, xr[k].w));
                    reinterpret_cast<float4*>(sq4)[i] = q;
                    if (k == 0) sq0 = q;
                }
            }
            consumer_sync();
            if (*abort_flag) return;
            float sumsq;
            if (op.cols <= 4 * kNC) {
                sumsq = sum_in_order_par<kNC>(sq0, sq4, static_cast<int>(op.cols), tid, *sum_ws,
                                              [] { consumer_sync(); });
            } else {
                if (tid == 0) *total_s = sum_in_order(sq4, static_cast<int>(op.cols));
                consumer_sync();
                sumsq = *total_s;
            }
            const float scale =
                __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, static_cast<float>(op.cols)), m.epsilon)));
#pragma unroll
            for (int k = kNormXVec; k < kXVec; ++k) xr[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int k = 0; k < kNormXVec; ++k) {
                const int64_t i = tid + (int64_t)k * kNC;
                if (i < vecs) {
                    const float4 w = nw[k];
                    float4 v = xr[k];
                    v.x = __fadd_rn(__fmul_rn(__fmul_rn(v.x, scale), w.x), 0.0f);
                    v.y = __fadd_rn(__fmul_rn(__fmul_rn(v.y, scale), w.y), 0.0f);
                    v.z = __fadd_rn(__fmul_rn(__fmul_rn(v.z, scale), w.z), 0.0f);
                    v.w = __fadd_rn(__fmul_rn(__fmul_rn(v.w, scale), w.w), 0.0f);
                    xr[k] = v;
                }
            }
        }
        // Residual inputs of this warp's rows, one lane per row block (the
        // hidden vector is complete: this op's input was derived from it).
        // The word is requested now and its tag checked after the
        // quantisation, so the load's latency hides behind it.
        int64_t resid_r = -1;
        uint64_t resid_word0 = 0, resid_word1 = 0;
        if (op.epi == kEpiResidTagged && rows_in_regs && ok && group + kGroups * lane < g.nblocks) {
            const int64_t r = g.row0 + (int64_t)(group + kGroups * lane) * kRowsPerStage + 2 * wi;
            if (r < g.row1) {
                resid_r = r;
                resid_word0 = load_tagged(op.resid_ll + r);
                if (r + 1 < g.row1) resid_word1 = load_tagged(op.resid_ll + r + 1);
            }
        }
        // Per-token INT8 quantisation of x (decoder.cpp:1028-1038).
        float mx = 0.0f;
#pragma unroll
        for (int k = 0; k < kXVec; ++k)
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(xr[k].x), fabsf(xr[k].y)), fmaxf(fabsf(xr[k].z), fabsf(xr[k].w))));
        mx = warp_max_f32(mx);
        if (lane == 0) partial_max[warp] = mx;
        consumer_sync();  // also: every warp has finished the previous linear
        if (*abort_flag) return;
        const float absmax = warp_max_f32(partial_max[lane & (kConsumerWarps - 1)]);
        const float xscale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
        const float mul = __fdiv_rn(1.0f, xscale);
        char4* out4 = reinterpret_cast<char4*>(codes);
#pragma unroll
        for (int k = 0; k < kXVec; ++k) {
            const int64_t i = tid + (int64_t)k * kNC;
            if (i < vecs)
                out4[i] = make_char4(to_code(xr[k].x, mul), to_code(xr[k].y, mul), to_code(xr[k].z, mul),
                                     to_code(xr[k].w, mul));
        }
        consumer_sync();
        float2 row_resid = make_float2(0.0f, 0.0f);
        if (resid_r >= 0) {
            if (static_cast<uint32_t>(resid_word0 >> 32) == tag) {
                row_resid.x = __uint_as_float(static_cast<uint32_t>(resid_word0));
            } else if (ok && !wait_tagged(op.resid_ll + resid_r, tag, row_resid.x)) {
                ok = false;
                *abort_flag = 1;
            }
            if (resid_r + 1 < g.row1) {
                if (static_cast<uint32_t>(resid_word1 >> 32) == tag) {
                    row_resid.y = __uint_as_float(static_cast<uint32_t>(resid_word1));
                } else if (ok && !wait_tagged(op.resid_ll + resid_r + 1, tag, row_resid.y)) {
                    ok = false;
                    *abort_flag = 1;
                }
            }
        }
        const int cols = static_cast<int>(op.cols);
        float best = -INFINITY;
        int32_t best_r = 0x7fffffff;
        for (int rb = 0; rb < g.nblocks; ++rb) {
            const int live_rows = block_rows(g, rb);
            const uint32_t start = cursor.place(static_cast<uint32_t>(live_rows * cols));
            if (rb % kGroups != group) continue;
            const int st = s + rb;
            const int b = st % kStageBarriers;
            if (ok && !mbar_wait(&full[b], (st / kStageBarriers) & 1, kSiteDecodeFull)) {
                ok = false;
                *abort_flag = 1;
            }
            // This warp's rows 2 wi and 2 wi + 1 of the stage, side by side.
            const bool live0 = 2 * wi < live_rows, live1 = 2 * wi + 1 < live_rows;
            int a0 = 0, a0b = 0, a1 = 0, a1b = 0;
            if (ok && live0) {
                const uint8_t* w0 = ring + start + (size_t)(2 * wi) * cols;
                if (live1) {
                    const uint8_t* w1 = w0 + cols;
#pragma unroll 4
                    for (int off = lane * 16; off < cols; off += 512) {
                        const int4 qv = *reinterpret_cast<const int4*>(codes + off);
                        const int4 u = *reinterpret_cast<const int4*>(w0 + off);
                        const int4 v = *reinterpret_cast<const int4*>(w1 + off);
                        a0 = dp4a(u.x, qv.x, a0);
                        a0b = dp4a(u.y, qv.y, a0b);
                        a0 = dp4a(u.z, qv.z, a0);
                        a0b = dp4a(u.w, qv.w, a0b);
                        a1 = dp4a(v.x, qv.x, a1);
                        a1b = dp4a(v.y, qv.y, a1b);
                        a1 = dp4a(v.z, qv.z, a1);
                        a1b = dp4a(v.w, qv.w, a1b);
                    }
                } else {
#pragma unroll 4
                    for (int off = lane * 16; off < cols; off += 512) {
                        const int4 qv = *reinterpret_cast<const int4*>(codes + off);
                        const int4 u = *reinterpret_cast<const int4*>(w0 + off);
                        a0 = dp4a(u.x, qv.x, a0);
                        a0b = dp4a(u.y, qv.y, a0b);
                        a0 = dp4a(u.z, qv.z, a0);
                        a0b = dp4a(u.w, qv.w, a0b);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[b]);
            // Both rows' sums by two independent warp reductions (integer sums:
            // any order); lanes 0-15 continue with row 2 wi, lanes 16-31 with
            // row 2 wi + 1.
            const int sum0 = __reduce_add_sync(0xffffffffu, a0 + a0b);
            const int sum1 = __reduce_add_sync(0xffffffffu, a1 + a1b);
            const bool hi = lane >= 16;
            const int acc = hi ? sum1 : sum0;
            const int64_t row = g.row0 + (int64_t)rb * kRowsPerStage + 2 * wi + (hi ? 1 : 0);
            const int src = (rb / kGroups) & 31;
            const float sw0 = __shfl_sync(0xffffffffu, row_scale.x, src);
            const float sw1 = __shfl_sync(0xffffffffu, row_scale.y, src);
            const float rs0 = __shfl_sync(0xffffffffu, row_resid.x, src);
            const float rs1 = __shfl_sync(0xffffffffu, row_resid.y, src);
            const bool live = hi ? live1 : live0;
            float y = 0.0f;
            if (live) {
                const float sw = rows_in_regs ? (hi ? sw1 : sw0) : __ldg(op.ws + row);
                const float product = __fmul_rn(__int2float_rn(acc), xscale);
                y = __fadd_rn(__fmaf_rn(product, sw, 0.0f), 0.0f);  // + (no bias)
            }
            if (op.epi == kEpiSiluPair) {
                // Rows 2 wi (gate) and 2 wi + 1 (up): lane 0 gets the up value.
                const float up = __shfl_sync(0xffffffffu, y, 16);
                if (ok && live0 && lane == 0) {
                    const float gate = y;
                    const float act = __fmul_rn(up, __fdiv_rn(gate, __fadd_rn(1.0f, expf_libm(-gate, *tab_s))));
                    store_tagged(op.y_ll + row / 2, act, tag);
                }
                continue;
            }
            if (!(ok && live && (lane & 15) == 0)) continue;
            if (op.epi == kEpiTagged) {
                store_tagged(op.y_ll + row, y, tag);
            } else if (op.epi == kEpiResidEmbed) {
                store_tagged(op.y_ll + row, __fadd_rn(embed_value(m, id, row), y), tag);
            } else if (op.epi == kEpiResidTagged) {
                float hin = hi ? rs1 : rs0;
                if (!rows_in_regs && !wait_tagged(op.resid_ll + row, tag, hin)) {
                    ok = false;
                    *abort_flag = 1;
                }
                const float v = op.add_zero ? __fadd_rn(y, 0.0f) : y;
                store_tagged(op.y_ll + row, __fadd_rn(hin, v), tag);
            } else {  // logits
                if (m.logits) m.logits[row] = y;
                if (y > best || best_r == 0x7fffffff) {
                    best = y;
                    best_r = static_cast<int32_t>(row);
                }
            }
        }
        s += g.nblocks;
        if (op.epi == kEpiLogits) {
            // Block argmax folded into the launch's 64-bit key: larger value
            // first, then the smaller row (std::max_element keeps the first).
            // Lane 16's rows into lane 0's: larger value, then the smaller row.
            const float ov = __shfl_sync(0xffffffffu, best, 16);
            const int32_t orow = __shfl_sync(0xffffffffu, best_r, 16);
            if (lane == 0) {
                if (orow != 0x7fffffff && (best_r == 0x7fffffff || ov > best || (ov == best && orow < best_r))) {
                    best = ov;
                    best_r = orow;
                }
                best_v[warp] = best;
                best_row[warp] = best_r;
            }
            consumer_sync();
            if (tid == 0) {
                float bv = -INFINITY;
                int32_t br = 0x7fffffff;
                for (int w = 0; w < kConsumerWarps; ++w)
                    if (best_row[w] != 0x7fffffff && (br == 0x7fffffff || best_v[w] > bv ||
                                                      (best_v[w] == bv && best_row[w] < br))) {
                        bv = best_v[w];
                        br = best_row[w];
                    }
                if (br != 0x7fffffff) {
                    const uint32_t bits = __float_as_uint(bv);
                    const uint32_t ordered = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
                    const unsigned long long key =
                        (static_cast<unsigned long long>(ordered) << 32) | (0xffffffffu - static_cast<uint32_t>(br));
                    atomicMax(reinterpret_cast<unsigned long long*>(m.sync + 2), key);
                }
            }
        }
    }
    // Last block out publishes the next token and advances the launch tag.
    consumer_sync();
    if (tid == 0 && ok && !*abort_flag) {
        __threadfence();
        const uint32_t done = atomicAdd(m.sync + 1, 1u);
        if (done == gridDim.x - 1) {
            __threadfence();
            unsigned long long* keyp = reinterpret_cast<unsigned long long*>(m.sync + 2);
            const unsigned long long key = atomicAdd(keyp, 0ull);
            const int32_t next = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffu));
            *m.ids = next;
            if (m.history) m.history[pos + 1] = next;
            *m.position = static_cast<int32_t>(pos + 1);
            *keyp = 0ull;
            m.sync[1] = 0;
            m.sync[0] = tag + 1 == 0 ? 1 : tag + 1;
        }
    }
}

struct ModelPlan {
    MOp* ops = nullptr;
    int nops = 0;
    uint32_t* sync = nullptr;
    uint64_t* buffers = nullptr;
    Model model = {};
    int device = 0;
};

}  // namespace
}  // namespace leafq

using namespace leafq;

extern "C" {

struct leafq_model_plan_t {
    ModelPlan plan;
};

int leafq_model_plan_create(const leafq_model_desc* d, leafq_model_plan_t** out) {
    clear_error();
    if (!d || !out || !d->layer || d->layers <= 0) {
        set_error("leafq_model_plan_create: null description or no layers");
        return LEAFQ_ERR_INVALID;
    }
    *out = nullptr;
    const int64_t h = d->hidden, f = d->intermediate, dim = d->head_dim;
    const int64_t qkv_rows = (int64_t)(d->heads + 2 * d->kv_heads) * dim;
    if (h <= 0 || f <= 0 || d->heads <= 0 || d->kv_heads <= 0 || d->heads % d->kv_heads ||
        d->heads * dim != h || dim % 4 || dim > kMaxDim || d->vocab <= 0 || d->capacity <= 0 ||
        d->capacity > kMaxCapacity || h > kScratchFloats || h % 16 || f % 16 || f > kMaxCols ||
        h > kMaxCols || 5 * d->layers + 1 > kMaxOps || d->heads > sm_count() ||
        !(d->attn_scale > 0.0f)) {
        set_error("leafq_model_plan_create: unsupported geometry (hidden and intermediate multiples of "
                  "16 and <= 4096 / 6144, heads * head_dim == hidden, head_dim a multiple of 4 and <= 256, "
                  "capacity <= 2048, heads <= SMs)");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    if (!d->embed || !d->embed_scales || !d->final_norm || !d->lm_head || !d->lm_head_scales ||
        !d->cos_table || !d->sin_table || !d->ids || !d->position) {
        set_error("leafq_model_plan_create: null model pointer");
        return LEAFQ_ERR_INVALID;
    }
    for (int l = 0; l < d->layers; ++l) {
        const leafq_model_layer& L = d->layer[l];
        if (!L.input_norm || !L.post_norm || !L.qkv || !L.qkv_scales || !L.o || !L.o_scales ||
            !L.gate_up || !L.gate_up_scales || !L.down || !L.down_scales || !L.k_cache || !L.v_cache ||
            !aligned16(L.qkv) || !aligned16(L.o) || !aligned16(L.gate_up) || !aligned16(L.down) ||
            !aligned16(L.input_norm) || !aligned16(L.post_norm)) {
            set_error("leafq_model_plan_create: null or unaligned pointer in layer " + std::to_string(l));
            return LEAFQ_ERR_INVALID;
        }
    }
    if (!aligned16(d->lm_head) || !aligned16(d->final_norm)) {
        set_error("leafq_model_plan_create: unaligned lm_head or final norm");
        return LEAFQ_ERR_INVALID;
    }
    // Tagged buffers per layer: qkv, attn, h1, act, h2.
    const size_t per_layer = (size_t)qkv_rows + h + h + f + h;
    const size_t words = per_layer * d->layers;
    auto* handle = new leafq_model_plan_t();
    ModelPlan& p = handle->plan;
    cudaGetDevice(&p.device);
    std::vector<MOp> host;
    cudaError_t err = cudaMalloc(&p.buffers, words * sizeof(uint64_t));
    if (err == cudaSuccess) err = cudaMemset(p.buffers, 0, words * sizeof(uint64_t));
    if (err == cudaSuccess) err = cudaMalloc(&p.sync, 4 * sizeof(uint32_t));
    const uint32_t sync_init[4] = {1u, 0u, 0u, 0u};
    if (err == cudaSuccess) err = cudaMemcpy(p.sync, sync_init, sizeof(sync_init), cudaMemcpyHostToDevice);
    if (err == cudaSuccess) {
        const uint64_t* prev_h2 = nullptr;
        for (int l = 0; l < d->layers; ++l) {
            const leafq_model_layer& L = d->layer[l];
            uint64_t* base = p.buffers + per_layer * l;
            uint64_t* qkv = base;
            uint64_t* attn = qkv + qkv_rows;
            uint64_t* h1 = attn + h;
            uint64_t* act = h1 + h;
            uint64_t* h2 = act + f;
            MOp op = {};
            // q|k|v = linear(RMSNorm(h))
            op = {};
            op.kind = kOpLinear;
            op.xsrc = l == 0 ? kXNormEmbed : kXNormTagged;
            op.x_ll = prev_h2;
            op.norm_w = L.input_norm;
            op.epi = kEpiTagged;
            op.y_ll = qkv;
            op.w = L.qkv;
            op.ws = L.qkv_scales;
            op.rows = qkv_rows;
            op.cols = h;
            host.push_back(op);
            // attention
            op = {};
            op.kind = kOpAttention;
            op.x_ll = qkv;
            op.y_ll = attn;
            op.k_cache = L.k_cache;
            op.v_cache = L.v_cache;
            host.push_back(op);
            // h1 = h + o(attn)
            op = {};
            op.kind = kOpLinear;
            op.xsrc = kXTagged;
            op.x_ll = attn;
            op.epi = l == 0 ? kEpiResidEmbed : kEpiResidTagged;
            op.resid_ll = prev_h2;
            op.y_ll = h1;
            op.w = L.o;
            op.ws = L.o_scales;
            op.rows = h;
            op.cols = h;
            host.push_back(op);
            // act = silu(gate) * up of linear(RMSNorm(h1))
            op = {};
            op.kind = kOpLinear;
            op.xsrc = kXNormTagged;
            op.x_ll = h1;
            op.norm_w = L.post_norm;
            op.epi = kEpiSiluPair;
            op.y_ll = act;
            op.w = L.gate_up;
            op.ws = L.gate_up_scales;
            op.rows = 2 * f;
            op.cols = h;
            host.push_back(op);
            // h2 = h1 + (down(act) + 0)
            op = {};
            op.kind = kOpLinear;
            op.xsrc = kXTagged;
            op.x_ll = act;
            op.epi = kEpiResidTagged;
            op.add_zero = 1;
            op.resid_ll = h1;
            op.y_ll = h2;
            op.w = L.down;
            op.ws = L.down_scales;
            op.rows = h;
            op.cols = f;
            host.push_back(op);
            prev_h2 = h2;
        }
        MOp op = {};
        op.kind = kOpLinear;
        op.xsrc = kXNormTagged;
        op.x_ll = prev_h2;
        op.norm_w = d->final_norm;
        op.epi = kEpiLogits;
        op.w = d->lm_head;
        op.ws = d->lm_head_scales;
        op.rows = d->vocab;
        op.cols = h;
        host.push_back(op);
        p.nops = static_cast<int>(host.size());
        err = cudaMalloc(&p.ops, sizeof(MOp) * host.size());
        if (err == cudaSuccess)
            err = cudaMemcpy(p.ops, host.data(), sizeof(MOp) * host.size(), cudaMemcpyHostToDevice);
    }
    if (err != cudaSuccess) {
        cudaFree(p.ops);
        cudaFree(p.sync);
        cudaFree(p.buffers);
        delete handle;
        return cuda_status(err, "leafq_model_plan_create");
    }
    Model& m = p.model;
    m.embed = d->embed;
    m.embed_scales = d->embed_scales;
    m.cos_table = d->cos_table;
    m.sin_table = d->sin_table;
    m.ids = d->ids;
    m.position = d->position;
    m.history = d->history;
    m.logits = d->logits;
    m.sync = p.sync;
    m.capacity = d->capacity;
    m.embedding_scale = d->embedding_scale;
    m.epsilon = d->epsilon;
    m.attn_scale = d->attn_scale;
    m.hidden = d->hidden;
    m.heads = d->heads;
    m.kv_heads = d->kv_heads;
    m.dim = d->head_dim;
    m.vocab = d->vocab;
    m.tab = exp_table();
    *out = handle;
    return LEAFQ_OK;
}

int leafq_model_plan_run(void* stream, leafq_model_plan_t* plan) {
    clear_error();
    if (!plan) {
        set_error("leafq_model_plan_run: null plan");
        return LEAFQ_ERR_INVALID;
    }
    int st = allow_smem(reinterpret_cast<const void*>(decode_model_kernel), kSmemBytes, "decode_model");
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
    const cudaError_t err = cudaLaunchKernelEx(&config, decode_model_kernel,
                                               static_cast<const MOp*>(plan->plan.ops), plan->plan.nops,
                                               plan->plan.model);
    return cuda_status(err, "leafq_model_plan_run");
}

int leafq_model_plan_destroy(leafq_model_plan_t* plan) {
    clear_error();
    if (!plan) return LEAFQ_OK;
    cudaFree(plan->plan.ops);
    cudaFree(plan->plan.sync);
    cudaFree(plan->plan.buffers);
    delete plan;
    return LEAFQ_OK;
}

}  // extern "C"
