// The decoder's non-linear operators around the quantised linears
// (Decoder::Impl::forward_into, decoder.cpp:1282-1452), on the GPU.
//
//   embed_kernel          embedding rows Weight::value(id, col) * embedding_scale
//                         (decoder.cpp:1293-1304, :241-250)
//   rmsnorm_kernel        optional residual add, then RMSNorm (norm(),
//                         decoder.cpp:706-727) with the reference's epilogue
//                         order (x * scale) * weight + 0
//   rotary_append_kernel  RoPE on q and k from host-computed tables
//                         (decoder.cpp:1234-1281), q to head-major order, k and
//                         v appended to the per-layer cache (kv_cache.cpp:21-59)
//   attention_kernel      causal GQA attention (KVCache::attend ->
//                         transformer.cpp:93-145): q.k, scaled twice, softmax,
//                         probability-weighted V
//   silu_gate_kernel      up * (gate / (1 + expf(-gate))) (decoder.cpp:982-988)
//   argmax_kernel         first index of the largest logit
//                         (main_decoder.cpp:101, std::max_element)
//
// Every result is bit-identical to the reference decoder's (built as
// leaf/cli.py:66 builds it, on Linux):
// * sums run in the reference's order: RMSNorm's sum of squares, the
//   attention dot product (transformer.cpp is built without -mavx2, so
//   fast_dot is the sequential scalar_dot), the softmax denominator and each
//   output element's probability-weighted sum over keys are sequential;
// * the exponential is libm's expf (attention transformer.cpp:130, SiLU
//   decoder.cpp:983; the vector SiLU kernel is enabled on Windows builds
//   only, decoder_config.h:5-11).  expf_libm restates the algorithm of the
//   system libm (GNU C Library 2.39 expf, from Arm's optimized-routines):
//   k = round(x * 32 / ln 2), r = x * 32 / ln 2 - k, 2^(k/32) from a
//   32-entry table of 2^(i/32), a cubic in r, all in double, one rounding
//   to float.  The table is computed on the host (2^(i/32) rounded to
//   double) and passed as a kernel parameter.  The restatement was checked
//   against libm expf on all 2^32 float inputs.
// Sequential sums cost latency (a 2048-element sum of squares is a chain of
// 2048 dependent additions); they are the price of identical greedy tokens:
// the random-init decoders amplify a last-bit difference anywhere into
// different logits within a few layers.
#include <cmath>
#include <cstring>

#include "decoder_math.cuh"
#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnThreads = 128;
constexpr int kArgmaxThreads = 1024;

__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max_f32(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < static_cast<int>(blockDim.x >> 5) ? scratch[lane] : -INFINITY;
        v = warp_max_f32(v);
        if (lane == 0) scratch[32] = v;
    }
    __syncthreads();
    return scratch[32];
}

// ------------------------------------------------------------------ embed
__global__ void embed_kernel(const int32_t* __restrict__ ids, const void* __restrict__ table,
                             const float* __restrict__ scales, int bits, int64_t group, int64_t vocab,
                             int64_t hidden, float embedding_scale, float* __restrict__ out,
                             int32_t* __restrict__ error_flag) {
    const int64_t t = blockIdx.x;
    int64_t id = ids[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0 && error_flag) atomicExch(error_flag, 1);
        id = 0;
    }
    for (int64_t c = threadIdx.x; c < hidden; c += blockDim.x) {
        const int64_t index = id * hidden + c;
        float v;
        if (bits == 32) {
            v = static_cast<const float*>(table)[index];
        } else {
            int q;
            if (bits == 8) {
                q = static_cast<const int8_t*>(table)[index];
            } else {
                q = (static_cast<const uint8_t*>(table)[index / 2] >> ((index % 2) * 4)) & 15;
                if (q >= 8) q -= 16;
            }
            v = __fmul_rn(static_cast<float>(q), scales[id * (hidden / group) + c / group]);
        }
        out[t * hidden + c] = __fmul_rn(v, embedding_scale);
    }
}

// ---------------------------------------------------------------- rmsnorm
// hidden[t] (+)= delta[t] (+ 0 when add_zero), written back; then
// out[t] = (hidden * (1 / sqrt(sum(h^2) / width + eps))) * weight + 0, the
// sum of squares accumulated left to right as norm() does.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(
    float* __restrict__ hidden, const float* __restrict__ delta, int add_zero, int64_t width,
    const float* __restrict__ weight, float epsilon, float* __restrict__ out) {
    extern __shared__ float row[];  // [width] values, then [width] squares
    float* squares = row + width;
    __shared__ float sequential_total;  // the sum of squares
    const int64_t t = blockIdx.x;
    float* h = hidden + t * width;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) {
        float v = h[c];
        if (delta) {
            float d = delta[t * width + c];
            if (add_zero) d = __fadd_rn(d, 0.0f);
            v = __fadd_rn(v, d);
            h[c] = v;
        }
        row[c] = v;
        squares[c] = __fmul_rn(v, v);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if ((width & 3) == 0) {
            sequential_total = sum_in_order(squares, static_cast<int>(width));
        } else {
            float sq = 0.0f;
            for (int64_t c = 0; c < width; ++c) sq = __fadd_rn(sq, squares[c]);
            sequential_total = sq;
        }
    }
    __syncthreads();
    const float total = sequential_total;
    const float scale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(width)), epsilon)));
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x)
        out[t * width + c] = __fadd_rn(__fmul_rn(__fmul_rn(row[c], scale), weight[c]), 0.0f);
}

// The same operator for rows of width % 4 == 0, width <= 4 * 2 * kNormVecThreads,
// 16-byte aligned: each thread keeps its (up to 8) values in registers, so
// the row is read once with all loads in flight; rows of up to 2048 values
// sum their squares with the whole block (sum_in_order_par).  Optionally the
// normalised row is quantised to per-token INT8 codes in the same pass (the
// quantiser of leafq_quantize_act, bit for bit), for a W8A8 linear that
// follows.
constexpr int kNormVec = 2;
constexpr int kNormVecThreads = 512;

__global__ void __launch_bounds__(kNormVecThreads) rmsnorm_vec_kernel(
    float* __restrict__ hidden, const float* __restrict__ delta, int add_zero, int64_t width,
    const float* __restrict__ weight, float epsilon, float* __restrict__ out, int8_t* __restrict__ codes,
    float* __restrict__ code_scales) {
    extern __shared__ __align__(16) float squares[];  // [width]
    __shared__ float scratch[33];
    __shared__ OrderedSumScratch<kNormVecThreads> sum_ws;
    const int64_t t = blockIdx.x;
    const int n4 = static_cast<int>(width / 4);
    float4* h4 = reinterpret_cast<float4*>(hidden + t * width);
    const float4* d4 = delta ? reinterpret_cast<const float4*>(delta + t * width) : nullptr;
    const float4* w4 = reinterpret_cast<const float4*>(weight);
    float4 v[kNormVec], w[kNormVec], dv[kNormVec];
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int c = threadIdx.x + j * kNormVecThreads;
        if (c < n4) {
            v[j] = h4[c];
            if (d4) dv[j] = __ldg(d4 + c);
            w[j] = __ldg(w4 + c);
        }
    }
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int c = threadIdx.x + j * kNormVecThreads;
        if (c < n4) {
            if (d4) {
                float4 d = dv[j];
                if (add_zero) d = make_float4(__fadd_rn(d.x, 0.0f), __fadd_rn(d.y, 0.0f), __fadd_rn(d.z, 0.0f),
                                              __fadd_rn(d.w, 0.0f));
                v[j] = make_float4(__fadd_rn(v[j].x, d.x), __fadd_rn(v[j].y, d.y), __fadd_rn(v[j].z, d.z),
                                   __fadd_rn(v[j].w, d.w));
                h4[c] = v[j];
            }
            reinterpret_cast<float4*>(squares)[c] =
                make_float4(__fmul_rn(v[j].x, v[j].x), __fmul_rn(v[j].y, v[j].y), __fmul_rn(v[j].z, v[j].z),
                            __fmul_rn(v[j].w, v[j].w));
        }
    }
    __syncthreads();
    float total;
    if (width <= 4 * kNormVecThreads) {
        const float4 sq0 = threadIdx.x < n4 ? reinterpret_cast<const float4*>(squares)[threadIdx.x]
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
        total = sum_in_order_par<kNormVecThreads>(sq0, squares, static_cast<int>(width), threadIdx.x, sum_ws,
                                                  [] { __syncthreads(); });
    } else {
        if (threadIdx.x == 0) scratch[32] = sum_in_order(squares, static_cast<int>(width));
        __syncthreads();
        total = scratch[32];
    }
    const float scale =
        __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(width)), epsilon)));
    float4 o[kNormVec];
    float absmax = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int c = threadIdx.x + j * kNormVecThreads;
        if (c < n4) {
            o[j] = make_float4(__fadd_rn(__fmul_rn(__fmul_rn(v[j].x, scale), w[j].x), 0.0f),
                               __fadd_rn(__fmul_rn(__fmul_rn(v[j].y, scale), w[j].y), 0.0f),
                               __fadd_rn(__fmul_rn(__fmul_rn(v[j].z, scale), w[j].z), 0.0f),
                               __fadd_rn(__fmul_rn(__fmul_rn(v[j].w, scale), w[j].w), 0.0f));
            if (out) reinterpret_cast<float4*>(out + t * width)[c] = o[j];
            absmax = fmaxf(absmax, fmaxf(fmaxf(fabsf(o[j].x), fabsf(o[j].y)), fmaxf(fabsf(o[j].z), fabsf(o[j].w))));
        }
    }
    if (!codes) return;  // uniform across the block
    absmax = block_max(absmax, scratch);
    const float qscale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
    const float multiplier = __fdiv_rn(1.0f, qscale);
    if (threadIdx.x == 0) code_scales[t] = qscale;
    char4* c4 = reinterpret_cast<char4*>(codes + t * width);
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
        const int c = threadIdx.x + j * kNormVecThreads;
        if (c < n4)
            c4[c] = make_char4(act_code(o[j].x, multiplier), act_code(o[j].y, multiplier),
                               act_code(o[j].z, multiplier), act_code(o[j].w, multiplier));
    }
}

// ------------------------------------------------------ rotary + KV append
// Sequence s of a batch owns rows s*tokens .. s*tokens+tokens-1 of qkv, its
// own cache [kv_heads][capacity][dim] at s * kv_heads * capacity * dim, and
// its own start position positions[s].  qkv[row] = [q (heads*dim) | k
// (kv*dim) | v (kv*dim)].  Blocks (t, s, *) rotate every q head (to
// q_heads[s][head][t]) and k head (to the k cache) of its row and copies v
// to the v cache, spread over blockIdx.z.  A position past the cache is recorded in the device
// error word and skipped.
__global__ void rotary_append_kernel(const float* __restrict__ qkv, int64_t tokens, int heads,
                                     int kv_heads, int dim, int rotary_dim,
                                     const float* __restrict__ cos_table,
                                     const float* __restrict__ sin_table,
                                     const int32_t* __restrict__ positions,
                                     float* __restrict__ q_heads, float* __restrict__ k_cache,
                                     float* __restrict__ v_cache, int64_t capacity) {
    const int64_t t = blockIdx.x;
    const int64_t seq = blockIdx.y;
    const int64_t width = (int64_t)(heads + 2 * kv_heads) * dim;
    const int64_t start = positions[seq];
    const int64_t pos = start + t;
    if (start < 0 || start + tokens > capacity) {
        if (threadIdx.x == 0 && t == 0) record_device_error(kSiteCacheRange);
        return;
    }
    const int half = rotary_dim / 2;
    const float* row = qkv + (seq * tokens + t) * width;
    const int64_t cache = seq * kv_heads * capacity * dim;
    const float* cs = cos_table + pos * half;
    const float* sn = sin_table + pos * half;
    // Items of the row, one per thread: a rotation pair or a copied element
    // of each q / k head, then each v element.
    const int rotated = heads + kv_heads;
    const int per_head = half + (dim - rotary_dim);
    const int rot_items = rotated * per_head;
    const int idx = blockIdx.z * blockDim.x + threadIdx.x;
    if (idx < rot_items) {
        const int head = idx / per_head, j = idx - head * per_head;
        const float* src = row + (int64_t)head * dim;
        float* dst = head < heads ? q_heads + ((seq * heads + head) * tokens + t) * dim
                                  : k_cache + cache + ((int64_t)(head - heads) * capacity + pos) * dim;
        if (j < half) {
            const float c = cs[j], sv = sn[j];
            const float a = src[j], b = src[j + half];
            dst[j] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sv));
            dst[j + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, sv));
        } else {
            const int i = rotary_dim + (j - half);
            dst[i] = src[i];
        }
    } else if (idx < rot_items + kv_heads * dim) {
        const int e = idx - rot_items;
        const int kvh = e / dim, i = e - kvh * dim;
        v_cache[cache + ((int64_t)kvh * capacity + pos) * dim + i] = row[(int64_t)rotated * dim + e];
    }
}

// -------------------------------------------------------------- attention
// Both kernels compute, for query t of sequence s and head h (kv head
// kvh = h / (heads / kv_heads)), over keys 0 .. positions[s] + t
// (attention_impl, transformer.cpp:93-145):
//   score_k = (dot(q, k_k) * scale) * scale, the dot summed over d in order;
//   e_k = expf(score_k - max_k score);  den = e_0 + e_1 + ... in key order;
//   out[d] = sum over keys in order of (e_k / den) * v_k[d].
// out[(s*tokens + t)][h*dim + d].
//
// attention_kernel: block (head, t, s), threads over keys for the dots, one
// thread for the denominator, threads over d for the weighted sum; the form
// for one or a few queries per sequence (decode).
// Shared memory: q [dim], then scores [capacity].
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(
    const float* __restrict__ q_heads, const float* __restrict__ k_cache,
    const float* __restrict__ v_cache, int64_t tokens, int heads, int kv_heads, int dim,
    const int32_t* __restrict__ positions, int64_t capacity, float scale, float* __restrict__ out,
    const __grid_constant__ ExpTable tab_g) {
    // The table in shared memory: lanes index it with different k, which the
    // constant bank would serialise.
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __syncthreads();
    extern __shared__ float smem[];
    float* q = smem;
    float* scores = smem + dim;
    __shared__ float scratch[33];
    __shared__ float denominator_s;
    const int head = blockIdx.x;
    const int64_t t = blockIdx.y;
    const int64_t seq = blockIdx.z;
    const int kvh = head / (heads / kv_heads);
    const int64_t start = positions[seq];
    if (start < 0 || start + tokens > capacity) {
        if (threadIdx.x == 0 && t == 0 && head == 0) record_device_error(kSiteCacheRange);
        return;
    }
    const int64_t keys = start + t + 1;
    const float* qrow = q_heads + ((seq * heads + head) * tokens + t) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) q[i] = qrow[i];
    __syncthreads();
    const int64_t cache = seq * kv_heads * capacity * dim;
    const float* kbase = k_cache + cache + (int64_t)kvh * capacity * dim;
    const float* vbase = v_cache + cache + (int64_t)kvh * capacity * dim;
    float local_max = -INFINITY;
    for (int64_t k = threadIdx.x; k < keys; k += blockDim.x) {
        const float* krow = kbase + k * dim;
        float dot = 0.0f;
        for (int d = 0; d < dim; ++d) dot = __fadd_rn(dot, __fmul_rn(q[d], krow[d]));
        const float s = __fmul_rn(__fmul_rn(dot, scale), scale);
        scores[k] = s;
        local_max = fmaxf(local_max, s);
    }
    const float maximum = block_max(local_max, scratch);
    for (int64_t k = threadIdx.x; k < keys; k += blockDim.x)
        scores[k] = expf_libm(__fsub_rn(scores[k], maximum), tab);
    __syncthreads();
    if (threadIdx.x == 0) {
        float den = 0.0f;
        for (int64_t k = 0; k < keys; ++k) den = __fadd_rn(den, scores[k]);
        denominator_s = den;
    }
    __syncthreads();
    const float denominator = denominator_s;
    for (int64_t k = threadIdx.x; k < keys; k += blockDim.x) scores[k] = __fdiv_rn(scores[k], denominator);
    __syncthreads();
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int64_t k = 0; k < keys; ++k) acc = __fadd_rn(acc, __fmul_rn(scores[k], vbase[k * dim + d]));
        out[((seq * tokens + t) * heads + head) * (int64_t)dim + d] = acc;
    }
}

// attention_group_kernel: the decode form.  Block (t, kv head, s) serves
// the query heads that share one kv head (all of them, or half when the
// grid would be small: head_split), so each key and value row
// is staged in shared memory once for all of them (coalesced loads; the next
// chunk is loaded into registers while the current one is used).
//   dots:  thread (h, k) of a chunk of min(64, kGroupThreads / group) keys,
//          its dot over d in order, the query in registers (key rows padded
//          to DIM + 4 floats: conflict-free float4 reads);
//   softmax: exponentials by all threads, one thread per head for the
//          denominator in key order, division by all threads;
//   values: thread (h, d), its sum over keys in order.
// Dynamic shared memory: scores [group][ld], ld = capacity rounded up to 4.
constexpr int kGroupThreads = 256;
constexpr int kGroupMaxHeads = 8;  // query heads per kv head served by this form
constexpr int kGroupRows = 64;     // rows per staged chunk, at most

template <int DIM>
__device__ __forceinline__ void fetch_rows(float4 (&buf)[(kGroupRows * DIM / 4 + kGroupThreads - 1) / kGroupThreads],
                                           const float* __restrict__ base, int n) {
    constexpr int kF4 = (kGroupRows * DIM / 4 + kGroupThreads - 1) / kGroupThreads;
#pragma unroll
    for (int j = 0; j < kF4; ++j) {
        const int i = threadIdx.x + j * kGroupThreads;
        if (i < n * (DIM / 4)) buf[j] = __ldg(reinterpret_cast<const float4*>(base) + i);
    }
}

template <int DIM>
__global__ void __launch_bounds__(kGroupThreads) attention_group_kernel(
    const float* __restrict__ q_heads, const float* __restrict__ k_cache,
    const float* __restrict__ v_cache, int64_t tokens, int heads, int kv_heads,
    const int32_t* __restrict__ positions, int64_t capacity, float scale, float* __restrict__ out,
    int head_split, const __grid_constant__ ExpTable tab_g) {
    // The table in shared memory: lanes index it with different k, which the
    // constant bank would serialise.
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __syncthreads();
    constexpr int kRowF4 = DIM / 4;
    constexpr int kF4 = (kGroupRows * kRowF4 + kGroupThreads - 1) / kGroupThreads;
    extern __shared__ __align__(16) float scores[];
    __shared__ float q_s[kGroupMaxHeads * DIM];
    constexpr int kLd = DIM + 4;  // padded key row: 16-byte aligned, conflict-free float4 reads
    __shared__ __align__(16) float rows_s[kGroupRows * kLd];
    __shared__ float red[kGroupThreads / 32];
    __shared__ float max_s[kGroupMaxHeads], den_s[kGroupMaxHeads];
    // head_split blocks share one kv head, each serving `group` of its
    // query heads (more blocks in flight when sequences x kv heads is small).
    const int group = heads / kv_heads / head_split;
    const int chunk = min(kGroupRows, kGroupThreads / group);  // 32 or 64 keys
    const int64_t t = blockIdx.x / head_split;
    const int kvh = blockIdx.y;
    const int head0 = kvh * group * head_split + static_cast<int>(blockIdx.x % head_split) * group;
    const int64_t seq = blockIdx.z;
    const int64_t start = positions[seq];
    if (start < 0 || start + tokens > capacity) {
        if (threadIdx.x == 0 && t == 0 && kvh == 0) record_device_error(kSiteCacheRange);
        return;
    }
    const int64_t keys = start + t + 1;
    const int64_t ld = (capacity + 3) & ~static_cast<int64_t>(3);
    const int64_t cache = (seq * kv_heads + kvh) * capacity * DIM;
    const float* kbase = k_cache + cache;
    const float* vbase = v_cache + cache;
    const int tid = threadIdx.x;
    if (tid < 2) {
        // The whole key (thread 0) or value (thread 1) range into L2 now, so
        // the chunk loads below wait on L2 rather than on HBM.
        const uint8_t* src = reinterpret_cast<const uint8_t*>(tid == 0 ? kbase : vbase);
        const int64_t bytes = keys * DIM * static_cast<int64_t>(sizeof(float));
        for (int64_t off = 0; off < bytes; off += 32768)
            bulk_prefetch_l2(src + off, static_cast<uint32_t>(min64(32768, bytes - off)));
    }
    for (int i = tid; i < group * DIM; i += kGroupThreads) {
        const int h = i / DIM, d = i % DIM;
        q_s[i] = q_heads[((seq * heads + head0 + h) * tokens + t) * DIM + d];
    }
    // ---- dots
    const int my_h = tid / chunk, my_k = tid % chunk;
    const bool dotter = my_h < group;
    __syncthreads();
    float q[DIM];
#pragma unroll
    for (int d = 0; d < DIM; ++d) q[d] = q_s[(dotter ? my_h : 0) * DIM + d];
    float4 pre[kF4];
    fetch_rows<DIM>(pre, kbase, static_cast<int>(min64(chunk, keys)));
    float local_max = -INFINITY;
    for (int64_t c0 = 0; c0 < keys; c0 += chunk) {
        const int n = static_cast<int>(min64(chunk, keys - c0));
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kF4; ++j) {
            const int i = tid + j * kGroupThreads;
            if (i < n * kRowF4)
                *reinterpret_cast<float4*>(rows_s + (i / kRowF4) * kLd + (i % kRowF4) * 4) = pre[j];
        }
        __syncthreads();
        if (c0 + chunk < keys)
            fetch_rows<DIM>(pre, kbase + (c0 + chunk) * DIM, static_cast<int>(min64(chunk, keys - c0 - chunk)));
        if (dotter && my_k < n) {
            const float* kr = rows_s + my_k * kLd;
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < DIM; d += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
                dot = __fadd_rn(dot, __fmul_rn(q[d], k4.x));
                dot = __fadd_rn(dot, __fmul_rn(q[d + 1], k4.y));
                dot = __fadd_rn(dot, __fmul_rn(q[d + 2], k4.z));
                dot = __fadd_rn(dot, __fmul_rn(q[d + 3], k4.w));
            }
            const float sc = __fmul_rn(__fmul_rn(dot, scale), scale);
            scores[my_h * ld + c0 + my_k] = sc;
            local_max = fmaxf(local_max, sc);
        }
    }
    // ---- per-head maximum (each warp lies within one head: chunk >= 32)
    local_max = warp_max_f32(local_max);
    if ((tid & 31) == 0) red[tid >> 5] = local_max;
    // Start the first value chunk while the softmax runs.
    fetch_rows<DIM>(pre, vbase, static_cast<int>(min64(kGroupRows, keys)));
    __syncthreads();
    if (tid < group) {
        const int warps_per_head = chunk / 32;
        float m = -INFINITY;
        for (int w = 0; w < warps_per_head; ++w) m = fmaxf(m, red[tid * warps_per_head + w]);
        max_s[tid] = m;
    }
    __syncthreads();
    for (int i = tid; i < group * chunk; i += kGroupThreads) {
        const int h = i / chunk;
        const float m = max_s[h];
        for (int64_t k = i % chunk; k < keys; k += chunk)
            scores[h * ld + k] = expf_libm(__fsub_rn(scores[h * ld + k], m), tab);
    }
    __syncthreads();
    if (tid < group) {
        const float* row = scores + tid * ld;
        const int64_t body = keys & ~static_cast<int64_t>(3);
        float den = sum_in_order(row, static_cast<int>(body));
        for (int64_t k = body; k < keys; ++k) den = __fadd_rn(den, row[k]);
        den_s[tid] = den;
    }
    __syncthreads();
    for (int i = tid; i < group * chunk; i += kGroupThreads) {
        const int h = i / chunk;
        const float den = den_s[h];
        for (int64_t k = i % chunk; k < keys; k += chunk) scores[h * ld + k] = __fdiv_rn(scores[h * ld + k], den);
    }
    // ---- probability-weighted values: thread (h, d) for h = h0, h0 + kPass, ...
    constexpr int kPass = kGroupThreads / DIM;  // heads per pass of the block
    constexpr int kAcc = (kGroupMaxHeads + kPass - 1) / kPass;
    const int d = tid % DIM, h0 = tid / DIM;
    float acc[kAcc];
#pragma unroll
    for (int j = 0; j < kAcc; ++j) acc[j] = 0.0f;
    for (int64_t c0 = 0; c0 < keys; c0 += kGroupRows) {
        const int n = static_cast<int>(min64(kGroupRows, keys - c0));
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kF4; ++j) {
            const int i = tid + j * kGroupThreads;
            if (i < n * kRowF4) reinterpret_cast<float4*>(rows_s)[i] = pre[j];
        }
        __syncthreads();
        if (c0 + kGroupRows < keys)
            fetch_rows<DIM>(pre, vbase + (c0 + kGroupRows) * DIM,
                            static_cast<int>(min64(kGroupRows, keys - c0 - kGroupRows)));
        // Four keys per step: each head's four probabilities in one 16-byte
        // load (c0 and k are multiples of 4, ld too), the additions in key order.
        int k = 0;
        for (; k + 4 <= n; k += 4) {
            const float v0 = rows_s[k * DIM + d], v1 = rows_s[(k + 1) * DIM + d];
            const float v2 = rows_s[(k + 2) * DIM + d], v3 = rows_s[(k + 3) * DIM + d];
#pragma unroll
            for (int j = 0; j < kAcc; ++j) {
                const int h = h0 + j * kPass;
                if (h < group) {
                    const float4 p = *reinterpret_cast<const float4*>(scores + h * ld + c0 + k);
                    float a = acc[j];
                    a = __fadd_rn(a, __fmul_rn(p.x, v0));
                    a = __fadd_rn(a, __fmul_rn(p.y, v1));
                    a = __fadd_rn(a, __fmul_rn(p.z, v2));
                    a = __fadd_rn(a, __fmul_rn(p.w, v3));
                    acc[j] = a;
                }
            }
        }
        for (; k < n; ++k) {
            const float v = rows_s[k * DIM + d];
#pragma unroll
            for (int j = 0; j < kAcc; ++j) {
                const int h = h0 + j * kPass;
                if (h < group) acc[j] = __fadd_rn(acc[j], __fmul_rn(scores[h * ld + c0 + k], v));
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kAcc; ++j) {
        const int h = h0 + j * kPass;
        if (h < group) out[((seq * tokens + t) * heads + head0 + h) * (int64_t)DIM + d] = acc[j];
    }
}

// attention_tile_kernel: the form for prompts (many queries per sequence).
// One thread per (query, head) pair: a block takes kTileThreads / group
// consecutive queries of one sequence and the `group` query heads of one kv
// head, so every key and value row staged in shared memory serves all of
// them.  Each thread keeps its query (DIM registers) for the dots and its
// DIM output sums in registers, and runs its own denominator and output
// sums in key order.  Scores, then exponentials, go to a per-block slice of
// the global workspace, [max_keys][kTileThreads] (pair fastest: coalesced).
// Blocks loop over (sequence, kv head, query tile) jobs.
constexpr int kTileThreads = 128;
constexpr int kTileKeys = 32;  // keys per staged chunk

template <int DIM>
__device__ __forceinline__ void stage_rows(float* __restrict__ dst, const float* __restrict__ src,
                                           int rows) {
    // rows x DIM floats, row-contiguous in both; float4 per thread.
    const int n4 = rows * DIM / 4;
    for (int i = threadIdx.x; i < n4; i += kTileThreads)
        reinterpret_cast<float4*>(dst)[i] = __ldg(reinterpret_cast<const float4*>(src) + i);
}

template <int DIM>
__global__ void __launch_bounds__(kTileThreads, 3) attention_tile_kernel(
    const float* __restrict__ q_heads, const float* __restrict__ k_cache,
    const float* __restrict__ v_cache, int sequences, int64_t tokens, int heads, int kv_heads,
    const int32_t* __restrict__ positions, int64_t capacity, int64_t max_keys, float scale,
    float* __restrict__ out, float* __restrict__ workspace, const __grid_constant__ ExpTable tab_g) {
    // The table in shared memory: lanes index it with different k, which the
    // constant bank would serialise.
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __syncthreads();
    __shared__ __align__(16) float rows_s[kTileKeys * DIM];
    const int group = heads / kv_heads;
    const int tq = kTileThreads / group;
    const int pair_query = threadIdx.x / group, pair_head = threadIdx.x % group;
    const int64_t tiles = (tokens + tq - 1) / tq;
    const int64_t jobs = (int64_t)sequences * kv_heads * tiles;
    float* mine = workspace + (int64_t)blockIdx.x * max_keys * kTileThreads + threadIdx.x;
    for (int64_t job = blockIdx.x; job < jobs; job += gridDim.x) {
        const int64_t tile = job % tiles;
        const int kvh = static_cast<int>((job / tiles) % kv_heads);
        const int64_t seq = job / tiles / kv_heads;
        const int64_t start = positions[seq];
        if (start < 0 || start + tokens > capacity || start + tokens > max_keys) {
            if (threadIdx.x == 0) record_device_error(kSiteCacheRange);
            continue;  // uniform across the block
        }
        const int64_t t = tile * tq + pair_query;
        const bool live = t < tokens;
        const int64_t block_keys = start + min64(tile * tq + tq, tokens);
        const int64_t keys = live ? start + t + 1 : 0;
        const int head = kvh * group + pair_head;
        const int64_t cache = (seq * kv_heads + kvh) * capacity * DIM;

        // Pass 1: scores to the workspace, and their maximum.
        float q[DIM];
        {
            const float* qrow = q_heads + ((seq * heads + head) * tokens + (live ? t : 0)) * DIM;
#pragma unroll
            for (int d = 0; d < DIM; d += 4) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(qrow + d));
                q[d] = v.x, q[d + 1] = v.y, q[d + 2] = v.z, q[d + 3] = v.w;
            }
        }
        float maximum = -INFINITY;
        for (int64_t c0 = 0; c0 < block_keys; c0 += kTileKeys) {
            const int n = static_cast<int>(min64(kTileKeys, block_keys - c0));
            __syncthreads();
            stage_rows<DIM>(rows_s, k_cache + cache + c0 * DIM, n);
            __syncthreads();
            for (int kk = 0; kk < n; kk += 4) {
                float dot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int d = 0; d < DIM; d += 4) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // Rows past n hold stale values; their dots are dropped below.
                        const float4 k = *reinterpret_cast<const float4*>(rows_s + (kk + j) * DIM + d);
                        dot[j] = __fadd_rn(dot[j], __fmul_rn(q[d], k.x));
                        dot[j] = __fadd_rn(dot[j], __fmul_rn(q[d + 1], k.y));
                        dot[j] = __fadd_rn(dot[j], __fmul_rn(q[d + 2], k.z));
                        dot[j] = __fadd_rn(dot[j], __fmul_rn(q[d + 3], k.w));
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int64_t key = c0 + kk + j;
                    if (key < keys) {
                        const float s = __fmul_rn(__fmul_rn(dot[j], scale), scale);
                        mine[key * kTileThreads] = s;
                        maximum = fmaxf(maximum, s);
                    }
                }
            }
        }
        // Pass 2: exponentials and the denominator, in key order; the scores
        // of the next 16 keys are loaded while the current 16 are used.
        float den = 0.0f;
        {
            constexpr int kB = 16;
            float cur[kB], nxt[kB];
#pragma unroll
            for (int j = 0; j < kB; ++j) cur[j] = j < keys ? mine[j * kTileThreads] : 0.0f;
            for (int64_t k0 = 0; k0 < keys; k0 += kB) {
#pragma unroll
                for (int j = 0; j < kB; ++j) nxt[j] = k0 + kB + j < keys ? mine[(k0 + kB + j) * kTileThreads] : 0.0f;
#pragma unroll
                for (int j = 0; j < kB; ++j) {
                    if (k0 + j < keys) {
                        const float e = expf_libm(__fsub_rn(cur[j], maximum), tab);
                        den = __fadd_rn(den, e);
                        mine[(k0 + j) * kTileThreads] = e;
                    }
                }
#pragma unroll
                for (int j = 0; j < kB; ++j) cur[j] = nxt[j];
            }
        }
        // Pass 3: probability-weighted values, each output element in key order.
        float acc[DIM];
#pragma unroll
        for (int d = 0; d < DIM; ++d) acc[d] = 0.0f;
        for (int64_t c0 = 0; c0 < block_keys; c0 += kTileKeys) {
            const int n = static_cast<int>(min64(kTileKeys, block_keys - c0));
            __syncthreads();
            stage_rows<DIM>(rows_s, v_cache + cache + c0 * DIM, n);
            __syncthreads();
            const int mine_n = static_cast<int>(max64(0, min64(n, keys - c0)));
            float e_next = mine_n > 0 ? mine[c0 * kTileThreads] : 0.0f;
            for (int kk = 0; kk < mine_n; ++kk) {
                const float e = e_next;
                if (kk + 1 < mine_n) e_next = mine[(c0 + kk + 1) * kTileThreads];
                const float p = __fdiv_rn(e, den);
#pragma unroll
                for (int d = 0; d < DIM; d += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(rows_s + kk * DIM + d);
                    acc[d] = __fadd_rn(acc[d], __fmul_rn(p, v.x));
                    acc[d + 1] = __fadd_rn(acc[d + 1], __fmul_rn(p, v.y));
                    acc[d + 2] = __fadd_rn(acc[d + 2], __fmul_rn(p, v.z));
                    acc[d + 3] = __fadd_rn(acc[d + 3], __fmul_rn(p, v.w));
                }
            }
        }
        if (live) {
            float* orow = out + ((seq * tokens + t) * heads + head) * (int64_t)DIM;
#pragma unroll
            for (int d = 0; d < DIM; d += 4)
                *reinterpret_cast<float4*>(orow + d) = make_float4(acc[d], acc[d + 1], acc[d + 2], acc[d + 3]);
        }
    }
}

// -------------------------------------------------------------- silu gate
// gate_up[t] = [g0, u0, g1, u1, ...] (gate and up rows interleaved);
// out[t][j] = u_j * (g_j / (1 + expf(-g_j))).
__device__ __forceinline__ float silu_gate_one(float g, float u, const ExpTable& tab) {
    return __fmul_rn(u, __fdiv_rn(g, __fadd_rn(1.0f, expf_libm(-g, tab))));
}

// Outputs are consecutive in memory (out [tokens][width] row-major and
// gate_up its interleaved pairs), so the flat index i covers every token.
__global__ void silu_gate_kernel(const float* __restrict__ gate_up, int64_t tokens, int64_t width,
                                 float* __restrict__ out, int vec, const __grid_constant__ ExpTable tab_g) {
    // The table in shared memory: lanes index it with different k, which the
    // constant bank would serialise.
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __syncthreads();
    const int64_t n = tokens * width;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        // Four outputs per thread and step: two float4 loads, one float4 store.
        const float4* gu4 = reinterpret_cast<const float4*>(gate_up);
        float4* o4 = reinterpret_cast<float4*>(out);
        for (int64_t i = first; i < n / 4; i += stride) {
            const float4 a = __ldg(gu4 + 2 * i), b = __ldg(gu4 + 2 * i + 1);
            o4[i] = make_float4(silu_gate_one(a.x, a.y, tab), silu_gate_one(a.z, a.w, tab),
                                silu_gate_one(b.x, b.y, tab), silu_gate_one(b.z, b.w, tab));
        }
        return;
    }
    for (int64_t i = first; i < n; i += stride) {
        const float2 gu = reinterpret_cast<const float2*>(gate_up)[i];
        out[i] = silu_gate_one(gu.x, gu.y, tab);
    }
}

// The SiLU gate with the per-token INT8 quantisation of the down
// projection's input fused in: block t computes row t's activations (kept in
// registers, up to kSiluQuantPer per thread), their absmax, and the codes and
// scale leafq_quantize_act would produce from them.  act (may be NULL) also
// receives the fp32 activations.
constexpr int kSiluQuantThreads = 512;
constexpr int kSiluQuantPer = 12;  // width <= 512 * 12 = 6144

__global__ void __launch_bounds__(kSiluQuantThreads) silu_gate_quantize_kernel(
    const float* __restrict__ gate_up, int64_t width, float* __restrict__ act, int8_t* __restrict__ codes,
    float* __restrict__ code_scales, const __grid_constant__ ExpTable tab_g) {
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __shared__ float scratch[33];
    __syncthreads();
    const int64_t t = blockIdx.x;
    const float2* gu = reinterpret_cast<const float2*>(gate_up) + t * width;
    float v[kSiluQuantPer];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < kSiluQuantPer; ++j) {
        const int64_t c = threadIdx.x + (int64_t)j * kSiluQuantThreads;
        if (c < width) {
            const float2 p = __ldg(gu + c);
            v[j] = silu_gate_one(p.x, p.y, tab);
            if (act) act[t * width + c] = v[j];
            m = fmaxf(m, fabsf(v[j]));
        }
    }
    const float absmax = block_max(m, scratch);
    const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
    const float multiplier = __fdiv_rn(1.0f, scale);
    if (threadIdx.x == 0) code_scales[t] = scale;
#pragma unroll
    for (int j = 0; j < kSiluQuantPer; ++j) {
        const int64_t c = threadIdx.x + (int64_t)j * kSiluQuantThreads;
        if (c < width) codes[t * width + c] = act_code(v[j], multiplier);
    }
}

// Fewer tokens than SMs: a cluster of kSiluCtas CTAs per token, each taking
// a contiguous quarter of the row; the row's absmax is the maximum of the
// four CTA maxima, read through distributed shared memory between two
// cluster barriers (the second keeps every CTA resident until the others
// have read its maximum).  Values, scale and codes are those of
// silu_gate_quantize_kernel (the maximum is order-free).
constexpr int kSiluCtas = 4;
constexpr int kSiluCtaThreads = 256;
constexpr int kSiluCtaPer = (kSiluQuantThreads * kSiluQuantPer) / (kSiluCtas * kSiluCtaThreads);  // 6

__global__ void __cluster_dims__(kSiluCtas, 1, 1) __launch_bounds__(kSiluCtaThreads)
    silu_gate_quantize_cluster_kernel(const float* __restrict__ gate_up, int64_t width, float* __restrict__ act,
                                      int8_t* __restrict__ codes, float* __restrict__ code_scales,
                                      const __grid_constant__ ExpTable tab_g) {
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __shared__ float scratch[33];
    __syncthreads();
    const int64_t t = blockIdx.x / kSiluCtas;
    const uint32_t part = cluster_ctarank();
    const int64_t c0 = width * part / kSiluCtas, c1 = width * (part + 1) / kSiluCtas;
    const float2* gu = reinterpret_cast<const float2*>(gate_up) + t * width;
    float v[kSiluCtaPer];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < kSiluCtaPer; ++j) {
        const int64_t c = c0 + threadIdx.x + (int64_t)j * kSiluCtaThreads;
        if (c < c1) {
            const float2 p = __ldg(gu + c);
            v[j] = silu_gate_one(p.x, p.y, tab);
            if (act) act[t * width + c] = v[j];
            m = fmaxf(m, fabsf(v[j]));
        }
    }
    block_max(m, scratch);  // this CTA's maximum in scratch[32]
    cluster_sync_all();
    float absmax = 0.0f;
#pragma unroll
    for (int r = 0; r < kSiluCtas; ++r)
        absmax = fmaxf(absmax, ld_shared_cluster_f32(mapa_shared(smem_u32(&scratch[32]), r)));
    cluster_sync_all();
    const float scale = fmaxf(__fdiv_rn(absmax, 127.0f), 1e-12f);
    const float multiplier = __fdiv_rn(1.0f, scale);
    if (part == 0 && threadIdx.x == 0) code_scales[t] = scale;
#pragma unroll
    for (int j = 0; j < kSiluCtaPer; ++j) {
        const int64_t c = c0 + threadIdx.x + (int64_t)j * kSiluCtaThreads;
        if (c < c1) codes[t * width + c] = act_code(v[j], multiplier);
    }
}

// ----------------------------------------------------------------- argmax
__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* __restrict__ logits,
                                                                 int64_t width,
                                                                 int32_t* __restrict__ ids) {
    __shared__ float best_v[kArgmaxThreads / 32];
    __shared__ int best_i[kArgmaxThreads / 32];
    const float* row = logits + (int64_t)blockIdx.x * width;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int64_t c = threadIdx.x; c < width; c += blockDim.x) {
        const float x = row[c];
        if (x > v || idx == 0x7fffffff) {
            v = x;
            idx = static_cast<int>(c);
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
            v = ov;
            idx = oi;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        best_v[warp] = v;
        best_i[warp] = idx;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bv = best_v[0];
        int bi = best_i[0];
        for (int w = 1; w < kArgmaxThreads / 32; ++w)
            if (best_v[w] > bv || (best_v[w] == bv && best_i[w] < bi)) {
                bv = best_v[w];
                bi = best_i[w];
            }
        ids[blockIdx.x] = bi;
    }
}

__global__ void advance_kernel(int32_t* positions, int sequences, int32_t count) {
    for (int i = threadIdx.x; i < sequences; i += blockDim.x) positions[i] += count;
}

__global__ void expf_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ y,
                            const __grid_constant__ ExpTable tab_g) {
    // The table in shared memory: lanes index it with different k, which the
    // constant bank would serialise.
    __shared__ ExpTable tab;
    if (threadIdx.x < 32) tab.bits[threadIdx.x] = tab_g.bits[threadIdx.x];
    __syncthreads();
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        y[i] = expf_libm(x[i], tab);
}

}  // namespace
}  // namespace leafq

using namespace leafq;

extern "C" {

int leafq_embed(void* stream, const int32_t* ids, int64_t tokens, const void* table,
                const float* scales, int bits, int64_t group, int64_t vocab, int64_t hidden,
                float embedding_scale, float* out, int32_t* error_flag) {
    clear_error();
    if (tokens < 0 || vocab <= 0 || hidden <= 0 || (bits != 32 && bits != 8 && bits != 4) ||
        (bits != 32 && (group <= 0 || hidden % group != 0 || !scales)) ||
        (bits == 4 && hidden % 2 != 0)) {
        set_error("leafq_embed: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0) return LEAFQ_OK;
    if (!ids || !table || !out || tokens > 0x7fffffff) {
        set_error("leafq_embed: null pointer or too many tokens");
        return LEAFQ_ERR_INVALID;
    }
    return launch(embed_kernel, dim3(static_cast<unsigned>(tokens)), dim3(256), 0,
                  static_cast<cudaStream_t>(stream), false, "embed", ids, table, scales, bits, group,
                  vocab, hidden, embedding_scale, out, error_flag);
}

int leafq_rmsnorm_quantize(void* stream, float* hidden, const float* delta, int add_zero, int64_t tokens,
                           int64_t width, const float* weight, float epsilon, float* out, int8_t* codes,
                           float* code_scales) {
    clear_error();
    if (tokens < 0 || width <= 0 || width > 16384 || tokens > 0x7fffffff) {
        set_error("leafq_rmsnorm: width must be 1..16384");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0) return LEAFQ_OK;
    if (!hidden || !weight || (!out && !codes) || (codes && !code_scales)) {
        set_error("leafq_rmsnorm: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool vec = width % 4 == 0 && width <= 4 * kNormVec * kNormVecThreads && aligned16(hidden) &&
                     (!delta || aligned16(delta)) && aligned16(weight) && (!out || aligned16(out)) &&
                     (!codes || reinterpret_cast<uintptr_t>(codes) % 4 == 0);
    const size_t smem = static_cast<size_t>(width) * sizeof(float);
    if (vec) {
        int st = allow_smem(reinterpret_cast<const void*>(rmsnorm_vec_kernel), smem, "rmsnorm");
        if (st) return st;
        return launch(rmsnorm_vec_kernel, dim3(static_cast<unsigned>(tokens)), dim3(kNormVecThreads), smem, s, false,
                      "rmsnorm", hidden, delta, add_zero, width, weight, epsilon, out, codes, code_scales);
    }
    if (codes) {
        set_error("leafq_rmsnorm_quantize: codes need width % 4 == 0, width <= 4096 and aligned rows");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    int st = allow_smem(reinterpret_cast<const void*>(rmsnorm_kernel), 2 * smem, "rmsnorm");
    if (st) return st;
    return launch(rmsnorm_kernel, dim3(static_cast<unsigned>(tokens)), dim3(kNormThreads), 2 * smem, s, false,
                  "rmsnorm", hidden, delta, add_zero, width, weight, epsilon, out);
}

int leafq_rmsnorm(void* stream, float* hidden, const float* delta, int add_zero, int64_t tokens,
                  int64_t width, const float* weight, float epsilon, float* out) {
    if (!out) {
        clear_error();
        set_error("leafq_rmsnorm: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    return leafq_rmsnorm_quantize(stream, hidden, delta, add_zero, tokens, width, weight, epsilon, out, nullptr,
                                  nullptr);
}

int leafq_rope_tables(float theta, int rotary_dim, int64_t positions, float* cos_out,
                      float* sin_out) {
    clear_error();
    if (!(theta > 0.0f) || rotary_dim <= 0 || rotary_dim % 2 || positions < 0 || !cos_out || !sin_out) {
        set_error("leafq_rope_tables: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    // decoder.cpp:929-933 and :1248-1256, with the same float libm calls.
    const int half = rotary_dim / 2;
    for (int i = 0; i < half; ++i) {
        const float frequency =
            1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(rotary_dim));
        for (int64_t p = 0; p < positions; ++p) {
            const float angle = static_cast<float>(p) * frequency;
            cos_out[p * half + i] = std::cos(angle);
            sin_out[p * half + i] = std::sin(angle);
        }
    }
    return LEAFQ_OK;
}

int leafq_rotary_append_batch(void* stream, const float* qkv, int sequences, int64_t tokens, int heads,
                              int kv_heads, int dim, int rotary_dim, const float* cos_table,
                              const float* sin_table, const int32_t* positions, float* q_heads,
                              float* k_cache, float* v_cache, int64_t capacity) {
    clear_error();
    if (sequences < 0 || sequences > 65535 || tokens < 0 || heads <= 0 || kv_heads <= 0 ||
        heads % kv_heads || dim <= 0 || rotary_dim < 0 || rotary_dim > dim || rotary_dim % 2 ||
        capacity <= 0 || tokens > 65535) {
        set_error("leafq_rotary_append: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0 || sequences == 0) return LEAFQ_OK;
    if (!qkv || !positions || !q_heads || !k_cache || !v_cache || (rotary_dim && (!cos_table || !sin_table))) {
        set_error("leafq_rotary_append: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    const int items = (heads + kv_heads) * (rotary_dim / 2 + dim - rotary_dim) + kv_heads * dim;
    return launch(rotary_append_kernel,
                  dim3(static_cast<unsigned>(tokens), static_cast<unsigned>(sequences), (items + 255) / 256),
                  dim3(256), 0, static_cast<cudaStream_t>(stream), false, "rotary_append", qkv,
                  tokens, heads, kv_heads, dim, rotary_dim, cos_table, sin_table, positions, q_heads,
                  k_cache, v_cache, capacity);
}

int leafq_rotary_append(void* stream, const float* qkv, int64_t tokens, int heads, int kv_heads,
                        int dim, int rotary_dim, const float* cos_table, const float* sin_table,
                        const int32_t* position, float* q_heads, float* k_cache, float* v_cache,
                        int64_t capacity) {
    return leafq_rotary_append_batch(stream, qkv, 1, tokens, heads, kv_heads, dim, rotary_dim, cos_table,
                                     sin_table, position, q_heads, k_cache, v_cache, capacity);
}

namespace {
// The tile form serves prompts: enough queries per sequence to fill a
// block's pairs, a head size it is compiled for, and 16-byte rows.
bool attention_tile_form(int64_t tokens, int heads, int kv_heads, int dim) {
    const int group = heads / kv_heads;
    return (dim == 32 || dim == 64) && kTileThreads % group == 0 && tokens >= 16;
}

int64_t attention_tile_grid(int sequences, int64_t tokens, int heads, int kv_heads) {
    const int tq = kTileThreads / (heads / kv_heads);
    const int64_t jobs = (int64_t)sequences * kv_heads * ((tokens + tq - 1) / tq);
    return std::min<int64_t>(jobs, static_cast<int64_t>(sm_count()) * 3);
}
}  // namespace

int64_t leafq_attention_workspace_bytes(int sequences, int64_t tokens, int heads, int kv_heads, int dim,
                                        int64_t max_keys) {
    if (sequences <= 0 || tokens <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || max_keys <= 0)
        return 0;
    if (!attention_tile_form(tokens, heads, kv_heads, dim)) return 0;
    return attention_tile_grid(sequences, tokens, heads, kv_heads) * max_keys * kTileThreads *
           static_cast<int64_t>(sizeof(float));
}

int leafq_attention_batch(void* stream, const float* q_heads, const float* k_cache, const float* v_cache,
                          int sequences, int64_t tokens, int heads, int kv_heads, int dim,
                          const int32_t* positions, int64_t capacity, int64_t max_keys, float scale,
                          float* out, void* workspace, int64_t workspace_bytes) {
    clear_error();
    if (sequences < 0 || sequences > 65535 || tokens < 0 || heads <= 0 || kv_heads <= 0 ||
        heads % kv_heads || dim <= 0 || dim > 1024 || capacity <= 0 || tokens > 65535 ||
        !(scale > 0.0f) || max_keys < tokens || max_keys > capacity) {
        set_error("leafq_attention: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0 || sequences == 0) return LEAFQ_OK;
    if (!q_heads || !k_cache || !v_cache || !positions || !out) {
        set_error("leafq_attention: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t need = leafq_attention_workspace_bytes(sequences, tokens, heads, kv_heads, dim, max_keys);
    if (need > 0 && aligned16(q_heads) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out)) {
        if (!workspace || workspace_bytes < need || !aligned16(workspace)) {
            set_error("leafq_attention: workspace smaller than leafq_attention_workspace_bytes");
            return LEAFQ_ERR_INVALID;
        }
        const int grid = static_cast<int>(attention_tile_grid(sequences, tokens, heads, kv_heads));
        float* ws = static_cast<float*>(workspace);
        if (dim == 32)
            return launch(attention_tile_kernel<32>, dim3(grid), dim3(kTileThreads), 0, s, false, "attention",
                          q_heads, k_cache, v_cache, sequences, tokens, heads, kv_heads, positions, capacity,
                          max_keys, scale, out, ws, exp_table());
        return launch(attention_tile_kernel<64>, dim3(grid), dim3(kTileThreads), 0, s, false, "attention",
                      q_heads, k_cache, v_cache, sequences, tokens, heads, kv_heads, positions, capacity,
                      max_keys, scale, out, ws, exp_table());
    }
    const int group = heads / kv_heads;
    const int64_t ld = (capacity + 3) & ~static_cast<int64_t>(3);
    const size_t group_smem = static_cast<size_t>(group) * ld * sizeof(float);
    if ((dim == 32 || dim == 64) && group <= kGroupMaxHeads && aligned16(k_cache) && aligned16(v_cache) &&
        group_smem + 24 * 1024 <= static_cast<size_t>(max_smem_per_block())) {
        // Two blocks per kv head (each with half of its query heads) when one
        // per kv head would leave most SMs idle (measured: a gain for 8
        // sequences, a loss for 64).
        const int head_split =
            (group % 2 == 0 && 2 * tokens * kv_heads * sequences <= static_cast<int64_t>(sm_count())) ? 2 : 1;
        const dim3 grid(static_cast<unsigned>(tokens * head_split), kv_heads, static_cast<unsigned>(sequences));
        if (dim == 32) {
            int st = allow_smem(reinterpret_cast<const void*>(attention_group_kernel<32>), group_smem, "attention");
            if (st) return st;
            return launch(attention_group_kernel<32>, grid, dim3(kGroupThreads), group_smem, s, false,
                          "attention", q_heads, k_cache, v_cache, tokens, heads, kv_heads, positions, capacity,
                          scale, out, head_split, exp_table());
        }
        int st = allow_smem(reinterpret_cast<const void*>(attention_group_kernel<64>), group_smem, "attention");
        if (st) return st;
        return launch(attention_group_kernel<64>, grid, dim3(kGroupThreads), group_smem, s, false, "attention",
                      q_heads, k_cache, v_cache, tokens, heads, kv_heads, positions, capacity, scale, out,
                      head_split, exp_table());
    }
    const size_t smem = (static_cast<size_t>(dim) + capacity) * sizeof(float);
    if (smem > static_cast<size_t>(max_smem_per_block())) {
        set_error("leafq_attention: context capacity exceeds shared memory");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    int st = allow_smem(reinterpret_cast<const void*>(attention_kernel), smem, "attention");
    if (st) return st;
    return launch(attention_kernel,
                  dim3(heads, static_cast<unsigned>(tokens), static_cast<unsigned>(sequences)),
                  dim3(kAttnThreads), smem, s, false, "attention", q_heads, k_cache, v_cache, tokens, heads,
                  kv_heads, dim, positions, capacity, scale, out, exp_table());
}

int leafq_attention(void* stream, const float* q_heads, const float* k_cache, const float* v_cache,
                    int64_t tokens, int heads, int kv_heads, int dim, const int32_t* position,
                    int64_t capacity, float scale, float* out) {
    // Without a workspace: the per-query form.
    clear_error();
    if (tokens < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || dim <= 0 || dim > 1024 ||
        capacity <= 0 || tokens > 65535 || !(scale > 0.0f)) {
        set_error("leafq_attention: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0) return LEAFQ_OK;
    if (!q_heads || !k_cache || !v_cache || !position || !out) {
        set_error("leafq_attention: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    const size_t smem = (static_cast<size_t>(dim) + capacity) * sizeof(float);
    if (smem > static_cast<size_t>(max_smem_per_block())) {
        set_error("leafq_attention: context capacity exceeds shared memory");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    int st = allow_smem(reinterpret_cast<const void*>(attention_kernel), smem, "attention");
    if (st) return st;
    return launch(attention_kernel, dim3(heads, static_cast<unsigned>(tokens), 1), dim3(kAttnThreads), smem,
                  static_cast<cudaStream_t>(stream), false, "attention", q_heads, k_cache, v_cache, tokens,
                  heads, kv_heads, dim, position, capacity, scale, out, exp_table());
}

int leafq_silu_gate(void* stream, const float* gate_up, int64_t tokens, int64_t width, float* out) {
    clear_error();
    if (tokens < 0 || width <= 0) {
        set_error("leafq_silu_gate: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0) return LEAFQ_OK;
    if (!gate_up || !out) {
        set_error("leafq_silu_gate: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    const int64_t n = tokens * width;
    const int vec = (n % 4 == 0) && aligned16(gate_up) && aligned16(out);
    const int64_t items = vec ? n / 4 : n;
    const int64_t blocks = std::min<int64_t>((items + 255) / 256, static_cast<int64_t>(sm_count()) * 8);
    return launch(silu_gate_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                  static_cast<cudaStream_t>(stream), false, "silu_gate", gate_up, tokens, width, out, vec,
                  exp_table());
}

int leafq_silu_gate_quantize(void* stream, const float* gate_up, int64_t tokens, int64_t width, float* act,
                             int8_t* codes, float* code_scales) {
    clear_error();
    if (tokens < 0 || tokens > 0x7fffffff || width <= 0 || width > kSiluQuantThreads * kSiluQuantPer) {
        set_error("leafq_silu_gate_quantize: width must be 1..6144");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0) return LEAFQ_OK;
    if (!gate_up || !codes || !code_scales) {
        set_error("leafq_silu_gate_quantize: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens < sm_count())
        return launch(silu_gate_quantize_cluster_kernel, dim3(static_cast<unsigned>(tokens * kSiluCtas)),
                      dim3(kSiluCtaThreads), 0, static_cast<cudaStream_t>(stream), false, "silu_gate", gate_up,
                      width, act, codes, code_scales, exp_table());
    return launch(silu_gate_quantize_kernel, dim3(static_cast<unsigned>(tokens)), dim3(kSiluQuantThreads), 0,
                  static_cast<cudaStream_t>(stream), false, "silu_gate", gate_up, width, act, codes, code_scales,
                  exp_table());
}

int leafq_argmax(void* stream, const float* logits, int64_t rows, int64_t width, int32_t* ids) {
    clear_error();
    if (rows < 0 || width <= 0 || width > 0x7fffffff || rows > 0x7fffffff) {
        set_error("leafq_argmax: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (rows == 0) return LEAFQ_OK;
    if (!logits || !ids) {
        set_error("leafq_argmax: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    return launch(argmax_kernel, dim3(static_cast<unsigned>(rows)), dim3(kArgmaxThreads), 0,
                  static_cast<cudaStream_t>(stream), false, "argmax", logits, width, ids);
}

int leafq_expf(void* stream, const float* x, int64_t n, float* y) {
    clear_error();
    if (n < 0 || (n > 0 && (!x || !y))) {
        set_error("leafq_expf: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (n == 0) return LEAFQ_OK;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, static_cast<int64_t>(sm_count()) * 16);
    return launch(expf_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                  static_cast<cudaStream_t>(stream), false, "expf", x, n, y, exp_table());
}

int leafq_advance_positions(void* stream, int32_t* positions, int sequences, int32_t count) {
    clear_error();
    if (!positions || count < 0 || sequences < 0) {
        set_error("leafq_advance_position: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (sequences == 0) return LEAFQ_OK;
    return launch(advance_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), false,
                  "advance_position", positions, sequences, count);
}

int leafq_advance_position(void* stream, int32_t* position, int32_t count) {
    return leafq_advance_positions(stream, position, 1, count);
}

}  // extern "C"
