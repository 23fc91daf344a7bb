// Graph executor INT8 GEMM with per-output-channel weight scales,
// leaf::kernels::gemm_i8_per_channel (kernels/gemm.cpp:99-166): a [m, k]
// int8, b [k, n] int8 (n contiguous, the ONNX MatMul layout), out [m, n].
//
// Shapes whose row strides are multiples of 16 bytes run on the tensor
// cores (graph_gemm_tc_kernel below).  The others take the CUDA-core
// kernel: 64x64 output tile per 256-thread block, 64-byte K steps staged in shared
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
    int activation;   // 0 none, 1 Relu, 2 Silu, 3 Gelu (tanh form)
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
    if (g.activation == 3) value = gelu_tanh_libm(value);
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

// ------------------------------------------------------------------------
// The same GEMM on the tensor cores: tcgen05.mma kind::i8 with int32
// accumulators in tensor memory, operands staged by TMA with 128-byte
// swizzle.  A (codes [m, k]) is K-major.  B is the weight as the graph
// stores it: [k, n] with n contiguous (ONNX MatMul / Gemm without transB),
// which the MMA reads MN-major -- each stage holds BN / 128 boxes of
// [128 rows of k, 128 columns of n] -- or [n, k] (transB), read K-major.
// Tile D[128 rows of a, BN columns], BN 256 or 128; warp roles as the
// prefill GEMM (warp 0 TMA, warp 1 TMEM + MMA issue, warps 2-9 epilogue --
// two per TMEM sub-partition on alternating 32-column blocks -- persistent
// over tiles, two accumulators).  The int32 sums are exact, and the epilogue
// is the reference's, element by element; its outputs leave through 32 x 32
// shared-memory blocks and TMA stores when the output rows are 16-byte
// aligned.
constexpr int GBM = 128, GBK = 128, GUMMA_K = 32;
constexpr int GEpiWarps = 8;
constexpr int GThreads = (2 + GEpiWarps) * 32;
constexpr int GEpiBar = 1;  // named barrier of the epilogue warps

template <int BN>
struct GraphTc {
    static constexpr int kABytes = GBM * GBK;
    static constexpr int kBBytes = BN * GBK;
    static constexpr int kTmemCols = 2 * BN;
    // The tile's [scale | bias][BN], rounded to 1 KB (the output blocks behind
    // it stay 1024-byte aligned for the 128-byte swizzle).
    static constexpr size_t kColBytes = (2 * BN * sizeof(float) + 1023) / 1024 * 1024;
    static constexpr size_t kYBytes = (size_t)GEpiWarps * 32 * 32 * sizeof(float);
    static constexpr size_t kFixed = 1024 + kColBytes + kYBytes + 1024;
    static constexpr int kPrefStages = BN == 256 ? 4 : 6;
    static constexpr int kFitStages = static_cast<int>((227 * 1024 - kFixed) / (kABytes + kBBytes));
    static constexpr int kStages = kPrefStages < kFitStages ? kPrefStages : kFitStages;
    static constexpr size_t kSmemBytes = (size_t)kStages * (kABytes + kBBytes) + kFixed;
};

struct GraphTcArgs {
    const float* ws;
    const float* bias;
    float* out;
    float input_scale;
    int relu;
    int64_t m, n, k;
    int m_tiles, n_tiles;
    int tma_store;  // n % 4 == 0 and a 16-byte aligned output: stores through map_y
    GraphGlue glue;
};

template <int BN, bool kMnB>
__global__ void __launch_bounds__(GThreads, 1)
graph_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_y, const GraphTcArgs g,
                     const __grid_constant__ ExpTable tab_g) {
    using Cfg = GraphTc<BN>;
    constexpr int kStages = Cfg::kStages;
    constexpr int kABytes = Cfg::kABytes;
    constexpr int kBBytes = Cfg::kBBytes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + (size_t)kStages * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(b_tiles + (size_t)kStages * kBBytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
    ExpTable* tab = reinterpret_cast<ExpTable*>(tmem_holder + 2);
    float* col_s = reinterpret_cast<float*>(b_tiles + (size_t)kStages * kBBytes + 1024);
    float* y_stage = col_s + Cfg::kColBytes / sizeof(float);  // [8 warps][32 x 32], 1024-byte aligned

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = static_cast<int>((g.k + GBK - 1) / GBK);
    const int tiles = g.m_tiles * g.n_tiles;
    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], GEpiWarps);
        }
        fence_barrier_init();
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
    }
    if (warp == 2) tab->bits[lane] = tab_g.bits[lane];
    if (warp == 1) {
        tmem_alloc(tmem_holder, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tcgen05_fence_before();
    __syncthreads();
    tcgen05_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    grid_dependency_wait();  // the codes come from the previous kernel

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one_sync()) {
            const uint64_t keep = l2_policy_evict_last();
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile % g.m_tiles) * GBM;
                const int n0 = (tile / g.m_tiles) * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, kSiteGemmEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
                    tma_load_2d(a_tiles + (size_t)s * kABytes, &map_a, kb * GBK, m0, &full[s], keep);
                    uint8_t* bt = b_tiles + (size_t)s * kBBytes;
                    if (kMnB) {
#pragma unroll
                        for (int j = 0; j < BN / 128; ++j)
                            tma_load_2d(bt + j * 128 * GBK, &map_b, n0 + 128 * j, kb * GBK, &full[s], keep);
                    } else {
                        tma_load_2d(bt, &map_b, kb * GBK, n0, &full[s], keep);
                    }
                }
            }
            for (int back = 0; back < kStages && back < it; ++back) {
                const int i = it - 1 - back;
                mbar_wait(&full[i % kStages], (i / kStages) & 1, kSiteGemmFull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one_sync()) {
            const uint32_t idesc = kMnB ? umma_idesc_i8_bmn(GBM, BN) : umma_idesc_i8(GBM, BN);
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                if (local >= 2 && !mbar_wait(&acc_empty[acc], ((local >> 1) - 1) & 1, kSiteGemmAccEmpty)) break;
                tcgen05_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&full[s], (it / kStages) & 1, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tcgen05_fence_after();
                    const uint64_t adesc = umma_desc_k_sw128(smem_u32(a_tiles + (size_t)s * kABytes));
                    const uint32_t b_addr = smem_u32(b_tiles + (size_t)s * kBBytes);
#pragma unroll
                    for (int k = 0; k < GBK / GUMMA_K; ++k) {
                        // K-major A: the next 32 bytes of each row.  B: MN-major,
                        // the next 32 rows of k (32 x 128 bytes), or K-major as A.
                        const uint64_t bdesc = kMnB ? umma_desc_mn_sw128(b_addr + k * GUMMA_K * 128, 128 * GBK)
                                                    : umma_desc_k_sw128(b_addr) + 2 * k;
                        umma_i8(d_tmem, adesc + 2 * k, bdesc, idesc, (kb | k) != 0);
                    }
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[acc]);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2-9)
        const int ew = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = rows of a
        const int part = ew >> 2;      // 32-column blocks part, part + 2, ...
        int local = 0;
        bool ok = true;  // a failed wait leaves the warps on the same barrier sequence
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const int64_t m0 = (int64_t)(tile % g.m_tiles) * GBM;
            const int64_t n0 = (int64_t)(tile / g.m_tiles) * BN;
            float* ws_s = col_s;
            float* bias_s = ws_s + BN;
            bar_sync(GEpiBar, GEpiWarps * 32);  // every epilogue warp is done with the previous tile
            for (int i = ew * 32 + lane; i < BN; i += GEpiWarps * 32) {
                const int64_t n = n0 + i < g.n ? n0 + i : g.n - 1;
                ws_s[i] = __ldg(g.ws + n);
                bias_s[i] = g.bias ? __ldg(g.bias + n) : 0.0f;
            }
            bar_sync(GEpiBar, GEpiWarps * 32);
            if (ok && !mbar_wait(&acc_full[acc], (local >> 1) & 1, kSiteGemmAccFull)) ok = false;
            tcgen05_fence_after();
            const int64_t mb = m0 + quarter * 32;
            const int64_t row = mb + lane;
            const bool live = row < g.m;
            float* out = g.out + row * g.n;
            for (int c = part * 32; c < BN; c += 64) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + acc * BN + c + ((uint32_t)(quarter * 32) << 16), r);
                tmem_wait_ld();
                const int64_t nb = n0 + c;
                if (!g.tma_store && (!live || nb >= g.n)) continue;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    // (float(acc) * input_scale) * weight_scales[col] (+ bias), gemm.cpp:150-160.
                    float value = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), g.input_scale),
                                            ws_s[c + j]);
                    if (g.bias) value = __fadd_rn(value, bias_s[c + j]);
                    if (g.relu) value = value < 0.0f ? 0.0f : value;
                    if (g.glue.on && live && nb + j < g.n) value = graph_glue(value, g.glue, row, nb + j, g.n, *tab);
                    v[j] = value;
                }
                if (g.tma_store) {
                    // Rows past m and columns past n are not written by the store.
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    store_block_32x32(y_stage + ew * 1024, v, lane, &map_y, static_cast<int32_t>(nb),
                                      static_cast<int32_t>(mb), nb < g.n && mb < g.m, true);
                } else if (nb + 32 <= g.n && ((reinterpret_cast<uintptr_t>(out + nb) & 15u) == 0)) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(out + nb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (nb + j < g.n) out[nb + j] = v[j];
                }
            }
            tcgen05_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        if (lane == 0) bulk_wait_all();  // this warp's output stores are done
    }
    tcgen05_fence_before();
    __syncthreads();
    if (warp == 1) {
        tcgen05_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// The tensor-core path takes the shapes TMA can describe: every row stride
// (k for the codes and a [n, k] weight, n for a [k, n] weight) a multiple of
// 16 bytes, 16-byte aligned bases.
bool graph_gemm_tc_supported(const int8_t* a, const int8_t* b, int64_t k, int64_t n, int b_kmajor) {
    return k % 16 == 0 && (b_kmajor || n % 16 == 0) && aligned16(a) && aligned16(b);
}

template <int BN, bool kMnB>
int run_graph_tc(cudaStream_t s, const int8_t* a, const int8_t* b, GraphTcArgs g) {
    CUtensorMap map_a, map_b;
    int st = make_tma_map_u8(&map_a, a, g.k, g.m, GBK, GBM);
    if (st) return st;
    st = kMnB ? make_tma_map_u8(&map_b, b, g.n, g.k, 128, GBK) : make_tma_map_u8(&map_b, b, g.k, g.n, GBK, BN);
    if (st) return st;
    g.n_tiles = static_cast<int>((g.n + BN - 1) / BN);
    CUtensorMap map_y = map_a;  // unused unless tma_store
    g.tma_store = g.n % 4 == 0 && aligned16(g.out);
    if (g.tma_store) {
        st = make_tma_map_f32_out(&map_y, g.out, g.n, g.m, 32);
        if (st) return st;
    }
    const int64_t tiles = (int64_t)g.m_tiles * g.n_tiles;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    constexpr size_t smem = GraphTc<BN>::kSmemBytes;
    st = allow_smem(reinterpret_cast<const void*>(graph_gemm_tc_kernel<BN, kMnB>), smem, "graph_gemm_tc");
    if (st) return st;
    return launch(graph_gemm_tc_kernel<BN, kMnB>, dim3(grid), dim3(GThreads), smem, s, false, "graph_gemm_tc",
                  map_a, map_b, map_y, g, exp_table());
}

int launch_graph_tc(cudaStream_t s, const int8_t* a, const int8_t* b, int b_kmajor, const float* bias,
                    float input_scale, const float* ws, float* out, int64_t m, int64_t k, int64_t n, int relu,
                    const GraphGlue& glue) {
    GraphTcArgs g;
    g.ws = ws;
    g.bias = bias;
    g.out = out;
    g.input_scale = input_scale;
    g.relu = relu;
    g.m = m;
    g.n = n;
    g.k = k;
    g.m_tiles = static_cast<int>((m + GBM - 1) / GBM);
    g.n_tiles = 0;
    g.glue = glue;
    const bool wide = (int64_t)g.m_tiles * ((n + 255) / 256) >= sm_count();
    if (b_kmajor) return wide ? run_graph_tc<256, false>(s, a, b, g) : run_graph_tc<128, false>(s, a, b, g);
    return wide ? run_graph_tc<256, true>(s, a, b, g) : run_graph_tc<128, true>(s, a, b, g);
}

}  // namespace

int launch_gemm_i8_per_channel(cudaStream_t s, const int8_t* a, const int8_t* b,
                               const float* bias, float input_scale, const float* wscales,
                               float* out, int64_t m, int64_t k, int64_t n, int activation) {
    if (m == 0 || n == 0) return LEAFQ_OK;
    const GraphGlue none{0, 1.0f, 0.0f, nullptr, 0, 0};
    if (k > 0 && graph_gemm_tc_supported(a, b, k, n, 0))
        return launch_graph_tc(s, a, b, 0, bias, input_scale, wscales, out, m, k, n, activation == 1 ? 1 : 0, none);
    const dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
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
    if (graph_gemm_tc_supported(codes, weight, k, n, trans_b ? 1 : 0))
        return launch_graph_tc(s, codes, weight, trans_b ? 1 : 0, nullptr, input_scale, wscales, out, m, k, n, 0,
                               glue);
    const dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
    return launch(gemm_i8_per_channel_kernel, grid, dim3(256), 0, s, false, "gemm_i8_per_channel", codes,
                  weight, static_cast<const float*>(nullptr), input_scale, wscales, out, m, k, n, 0,
                  trans_b ? 1 : 0, glue, exp_table());
}

}  // namespace leafq
