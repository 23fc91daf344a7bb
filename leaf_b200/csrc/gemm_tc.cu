// W8A8 prefill GEMM on the 5th-generation tensor cores (tcgen05.mma
// kind::i8, int32 accumulators in tensor memory).
//
// Replaces the prefill branch of Decoder::Impl::linear for per-row INT8
// weights: the VNNI 2x4 tile (decoder.cpp:661-702) or the AVX2 4x2 tile
// (:571-617) over all rows, with the per-token codes produced beforehand by
// quantize_act_kernel.  Both CPU tiles and this kernel produce the exact
// int32 dot product of every (token, row), and the same epilogue:
//   y = fma(float(acc) * sx[token], sw[row], 0.0f) + (bias[row] or 0.0f).
//
// Tiling: D[128 tokens, BN rows] per tile (one UMMA of M=128, N=BN, K=32
// per instruction, four per 128-byte K block).  More than 64 tokens: BN of
// 256, 160, 128, 64 or 32, whichever needs the fewest rounds of tiles x
// width (so M=512 x N=5632 runs one round of 144 tiles 160 wide).  At most
// 64 tokens (prefill chunks, batched decode of a few dozen sequences, where
// the weight stream must come through most SMs): 256 or 128 when their
// tiles give every SM one, else 64 when its tiles cover about 4/5 of the
// SMs, else 32.  Operands are K-major: the
// codes [tokens, cols] and the weights [rows, cols] are both row-major with
// K contiguous, loaded by TMA with 128-byte swizzle into a ring of 4 to 10
// stages (about 200 KB); with at most 64 tokens the code box is cut to 32 or
// 64 rows.  Warp roles (192 threads, persistent over tiles):
//   warp 0: TMA producer (one elected lane), no multicast;
//   warp 1: allocates 512 TMEM columns (two 256-column accumulators so the
//           epilogue of one tile overlaps the MMAs of the next) and issues
//           the MMAs from one elected lane;
//   warps 2-5: epilogue, each reading its 32 TMEM lanes (= tokens) with
//           tcgen05.ld and writing 32 consecutive fp32 outputs per load.
// Every mbarrier wait is bounded; on a timeout the roles stop, the TMEM is
// freed and the kernel returns with the device error word set.
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (= int8 elements) of K per stage
constexpr int UMMA_K = 32;
constexpr int kThreads = 192;      // CTA-pair kernel: producer, MMA, 4 epilogue warps
constexpr int kEpiWarps = 8;       // one-CTA kernel: two epilogue warps per TMEM sub-partition
constexpr int kThreadsOne = (2 + kEpiWarps) * 32;
constexpr int kEpiBar = 1;         // named barrier of the one-CTA kernel's epilogue warps
constexpr int kABytes = BM * BK;  // 16 KB
// Output staging: one 32 x 32 fp32 block (4 KB, 128-byte swizzle) per
// epilogue warp, written to global memory by a TMA store.
constexpr size_t kYStageBytes = 4 * 32 * 32 * sizeof(float);
constexpr size_t kYStageBytesOne = kEpiWarps * 32 * 32 * sizeof(float);

// kThin (at most 64 tokens, one M tile): each stage holds only 64 rows of
// codes, so twice as many stages fit and a whole K of 2048 is in flight at
// once, and the MMAs are M = 64 (tcgen05.mma kind::i8 128 x N would read
// past the stage).  The M = 64 accumulator occupies TMEM lanes 0-15 of each
// 32-lane sub-partition: row 16q + i in lane 32q + i, so epilogue warp q
// owns rows 16q .. 16q + 15 and stores them through a 16-row TMA box.
template <int BN, bool kThin>
struct TileCfg {
    // Thin launches take two 128-byte K boxes per stage: half as many stages
    // (each costs the MMA thread a wait, a commit and a round trip to the
    // producer), the same bytes in flight.
    static constexpr int kBoxes = kThin ? 2 : 1;
    static constexpr int kABox = kThin ? 64 * BK : kABytes;
    static constexpr int kBBox = BN * BK;
    static constexpr int kAStage = kABox * kBoxes;
    static constexpr int kBBytes = kBBox * kBoxes;
    // The tile's [scale | bias][BN], rounded to 1 KB: the output staging
    // blocks behind it must stay 1024-byte aligned for the 128-byte swizzle.
    static constexpr size_t kColBytes = (2 * BN * sizeof(float) + 1023) / 1024 * 1024;
    static constexpr size_t kFixed = 1024 /*barriers*/ + kColBytes + kYStageBytesOne + 1024 /*align*/;
    // The preferred ring depth, cut to what fits in 227 KB beside the rest.
    static constexpr int kPrefStages =
        kThin ? 16 : (BN == 256 ? 4 : BN == 160 ? 5 : BN == 128 ? 6 : BN == 64 ? 8 : 10);
    static constexpr int kFitStages = static_cast<int>((227 * 1024 - kFixed) / (kAStage + kBBytes));
    static constexpr int kStages = kPrefStages < kFitStages ? kPrefStages : kFitStages;
    static constexpr int kAccCols = BN;  // TMEM columns per accumulator
    // Allocated TMEM columns: a power of two covering both accumulators.
    static constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128 : 2 * kAccCols <= 256 ? 256 : 512;
    static constexpr size_t kSmemBytes = (size_t)kStages * (kAStage + kBBytes) + kFixed;
};

struct GemmArgs {
    const float* sx;
    const float* ws;
    const float* bias;
    float* y;
    int64_t tokens;
    int64_t rows;
    int64_t cols;
    int m_tiles;
    int n_tiles;
    uint32_t a_box_bytes;  // bytes one A load brings (box rows x 128): fewer rows for few tokens
    int tma_store;         // outputs through map_y (rows % 4 == 0, 16-byte aligned y)
};

template <int BN, bool kThin>
__global__ void __launch_bounds__(kThreadsOne, 1)
gemm_w8a8_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_w,
                    const __grid_constant__ CUtensorMap map_y, const GemmArgs a) {
    using Cfg = TileCfg<BN, kThin>;
    constexpr int kStages = Cfg::kStages;
    constexpr int kAccCols = Cfg::kAccCols;
    constexpr int kTmemCols = Cfg::kTmemCols;
    constexpr int kBBytes = Cfg::kBBytes;
    constexpr int kABytes = Cfg::kAStage;  // bytes of one stage's code tile
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte alignment for the swizzled operand tiles.
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + (size_t)kStages * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(b_tiles + (size_t)kStages * kBBytes);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
    // The tile's row scales and bias, staged once per tile by the epilogue
    // warps together.
    float* col_s = reinterpret_cast<float*>(b_tiles + (size_t)kStages * kBBytes + 1024);
    float* y_stage = col_s + Cfg::kColBytes / sizeof(float);  // [8 warps][32 x 32], 1024-byte aligned

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kBoxes = Cfg::kBoxes;
    constexpr int kStageK = BK * kBoxes;  // bytes of K per stage
    const int kblocks = static_cast<int>((a.cols + kStageK - 1) / kStageK);
    const int tiles = a.m_tiles * a.n_tiles;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);  // one arrival per epilogue warp
        }
        fence_barrier_init();
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tcgen05_fence_before();
    __syncthreads();
    tcgen05_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    grid_launch_dependents();

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (elect_one_sync()) {
            const uint64_t keep = l2_policy_evict_last();
            // The weights do not depend on the previous kernel: the first
            // tile's first stages of weight rows are requested before waiting
            // for it (with programmatic dependent launch this overlaps its tail).
            const int early = blockIdx.x < tiles ? (kblocks < kStages ? kblocks : kStages) : 0;
            {
                const int n0 = (blockIdx.x / a.m_tiles) * BN;
                for (int kb = 0; kb < early; ++kb) {
                    mbar_arrive_expect_tx(&full[kb], kBoxes * a.a_box_bytes + kBBytes);
                    for (int h = 0; h < kBoxes; ++h)
                        tma_load_2d(b_tiles + (size_t)kb * kBBytes + h * Cfg::kBBox, &map_w, kb * kStageK + h * BK, n0,
                                    &full[kb], keep);
                }
            }
            grid_dependency_wait();  // the codes come from the previous kernel
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile % a.m_tiles) * BM;
                const int n0 = (tile / a.m_tiles) * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (it < early) {  // weights already requested
                        for (int h = 0; h < kBoxes; ++h)
                            tma_load_2d(a_tiles + (size_t)s * kABytes + h * Cfg::kABox, &map_q, kb * kStageK + h * BK,
                                        m0, &full[s], keep);
                        continue;
                    }
                    if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1, kSiteGemmEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kBoxes * a.a_box_bytes + kBBytes);
                    for (int h = 0; h < kBoxes; ++h) {
                        tma_load_2d(a_tiles + (size_t)s * kABytes + h * Cfg::kABox, &map_q, kb * kStageK + h * BK, m0,
                                    &full[s], keep);
                        tma_load_2d(b_tiles + (size_t)s * kBBytes + h * Cfg::kBBox, &map_w, kb * kStageK + h * BK, n0,
                                    &full[s], keep);
                    }
                }
            }
            // Drain: the last use of every stage must have landed before the
            // block can exit (normally already true).
            for (int back = 0; back < kStages && back < it; ++back) {
                const int i = it - 1 - back;
                mbar_wait(&full[i % kStages], (i / kStages) & 1, kSiteGemmFull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one_sync()) {
            const uint32_t idesc = umma_idesc_i8(kThin ? 64 : BM, BN);
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                if (local >= 2 && !mbar_wait(&acc_empty[acc], ((local >> 1) - 1) & 1, kSiteGemmAccEmpty)) break;
                tcgen05_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kAccCols;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&full[s], (it / kStages) & 1, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tcgen05_fence_after();
                    const uint32_t a_st = smem_u32(a_tiles + (size_t)s * kABytes);
                    const uint32_t b_st = smem_u32(b_tiles + (size_t)s * kBBytes);
#pragma unroll
                    for (int k = 0; k < kBoxes * (BK / UMMA_K); ++k) {
                        // Box k / 4; advance its start address by (k % 4) * 32 bytes (>> 4).
                        // Zero-filled steps past the columns add nothing.
                        constexpr int kPer = BK / UMMA_K;
                        const uint64_t adesc = umma_desc_k_sw128(a_st + (k / kPer) * Cfg::kABox) + 2 * (k % kPer);
                        const uint64_t bdesc = umma_desc_k_sw128(b_st + (k / kPer) * Cfg::kBBox) + 2 * (k % kPer);
                        umma_i8(d_tmem, adesc, bdesc, idesc, (kb | k) != 0);
                    }
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&acc_full[acc]);
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2-9)
        // Warp w reads TMEM lanes 32 (w % 4) .. + 31 and takes the 32-column
        // blocks c / 32 = part, part + 2, ... (two warps per sub-partition, so
        // one's arithmetic overlaps the other's loads and stores).
        grid_dependency_wait();
        const int ew = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
        const int part = ew >> 2;
        constexpr int kWarpRows = kThin ? 16 : 32;  // accumulator rows in those lanes
        int local = 0;
        bool ok = true;  // a failed wait leaves the warps on the same barrier sequence
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const int m0 = (tile % a.m_tiles) * BM;
            const int n0 = (tile / a.m_tiles) * BN;
            // Stage this tile's row scales and bias (0 without bias: the
            // epilogue always adds it) while the MMAs run, after every
            // epilogue warp has finished the previous tile.
            float* ws_s = col_s;
            float* bias_s = ws_s + BN;
            bar_sync(kEpiBar, kEpiWarps * 32);
            for (int i = ew * 32 + lane; i < BN; i += kEpiWarps * 32) {
                const int64_t n = n0 + i < a.rows ? n0 + i : a.rows - 1;
                ws_s[i] = __ldg(a.ws + n);
                bias_s[i] = a.bias ? __ldg(a.bias + n) : 0.0f;
            }
            bar_sync(kEpiBar, kEpiWarps * 32);
            if (ok && !mbar_wait(&acc_full[acc], (local >> 1) & 1, kSiteGemmAccFull)) ok = false;
            tcgen05_fence_after();
            const int64_t mb = m0 + quarter * kWarpRows;  // this warp's first row
            const int64_t m = mb + lane;
            const bool row_live = lane < kWarpRows && m < a.tokens;
            const float token_scale = row_live ? __ldg(a.sx + m) : 0.0f;
            float* out = a.y + m * a.rows;
            const bool vec = (a.rows % 4) == 0;
            for (int c = part * 32; c < BN; c += 64) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + acc * kAccCols + c + ((uint32_t)(quarter * 32) << 16), r);
                tmem_wait_ld();
                const int64_t nb = n0 + c;
                if (!a.tma_store && (!row_live || nb >= a.rows)) continue;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 w4 = *reinterpret_cast<const float4*>(ws_s + c + j);
                    const float4 b4 = *reinterpret_cast<const float4*>(bias_s + c + j);
                    const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float product = __fmul_rn(__int2float_rn(static_cast<int>(r[j + u])), token_scale);
                        v[j + u] = __fadd_rn(__fmaf_rn(product, wv[u], 0.0f), bv[u]);
                    }
                }
                if (a.tma_store) {
                    // This warp's rows x 32 outputs through its staging tile
                    // (rows past the tokens and columns past the rows are not
                    // written by the store; with kThin the box is 16 rows and
                    // lanes 16-31 write nothing).
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    store_block_32x32(y_stage + ew * 1024, v, lane, &map_y, static_cast<int32_t>(nb),
                                      static_cast<int32_t>(mb), nb < a.rows && mb < a.tokens, lane < kWarpRows);
                } else if (vec && nb + 32 <= a.rows) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(out + nb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (nb + j < a.rows) out[nb + j] = v[j];
                }
            }
            tcgen05_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
    }

    if (warp >= 2 && lane == 0) bulk_wait_all();  // this warp's output stores are done
    tcgen05_fence_before();
    __syncthreads();
    if (warp == 1) {
        tcgen05_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ------------------------------------------------------------------------
// Many tokens: a pair of CTAs on two SMs (a cluster of 2) per 256 x 256 tile.
// Each CTA loads its own 128 rows of codes and 128 of the tile's 256 weight
// rows per stage (32 KB instead of 48 KB for a one-CTA 128 x 256 tile, so 6
// stages fit instead of 4); the leader's elected thread issues
// tcgen05.mma.cta_group::2 (M = 256, N = 256) over both CTAs' halves, and
// each CTA's TMEM holds its 128 tokens x 256 rows of int32 sums.  The
// follower's TMA loads count on the leader's `full` barrier; the MMA commits
// arrive on both CTAs' `empty` / `acc_full` barriers (multicast commit; no
// load uses multicast); both CTAs' epilogue warps release an accumulator on
// the leader's `acc_empty`.  Same epilogue and bits as the one-CTA kernel.
constexpr int kPairM = 256, kPairN = 256;
constexpr int kPairStages = 6;
constexpr int kPairABytes = 128 * BK;       // this CTA's half of M
constexpr int kPairBBytes = (kPairN / 2) * BK;  // this CTA's half of N
constexpr size_t kPairColBytes = 4 * 2 * 2 * kPairN * sizeof(float);
constexpr size_t kPairSmemBytes =
    (size_t)kPairStages * (kPairABytes + kPairBBytes) + 1024 + kPairColBytes + kYStageBytes + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_w8a8_tc2_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_w,
                     const __grid_constant__ CUtensorMap map_y, const GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + (size_t)kPairStages * kPairABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(b_tiles + (size_t)kPairStages * kPairBBytes);
    uint64_t* empty = full + kPairStages;
    uint64_t* acc_full = empty + kPairStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
    float* col_s = reinterpret_cast<float*>(b_tiles + (size_t)kPairStages * kPairBBytes + 1024);
    float* y_stage = col_s + kPairColBytes / sizeof(float);  // [4 warps][32 x 32], 1024-byte aligned

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int kblocks = static_cast<int>((a.cols + BK - 1) / BK);
    const int tiles = a.m_tiles * a.n_tiles;  // 256 x 256 tiles
    const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&full[s], 1);   // the leader's expect_tx; both CTAs' bytes
            mbar_init(&empty[s], 1);  // the leader's multicast commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);  // four epilogue warps of each CTA
        }
        fence_barrier_init();
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_holder, 512);
        tmem_relinquish_pair();
    }
    tcgen05_fence_before();
    __syncthreads();
    // The follower signals the leader's barriers: both CTAs' barriers must
    // be initialised before either CTA uses them.
    cluster_sync_all();
    tcgen05_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    grid_launch_dependents();

    if (warp == 0) {
        // ---------------------------------------- TMA producer (both CTAs)
        if (elect_one_sync()) {
            const uint64_t keep = l2_policy_evict_last();
            grid_dependency_wait();  // the codes come from the previous kernel
            int it = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs) {
                const int m0 = (tile % a.m_tiles) * kPairM + 128 * static_cast<int>(rank);
                const int n0 = (tile / a.m_tiles) * kPairN + (kPairN / 2) * static_cast<int>(rank);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (it >= kPairStages && !mbar_wait(&empty[s], ((it / kPairStages) - 1) & 1, kSiteGemmEmpty)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[s], 2u * (kPairABytes + kPairBBytes));
                    const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
                    tma_load_2d_pair(a_tiles + (size_t)s * kPairABytes, &map_q, kb * BK, m0, bar, keep);
                    tma_load_2d_pair(b_tiles + (size_t)s * kPairBBytes, &map_w, kb * BK, n0, bar, keep);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------- MMA issuer (leader only)
        if (leader && elect_one_sync()) {
            const uint32_t idesc = umma_idesc_i8(kPairM, kPairN);
            int it = 0, local = 0;
            bool ok = true;
            for (int tile = pair; tile < tiles && ok; tile += pairs, ++local) {
                const int acc = local & 1;
                if (local >= 2 && !mbar_wait(&acc_empty[acc], ((local >> 1) - 1) & 1, kSiteGemmAccEmpty)) break;
                tcgen05_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kPairN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (!mbar_wait(&full[s], (it / kPairStages) & 1, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tcgen05_fence_after();
                    const uint64_t adesc = umma_desc_k_sw128(smem_u32(a_tiles + (size_t)s * kPairABytes));
                    const uint64_t bdesc = umma_desc_k_sw128(smem_u32(b_tiles + (size_t)s * kPairBBytes));
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k)
                        umma_i8_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
                    umma_commit_pair(&empty[s], 0x3);
                }
                if (ok) umma_commit_pair(&acc_full[acc], 0x3);
            }
        }
    } else {
        // ---------------------------------------- epilogue (warps 2-5, both CTAs)
        grid_dependency_wait();
        const int quarter = warp & 3;
        const uint32_t leader_acc_empty[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0),
                                              mapa_shared(smem_u32(&acc_empty[1]), 0)};
        int local = 0;
        for (int tile = pair; tile < tiles; tile += pairs, ++local) {
            const int acc = local & 1;
            const int m0 = (tile % a.m_tiles) * kPairM + 128 * static_cast<int>(rank);
            const int n0 = (tile / a.m_tiles) * kPairN;
            float* ws_s = col_s + (quarter * 2 + acc) * 2 * kPairN;
            float* bias_s = ws_s + kPairN;
            for (int i = lane; i < kPairN; i += 32) {
                const int64_t n = n0 + i < a.rows ? n0 + i : a.rows - 1;
                ws_s[i] = __ldg(a.ws + n);
                bias_s[i] = a.bias ? __ldg(a.bias + n) : 0.0f;
            }
            __syncwarp();
            if (!mbar_wait(&acc_full[acc], (local >> 1) & 1, kSiteGemmAccFull)) break;
            tcgen05_fence_after();
            const int64_t m = m0 + quarter * 32 + lane;
            const bool row_live = m < a.tokens;
            const float token_scale = row_live ? __ldg(a.sx + m) : 0.0f;
            float* out = a.y + m * a.rows;
            const bool vec = (a.rows % 4) == 0;
            for (int c = 0; c < kPairN; c += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + acc * kPairN + c + ((uint32_t)(quarter * 32) << 16), r);
                tmem_wait_ld();
                const int64_t nb = n0 + c;
                if (!a.tma_store && (!row_live || nb >= a.rows)) continue;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 w4 = *reinterpret_cast<const float4*>(ws_s + c + j);
                    const float4 b4 = *reinterpret_cast<const float4*>(bias_s + c + j);
                    const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float product = __fmul_rn(__int2float_rn(static_cast<int>(r[j + u])), token_scale);
                        v[j + u] = __fadd_rn(__fmaf_rn(product, wv[u], 0.0f), bv[u]);
                    }
                }
                if (a.tma_store) {
                    // This warp's 32 rows x 32 outputs through its staging tile.
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    const int64_t mb = m - lane;
                    store_block_32x32(y_stage + quarter * 1024, v, lane, &map_y, static_cast<int32_t>(nb),
                                      static_cast<int32_t>(mb), nb < a.rows && mb < a.tokens, true);
                } else if (vec && nb + 32 <= a.rows) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(out + nb + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (nb + j < a.rows) out[nb + j] = v[j];
                }
            }
            tcgen05_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(leader_acc_empty[acc]);
        }
    }

    if (warp >= 2 && lane == 0) bulk_wait_all();  // this warp's output stores are done
    // Neither CTA may leave while the pair's MMAs can still read its shared
    // memory or the other CTA can still signal its barriers.
    tcgen05_fence_before();
    __syncthreads();
    cluster_sync_all();
    if (warp == 1) {
        tcgen05_fence_after();
        tmem_dealloc_pair(tmem_base, 512);
    }
}

// 2-D int8 map over a row-major [outer, inner] matrix, box [box_outer, 128].
int make_map(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_outer) {
    return make_tma_map_u8(map, base, inner, outer, BK, box_outer);
}

}  // namespace

// ------------------------------------------------------------ tensor maps
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
}  // namespace

int make_tma_map_u8(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_inner,
                    int box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return LEAFQ_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
    const cuuint32_t estrides[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                          box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string(static_cast<int>(r)));
        return LEAFQ_ERR_CUDA;
    }
    return LEAFQ_OK;
}

int make_tma_map_f32_out(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled is not available from the driver");
        return LEAFQ_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner) * 4};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estrides[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
                          estrides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (output) failed with CUresult " + std::to_string(static_cast<int>(r)));
        return LEAFQ_ERR_CUDA;
    }
    return LEAFQ_OK;
}

bool gemm_tc_supported(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                       const void* weight) {
    (void)tokens;
    (void)rows;
    return bits == 8 && group == cols && cols % 16 == 0 && cols >= BK && aligned16(weight);
}

namespace {
template <int BN, bool kThin>
int run_tiles(cudaStream_t s, const int8_t* q, const int8_t* weight, int64_t cols, int64_t tokens,
              int64_t rows, GemmArgs a, bool pdl) {
    CUtensorMap map_q, map_w;
    // With one M tile of few tokens the A box is cut to 32 or 64 rows: the
    // tile's other rows are never stored (their accumulator lanes are
    // dropped by the epilogue), so loading them would only cost bandwidth.
    const int a_rows = kThin ? (tokens <= 32 ? 32 : 64) : BM;
    a.a_box_bytes = static_cast<uint32_t>(a_rows * BK);
    int st = make_map(&map_q, q, cols, tokens, a_rows);
    if (st) return st;
    st = make_map(&map_w, weight, cols, rows, BN);
    if (st) return st;
    CUtensorMap map_y = map_q;  // unused unless tma_store
    a.tma_store = rows % 4 == 0 && aligned16(a.y);
    if (a.tma_store) {
        st = make_tma_map_f32_out(&map_y, a.y, rows, tokens, kThin ? 16 : 32);
        if (st) return st;
    }
    a.n_tiles = static_cast<int>((rows + BN - 1) / BN);
    const int64_t tiles = (int64_t)a.m_tiles * a.n_tiles;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    constexpr size_t smem = TileCfg<BN, kThin>::kSmemBytes;
    st = allow_smem(reinterpret_cast<const void*>(gemm_w8a8_tc_kernel<BN, kThin>), smem, "gemm_w8a8_tc");
    if (st) return st;
    return launch(gemm_w8a8_tc_kernel<BN, kThin>, dim3(grid), dim3(kThreadsOne), smem, s, pdl, "gemm_w8a8_tc",
                  map_q, map_w, map_y, a);
}

// Clusters of two that can be resident at once (an SM left unpaired in its
// GPC cannot host one), cached per device; 0 if the query fails.
int max_pair_clusters() {
    static std::mutex mutex;
    static std::unordered_map<int, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int clusters = 0;
    if (allow_smem(reinterpret_cast<const void*>(gemm_w8a8_tc2_kernel), kPairSmemBytes, "gemm_w8a8_tc2") ==
        LEAFQ_OK) {
        cudaLaunchConfig_t config = {};
        config.gridDim = dim3(2 * sm_count());
        config.blockDim = dim3(kThreads);
        config.dynamicSmemBytes = kPairSmemBytes;
        cudaLaunchAttribute attribute[1];
        attribute[0].id = cudaLaunchAttributeClusterDimension;
        attribute[0].val.clusterDim.x = 2;
        attribute[0].val.clusterDim.y = 1;
        attribute[0].val.clusterDim.z = 1;
        config.attrs = attribute;
        config.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_w8a8_tc2_kernel, &config) != cudaSuccess) {
            cudaGetLastError();
            clusters = 0;
        }
    }
    cache[dev] = clusters;
    return clusters;
}

int run_pairs(cudaStream_t s, const int8_t* q, const int8_t* weight, int64_t cols, int64_t tokens, int64_t rows,
              GemmArgs a, int pairs, bool pdl) {
    CUtensorMap map_q, map_w;
    int st = make_map(&map_q, q, cols, tokens, 128);
    if (st) return st;
    st = make_map(&map_w, weight, cols, rows, kPairN / 2);
    if (st) return st;
    CUtensorMap map_y = map_q;  // unused unless tma_store
    a.tma_store = rows % 4 == 0 && aligned16(a.y);
    if (a.tma_store) {
        st = make_tma_map_f32_out(&map_y, a.y, rows, tokens, 32);
        if (st) return st;
    }
    a.m_tiles = static_cast<int>((tokens + kPairM - 1) / kPairM);
    a.n_tiles = static_cast<int>((rows + kPairN - 1) / kPairN);
    a.a_box_bytes = kPairABytes;
    const int64_t tiles = (int64_t)a.m_tiles * a.n_tiles;
    const int grid = 2 * static_cast<int>(std::min<int64_t>(tiles, pairs));
    st = allow_smem(reinterpret_cast<const void*>(gemm_w8a8_tc2_kernel), kPairSmemBytes, "gemm_w8a8_tc2");
    if (st) return st;
    return launch(gemm_w8a8_tc2_kernel, dim3(grid), dim3(kThreads), kPairSmemBytes, s, pdl, "gemm_w8a8_tc2",
                  map_q, map_w, map_y, a);
}

}  // namespace

int launch_gemm_tc(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens, int64_t cols,
                   const int8_t* weight, const float* wscales, int64_t rows, const float* bias,
                   float* y, bool pdl) {
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    if (!aligned16(q) || !aligned16(weight) || cols % 16 != 0) return LEAFQ_ERR_UNSUPPORTED;
    GemmArgs a;
    a.sx = sx;
    a.ws = wscales;
    a.bias = bias;
    a.y = y;
    a.tokens = tokens;
    a.rows = rows;
    a.cols = cols;
    a.m_tiles = static_cast<int>((tokens + BM - 1) / BM);
    // 256- or 128-row tiles when they give every SM one; 64-row tiles when
    // they cover about 4/5 of the SMs (measured: one wave of those beats two
    // waves of 32-row tiles, while wide tiles short of one per SM lose to
    // narrower ones); else 32.
    const int64_t sms = sm_count();
    auto tiles = [&](int64_t bn) { return (int64_t)a.m_tiles * ((rows + bn - 1) / bn); };
    if (tokens <= 64) {
        if (tiles(256) >= sms) return run_tiles<256, true>(s, q, weight, cols, tokens, rows, a, pdl);
        if (tiles(128) >= sms) return run_tiles<128, true>(s, q, weight, cols, tokens, rows, a, pdl);
        if (tiles(64) * 5 >= sms * 4) return run_tiles<64, true>(s, q, weight, cols, tokens, rows, a, pdl);
        return run_tiles<32, true>(s, q, weight, cols, tokens, rows, a, pdl);
    }
    // Many tokens: CTA pairs on 256 x 256 tiles when they fill at least two
    // rounds of the pairs that fit (measured: at 1024 tokens, 88 pair tiles on
    // 74 pairs, the one-CTA tiles are faster; LEAFQ_GEMM_PAIRS=0 turns pairs
    // off).
    static const bool pairs_on = [] {
        const char* env = std::getenv("LEAFQ_GEMM_PAIRS");
        return !(env && env[0] == '0');
    }();
    if (pairs_on && tokens >= 2048 && rows >= kPairN) {
        const int pairs = max_pair_clusters();
        const int64_t pair_tiles = ((tokens + kPairM - 1) / kPairM) * ((rows + kPairN - 1) / kPairN);
        if (pairs > 0 && pair_tiles >= 2 * pairs) return run_pairs(s, q, weight, cols, tokens, rows, a, pairs, pdl);
    }
    // More tokens: the width with the least work per SM, counted as rounds of
    // tiles x (width + 32) -- a partial last round costs a whole one, and each
    // tile carries a fixed prologue / epilogue of about 32 columns' worth; the
    // wider on a tie.  M=512 x N=5632 takes 160 (144 tiles, one round) rather
    // than 128 (176 tiles: a second round 19 % full); large M keeps 256.
    const int widths[5] = {256, 160, 128, 64, 32};
    int best = 256;
    int64_t best_cost = -1;
    for (int bn : widths) {
        const int64_t rounds = (tiles(bn) + sms - 1) / sms;
        const int64_t cost = rounds * (bn + 32);
        if (best_cost < 0 || cost < best_cost) {
            best = bn;
            best_cost = cost;
        }
    }
    switch (best) {
        case 256: return run_tiles<256, false>(s, q, weight, cols, tokens, rows, a, pdl);
        case 160: return run_tiles<160, false>(s, q, weight, cols, tokens, rows, a, pdl);
        case 128: return run_tiles<128, false>(s, q, weight, cols, tokens, rows, a, pdl);
        case 64: return run_tiles<64, false>(s, q, weight, cols, tokens, rows, a, pdl);
        default: return run_tiles<32, false>(s, q, weight, cols, tokens, rows, a, pdl);
    }
}

}  // namespace leafq
