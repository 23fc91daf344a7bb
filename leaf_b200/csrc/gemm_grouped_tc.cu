// Many-token W8A8 linear with GROUPED INT8 weights on the tensor cores
// (int8_group_size export, export_decoder.py:315; Decoder::Impl::linear's
// integer branch with quant_tile_avx / quant_vnni_tile, decoder.cpp:571-617,
// 661-702).  Per token t, row n and group g of `group` columns the
// reference forms the exact int32 sum acc_g, then walks the groups in order:
//   result = fma(float(acc_g) * sx[t], sw[n][g], result)     (AVX2 + FMA)
//   result = result + (float(acc_g) * sx[t]) * sw[n][g]      (VNNI tile)
// from result = 0.0f, and stores result + bias[n] (:1229).
//
// One CTA per 128-token x 64-row tile (persistent over tiles), 320 threads:
//   warp 0      TMA producer: 256-byte K stages, each two 128-byte swizzled
//               boxes of codes (2 x 16 KB) and of weight rows (2 x 8 KB).
//   warp 1      MMA issuer: tcgen05.mma kind::i8, M = 128, N = 64, K = 32
//               per instruction.  Each group's K range accumulates into its
//               own 64-column TMEM slot (a ring of 8 slots, 512 columns), and
//               the slot is committed when the group's last MMA is issued, so
//               the tensor cores run up to 8 groups ahead of the epilogue.
//   warps 2-9   epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its 32
//               tokens) and columns 32 ((w - 2) / 4) .. + 31 of every slot
//               (its 32 rows), and keeps those 32 running sums in registers
//               across the groups (cvt, mul.f32x2 by the token scale, then
//               fma.f32x2 with the group scales staged in shared memory per
//               tile; the two-rounding form in scalar __fmul_rn / __fadd_rn).
//               Bias, then a 32 x 32 TMA store.
// Groups must be multiples of 32 codes (the MMA's K).  Every wait is bounded
// and reports through the device error word.
#include <algorithm>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr int kGBM = 128;
constexpr int kGBN = 64;
constexpr int kGBox = 128;  // bytes of K per TMA box (the 128-byte swizzle span)
constexpr int kGBoxes = 2;  // boxes per stage
constexpr int kGBK = kGBox * kGBoxes;  // bytes of K per stage
constexpr int kGUmmaK = 32;
constexpr int kGThreads = 320;
constexpr int kGEpiWarps = 8;
constexpr int kGSlots = 8;  // TMEM accumulator slots of kGBN columns
constexpr int kGTmemCols = kGSlots * kGBN;
constexpr int kGMaxStages = 8;
constexpr int kGMaxGroups = 256;  // group scales staged per tile: 64 x groups floats
constexpr uint32_t kGABox = kGBM * kGBox;
constexpr uint32_t kGBBox = kGBN * kGBox;
constexpr uint32_t kGABytes = kGABox * kGBoxes;
constexpr uint32_t kGBBytes = kGBBox * kGBoxes;
constexpr size_t kGYStageBytes = (size_t)kGEpiWarps * 32 * 32 * sizeof(float);
constexpr int kEpiBar = 1;  // named barrier of the epilogue warps
constexpr int kStageGeneric = -1;

struct GroupedArgs {
    const float* sx;
    const float* ws;  // [rows][groups]
    const float* bias;
    float* y;
    int64_t tokens, rows, cols;
    int group, groups;
    int m_tiles, n_tiles;
    int stages;
    int fused;      // 1: fma per group (AVX2 + FMA); 0: two roundings (VNNI tile)
    int tma_store;  // rows % 4 == 0 and y 16-byte aligned
    uint32_t scale_offset, ystage_offset, bar_offset;  // shared-memory layout (bytes from the aligned base)
};

// One full stage (8 MMAs of K = 32, two 128-byte boxes: descriptors a0/b0 and
// a1/b1) without branches between the tensor instructions (a branch beside
// each MMA, as a per-step group test makes, tripled the MMA thread's time per
// stage).  GS MMAs per group, GS in {1, 2, 4}: 8 / GS groups per stage; each
// box's accumulator slots are reserved before its first MMA, and each group
// is committed after its last MMA.
template <int GS>
__device__ __forceinline__ bool issue_stage_groups(uint32_t tmem_base, uint64_t a0, uint64_t a1, uint64_t b0,
                                                   uint64_t b1, uint32_t idesc, uint32_t& gc, uint64_t* acc_full,
                                                   uint64_t* acc_empty) {
    constexpr int kPerBox = 4 / GS;  // groups in each 128-byte box
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        // Reserve the box's slots, then issue its MMAs (the other box's slots
        // may still be in the epilogue's hands).
#pragma unroll
        for (int g = 0; g < kPerBox; ++g) {
            const uint32_t c = gc + h * kPerBox + g;
            if (c >= kGSlots && !mbar_wait(&acc_empty[c % kGSlots], ((c / kGSlots) - 1) & 1, kSiteGemmAccEmpty))
                return false;
        }
        tcgen05_fence_after();
        const uint64_t ad = h == 0 ? a0 : a1, bd = h == 0 ? b0 : b1;
#pragma unroll
        for (int g = 0; g < kPerBox; ++g) {
            const uint32_t slot = (gc + h * kPerBox + g) % kGSlots;
            const uint32_t d = tmem_base + slot * kGBN;
#pragma unroll
            for (int j = 0; j < GS; ++j) {
                const int k = g * GS + j;  // MMA within the box
                umma_i8(d, ad + 2 * k, bd + 2 * k, idesc, j != 0 ? 1u : 0u);
            }
            umma_commit(&acc_full[slot]);
        }
    }
    gc += 2 * kPerBox;
    return true;
}

// One full stage inside a group of whole stages; kFirst: the group's first
// stage (its first MMA starts the accumulator).
template <bool kFirst>
__device__ __forceinline__ void issue_stage_whole(uint32_t d, uint64_t a0, uint64_t a1, uint64_t b0, uint64_t b1,
                                                  uint32_t idesc) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
        umma_i8(d, (k < 4 ? a0 : a1) + 2 * (k % 4), (k < 4 ? b0 : b1) + 2 * (k % 4), idesc,
                (kFirst && k == 0) ? 0u : 1u);
}

__global__ void __launch_bounds__(kGThreads, 1)
gemm_w8a8_grouped_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_w,
                            const __grid_constant__ CUtensorMap map_y, const GroupedArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const int S = a.stages;
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + (size_t)S * kGABytes;
    float* scales_s = reinterpret_cast<float*>(smem + a.scale_offset);  // [groups][kGBN]
    float* y_stage = reinterpret_cast<float*>(smem + a.ystage_offset);  // [8 warps][32 x 32]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.bar_offset);
    uint64_t* empty = full + kGMaxStages;
    uint64_t* acc_full = empty + kGMaxStages;
    uint64_t* acc_empty = acc_full + kGSlots;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + kGSlots);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = static_cast<int>((a.cols + kGBK - 1) / kGBK);
    const int ksteps = static_cast<int>(a.cols / kGUmmaK);  // cols is a multiple of the group, so of 32
    const int group_steps = a.group / kGUmmaK;
    const int tiles = a.m_tiles * a.n_tiles;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < kGSlots; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kGEpiWarps);
        }
        fence_barrier_init();
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_w);
    }
    if (warp == 1) {
        tmem_alloc(tmem_holder, kGTmemCols);
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
            // Weights do not depend on the previous kernel: the first tile's
            // first stages of weight rows go out before the wait.
            const int early = blockIdx.x < tiles ? (kblocks < S ? kblocks : S) : 0;
            {
                const int n0 = (blockIdx.x / a.m_tiles) * kGBN;
                for (int kb = 0; kb < early; ++kb) {
                    mbar_arrive_expect_tx(&full[kb], kGABytes + kGBBytes);
                    for (int h = 0; h < kGBoxes; ++h)
                        tma_load_2d(b_tiles + (size_t)kb * kGBBytes + h * kGBBox, &map_w, kb * kGBK + h * kGBox, n0,
                                    &full[kb], keep);
                }
            }
            grid_dependency_wait();
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile % a.m_tiles) * kGBM;
                const int n0 = (tile / a.m_tiles) * kGBN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % S;
                    if (it < early) {
                        for (int h = 0; h < kGBoxes; ++h)
                            tma_load_2d(a_tiles + (size_t)s * kGABytes + h * kGABox, &map_q, kb * kGBK + h * kGBox, m0,
                                        &full[s], keep);
                        continue;
                    }
                    if (it >= S && !mbar_wait(&empty[s], ((it / S) - 1) & 1, kSiteGemmEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kGABytes + kGBBytes);
                    for (int h = 0; h < kGBoxes; ++h) {
                        tma_load_2d(a_tiles + (size_t)s * kGABytes + h * kGABox, &map_q, kb * kGBK + h * kGBox, m0,
                                    &full[s], keep);
                        tma_load_2d(b_tiles + (size_t)s * kGBBytes + h * kGBBox, &map_w, kb * kGBK + h * kGBox, n0,
                                    &full[s], keep);
                    }
                }
            }
            for (int back = 0; back < S && back < it; ++back) {
                const int i = it - 1 - back;
                mbar_wait(&full[i % S], (i / S) & 1, kSiteGemmFull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (elect_one_sync()) {
            const uint32_t idesc = umma_idesc_i8(kGBM, kGBN);
            // The full stages' group pattern: 1, 2 or 4 MMAs per group, 0 for
            // groups of whole stages, else the generic per-step path.
            constexpr int kSteps = kGBK / kGUmmaK;
            const int stage_kind = (group_steps == 1 || group_steps == 2 || group_steps == 4) ? group_steps
                                   : group_steps % kSteps == 0                                 ? 0
                                                                                                : kStageGeneric;
            const int stages_per_group = group_steps / kSteps > 0 ? group_steps / kSteps : 1;
            int it = 0;
            uint32_t gc = 0;  // groups started so far (slot = gc % kGSlots)
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                uint32_t d_tmem = tmem_base;
                for (int kb = 0; kb < kblocks && ok; ++kb, ++it) {
                    const int s = it % S;
                    if (!mbar_wait(&full[s], (it / S) & 1, kSiteGemmFull)) {
                        ok = false;
                        break;
                    }
                    tcgen05_fence_after();
                    const uint32_t a_st = smem_u32(a_tiles + (size_t)s * kGABytes);
                    const uint32_t b_st = smem_u32(b_tiles + (size_t)s * kGBBytes);
                    const uint64_t a0 = umma_desc_k_sw128(a_st), a1 = umma_desc_k_sw128(a_st + kGABox);
                    const uint64_t b0 = umma_desc_k_sw128(b_st), b1 = umma_desc_k_sw128(b_st + kGBBox);
                    if ((kb + 1) * (kGBK / kGUmmaK) <= ksteps && stage_kind != kStageGeneric) {
                        if (stage_kind == 1) {
                            ok = issue_stage_groups<1>(tmem_base, a0, a1, b0, b1, idesc, gc, acc_full, acc_empty);
                        } else if (stage_kind == 2) {
                            ok = issue_stage_groups<2>(tmem_base, a0, a1, b0, b1, idesc, gc, acc_full, acc_empty);
                        } else if (stage_kind == 4) {
                            ok = issue_stage_groups<4>(tmem_base, a0, a1, b0, b1, idesc, gc, acc_full, acc_empty);
                        } else {  // whole stages per group
                            const int pos = kb % stages_per_group;
                            if (pos == 0) {
                                const uint32_t slot = gc % kGSlots;
                                if (gc >= kGSlots &&
                                    !mbar_wait(&acc_empty[slot], ((gc / kGSlots) - 1) & 1, kSiteGemmAccEmpty))
                                    ok = false;
                                tcgen05_fence_after();
                                d_tmem = tmem_base + slot * kGBN;
                                if (ok) issue_stage_whole<true>(d_tmem, a0, a1, b0, b1, idesc);
                            } else {
                                issue_stage_whole<false>(d_tmem, a0, a1, b0, b1, idesc);
                            }
                            if (ok && pos == stages_per_group - 1) {
                                umma_commit(&acc_full[gc % kGSlots]);
                                ++gc;
                            }
                        }
                    } else {
                        // Partial last stage, or a group size outside the patterns above.
#pragma unroll
                        for (int k = 0; k < kGBK / kGUmmaK; ++k) {
                            const int step = kb * (kGBK / kGUmmaK) + k;
                            if (step >= ksteps) break;  // the last stage's zero-filled tail
                            const int in_group = step % group_steps;
                            if (in_group == 0) {
                                const uint32_t slot = gc % kGSlots;
                                if (gc >= kGSlots &&
                                    !mbar_wait(&acc_empty[slot], ((gc / kGSlots) - 1) & 1, kSiteGemmAccEmpty)) {
                                    ok = false;
                                    break;
                                }
                                tcgen05_fence_after();
                                d_tmem = tmem_base + slot * kGBN;
                            }
                            umma_i8(d_tmem, (k < 4 ? a0 : a1) + 2 * (k % 4), (k < 4 ? b0 : b1) + 2 * (k % 4), idesc,
                                    in_group != 0);
                            if (in_group == group_steps - 1) {
                                umma_commit(&acc_full[gc % kGSlots]);
                                ++gc;
                            }
                        }
                    }
                    umma_commit(&empty[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2-9)
        grid_dependency_wait();
        const int ew = warp - 2;
        const int quarter = warp & 3;  // TMEM lanes 32 * quarter .. + 31
        const int half = ew >> 2;      // columns 32 * half .. + 31 of each slot
        const int etid = ew * 32 + lane;
        uint32_t gc = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            const int m0 = (tile % a.m_tiles) * kGBM;
            const int n0 = (tile / a.m_tiles) * kGBN;
            // This tile's group scales, transposed to [group][row] (rows past
            // the weight repeat the last one; their outputs are not stored).
            bar_sync(kEpiBar, kGEpiWarps * 32);  // every warp is done with the previous tile's
            for (int i = etid; i < a.groups * kGBN; i += kGEpiWarps * 32) {
                const int g = i / kGBN, c = i % kGBN;
                const int64_t n = n0 + c < a.rows ? n0 + c : a.rows - 1;
                scales_s[i] = __ldg(a.ws + n * a.groups + g);
            }
            bar_sync(kEpiBar, kGEpiWarps * 32);
            const int64_t m = m0 + quarter * 32 + lane;
            const float sx = m < a.tokens ? __ldg(a.sx + m) : 0.0f;
            const unsigned long long sx2 = pack2(sx, sx);
            unsigned long long res[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) res[j] = 0ull;  // (+0.0f, +0.0f)
            for (int g = 0; g < a.groups; ++g, ++gc) {
                const uint32_t slot = gc % kGSlots;
                if (ok && !mbar_wait(&acc_full[slot], (gc / kGSlots) & 1, kSiteGemmAccFull)) ok = false;
                tcgen05_fence_after();
                uint32_t r[32];
                tmem_ld_32x32b_x32(tmem_base + slot * kGBN + half * 32 + ((uint32_t)(quarter * 32) << 16), r);
                tmem_wait_ld();
                tcgen05_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[slot]);
                const float4* sc4 = reinterpret_cast<const float4*>(scales_s + g * kGBN + half * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 w4 = sc4[j];
                    const unsigned long long p0 =
                        mul2(pack2(__int2float_rn(static_cast<int>(r[4 * j])),
                                   __int2float_rn(static_cast<int>(r[4 * j + 1]))), sx2);
                    const unsigned long long p1 =
                        mul2(pack2(__int2float_rn(static_cast<int>(r[4 * j + 2])),
                                   __int2float_rn(static_cast<int>(r[4 * j + 3]))), sx2);
                    const unsigned long long s0 = pack2(w4.x, w4.y), s1 = pack2(w4.z, w4.w);
                    if (a.fused) {
                        res[2 * j] = fma2(p0, s0, res[2 * j]);
                        res[2 * j + 1] = fma2(p1, s1, res[2 * j + 1]);
                    } else {
                        // Two roundings, in scalar __fmul_rn / __fadd_rn: the
                        // paired mul + add came out as one fused operation.
                        const float2 q0 = unpack2(p0), q1 = unpack2(p1);
                        const float2 r0 = unpack2(res[2 * j]), r1 = unpack2(res[2 * j + 1]);
                        res[2 * j] =
                            pack2(__fadd_rn(r0.x, __fmul_rn(q0.x, w4.x)), __fadd_rn(r0.y, __fmul_rn(q0.y, w4.y)));
                        res[2 * j + 1] =
                            pack2(__fadd_rn(r1.x, __fmul_rn(q1.x, w4.z)), __fadd_rn(r1.y, __fmul_rn(q1.y, w4.w)));
                    }
                }
            }
            // result + bias (or + 0.0f), then this warp's 32 x 32 block out.
            const int64_t nb = n0 + half * 32;
            float v[32];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float2 f = unpack2(res[j]);
                const int64_t c0 = nb + 2 * j, c1 = c0 + 1;
                const float b0 = a.bias && c0 < a.rows ? __ldg(a.bias + c0) : 0.0f;
                const float b1 = a.bias && c1 < a.rows ? __ldg(a.bias + c1) : 0.0f;
                v[2 * j] = __fadd_rn(f.x, b0);
                v[2 * j + 1] = __fadd_rn(f.y, b1);
            }
            if (a.tma_store) {
                if (lane == 0) bulk_wait_read_all();
                __syncwarp();
                const int64_t mb = m0 + quarter * 32;
                store_block_32x32(y_stage + ew * 1024, v, lane, &map_y, static_cast<int32_t>(nb),
                                  static_cast<int32_t>(mb), nb < a.rows && mb < a.tokens, true);
            } else if (m < a.tokens) {
                float* out = a.y + m * a.rows;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (nb + j < a.rows) out[nb + j] = v[j];
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    tcgen05_fence_before();
    __syncthreads();
    if (warp == 1) {
        tcgen05_fence_after();
        tmem_dealloc(tmem_base, kGTmemCols);
    }
}

}  // namespace

bool gemm_grouped_tc_supported(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                               const void* weight, const int8_t* q) {
    (void)rows;
    return bits == 8 && tokens > 8 && group < cols && group % kGUmmaK == 0 && cols % group == 0 &&
           cols >= kGBox && cols / group <= kGMaxGroups && aligned16(weight) && aligned16(q);
}

int launch_gemm_grouped_tc(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens, int64_t cols,
                           const int8_t* weight, const float* wscales, int64_t rows, int64_t group,
                           const float* bias, float* y, bool fused, bool pdl) {
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    GroupedArgs a{};
    a.sx = sx;
    a.ws = wscales;
    a.bias = bias;
    a.y = y;
    a.tokens = tokens;
    a.rows = rows;
    a.cols = cols;
    a.group = static_cast<int>(group);
    a.groups = static_cast<int>(cols / group);
    a.m_tiles = static_cast<int>((tokens + kGBM - 1) / kGBM);
    a.n_tiles = static_cast<int>((rows + kGBN - 1) / kGBN);
    a.fused = fused ? 1 : 0;
    a.tma_store = rows % 4 == 0 && aligned16(y);
    // Shared memory: stages, the tile's group scales, the output staging
    // tiles, barriers; as many stages (up to 8) as fit in 227 KB.
    const size_t scale_bytes = ((size_t)a.groups * kGBN * sizeof(float) + 1023) & ~size_t(1023);
    const size_t fixed = scale_bytes + kGYStageBytes + 1024 /*barriers*/ + 1024 /*alignment*/;
    const size_t budget = 227 * 1024;
    const int stages = static_cast<int>(std::min<size_t>(kGMaxStages, (budget - fixed) / (kGABytes + kGBBytes)));
    if (stages < 2) {
        set_error("grouped INT8 tensor-core GEMM: too many groups for shared memory");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    a.stages = stages;
    a.scale_offset = static_cast<uint32_t>((size_t)stages * (kGABytes + kGBBytes));
    a.ystage_offset = static_cast<uint32_t>(a.scale_offset + scale_bytes);
    a.bar_offset = static_cast<uint32_t>(a.ystage_offset + kGYStageBytes);
    const size_t smem = (size_t)a.bar_offset + 1024 + 1024;

    CUtensorMap map_q, map_w, map_y;
    int st = make_tma_map_u8(&map_q, q, cols, tokens, kGBox, kGBM);
    if (st) return st;
    st = make_tma_map_u8(&map_w, weight, cols, rows, kGBox, kGBN);
    if (st) return st;
    map_y = map_q;  // unused unless tma_store
    if (a.tma_store) {
        st = make_tma_map_f32_out(&map_y, y, rows, tokens, 32);
        if (st) return st;
    }
    const int64_t tiles = (int64_t)a.m_tiles * a.n_tiles;
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    st = allow_smem(reinterpret_cast<const void*>(gemm_w8a8_grouped_tc_kernel), smem, "gemm_w8a8_grouped_tc");
    if (st) return st;
    return launch(gemm_w8a8_grouped_tc_kernel, dim3(grid), dim3(kGThreads), smem, s, pdl, "gemm_w8a8_grouped_tc",
                  map_q, map_w, map_y, a);
}

}  // namespace leafq
