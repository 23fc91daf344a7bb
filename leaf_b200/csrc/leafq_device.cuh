// Device-side helpers shared by the leafq kernels (sm_100a only).
//
// Inline PTX for: mbarriers with bounded waits, 1-D bulk copies (TMA without
// a tensor map), tiled tensor copies, programmatic dependent launch, and the
// tcgen05 tensor-memory / MMA instructions.  No copy here uses cluster
// multicast.
//
// Every wait in this library is bounded.  A wait that gives up records where
// it stopped in leafq_device_error (see leafq_internal.h) and the kernel
// returns; the host reports LEAFQ_ERR_TIMEOUT from leafq_device_status().
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "leafq_internal.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "leafq kernels are written for sm_100a only"
#endif

namespace leafq {

// Error word written by kernels whose waits time out (first writer wins).
// Codes: 0 = fine; otherwise (site << 16) | (blockIdx.x & 0xffff).
extern __device__ unsigned int g_device_error;

// A wait gives up after g_wait_limit_ns nanoseconds of %globaltimer: by
// default 2 s, far longer than any legitimate wait in these kernels, short
// enough that a broken pipeline ends on its own.  The host can change it
// per device (leafq_set_wait_limit_ns), e.g. to drive a wait to its limit
// in a test.
constexpr unsigned long long kDefaultWaitLimitNs = 2000000000ull;
extern __device__ unsigned long long g_wait_limit_ns;

__device__ __forceinline__ unsigned long long wait_limit_ns() { return g_wait_limit_ns; }

enum WaitSite : unsigned {
    kSiteGemvFull = 1,
    kSiteGemvEmpty = 2,
    kSiteGemmFull = 3,
    kSiteGemmEmpty = 4,
    kSiteGemmAccFull = 5,
    kSiteGemmAccEmpty = 6,
    kSiteW4Full = 7,
    kSiteW4Empty = 8,
    kSiteDecodeFull = 9,
    kSiteDecodeEmpty = 10,
    kSiteDecodeDependency = 11,
    kSiteDecodeCodes = 12,
    kSiteAllGather = 13,
    kSiteCacheRange = 14,  // not a wait: a position outside the KV cache
};

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_device_error(unsigned site) {
    atomicCAS(&g_device_error, 0u, (site << 16) | (blockIdx.x & 0xffffu));
}

__device__ __forceinline__ bool device_error_raised() {
    return *((volatile unsigned int*)&g_device_error) != 0u;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 16-byte asynchronous global -> shared copies (cp.async, L1 bypassed); a
// thread's copies complete at its wait_async_copies().
__device__ __forceinline__ void async_copy16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void commit_async_copies() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void wait_async_copies() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `site`) when the limit passes or another block has
// already reported an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned site) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long start = global_timer_ns();
    for (uint32_t spins = 1;; ++spins) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spins & 255u) == 0u) {
            if (device_error_raised()) return false;
            if (global_timer_ns() - start > wait_limit_ns()) {
                record_device_error(site);
                return false;
            }
        }
    }
}

// ------------------------------------------------------ bulk (TMA) copies
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// 1-D bulk copy global -> shared, completing `bytes` on `bar`.  Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled tensor copy global -> shared (no multicast).  c0 is the inner
// (contiguous) coordinate in elements, c1 the row.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t c0,
                                            int32_t c1, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 2-D tiled tensor store shared -> global (bulk group).  c0 is the inner
// coordinate in elements (its byte offset a multiple of 16), c1 the row;
// both non-negative.  Elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t c0, int32_t c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
                 "r"(c1), "r"(smem_u32(smem_src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until this thread's committed bulk stores have finished reading
// shared memory (the source may be rewritten) / have completed.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// One 32 x 32 fp32 block of an output tile: lane r of the warp holds row r's
// 32 values (v), written into a 4 KB shared-memory tile in the 128-byte
// swizzled layout a TMA store reads (16-byte chunk i of row r at chunk
// i ^ (r % 8): the lanes of each float4 store hit all 32 banks), then
// stored by one TMA from lane 0.  With a 16-row box (map), only lanes 0-15
// hold rows and pass `live`.  The tile's previous store must have finished
// reading (the caller waits before writing again).
__device__ __forceinline__ void store_block_32x32(float* tile, const float (&v)[32], int lane,
                                                  const CUtensorMap* map, int32_t c0, int32_t c1, bool issue,
                                                  bool live) {
    uint8_t* row = reinterpret_cast<uint8_t*>(tile) + lane * 128;
    if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(row + ((i ^ (lane & 7)) << 4)) =
                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && issue) {
        tma_store_2d(map, tile, c0, c1);
        bulk_commit_group();
    }
}

// Prefetch `bytes` (multiple of 16, 16-byte aligned) of global memory into L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------- programmatic dependent launch
// Block until the grid this one depends on has completed and its writes are
// visible.  A no-op when the kernel was launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Let the next grid in the stream start launching (its own
// grid_dependency_wait still waits for this whole grid to finish).
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ bool elect_one_sync() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
        "elect.sync r|p, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Per-token dynamic INT8 code (decoder.cpp:618-627): round half to even of
// value * multiplier, saturated; multiplier = 1 / max(absmax / 127, 1e-12).
__device__ __forceinline__ int8_t act_code(float value, float multiplier) {
    int r = __float2int_rn(__fmul_rn(value, multiplier));
    r = r > 127 ? 127 : (r < -128 ? -128 : r);
    return static_cast<int8_t>(r);
}

// ------------------------------------------------------ packed FP32 pairs
// Two floats in one 64-bit register and the sm_100 paired instructions:
// each half is an IEEE round-to-nearest operation of its own (no
// contraction, subnormals kept), two results per issue slot.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 unpack2(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// Named barriers (ids 1-15; 0 is __syncthreads): `count` threads, whole warps.
__device__ __forceinline__ void bar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// --------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, signed int8 inputs, int32 accumulators.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tcgen05_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tcgen05_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
// Fields (sm_100 UMMA smem descriptor): start address >> 4 in [0,14),
// leading byte offset (unused for swizzled K-major, 1) in [16,30), stride
// byte offset 1024 >> 4 in [32,46), version 1 in [46,48), base offset 0,
// layout type 2 (128-byte swizzle) in [61,64).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((smem_addr >> 4) & 0x3fffu);
    desc |= static_cast<uint64_t>(1u) << 16;
    desc |= static_cast<uint64_t>(1024u >> 4) << 32;
    desc |= static_cast<uint64_t>(1u) << 46;
    desc |= static_cast<uint64_t>(2u) << 61;
    return desc;
}

// Instruction descriptor for kind::i8: int32 accumulator (2) in [4,6), A and
// B signed int8 (1) in [7,10) and [10,13), both K-major (bits 15, 16 = 0),
// N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_i8(uint32_t m, uint32_t n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ------------------------------------------------ CTA pairs (2-SM MMA)
// A cluster of two CTAs on two SMs: the leader (rank 0) issues
// tcgen05.mma.cta_group::2 over both CTAs' shared-memory halves.  No copy
// here uses multicast; only tcgen05.commit multicasts its arrival.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Shared::cluster address of `local` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// Maximum over the full warp (every lane must call it).  Like fmaxf, a NaN
// operand is dropped in favour of a number.
__device__ __forceinline__ float warp_max_f32(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// A float in the shared memory of a CTA of this cluster (shared::cluster
// address from mapa_shared).
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// All threads of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// 2-D tiled load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (`mbar` a shared::cluster
// address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint32_t mbar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
        "l"(map), "r"(c0), "r"(c1), "r"(mbar), "l"(policy)
        : "memory");
}

// Arrive on an mbarrier of either CTA (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t mbar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(mbar) : "memory");
}

// TMEM allocation for a CTA pair: one warp of each CTA, the same warp index
// and the same destination offset in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[each CTA's half of M] * B[both CTAs' halves of N]^T.
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask`
// when the pair's previously issued MMAs have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// 2-D tensor map over a row-major uint8 [outer, inner] matrix (inner
// contiguous, a multiple of 16 bytes) with 128-byte swizzle and box
// [box_outer, box_inner]; out-of-range elements load as zero.  Host side.
int make_tma_map_u8(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_inner,
                    int box_outer);
// The same for a row-major fp32 [outer, inner] matrix (inner a multiple of
// 4), box [box_rows (16 or 32) rows, 32 floats], 128-byte swizzle: the
// output blocks of store_block_32x32.
int make_tma_map_f32_out(CUtensorMap* map, const void* base, int64_t inner, int64_t outer, int box_rows);

// Instruction descriptor for kind::i8 with the B operand MN-major (bit 16):
// B tiles hold rows of N contiguous, as a [k, n] matrix is stored.
__host__ __device__ constexpr uint32_t umma_idesc_i8_bmn(uint32_t m, uint32_t n) {
    return umma_idesc_i8(m, n) | (1u << 16);
}

// Shared-memory descriptor for an MN-major operand tile written by TMA with
// 128-byte swizzle in boxes of [rows of K, 128 bytes of N]: 8-row K groups
// 1024 bytes apart (stride byte offset), 128-column N blocks `lbo` bytes
// apart (leading byte offset), layout type 2.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t smem_addr, uint32_t lbo) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((smem_addr >> 4) & 0x3fffu);
    desc |= static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16;
    desc |= static_cast<uint64_t>(1024u >> 4) << 32;
    desc |= static_cast<uint64_t>(1u) << 46;
    desc |= static_cast<uint64_t>(2u) << 61;
    return desc;
}

// ------------------------------------------------ peer-memory all-gather
// One flag-in-data word {value, tag} of gathered element (token, local_row),
// stored into every rank's receive buffer.  The 8-byte store is single-copy
// atomic, so a reader that sees the tag also sees the value; no fence.
__device__ __forceinline__ void peer_store(const PeerStore& p, uint32_t tag, int64_t token,
                                           int64_t local_row, float v) {
    const int64_t idx = (int64_t)(tag & 1u) * p.half + token * p.rows + p.row_offset + local_row;
    const unsigned long long word =
        (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v);
    for (int g = 0; g < p.world; ++g)
        asm volatile("st.volatile.global.b64 [%0], %1;" ::"l"(p.dst[g] + idx), "l"(word) : "memory");
}

}  // namespace leafq
