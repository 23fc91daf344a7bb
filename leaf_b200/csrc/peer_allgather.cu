// Peer-memory all-gather along N for N-sharded linears (one process per GPU).
//
// Every rank owns rows [row_begin, row_begin + local_rows) of a linear's
// output (output rows are independent, decoder.cpp:1109, so the split is
// bit-exact).  Instead of a separate collective, the kernel that produces a
// row stores it straight into every rank's receive buffer over NVLink as one
// 8-byte flag-in-data word {fp32 value, 32-bit run tag}.  A small collect
// kernel on each rank polls its own buffer until every word of the gathered
// [tokens, rows] output carries the current run's tag (bounded: 2 s, then
// the device error word is set and NaN is written), unpacks the values, and
// its last block advances the rank's run counter.
//
// Receive buffers are plain cudaMalloc memory shared through CUDA IPC
// handles; nothing here uses multicast objects or TMA.  Two halves alternate
// with the tag's parity: rank A can start run k+2 (which rewrites half k&1
// on rank B) only after its run k+1 collected B's rows of run k+1, which B
// stores only after its run k finished reading half k&1.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "leafq_device.cuh"
#include "leafq_internal.h"

static_assert(sizeof(cudaIpcMemHandle_t) == LEAFQ_IPC_HANDLE_BYTES, "IPC handle size");

struct leafq_allgather {  // leafq_allgather_t
    int rank = 0;
    int world = 0;
    int device = 0;
    int64_t max_elements = 0;
    unsigned long long* recv = nullptr;  // [2][max_elements] tagged words
    unsigned int* counters = nullptr;    // [0] run tag, [1] collect blocks done
    float* scratch = nullptr;            // local rows of the unfused path
    void* opened[leafq::kMaxPeers] = {};
    unsigned long long* dst[leafq::kMaxPeers] = {};
    bool connected = false;
};

namespace leafq {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t n) {
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 4;
    return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

__global__ void __launch_bounds__(kThreads) allgather_send_kernel(const float* __restrict__ local,
                                                                  int64_t tokens, int64_t local_rows,
                                                                  const PeerStore p) {
    const uint32_t tag = *reinterpret_cast<const volatile uint32_t*>(p.epoch);
    const int64_t n = tokens * local_rows;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / local_rows;
        peer_store(p, tag, t, i - t * local_rows, __ldg(local + i));
    }
}

__global__ void __launch_bounds__(kThreads) allgather_collect_kernel(
    const unsigned long long* __restrict__ recv, int64_t half, int64_t n, float* __restrict__ out,
    unsigned int* counters) {
    const uint32_t tag = *reinterpret_cast<volatile uint32_t*>(counters);
    const unsigned long long* base = recv + (int64_t)(tag & 1u) * half;
    const unsigned long long start = global_timer_ns();
    bool gave_up = false;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        unsigned long long w;
        while (true) {
            asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(w) : "l"(base + i) : "memory");
            if (static_cast<uint32_t>(w >> 32) == tag) break;
            if (gave_up || global_timer_ns() - start > wait_limit_ns()) {
                if (!gave_up) record_device_error(kSiteAllGather);
                gave_up = true;
                w = 0x7fc00000ull;  // NaN: a peer never stored this word
                break;
            }
        }
        out[i] = __uint_as_float(static_cast<uint32_t>(w));
    }
    // Every block has read the tag; the last one to finish advances it.
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&counters[1], 1u) == gridDim.x - 1) {
            counters[1] = 0;
            atomicAdd(&counters[0], 1u);
        }
    }
}

PeerStore peer_for(const leafq_allgather* ag, int64_t row_begin, int64_t rows) {
    PeerStore p = {};
    for (int g = 0; g < ag->world; ++g) p.dst[g] = ag->dst[g];
    p.epoch = ag->counters;
    p.world = ag->world;
    p.half = ag->max_elements;
    p.row_offset = row_begin;
    p.rows = rows;
    return p;
}

int check_run(const leafq_allgather* ag, int64_t tokens, int64_t local_rows, int64_t row_begin,
              int64_t rows, const void* out, const char* who) {
    if (!ag || !ag->connected) {
        set_error(std::string(who) + ": all-gather is not connected");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens < 0 || rows < 0 || local_rows < 0 || row_begin < 0 || row_begin + local_rows > rows) {
        set_error(std::string(who) + ": rows [row_begin, row_begin + local_rows) must lie in [0, rows)");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens * rows > ag->max_elements) {
        set_error(std::string(who) + ": tokens x rows exceeds the all-gather capacity of " +
                  std::to_string(ag->max_elements));
        return LEAFQ_ERR_INVALID;
    }
    if (tokens * rows > 0 && !out) {
        set_error(std::string(who) + ": null output");
        return LEAFQ_ERR_INVALID;
    }
    int dev = -1;
    cudaGetDevice(&dev);
    if (dev != ag->device) {
        set_error(std::string(who) + ": the current device is not the all-gather's device");
        return LEAFQ_ERR_INVALID;
    }
    return LEAFQ_OK;
}

int collect(cudaStream_t s, leafq_allgather* ag, int64_t n, float* out) {
    return launch(allgather_collect_kernel, dim3(grid_for(n)), dim3(kThreads), 0, s, false,
                  "allgather_collect", ag->recv, ag->max_elements, n, out, ag->counters);
}

}  // namespace
}  // namespace leafq

using namespace leafq;

extern "C" {

int leafq_allgather_init(int rank, int world, int64_t max_elements, leafq_allgather** out,
                         void* ipc_handle) {
    clear_error();
    if (!out || !ipc_handle || world < 1 || world > kMaxPeers || rank < 0 || rank >= world ||
        max_elements < 1) {
        set_error("leafq_allgather_init: invalid arguments (world 1..8, rank < world, capacity > 0)");
        return LEAFQ_ERR_INVALID;
    }
    *out = nullptr;
    auto* ag = new leafq_allgather();
    ag->rank = rank;
    ag->world = world;
    ag->max_elements = max_elements;
    cudaGetDevice(&ag->device);
    const size_t recv_bytes = 2 * static_cast<size_t>(max_elements) * sizeof(unsigned long long);
    int st = cuda_status(cudaMalloc(&ag->recv, recv_bytes), "leafq_allgather_init");
    if (!st) st = cuda_status(cudaMalloc(&ag->counters, 2 * sizeof(unsigned int)), "leafq_allgather_init");
    if (!st) st = cuda_status(cudaMalloc(&ag->scratch, static_cast<size_t>(max_elements) * sizeof(float)),
                              "leafq_allgather_init");
    // Tags start at 1 so the zeroed buffer never reads as delivered.
    const unsigned int init[2] = {1u, 0u};
    if (!st) st = cuda_status(cudaMemset(ag->recv, 0, recv_bytes), "leafq_allgather_init");
    if (!st) st = cuda_status(cudaMemcpy(ag->counters, init, sizeof(init), cudaMemcpyHostToDevice),
                              "leafq_allgather_init");
    cudaIpcMemHandle_t handle;
    if (!st) st = cuda_status(cudaIpcGetMemHandle(&handle, ag->recv), "leafq_allgather_init");
    if (!st) st = cuda_status(cudaDeviceSynchronize(), "leafq_allgather_init");
    if (st) {
        cudaFree(ag->recv);
        cudaFree(ag->counters);
        cudaFree(ag->scratch);
        delete ag;
        return st;
    }
    std::memcpy(ipc_handle, &handle, sizeof(handle));
    ag->dst[rank] = ag->recv;
    *out = ag;
    return LEAFQ_OK;
}

int leafq_allgather_connect(leafq_allgather* ag, const void* handles) {
    clear_error();
    if (!ag || !handles || ag->connected) {
        set_error("leafq_allgather_connect: invalid arguments or already connected");
        return LEAFQ_ERR_INVALID;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ag->device);
    int st = LEAFQ_OK;
    for (int g = 0; g < ag->world && !st; ++g) {
        if (g == ag->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)g * LEAFQ_IPC_HANDLE_BYTES,
                    sizeof(h));
        void* p = nullptr;
        st = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess),
                         "leafq_allgather_connect");
        if (!st) {
            ag->opened[g] = p;
            ag->dst[g] = static_cast<unsigned long long*>(p);
        }
    }
    if (st) {
        for (int g = 0; g < ag->world; ++g)
            if (ag->opened[g]) {
                cudaIpcCloseMemHandle(ag->opened[g]);
                ag->opened[g] = nullptr;
                ag->dst[g] = nullptr;
            }
    } else {
        ag->connected = true;
    }
    cudaSetDevice(prev);
    return st;
}

int leafq_allgather_run(void* stream, leafq_allgather* ag, const float* local, int64_t tokens,
                        int64_t local_rows, int64_t row_begin, int64_t rows, float* out) {
    clear_error();
    int st = check_run(ag, tokens, local_rows, row_begin, rows, out, "leafq_allgather_run");
    if (st) return st;
    if (tokens * local_rows > 0 && !local) {
        set_error("leafq_allgather_run: null local rows");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (tokens * local_rows > 0) {
        const PeerStore p = peer_for(ag, row_begin, rows);
        st = launch(allgather_send_kernel, dim3(grid_for(tokens * local_rows)), dim3(kThreads), 0, s,
                    false, "allgather_send", local, tokens, local_rows, p);
        if (st) return st;
    }
    return collect(s, ag, tokens * rows, out);
}

int leafq_linear_allgather(void* stream, leafq_allgather* ag, const float* x, int64_t tokens,
                           int64_t cols, const void* weight, const float* weight_scales,
                           int64_t local_rows, int64_t row_begin, int64_t rows, int bits,
                           int64_t group, int activation_bits, const float* bias, float* out,
                           void* workspace, size_t workspace_bytes, uint32_t flags) {
    clear_error();
    int st = check_run(ag, tokens, local_rows, row_begin, rows, out, "leafq_linear_allgather");
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    if (tokens > 0 && local_rows > 0 && activation_bits == 8 && weight && weight_scales && x &&
        gemv_w8a8_supported(tokens, cols, bits, group, weight, x)) {
        // Fused: the GEMV epilogue stores into every rank's receive buffer.
        const PeerStore p = peer_for(ag, row_begin, rows);
        st = launch_gemv_w8a8(s, x, tokens, cols, static_cast<const int8_t*>(weight), weight_scales,
                              local_rows, bias, nullptr, pdl, &p);
        if (st) return st;
        return collect(s, ag, tokens * rows, out);
    }
    // Other paths: the linear into local scratch, then the peer stores.
    st = leafq_linear(stream, x, tokens, cols, weight, weight_scales, local_rows, bits, group,
                      activation_bits, bias, ag->scratch, workspace, workspace_bytes, flags);
    if (st) return st;
    return leafq_allgather_run(stream, ag, ag->scratch, tokens, local_rows, row_begin, rows, out);
}

int leafq_allgather_destroy(leafq_allgather* ag) {
    clear_error();
    if (!ag) return LEAFQ_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ag->device);
    cudaDeviceSynchronize();
    for (int g = 0; g < ag->world; ++g)
        if (ag->opened[g]) cudaIpcCloseMemHandle(ag->opened[g]);
    cudaFree(ag->recv);
    cudaFree(ag->counters);
    cudaFree(ag->scratch);
    delete ag;
    cudaSetDevice(prev);
    return LEAFQ_OK;
}

}  // extern "C"
