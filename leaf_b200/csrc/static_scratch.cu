// leafq_linear_w8a8_static_scratch: the per-row W8A8 prefill linear
// (quantise into scratch, then the tcgen05 GEMM) for callers that cannot
// allocate device memory.
//
// Why: leafq_linear's many-token path needs a workspace for the int8 codes
// and token scales, and the caller has to allocate it.  Some callers cannot:
// a plugin running under a host runtime that owns all device memory and
// hands out none, a latency-critical serving loop that may not touch the
// allocator after start-up, or an embedder with a fixed memory budget where
// an allocation could fail mid-request.  This entry point keeps its scratch
// in a file-scope device array instead, so a call allocates nothing.
//
// Limits and sharing:
//   * codes: tokens * cols <= kStaticCodeBytes (8 MiB); token scales:
//     tokens <= kStaticMaxTokens (16384).  Larger calls are rejected with
//     LEAFQ_ERR_INVALID before anything is launched.
//   * Every GPU that loads the library holds the array (8 MiB + 64 KiB)
//     until the process exits.
//   * All calls on a device share the one array.  Each call overwrites the
//     part it uses before reading it (nothing has to start at zero), so
//     back-to-back calls on one stream are fine; calls that overlap on the
//     GPU (different streams, no ordering between them) race on the array.
//   * The array's host-side name is only a stand-in; its device address is
//     looked up once per device (cudaGetSymbolAddress, with that device
//     current) by the first call on that device.  Make that first call
//     before any stream capture.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr size_t kStaticCodeBytes = size_t(8) << 20;
constexpr size_t kStaticMaxTokens = 16384;
constexpr size_t kStaticScaleBytes = kStaticMaxTokens * sizeof(float);

static __device__ __align__(256) uint8_t g_static_scratch[kStaticCodeBytes + kStaticScaleBytes];

// Device address of g_static_scratch on the current device, looked up once
// per device.
int static_scratch_address(uint8_t** address) {
    static std::mutex mutex;
    static std::unordered_map<int, uint8_t*> cache;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return cuda_status(err, "leafq_linear_w8a8_static_scratch: cudaGetDevice");
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(device);
    if (it != cache.end()) {
        *address = it->second;
        return LEAFQ_OK;
    }
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess)
        return cuda_status(err, "leafq_linear_w8a8_static_scratch: cudaGetSymbolAddress");
    if (ptr == nullptr) {
        set_error("leafq_linear_w8a8_static_scratch: the scratch array has no device address");
        return LEAFQ_ERR_CUDA;
    }
    cache[device] = static_cast<uint8_t*>(ptr);
    *address = static_cast<uint8_t*>(ptr);
    return LEAFQ_OK;
}

}  // namespace
}  // namespace leafq

using namespace leafq;

extern "C" int leafq_linear_w8a8_static_scratch(void* stream, const float* x, int64_t tokens,
                                                int64_t cols, const int8_t* weight,
                                                const float* weight_scales, int64_t rows,
                                                const float* bias, float* y, uint32_t flags) {
    clear_error();
    if (tokens < 0 || cols <= 0 || rows < 0) {
        set_error("leafq_linear_w8a8_static_scratch: tokens and rows must be non-negative, cols positive");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    if (!x || !weight || !weight_scales || !y) {
        set_error("leafq_linear_w8a8_static_scratch: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    if (static_cast<size_t>(tokens) > kStaticMaxTokens ||
        static_cast<size_t>(tokens) * static_cast<size_t>(cols) > kStaticCodeBytes) {
        set_error("leafq_linear_w8a8_static_scratch: tokens * cols = " +
                  std::to_string(tokens * cols) + " exceeds the static scratch (at most " +
                  std::to_string(kStaticCodeBytes) + " code bytes and " +
                  std::to_string(kStaticMaxTokens) + " tokens); use leafq_linear with a workspace");
        return LEAFQ_ERR_INVALID;
    }
    if (!gemm_tc_supported(tokens, cols, rows, 8, cols, weight)) {
        set_error("leafq_linear_w8a8_static_scratch: needs per-row INT8 weights with cols a multiple "
                  "of 16, cols >= 128 and a 16-byte aligned weight");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    uint8_t* base = nullptr;
    int st = static_scratch_address(&base);
    if (st) return st;
    int8_t* q = reinterpret_cast<int8_t*>(base);
    float* sx = reinterpret_cast<float*>(base + kStaticCodeBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    st = launch_quantize_act(s, x, tokens, cols, q, sx, pdl);
    if (st) return st;
    return launch_gemm_tc(s, q, sx, tokens, cols, weight, weight_scales, rows, bias, y, pdl);
}
