// leafq_linear_w8a8_static_scratch: the per-row W8A8 linear for callers
// that cannot allocate device memory.
//
// Why: leafq_linear's many-token path needs a workspace for the int8 codes
// and token scales, and the caller has to allocate it.  Some callers cannot:
// a plugin running under a host runtime that owns all device memory and
// hands out none, a latency-critical serving loop that may not touch the
// allocator after start-up, or an embedder with a fixed memory budget where
// an allocation could fail mid-request.  This entry point keeps its scratch
// in a file-scope device array instead, so a call allocates nothing.
//
// It takes the kernels leafq_linear takes for the same call: the
// fused-quantisation decode GEMV (1-8 tokens, no scratch at all), else the
// codes and token scales quantised into the array and then the tcgen05 GEMM
// (more than 8 tokens) or the generic integer kernel.
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
//     looked up (cudaGetSymbolAddress, with the device current) by the first
//     call in each CUDA context and cached for that context.  Make that
//     first call before any stream capture.  A device reset destroys the
//     context; the next call then looks the address up again.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <map>
#include <utility>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {
namespace {

constexpr size_t kStaticCodeBytes = size_t(8) << 20;
constexpr size_t kStaticMaxTokens = 16384;
constexpr size_t kStaticScaleBytes = kStaticMaxTokens * sizeof(float);

static __device__ __align__(256) uint8_t g_static_scratch[kStaticCodeBytes + kStaticScaleBytes];

// The calling thread's current CUDA context (driver API through the
// runtime's entry-point query, so the library needs no -lcuda).
using CtxGetCurrentFn = int (*)(void**);

void* current_context() {
    static CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    void* ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != 0) return nullptr;
    return ctx;
}

// Device address of g_static_scratch in the current context, looked up once
// per (device, context).
int static_scratch_address(uint8_t** address) {
    static std::mutex mutex;
    static std::map<std::pair<int, void*>, uint8_t*> cache;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return cuda_status(err, "leafq_linear_w8a8_static_scratch: cudaGetDevice");
    // Before the runtime has made the device's context current there is none
    // (null key); the lookup below creates it, and the next call caches the
    // address again under the real context.
    const std::pair<int, void*> key(device, current_context());
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(key);
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
    cache[key] = static_cast<uint8_t*>(ptr);
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
    if (static_cast<size_t>(tokens) > kStaticMaxTokens) {
        set_error("leafq_linear_w8a8_static_scratch: " + std::to_string(tokens) +
                  " tokens exceed the static scratch's " + std::to_string(kStaticMaxTokens) +
                  " token scales; use leafq_linear with a workspace");
        return LEAFQ_ERR_INVALID;
    }
    // tokens * cols <= kStaticCodeBytes, without forming the product.
    if (static_cast<uint64_t>(cols) > kStaticCodeBytes / static_cast<uint64_t>(tokens)) {
        set_error("leafq_linear_w8a8_static_scratch: " + std::to_string(tokens) + " tokens of " +
                  std::to_string(cols) + " columns exceed the static scratch's " +
                  std::to_string(kStaticCodeBytes) + " code bytes; use leafq_linear with a workspace");
        return LEAFQ_ERR_INVALID;
    }
    if (cols > 131000) {
        set_error("leafq_linear_w8a8_static_scratch: integer accumulation exceeds safe input width");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    // Decode sizes: the fused GEMV quantises in shared memory and needs no
    // scratch.
    if (integer_path_takes_gemv(tokens, cols, 8, cols, weight, x))
        return launch_gemv_w8a8(s, x, tokens, cols, weight, weight_scales, rows, bias, y, pdl);
    uint8_t* base = nullptr;
    int st = static_scratch_address(&base);
    if (st) return st;
    int8_t* q = reinterpret_cast<int8_t*>(base);
    float* sx = reinterpret_cast<float*>(base + kStaticCodeBytes);
    st = launch_quantize_act(s, x, tokens, cols, q, sx, pdl);
    if (st) return st;
    if (integer_path_takes_gemm_tc(tokens, cols, rows, 8, cols, weight))
        return launch_gemm_tc(s, q, sx, tokens, cols, weight, weight_scales, rows, bias, y, pdl);
    return launch_linear_int_q(s, q, sx, tokens, cols, weight, weight_scales, rows, 8, cols, bias, y, nullptr,
                               (flags & LEAFQ_FLAG_VNNI_ROUNDING) == 0, pdl);
}
