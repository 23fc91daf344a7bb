// The C ABI (include/leafq.h): argument checks, path selection, status codes.
//
// Path selection follows Decoder::Impl::linear (decoder.cpp:1020-1232):
//   activation_bits 8, bits 8/4  -> integer path
//     tokens <= 8, per-row INT8     fused quantise + bulk-TMA GEMV
//     tokens  > 8, per-row INT8     quantise + tcgen05 GEMM
//     otherwise (groups, INT4)      quantise + grouped integer kernel
//   activation_bits 32           -> weight-only path in dot_avx order
//     one token, INT4, group 32/64/128  streaming W4A32 GEMV
//     otherwise                         generic exact-order kernel
// Nothing here allocates device memory; the two-kernel paths put the codes
// and token scales in the caller's workspace.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>
#include <string>
#include <unordered_map>

#include "leafq_device.cuh"
#include "leafq_internal.h"

namespace leafq {

__device__ unsigned int g_device_error = 0;
__device__ unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;

namespace {
thread_local std::string t_error;
constexpr int kGemvMaxTokens = 8;

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct DeviceInfo {
    int sms = 0;
    int smem = 0;
};

DeviceInfo& device_info() {
    static std::mutex mutex;
    static std::unordered_map<int, DeviceInfo> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mutex);
    DeviceInfo& info = cache[dev];
    if (info.sms == 0) {
        cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&info.smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (info.sms <= 0) info.sms = 1;
    }
    return info;
}

bool integer_path_uses_gemv(int64_t tokens, int64_t cols, int bits, int64_t group) {
    return bits == 8 && group == cols && tokens >= 1 && tokens <= kGemvMaxTokens && cols % 16 == 0 &&
           (tokens <= 1 ? 1 : tokens <= 2 ? 2 : tokens <= 4 ? 4 : 8) * cols <= 64 * 1024;
}

int check_weight(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                 int activation_bits) {
    if (tokens < 0 || cols <= 0 || rows < 0) {
        set_error("tokens, cols and rows must be non-negative (cols positive)");
        return LEAFQ_ERR_INVALID;
    }
    if (activation_bits != 8 && activation_bits != 32) {
        set_error("activation bits must be 8 or 32");  // decoder.cpp:750
        return LEAFQ_ERR_INVALID;
    }
    if (bits != 4 && bits != 8 && bits != 32) {
        set_error("weight bits must be 32, 8 or 4");
        return LEAFQ_ERR_INVALID;
    }
    if (bits == 32) return LEAFQ_OK;
    // decoder.cpp:864-868: a positive group dividing cols; INT4 needs even
    // cols and an even group.
    if (group <= 0 || cols % group != 0 || (bits == 4 && (cols % 2 != 0 || group % 2 != 0))) {
        set_error("invalid quantization group " + std::to_string(group) + " for width " +
                  std::to_string(cols));
        return LEAFQ_ERR_INVALID;
    }
    // decoder.cpp:1025: int32 accumulation is exact only up to this width.
    if (activation_bits == 8 && group > 131000) {
        set_error("integer accumulation exceeds safe input width");
        return LEAFQ_ERR_INVALID;
    }
    return LEAFQ_OK;
}

}  // namespace

bool integer_path_takes_gemv(int64_t tokens, int64_t cols, int bits, int64_t group, const void* weight,
                             const float* x) {
    return integer_path_uses_gemv(tokens, cols, bits, group) &&
           gemv_w8a8_supported(tokens, cols, bits, group, weight, x);
}

bool integer_path_takes_gemm_tc(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                                const void* weight) {
    return tokens > kGemvMaxTokens && gemm_tc_supported(tokens, cols, rows, bits, group, weight);
}

void set_error(const std::string& message) { t_error = message; }
void clear_error() { t_error.clear(); }

int cuda_status(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return LEAFQ_OK;
    set_error(std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")");
    return LEAFQ_ERR_CUDA;
}

int sm_count() { return device_info().sms; }
int max_smem_per_block() { return device_info().smem; }

int allow_smem(const void* kernel, size_t bytes, const char* what) {
    static std::mutex mutex;
    static std::unordered_map<const void*, size_t> done;
    int dev = 0;
    cudaGetDevice(&dev);
    const void* key = reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(kernel) ^
                                                    (static_cast<uintptr_t>(dev) << 56));
    {
        std::lock_guard<std::mutex> lock(mutex);
        auto it = done.find(key);
        if (it != done.end() && it->second >= bytes) return LEAFQ_OK;
    }
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(bytes));
    if (err != cudaSuccess) return cuda_status(err, what);
    std::lock_guard<std::mutex> lock(mutex);
    size_t& have = done[key];
    if (bytes > have) have = bytes;
    return LEAFQ_OK;
}

}  // namespace leafq

using namespace leafq;

extern "C" {

const char* leafq_last_error(void) { return t_error.c_str(); }

int leafq_version(void) { return 100; }

int leafq_device_status(void) {
    clear_error();
    cudaError_t err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return cuda_status(err, "leafq_device_status");
    unsigned int word = 0;
    err = cudaMemcpyFromSymbol(&word, g_device_error, sizeof(word));
    if (err != cudaSuccess) return cuda_status(err, "leafq_device_status");
    if (word == 0) return LEAFQ_OK;
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    if ((word >> 16) == kSiteCacheRange) {
        set_error("a cache position was outside the KV cache (block " + std::to_string(word & 0xffffu) +
                  "); the kernel skipped it");
        return LEAFQ_ERR_INVALID;
    }
    set_error("a device wait timed out (site " + std::to_string(word >> 16) + ", block " +
              std::to_string(word & 0xffffu) + ")");
    return LEAFQ_ERR_TIMEOUT;
}

int leafq_set_wait_limit_ns(uint64_t nanoseconds) {
    clear_error();
    const unsigned long long limit = nanoseconds == 0 ? kDefaultWaitLimitNs : nanoseconds;
    if (limit < 1000ull || limit > 60000000000ull) {
        set_error("leafq_set_wait_limit_ns: the limit must be 0 (default, 2 s) or 1 us .. 60 s");
        return LEAFQ_ERR_INVALID;
    }
    // Finish the kernels in flight first, so none sees the limit change in
    // the middle of a wait.
    cudaError_t err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_wait_limit_ns, &limit, sizeof(limit));
    return cuda_status(err, "leafq_set_wait_limit_ns");
}

int leafq_quantize_act(void* stream, const float* x, int64_t tokens, int64_t cols, int8_t* q,
                       float* scales) {
    clear_error();
    if (tokens < 0 || cols <= 0 || (tokens > 0 && (!x || !q || !scales))) {
        set_error("leafq_quantize_act: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens > 0x7fffffff) {
        set_error("leafq_quantize_act: too many tokens");
        return LEAFQ_ERR_INVALID;
    }
    return launch_quantize_act(static_cast<cudaStream_t>(stream), x, tokens, cols, q, scales, false);
}

size_t leafq_linear_workspace_bytes(int64_t tokens, int64_t cols, int bits, int64_t group,
                                    int activation_bits) {
    if (activation_bits != 8 || tokens <= 0 || cols <= 0) return 0;
    if (integer_path_uses_gemv(tokens, cols, bits, group)) return 0;
    return align256(static_cast<size_t>(tokens) * static_cast<size_t>(cols)) +
           align256(static_cast<size_t>(tokens) * sizeof(float));
}

int leafq_linear(void* stream, const float* x, int64_t tokens, int64_t cols, const void* weight,
                 const float* weight_scales, int64_t rows, int bits, int64_t group,
                 int activation_bits, const float* bias, float* y, void* workspace,
                 size_t workspace_bytes, uint32_t flags) {
    clear_error();
    int st = check_weight(tokens, cols, rows, bits, group, activation_bits);
    if (st) return st;
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    if (!x || !weight || !y || (bits != 32 && !weight_scales)) {
        set_error("leafq_linear: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    const bool fused = (flags & LEAFQ_FLAG_VNNI_ROUNDING) == 0;
    if (activation_bits == 8) {
        if (bits == 32) {
            set_error("W32A8 is not a reference path (FP32 weights always use FP32 activations)");
            return LEAFQ_ERR_INVALID;
        }
        if (integer_path_uses_gemv(tokens, cols, bits, group) &&
            gemv_w8a8_supported(tokens, cols, bits, group, weight, x))
            return launch_gemv_w8a8(s, x, tokens, cols, static_cast<const int8_t*>(weight),
                                    weight_scales, rows, bias, y, pdl);
        const size_t need = align256(static_cast<size_t>(tokens) * static_cast<size_t>(cols)) +
                            align256(static_cast<size_t>(tokens) * sizeof(float));
        if (!workspace || workspace_bytes < need ||
            (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
            set_error("leafq_linear: this shape needs " + std::to_string(need) +
                      " bytes of 256-byte aligned workspace");
            return LEAFQ_ERR_INVALID;
        }
        int8_t* q = static_cast<int8_t*>(workspace);
        float* sx = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                             align256(static_cast<size_t>(tokens) * cols));
        st = launch_quantize_act(s, x, tokens, cols, q, sx, pdl);
        if (st) return st;
        if (tokens > kGemvMaxTokens && gemm_tc_supported(tokens, cols, rows, bits, group, weight))
            return launch_gemm_tc(s, q, sx, tokens, cols, static_cast<const int8_t*>(weight),
                                  weight_scales, rows, bias, y, pdl);
        return launch_linear_int_q(s, q, sx, tokens, cols, weight, weight_scales, rows, bits, group,
                                   bias, y, nullptr, fused, pdl);
    }
    if (gemv_w4a32_fast_supported(tokens, cols, bits, group, weight, weight_scales) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0))
        return launch_gemv_w4a32_fast(s, x, cols, static_cast<const uint8_t*>(weight), weight_scales,
                                      rows, group, bias, y, pdl);
    return launch_linear_f32act(s, x, tokens, cols, weight, weight_scales, rows, bits, group, bias, y,
                                pdl);
}

int leafq_linear_int_q(void* stream, const int8_t* q, const float* scales, int64_t tokens,
                       int64_t cols, const void* weight, const float* weight_scales, int64_t rows,
                       int bits, int64_t group, const float* bias, float* y, int32_t* acc,
                       uint32_t flags) {
    clear_error();
    int st = check_weight(tokens, cols, rows, bits, group, 8);
    if (st) return st;
    if (bits == 32) {
        set_error("leafq_linear_int_q: weights must be INT8 or INT4");
        return LEAFQ_ERR_INVALID;
    }
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    if (!q || !scales || !weight || !weight_scales || !y) {
        set_error("leafq_linear_int_q: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    if (!acc && tokens > kGemvMaxTokens && gemm_tc_supported(tokens, cols, rows, bits, group, weight) &&
        aligned16(q))
        return launch_gemm_tc(s, q, scales, tokens, cols, static_cast<const int8_t*>(weight),
                              weight_scales, rows, bias, y, pdl);
    return launch_linear_int_q(s, q, scales, tokens, cols, weight, weight_scales, rows, bits, group,
                               bias, y, acc, (flags & LEAFQ_FLAG_VNNI_ROUNDING) == 0, pdl);
}

int leafq_graph_quantize(void* stream, const float* x, int64_t count, float scale, int8_t* q,
                         int32_t* error_flag) {
    clear_error();
    if (!std::isfinite(scale) || !(scale > 0.0f)) {
        set_error("invalid activation scale");  // executor.cpp:221
        return LEAFQ_ERR_INVALID;
    }
    if (count < 0 || (count > 0 && (!x || !q))) {
        set_error("leafq_graph_quantize: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    return launch_graph_quantize(static_cast<cudaStream_t>(stream), x, count, scale, q, error_flag);
}

int leafq_gemm_i8_per_channel(void* stream, const int8_t* a, const int8_t* b, const float* bias,
                              float input_scale, const float* weight_scales, float* out, int64_t m,
                              int64_t k, int64_t n, int activation) {
    clear_error();
    if (m < 0 || k < 0 || n < 0 || (m > 0 && n > 0 && (!a || !b || !weight_scales || !out))) {
        set_error("leafq_gemm_i8_per_channel: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    if (activation != 0 && activation != 1) {
        set_error("leafq_gemm_i8_per_channel: activation must be 0 (none) or 1 (ReLU)");
        return LEAFQ_ERR_INVALID;
    }
    if (m > 65535LL * 64) {
        set_error("leafq_gemm_i8_per_channel: m too large");
        return LEAFQ_ERR_INVALID;
    }
    // executor.cpp:573: int32 accumulation is exact only while
    // k <= INT32_MAX / (127 * 127); the reference switches to int64 beyond.
    if (k > 2147483647LL / (127 * 127)) {
        set_error("leafq_gemm_i8_per_channel: k exceeds the exact int32 range");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    return launch_gemm_i8_per_channel(static_cast<cudaStream_t>(stream), a, b, bias, input_scale,
                                      weight_scales, out, m, k, n, activation);
}

int leafq_scale_columns(void* stream, const float* x, int64_t tokens, int64_t cols, const float* col_scale,
                        float* y) {
    clear_error();
    if (tokens < 0 || cols <= 0 || (tokens > 0 && (!x || !col_scale || !y))) {
        set_error("leafq_scale_columns: invalid arguments");
        return LEAFQ_ERR_INVALID;
    }
    return launch_scale_columns(static_cast<cudaStream_t>(stream), x, tokens, cols, col_scale, y, false);
}

size_t leafq_linear_smooth_workspace_bytes(int64_t tokens, int64_t cols, int activation_bits) {
    if (tokens <= 0 || cols <= 0) return 0;
    if (activation_bits == 8)
        return align256(static_cast<size_t>(tokens) * static_cast<size_t>(cols)) +
               align256(static_cast<size_t>(tokens) * sizeof(float));
    return align256(static_cast<size_t>(tokens) * static_cast<size_t>(cols) * sizeof(float));
}

int leafq_linear_smooth(void* stream, const float* x, const float* input_scale, int64_t tokens, int64_t cols,
                        const void* weight, const float* weight_scales, int64_t rows, int bits, int64_t group,
                        int activation_bits, const float* bias, float* y, void* workspace,
                        size_t workspace_bytes, uint32_t flags) {
    if (!input_scale)
        return leafq_linear(stream, x, tokens, cols, weight, weight_scales, rows, bits, group, activation_bits,
                            bias, y, workspace, workspace_bytes, flags);
    clear_error();
    int st = check_weight(tokens, cols, rows, bits, group, activation_bits);
    if (st) return st;
    if (tokens == 0 || rows == 0) return LEAFQ_OK;
    if (!x || !weight || !y || (bits != 32 && !weight_scales)) {
        set_error("leafq_linear_smooth: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    if (activation_bits == 8 && bits == 32) {
        set_error("W32A8 is not a reference path (FP32 weights always use FP32 activations)");
        return LEAFQ_ERR_INVALID;
    }
    const size_t need = leafq_linear_smooth_workspace_bytes(tokens, cols, activation_bits);
    if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) {
        set_error("leafq_linear_smooth: this shape needs " + std::to_string(need) +
                  " bytes of 256-byte aligned workspace");
        return LEAFQ_ERR_INVALID;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool pdl = (flags & LEAFQ_FLAG_PDL) != 0;
    if (activation_bits == 8) {
        // The scaling runs inside the quantiser; then the integer linear.
        int8_t* q = static_cast<int8_t*>(workspace);
        float* sx = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) +
                                             align256(static_cast<size_t>(tokens) * cols));
        st = launch_quantize_act(s, x, tokens, cols, q, sx, pdl, input_scale);
        if (st) return st;
        if (tokens > kGemvMaxTokens && gemm_tc_supported(tokens, cols, rows, bits, group, weight))
            return launch_gemm_tc(s, q, sx, tokens, cols, static_cast<const int8_t*>(weight), weight_scales, rows,
                                  bias, y, pdl);
        return launch_linear_int_q(s, q, sx, tokens, cols, weight, weight_scales, rows, bits, group, bias, y,
                                   nullptr, (flags & LEAFQ_FLAG_VNNI_ROUNDING) == 0, pdl);
    }
    float* scaled = static_cast<float*>(workspace);
    st = launch_scale_columns(s, x, tokens, cols, input_scale, scaled, pdl);
    if (st) return st;
    if (gemv_w4a32_fast_supported(tokens, cols, bits, group, weight, weight_scales))
        return launch_gemv_w4a32_fast(s, scaled, cols, static_cast<const uint8_t*>(weight), weight_scales, rows,
                                      group, bias, y, pdl);
    return launch_linear_f32act(s, scaled, tokens, cols, weight, weight_scales, rows, bits, group, bias, y, pdl);
}

size_t leafq_graph_linear_workspace_bytes(int64_t m, int64_t k) {
    if (m <= 0 || k <= 0) return 0;
    return align256(static_cast<size_t>(m) * static_cast<size_t>(k));
}

int leafq_graph_linear(void* stream, const float* a, int64_t m, int64_t k, int trans_a, const int8_t* weight,
                       int64_t n, int trans_b, float input_scale, const float* weight_scales, float alpha,
                       float beta, const float* c, int c_kind, int activation, float* out, void* workspace,
                       size_t workspace_bytes, int32_t* error_flag) {
    clear_error();
    if (m < 0 || k <= 0 || n < 0 || m > 65535LL * 64) {
        set_error("leafq_graph_linear: invalid dimensions");
        return LEAFQ_ERR_INVALID;
    }
    if (!std::isfinite(input_scale) || !(input_scale > 0.0f)) {
        set_error("invalid activation scale");  // executor.cpp:221
        return LEAFQ_ERR_INVALID;
    }
    if (c && (c_kind < 1 || c_kind > 3)) {
        set_error("unsupported INT8 Gemm C broadcast shape");  // executor.cpp:601-603
        return LEAFQ_ERR_INVALID;
    }
    if (activation < 0 || activation > 3) {
        set_error("leaf::Executor: unsupported fused activation");  // executor.cpp:241
        return LEAFQ_ERR_INVALID;
    }
    if (k > 2147483647LL / (127 * 127)) {
        set_error("leafq_graph_linear: k exceeds the exact int32 range");
        return LEAFQ_ERR_UNSUPPORTED;
    }
    if (m == 0 || n == 0) return LEAFQ_OK;
    if (!a || !weight || !weight_scales || !out) {
        set_error("leafq_graph_linear: null pointer");
        return LEAFQ_ERR_INVALID;
    }
    if (!workspace || workspace_bytes < leafq_graph_linear_workspace_bytes(m, k)) {
        set_error("leafq_graph_linear: workspace smaller than leafq_graph_linear_workspace_bytes");
        return LEAFQ_ERR_INVALID;
    }
    return launch_graph_linear(static_cast<cudaStream_t>(stream), a, m, k, trans_a ? 1 : 0, weight, n,
                               trans_b ? 1 : 0, input_scale, weight_scales, alpha, beta, c, c_kind, activation,
                               out, static_cast<int8_t*>(workspace), error_flag);
}

}  // extern "C"
