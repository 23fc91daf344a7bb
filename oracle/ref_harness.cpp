// Test-only harness: appended (on the compiler's stdin) after the reference's
// unmodified engine/src/decoder.cpp so that its anonymous-namespace CPU kernels
// can be called from Python through a C ABI.  It lives at global scope and
// names the reference symbols with their qualified names.  Nothing here is
// part of the product; it is the "reference" CPU oracle and CPU baseline.
//
// The row loop below follows Decoder::Impl::linear (decoder.cpp:994-1233):
// per-token absmax scale (:1028-1032), quantisation with the reciprocal
// (:1035-1038), rows handed to the reference Workers pool in grains of 32
// (:1109), then the VNNI 2x4 tile (:1183-1200), the AVX2 4x2 tile (:1206-1219)
// or the per-row dot in blocks of 4 tokens (:1221-1231), plus the bias
// (:1229).  The kernels themselves are the reference's.

#include "leaf/kernels/gemm.h"

#include <cstddef>
#include <cstdint>
#include <exception>
#include <string>
#include <vector>

namespace {
namespace lr = leaf::runtime;

thread_local std::string harness_error;

void harness_scales(const float* x, std::size_t tokens, std::size_t cols, float* scales) {
    for (std::size_t t = 0; t < tokens; ++t) {
        float maximum = 0;
        for (std::size_t col = 0; col < cols; ++col)
            maximum = std::max(maximum, std::abs(x[t * cols + col]));
        scales[t] = std::max(maximum / 127.0f, 1e-12f);
    }
}

lr::Weight harness_weight(const void* data, const float* scales, std::size_t rows,
                          std::size_t cols, unsigned bits, std::size_t group) {
    lr::Weight w;
    w.rows = rows; w.cols = cols; w.bits = bits;
    w.group = bits == 32 ? 0 : group;
    w.data = static_cast<const std::uint8_t*>(data);
    w.scales = scales;
    return w;
}

// One persistent pool per thread count, like the decoder's own member pool
// (Decoder::Impl::workers); callers use the harness from one thread.
lr::Workers& harness_pool(unsigned threads) {
    static std::unique_ptr<lr::Workers> pool;
    static unsigned pool_threads = 0;
    if (!pool || pool_threads != threads) {
        pool.reset();
        pool = std::make_unique<lr::Workers>(threads);
        pool_threads = threads;
    }
    return *pool;
}

bool harness_vnni_available() {
#if LEAF_DECODER_VNNI
    return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma") &&
           __builtin_cpu_supports("avxvnni");
#else
    return false;
#endif
}
}  // namespace

extern "C" {

const char* leafref_last_error() { return harness_error.c_str(); }

int leafref_has_vnni() { return harness_vnni_available() ? 1 : 0; }

// Per-token scales plus the int16 codes quantize_input_avx writes (the decode
// and non-VNNI prefill container, decoder.cpp:618-627).
int leafref_quantize_i16(const float* x, std::size_t tokens, std::size_t cols,
                         std::int16_t* q, float* scales) {
    try {
        harness_scales(x, tokens, cols, scales);
        for (std::size_t t = 0; t < tokens; ++t)
            lr::quantize_input_avx(x + t * cols, q + t * cols, cols, 1.0f / scales[t]);
        return 0;
    } catch (const std::exception& e) { harness_error = e.what(); return 1; }
}

// The uint8 (q + 128) codes of quantize_input_bytes (VNNI prefill,
// decoder.cpp:648-660).
int leafref_quantize_u8(const float* x, std::size_t tokens, std::size_t cols,
                        std::uint8_t* q, float* scales) {
#if LEAF_DECODER_VNNI
    try {
        harness_scales(x, tokens, cols, scales);
        for (std::size_t t = 0; t < tokens; ++t)
            lr::quantize_input_bytes(x + t * cols, q + t * cols, cols, 1.0f / scales[t]);
        return 0;
    } catch (const std::exception& e) { harness_error = e.what(); return 1; }
#else
    (void)x; (void)tokens; (void)cols; (void)q; (void)scales;
    harness_error = "built without AVX-VNNI support"; return 2;
#endif
}

// W8A8 / W4A8 linear.  mode 0: the dispatch Impl::linear takes on this CPU
// (VNNI tile when tokens > 1 and bits == 8); mode 1: AVX2 only; mode 2: the
// portable scalar kernel.  Output is token-major [tokens, rows].
int leafref_linear_int(const float* x, std::size_t tokens, std::size_t cols,
                       const void* wdata, const float* wscales, std::size_t rows,
                       unsigned bits, std::size_t group, const float* bias, float* y,
                       unsigned threads, int mode) {
    try {
        lr::Weight w = harness_weight(wdata, wscales, rows, cols, bits, group);
        const bool vnni = mode == 0 && harness_vnni_available() && tokens > 1 && bits == 8 &&
                          group <= 65536;
        const bool avx = mode != 2;
        std::vector<float> scales(tokens);
        std::vector<std::int16_t> q16;
        std::vector<std::uint8_t> q8;
        harness_scales(x, tokens, cols, scales.data());
        if (vnni) {
#if LEAF_DECODER_VNNI
            q8.resize(tokens * cols);
            for (std::size_t t = 0; t < tokens; ++t)
                lr::quantize_input_bytes(x + t * cols, q8.data() + t * cols, cols, 1.0f / scales[t]);
            lr::prepare_signed_sums(w);
#endif
        } else {
            q16.resize(tokens * cols);
            for (std::size_t t = 0; t < tokens; ++t) {
                if (avx) lr::quantize_input_avx(x + t * cols, q16.data() + t * cols, cols, 1.0f / scales[t]);
                else
                    for (std::size_t col = 0; col < cols; ++col)
                        q16[t * cols + col] = static_cast<std::int16_t>(std::max(-127L, std::min(127L,
                            std::lrint(x[t * cols + col] / scales[t]))));
            }
        }
        lr::Workers& workers = harness_pool(threads);
        auto bias_at = [&](std::size_t row) { return bias ? bias[row] : 0.0f; };
        workers.run(rows, [&](std::size_t first, std::size_t last) {
            std::size_t row = first;
#if LEAF_DECODER_VNNI
            if (vnni) {
                float result[8];
                for (; row < last; row += 2) {
                    const std::size_t live = std::min<std::size_t>(2, last - row);
                    for (std::size_t token = 0; token < tokens; token += 4) {
                        const std::size_t count = std::min<std::size_t>(4, tokens - token);
                        lr::quant_vnni_tile(w, row, live, q8.data() + token * cols, count,
                                            scales.data() + token, result);
                        for (std::size_t r = 0; r < live; ++r)
                            for (std::size_t t = 0; t < count; ++t)
                                y[(token + t) * rows + row + r] = result[r * 4 + t] + bias_at(row + r);
                    }
                }
                return;
            }
#endif
            if (avx && tokens > 1) {
                float result[8];
                for (; row + 4 <= last; row += 4)
                    for (std::size_t token = 0; token < tokens; token += 2) {
                        const std::size_t count = std::min<std::size_t>(2, tokens - token);
                        lr::quant_tile_avx(w, row, q16.data() + token * cols, count,
                                           scales.data() + token, result);
                        for (std::size_t r = 0; r < 4; ++r)
                            for (std::size_t t = 0; t < count; ++t)
                                y[(token + t) * rows + row + r] = result[r * 2 + t] + bias_at(row + r);
                    }
            }
            float result[4];
            for (; row < last; ++row)
                for (std::size_t token = 0; token < tokens; token += 4) {
                    const std::size_t count = std::min<std::size_t>(4, tokens - token);
                    if (avx) lr::quant_dot_avx(w, row, q16.data() + token * cols, count,
                                               scales.data() + token, result);
                    else lr::quant_dot_scalar(w, row, q16.data() + token * cols, count,
                                              scales.data() + token, result);
                    for (std::size_t t = 0; t < count; ++t)
                        y[(token + t) * rows + row] = result[t] + bias_at(row);
                }
        });
        return 0;
    } catch (const std::exception& e) { harness_error = e.what(); return 1; }
}

// Weight-only linear with fp32 activations (W4A32 / W8A32 / FP32): the
// non-integer branch of Impl::linear (decoder.cpp:1221-1231) with the
// decoder's default dot (dot_avx, or dot_scalar when mode == 2).
int leafref_linear_float(const float* x, std::size_t tokens, std::size_t cols,
                         const void* wdata, const float* wscales, std::size_t rows,
                         unsigned bits, std::size_t group, const float* bias, float* y,
                         unsigned threads, int mode) {
    try {
        lr::Weight w = harness_weight(wdata, wscales, rows, cols, bits, group);
        lr::Workers& workers = harness_pool(threads);
        workers.run(rows, [&](std::size_t first, std::size_t last) {
            float result[4];
            for (std::size_t row = first; row < last; ++row)
                for (std::size_t token = 0; token < tokens; token += 4) {
                    const std::size_t count = std::min<std::size_t>(4, tokens - token);
                    if (mode == 2) lr::dot_scalar(w, row, x + token * cols, count, result);
                    else lr::dot_avx(w, row, x + token * cols, count, result);
                    for (std::size_t t = 0; t < count; ++t)
                        y[(token + t) * rows + row] = result[t] + (bias ? bias[row] : 0.0f);
                }
        });
        return 0;
    } catch (const std::exception& e) { harness_error = e.what(); return 1; }
}

// Graph-executor INT8 GEMM (engine/src/kernels/gemm.cpp:99-166), B is [K, N].
int leafref_gemm_i8_per_channel(const std::int8_t* a, const std::int8_t* b, const float* bias,
                                float input_scale, const float* weight_scales, float* output,
                                std::size_t m, std::size_t k, std::size_t n, int relu) {
    leaf::kernels::gemm_i8_per_channel(a, b, bias, input_scale, weight_scales, output, m, k, n,
        relu ? leaf::kernels::Activation::Relu : leaf::kernels::Activation::None);
    return 0;
}

int leafref_gemm_i8_reference(const std::int8_t* a, const std::int8_t* b, const float* bias,
                              float input_scale, const float* weight_scales, float* output,
                              std::size_t m, std::size_t k, std::size_t n, int relu) {
    leaf::kernels::gemm_i8_reference(a, b, bias, input_scale, weight_scales, output, m, k, n,
        relu ? leaf::kernels::Activation::Relu : leaf::kernels::Activation::None);
    return 0;
}

}  // extern "C"

