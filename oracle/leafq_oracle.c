/* CPU restatement of Leaf's quantised-linear path.  TEST INFRASTRUCTURE ONLY:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU legs load this
 * library, and only as the checker.  All arithmetic is scalar and in the
 * reference's order.  Built with -ffp-contract=off; every fused multiply-add
 * of the reference is written out as fmaf().
 *
 * Contraction in the reference: leaf/cli.py:66 builds decoder.cpp with
 * g++ -std=c++17 -O3, and GCC contracts a*b+c into one FMA inside functions
 * compiled for target("avx2,fma") (LEAF_AVX_TARGET, decoder.cpp:67).  So in
 * quant_dot_avx (:567), quant_tile_avx (:614) and dot_avx (:383, :386) the
 * accumulation `result += p * scale` is a single fused operation.  The VNNI
 * tile (target "avx2,avxvnni", :699) has no FMA and rounds twice; with one
 * group per row (the default per-row INT8 export) both agree bit for bit,
 * with several groups they can differ in the last bit.  This restatement
 * follows the AVX2/FMA path: the one every decode step (M = 1) and every
 * INT4 call takes. */
#include "leafq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Signed value of weight (row, col) before scaling: Weight::value without
 * the scale multiply (decoder.cpp:245-249).  int4: low nibble = even index,
 * sign by subtracting 16 from codes >= 8. */
static int weight_code(const void* w, size_t index, unsigned bits) {
    if (bits == 8) return ((const int8_t*)w)[index];
    int code = (((const uint8_t*)w)[index / 2] >> ((index % 2) * 4)) & 15;
    return code >= 8 ? code - 16 : code;
}

static float weight_float(const void* w, size_t index, unsigned bits) {
    if (bits == 32) return ((const float*)w)[index];
    return (float)weight_code(w, index, bits);
}

int oq_quantize_act(const float* x, size_t tokens, size_t cols, int8_t* q, float* sx) {
    for (size_t t = 0; t < tokens; ++t) {
        const float* row = x + t * cols;
        /* decoder.cpp:1030-1032: absmax over the row (a NaN never replaces the
         * running maximum, like std::max), IEEE division by 127, floor 1e-12. */
        float maximum = 0.0f;
        for (size_t c = 0; c < cols; ++c) {
            const float a = fabsf(row[c]);
            if (maximum < a) maximum = a;
        }
        float scale = maximum / 127.0f;
        if (scale < 1e-12f) scale = 1e-12f;
        sx[t] = scale;
        /* decoder.cpp:1035/1038 pass the reciprocal; quantize_input_avx
         * (:618-627) multiplies and rounds half-to-even (cvtps_epi32).  For
         * finite input |x * (1/s)| <= 127 + a few ulp, so the code is in
         * [-127, 127]. */
        const float multiplier = 1.0f / scale;
        for (size_t c = 0; c < cols; ++c) {
            const float v = row[c] * multiplier;
            long r = lrintf(v);
            if (r > 127) r = 127;
            if (r < -128) r = -128;
            q[t * cols + c] = (int8_t)r;
        }
    }
    return 0;
}

int oq_linear_int_q(const int8_t* q, const float* sx, size_t tokens, size_t cols,
                    const void* w, const float* ws, size_t rows, unsigned bits, size_t group,
                    const float* bias, float* y, int32_t* acc, int fused) {
    if ((bits != 8 && bits != 4) || group == 0 || cols % group) return 1;
    const size_t groups = cols / group;
    for (size_t t = 0; t < tokens; ++t) {
        for (size_t r = 0; r < rows; ++r) {
            /* quant_dot_avx / quant_tile_avx produce the exact int32 group sum,
             * then accumulate in group order from 0.0f:
             * result = fma(float(acc) * sx, sw, result)
             * (decoder.cpp:566-568, 612-615).  fused == 0 restates the VNNI
             * tile instead (:695-700): result + (float(acc) * sx) * sw. */
            float result = 0.0f;
            for (size_t g = 0; g < groups; ++g) {
                int32_t sum = 0;
                for (size_t c = g * group; c < (g + 1) * group; ++c)
                    sum += weight_code(w, r * cols + c, bits) * (int32_t)q[t * cols + c];
                if (acc) acc[(t * rows + r) * groups + g] = sum;
                const float product = (float)sum * sx[t];
                if (fused) result = fmaf(product, ws[r * groups + g], result);
                else result = result + product * ws[r * groups + g];
            }
            /* decoder.cpp:1229: bias (or 0.0f) added after the dot. */
            y[t * rows + r] = result + (bias ? bias[r] : 0.0f);
        }
    }
    return 0;
}

int oq_linear_int(const float* x, size_t tokens, size_t cols, const void* w, const float* ws,
                  size_t rows, unsigned bits, size_t group, const float* bias, float* y,
                  int32_t* acc, int fused) {
    int8_t* q = (int8_t*)malloc(tokens * cols ? tokens * cols : 1);
    float* sx = (float*)malloc((tokens ? tokens : 1) * sizeof(float));
    if (!q || !sx) { free(q); free(sx); return 2; }
    oq_quantize_act(x, tokens, cols, q, sx);
    const int status = oq_linear_int_q(q, sx, tokens, cols, w, ws, rows, bits, group, bias, y, acc,
                                       fused);
    free(q);
    free(sx);
    return status;
}

/* reduce() (decoder.cpp:294-298): lanes (i, i+4) first, then
 * (h0 + h2) + (h1 + h3). */
static float lane_tree(const float v[8]) {
    const float h0 = v[0] + v[4], h1 = v[1] + v[5], h2 = v[2] + v[6], h3 = v[3] + v[7];
    return (h0 + h2) + (h1 + h3);
}

/* One call of dot_avx (decoder.cpp:355-391) for `count` (1..4) tokens. */
static void dot_block(const void* w, const float* ws, size_t row, size_t cols, unsigned bits,
                      size_t group, const float* x, size_t count, float* result) {
    const size_t g_size = bits == 32 ? cols : group;
    const size_t groups = cols / g_size;
    for (size_t t = 0; t < count; ++t) result[t] = 0.0f;
    for (size_t g = 0; g < groups; ++g) {
        float chain[4][8];
        memset(chain, 0, sizeof chain);
        size_t col = g * g_size;
        const size_t end = col + g_size;
        const size_t base = row * cols;
        if (count == 1) {
            /* Four 8-lane FMA chains over 32-column blocks (:362-369). */
            for (; col + 32 <= end; col += 32)
                for (int j = 0; j < 4; ++j)
                    for (int l = 0; l < 8; ++l) {
                        const size_t c = col + 8 * j + l;
                        chain[j][l] = fmaf(weight_float(w, base + c, bits), x[c], chain[j][l]);
                    }
            for (int l = 0; l < 8; ++l)
                chain[0][l] = (chain[0][l] + chain[1][l]) + (chain[2][l] + chain[3][l]);
        }
        /* One 8-lane chain per token over 8-column steps (:372-378). */
        for (; col + 8 <= end; col += 8)
            for (int l = 0; l < 8; ++l) {
                const float value = weight_float(w, base + col + l, bits);
                for (size_t t = 0; t < count; ++t)
                    chain[t][l] = fmaf(value, x[t * cols + col + l], chain[t][l]);
            }
        float partial[4];
        for (size_t t = 0; t < 4; ++t) partial[t] = lane_tree(chain[t]);
        const float scale = bits == 32 ? 1.0f : ws[row * groups + g];
        /* Scalar tail: Weight::value(row, col) / scale (:381-384). */
        for (; col < end; ++col) {
            const float stored = bits == 32 ? weight_float(w, base + col, bits)
                                            : (float)weight_code(w, base + col, bits) * scale;
            const float value = stored / scale;
            for (size_t t = 0; t < count; ++t) partial[t] = fmaf(value, x[t * cols + col], partial[t]);
        }
        for (size_t t = 0; t < count; ++t) result[t] = fmaf(partial[t], scale, result[t]);
    }
}

int oq_linear_float(const float* x, size_t tokens, size_t cols, const void* w, const float* ws,
                    size_t rows, unsigned bits, size_t group, const float* bias, float* y) {
    if (bits != 4 && bits != 8 && bits != 32) return 1;
    if (bits != 32 && (group == 0 || cols % group)) return 1;
    for (size_t r = 0; r < rows; ++r)
        for (size_t token = 0; token < tokens; token += 4) {
            const size_t count = tokens - token < 4 ? tokens - token : 4;
            float result[4];
            dot_block(w, ws, r, cols, bits, group, x + token * cols, count, result);
            for (size_t t = 0; t < count; ++t)
                y[(token + t) * rows + r] = result[t] + (bias ? bias[r] : 0.0f);
        }
    return 0;
}

int oq_graph_quantize(const float* x, size_t count, float scale, int8_t* q) {
    /* executor.cpp:220-230: IEEE division (not a reciprocal), clamp to
     * [-127, 127], then nearbyint (half-to-even). */
    if (!isfinite(scale) || !(scale > 0.0f)) return 1;
    for (size_t i = 0; i < count; ++i) {
        if (!isfinite(x[i])) return 1;
        float v = x[i] / scale;
        if (v > 127.0f) v = 127.0f;
        if (v < -127.0f) v = -127.0f;
        q[i] = (int8_t)nearbyintf(v);
    }
    return 0;
}

void oq_gemm_i8_per_channel(const int8_t* a, const int8_t* b, const float* bias, float input_scale,
                            const float* weight_scales, float* out, size_t m, size_t k, size_t n,
                            int relu) {
    for (size_t row = 0; row < m; ++row)
        for (size_t col = 0; col < n; ++col) {
            int32_t sum = 0;
            for (size_t i = 0; i < k; ++i) sum += (int32_t)a[row * k + i] * (int32_t)b[i * n + col];
            /* gemm.cpp:89-95 / 151-156: (float(acc) * s_in) * s_w, + bias,
             * then ReLU as std::max(value, 0.0f), which keeps -0.0f and NaN
             * (gemm.cpp:14-16). */
            float value = ((float)sum * input_scale) * weight_scales[col];
            if (bias) value = value + bias[col];
            if (relu) value = value < 0.0f ? 0.0f : value;
            out[row * n + col] = value;
        }
}

/* libm expf over an array: the exponential the reference's attention
 * (transformer.cpp:130) and scalar SiLU (decoder.cpp:983) call on Linux. */
void oq_expf(const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = expf(x[i]);
}

/* The graph executor's fused Gelu (executor.cpp:236-240), tanh form, each
 * step one float rounding in C++'s left-to-right order:
 * (0.5f * v) * (1 + tanhf(c * (v + ((0.044715f * v) * v) * v))), libm tanhf. */
void oq_gelu(const float* x, float* y, size_t n) {
    const float root_two_over_pi = 0.7978845608028654f;
    for (size_t i = 0; i < n; ++i) {
        const float v = x[i];
        y[i] = 0.5f * v * (1.0f + tanhf(root_two_over_pi * (v + 0.044715f * v * v * v)));
    }
}

/* y[i] = tanhf(x[i]) (libm). */
void oq_tanhf(const float* x, float* y, size_t n) {
    for (size_t i = 0; i < n; ++i) y[i] = tanhf(x[i]);
}
