/* CPU restatement of Leaf's quantised-linear path (TEST INFRASTRUCTURE ONLY).
 *
 * This is the checker the parity tests and bench.py's cpu_baseline leg use.
 * The product (leaf_b200/, libleafq.so) never links or calls it.  Every
 * function cites the reference file:line whose arithmetic it restates; the
 * restatement is pinned against the reference's own compiled kernels
 * (oracle/_ref/libleafref.so) by tests/test_oracle_pinned.py and against the
 * committed golden vectors in tests/golden/.
 *
 * Layouts: activations x are token-major [tokens, cols] fp32.  Weights are
 * row-major [rows, cols]: int8 one byte per value, int4 two values per byte
 * (low nibble = even column), fp32 four bytes.  Scales are [rows, cols/group]
 * fp32.  Outputs are token-major [tokens, rows] fp32.
 */
#ifndef LEAFQ_ORACLE_H
#define LEAFQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Per-token dynamic scale and int8 codes (decoder.cpp:1028-1038, 618-627). */
int oq_quantize_act(const float* x, size_t tokens, size_t cols, int8_t* q, float* sx);

/* Integer linear from already-quantised activations: W8A8 (bits 8) or W4A8
 * (bits 4).  acc (optional, may be NULL) receives the int32 accumulator of
 * every (token, row, group), layout [tokens, rows, cols/group].  fused = 1:
 * the AVX2 kernels' fused group accumulation (decode, INT4, non-VNNI
 * prefill); fused = 0: the VNNI prefill tile's two-rounding accumulation.
 * With one group per row both give identical results. */
int oq_linear_int_q(const int8_t* q, const float* sx, size_t tokens, size_t cols,
                    const void* w, const float* ws, size_t rows, unsigned bits, size_t group,
                    const float* bias, float* y, int32_t* acc, int fused);

/* Quantise then run oq_linear_int_q: the whole integer branch of
 * Decoder::Impl::linear (decoder.cpp:1020-1044, 1109-1232). */
int oq_linear_int(const float* x, size_t tokens, size_t cols, const void* w, const float* ws,
                  size_t rows, unsigned bits, size_t group, const float* bias, float* y,
                  int32_t* acc, int fused);

/* Weight-only linear with fp32 activations (bits 4, 8 or 32), in the exact
 * summation order of dot_avx (decoder.cpp:355-391) as Impl::linear calls it
 * in blocks of four tokens (decoder.cpp:1221-1231). */
int oq_linear_float(const float* x, size_t tokens, size_t cols, const void* w, const float* ws,
                    size_t rows, unsigned bits, size_t group, const float* bias, float* y);

/* Graph executor static activation quantiser (executor.cpp:220-230).
 * Returns 1 (and writes nothing further) on a non-finite value or scale. */
int oq_graph_quantize(const float* x, size_t count, float scale, int8_t* q);

/* Graph executor INT8 GEMM with per-output-channel scales, B is [k, n]
 * (kernels/gemm.cpp:79-97 and 99-166). */
void oq_gemm_i8_per_channel(const int8_t* a, const int8_t* b, const float* bias, float input_scale,
                            const float* weight_scales, float* out, size_t m, size_t k, size_t n,
                            int relu);

/* y[i] = expf(x[i]) (libm): the reference decoder's attention and SiLU
 * exponential on Linux (transformer.cpp:130, decoder.cpp:983). */
void oq_expf(const float* x, float* y, size_t n);

/* y[i] = the graph executor's fused Gelu of x[i] (executor.cpp:236-240,
 * libm tanhf). */
void oq_gelu(const float* x, float* y, size_t n);

/* y[i] = tanhf(x[i]) (libm). */
void oq_tanhf(const float* x, float* y, size_t n);

#ifdef __cplusplus
}
#endif
#endif
