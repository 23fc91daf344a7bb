// Host-side plumbing shared by the leafq translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/leafq.h"

namespace leafq {

// Thread-local error text for leafq_last_error().
void set_error(const std::string& message);
void clear_error();

// Returns LEAFQ_ERR_CUDA (and records the text) when err is not cudaSuccess.
int cuda_status(cudaError_t err, const char* what);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();
// Opt-in dynamic shared memory per block of the current device (cached).
int max_smem_per_block();

// Launch `kernel` with grid/block/smem on `stream`, with the programmatic
// stream serialisation attribute when `pdl`.  Returns LEAFQ_OK or
// LEAFQ_ERR_CUDA.
template <typename... KernelArgs, typename... Args>
int launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t stream, bool pdl, const char* what, Args&&... args) {
    cudaLaunchConfig_t config = {};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = pdl ? 1 : 0;
    cudaError_t err = cudaLaunchKernelEx(&config, kernel, static_cast<KernelArgs>(args)...);
    return cuda_status(err, what);
}

// Raises the kernel's dynamic shared memory limit once per (kernel, size).
int allow_smem(const void* kernel, size_t bytes, const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------ peer-memory all-gather
// A kernel that ends an N-sharded linear can store its output rows straight
// into every rank's receive buffer (CUDA IPC mappings over NVLink) as
// flag-in-data words {fp32 value, 32-bit run tag}; the receiving rank polls
// its own buffer until every word carries the current tag.  Two halves
// alternate with the tag's parity, so a rank one run ahead never overwrites
// words a slower rank has still to read.
constexpr int kMaxPeers = 8;
struct PeerStore {
    unsigned long long* dst[kMaxPeers];  // receive buffers of ranks 0..world-1
    const unsigned int* epoch;           // this rank's run counter = the run's tag
    int world;                           // 0: no peer stores (plain output)
    long long half;                      // words per parity half
    long long row_offset;                // gathered row of local row 0
    long long rows;                      // rows of the gathered output
};

// ------------------------------------------------------------ launchers
// Each returns a LEAFQ_* status; arguments are validated by the caller.
int launch_quantize_act(cudaStream_t s, const float* x, int64_t tokens, int64_t cols, int8_t* q,
                        float* scales, bool pdl, const float* col_scale = nullptr);
// y[t][c] = x[t][c] * col_scale[c] (SmoothQuant input scaling for the
// float-activation path).
int launch_scale_columns(cudaStream_t s, const float* x, int64_t tokens, int64_t cols, const float* col_scale,
                         float* y, bool pdl);

// Fused act-quant + per-row W8A8 GEMV for tokens <= 8 (bulk-TMA weights).
bool gemv_w8a8_supported(int64_t tokens, int64_t cols, int bits, int64_t group,
                         const void* weight, const float* x);
// With `peer` (world > 0) the epilogue stores into the receive buffers
// instead of y.
int launch_gemv_w8a8(cudaStream_t s, const float* x, int64_t tokens, int64_t cols,
                     const int8_t* weight, const float* wscales, int64_t rows, const float* bias,
                     float* y, bool pdl, const PeerStore* peer = nullptr);

// The path leafq_linear takes for an integer call (activation bits 8): the
// fused-quantisation GEMV (no workspace), else codes into a workspace and
// then the tcgen05 GEMM when integer_path_takes_gemm_tc, else the generic
// integer kernel.
bool integer_path_takes_gemv(int64_t tokens, int64_t cols, int bits, int64_t group, const void* weight,
                             const float* x);
bool integer_path_takes_gemm_tc(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                                const void* weight);

// Generic integer linear from codes (any group, bits 8 / 4, any tokens).
int launch_linear_int_q(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens,
                        int64_t cols, const void* weight, const float* wscales, int64_t rows,
                        int bits, int64_t group, const float* bias, float* y, int32_t* acc,
                        bool fused, bool pdl);

// Weight-only linear with fp32 activations in dot_avx order.
bool gemv_w4a32_fast_supported(int64_t tokens, int64_t cols, int bits, int64_t group,
                               const void* weight, const float* wscales);
int launch_gemv_w4a32_fast(cudaStream_t s, const float* x, int64_t cols, const uint8_t* weight,
                           const float* wscales, int64_t rows, int64_t group, const float* bias,
                           float* y, bool pdl);
int launch_linear_f32act(cudaStream_t s, const float* x, int64_t tokens, int64_t cols,
                         const void* weight, const float* wscales, int64_t rows, int bits,
                         int64_t group, const float* bias, float* y, bool pdl);

// tcgen05 INT8 GEMM for per-row INT8 weights with many tokens.
bool gemm_tc_supported(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                       const void* weight);
int launch_gemm_tc(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens,
                   int64_t cols, const int8_t* weight, const float* wscales, int64_t rows,
                   const float* bias, float* y, bool pdl);

// tcgen05 INT8 GEMM for grouped INT8 weights (groups a multiple of 32 codes)
// with more than 8 tokens; `fused` picks the AVX2 + FMA group accumulation,
// else the VNNI tile's two roundings.
bool gemm_grouped_tc_supported(int64_t tokens, int64_t cols, int64_t rows, int bits, int64_t group,
                               const void* weight, const int8_t* q);
int launch_gemm_grouped_tc(cudaStream_t s, const int8_t* q, const float* sx, int64_t tokens, int64_t cols,
                           const int8_t* weight, const float* wscales, int64_t rows, int64_t group,
                           const float* bias, float* y, bool fused, bool pdl);

// Graph executor kernels.
int launch_graph_quantize(cudaStream_t s, const float* x, int64_t count, float scale, int8_t* q,
                          int32_t* error_flag);
// execute_quant_linear (executor.cpp:524-614): static quantisation of a
// (transposed first when trans_a) into codes [m, k], the per-channel GEMM
// against weight [k, n] or, with trans_b, [n, k], then alpha / beta * C /
// activation.
int launch_graph_linear(cudaStream_t s, const float* a, int64_t m, int64_t k, int trans_a,
                        const int8_t* weight, int64_t n, int trans_b, float input_scale,
                        const float* wscales, float alpha, float beta, const float* c, int c_kind,
                        int activation, float* out, int8_t* codes, int32_t* error_flag);
int launch_gemm_i8_per_channel(cudaStream_t s, const int8_t* a, const int8_t* b,
                               const float* bias, float input_scale, const float* wscales,
                               float* out, int64_t m, int64_t k, int64_t n, int activation);

}  // namespace leafq
