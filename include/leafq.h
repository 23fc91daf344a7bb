/* leafq -- B200 (sm_100a) quantised-linear operators behind a plain C ABI.
 *
 * Drop-in boundary for Leaf's quantised Linear: every entry point takes
 * device pointers, plain sizes and a cudaStream_t (passed as void*), returns
 * an int status, allocates nothing on the hot path and never throws.  All
 * calls are stream-ordered and asynchronous; results are ready when the
 * stream is.  Calls on different streams may run concurrently (the library
 * keeps no mutable per-call host state besides the thread-local error text).
 *
 * Layouts are the reference's:
 *   x       fp32 [tokens, cols] token-major (Decoder::Impl::linear input)
 *   weight  row-major [rows, cols]; bits 8: one int8 per value; bits 4: two
 *           signed nibbles per byte, low nibble = even column
 *           (decoder.cpp:236-251, tools/export_decoder.py:91-105); bits 32:
 *           fp32.  16-byte aligned base for the fast paths.
 *   scales  fp32 [rows, cols / group] (group == cols for per-row INT8)
 *   bias    fp32 [rows] or NULL
 *   y       fp32 [tokens, rows] token-major (decoder.cpp:1229)
 *
 * Status codes: LEAFQ_OK on success; anything else leaves the outputs
 * unspecified and leafq_last_error() describes the failure.
 */
#ifndef LEAFQ_H
#define LEAFQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LEAFQ_OK 0
#define LEAFQ_ERR_INVALID 1     /* bad argument: null pointer, shape, alignment */
#define LEAFQ_ERR_CUDA 2        /* a CUDA runtime call failed */
#define LEAFQ_ERR_UNSUPPORTED 3 /* valid for the reference, not built here */
#define LEAFQ_ERR_TIMEOUT 4     /* a bounded device-side wait gave up */
#define LEAFQ_ERR_NONFINITE 5   /* graph quantiser saw a non-finite value */

/* flags */
/* Accumulate per-group partial sums with two roundings, as the reference's
 * AVX-VNNI prefill tile does (decoder.cpp:695-700), instead of the fused
 * multiply-add of its AVX2 kernels (decoder.cpp:567, 614).  Only matters
 * with several groups per row. */
#define LEAFQ_FLAG_VNNI_ROUNDING 0x1u
/* Launch with programmatic dependent launch: the kernel may start, and
 * begin streaming weights, scales and bias, before the previous kernel in
 * the stream has finished; it still waits for that kernel before reading x
 * or writing y.  Only valid when the previous kernel does not write this
 * call's weights, scales or bias (true inside a decode step, where they are
 * read-only). */
#define LEAFQ_FLAG_PDL 0x2u

/* Human-readable description of this thread's last failure ("" if none). */
const char* leafq_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int leafq_version(void);

/* Reads and clears the device error word that bounded waits set when they
 * give up.  Synchronises the current device.  LEAFQ_OK or LEAFQ_ERR_TIMEOUT. */
int leafq_device_status(void);

/* How long a device-side wait (a pipeline barrier, a hand-off word another
 * block or rank writes) spins before it gives up, records the failure for
 * leafq_device_status() and lets its kernel return: 2 s by default (0
 * restores it), 1 us .. 60 s otherwise.  Applies to the current device;
 * synchronises it first.  The reference's counterpart is its bounded worker
 * spin (engine/include/leaf/runtime/host_support.h:185-197); a short limit
 * lets a test make a wait run out without hanging anything. */
int leafq_set_wait_limit_ns(uint64_t nanoseconds);

/* Per-token dynamic activation quantisation.
 * Replaces decoder.cpp:1028-1044 (scale = max(absmax / 127, 1e-12), codes =
 * round-half-even(x * (1 / scale)) as quantize_input_avx, :618-627).  q is
 * int8 [tokens, cols] (the reference's int16 container holds the same values
 * in [-127, 127]; its VNNI uint8 container holds q + 128), scales fp32
 * [tokens]. */
int leafq_quantize_act(void* stream, const float* x, int64_t tokens, int64_t cols, int8_t* q,
                       float* scales);

/* Bytes of caller-provided device workspace leafq_linear needs for this
 * shape (0 when the call needs none).  The workspace must be 256-byte
 * aligned. */
size_t leafq_linear_workspace_bytes(int64_t tokens, int64_t cols, int bits, int64_t group,
                                    int activation_bits);

/* The quantised Linear: Decoder::Impl::linear(input, tokens, name, output)
 * for one named weight (decoder.cpp:994-1233).
 *   activation_bits 8  + bits 8/4: W8A8 / W4A8 -- per-token dynamic int8
 *       activations, exact int32 group sums, then per group in order
 *       result = fma(float(acc) * sx, sw, result), plus bias.
 *   activation_bits 32 + bits 4/8/32: weight-only, fp32 activations, in the
 *       summation order of dot_avx (decoder.cpp:355-391).
 * workspace may be NULL when leafq_linear_workspace_bytes() returned 0. */
int leafq_linear(void* stream, const float* x, int64_t tokens, int64_t cols, const void* weight,
                 const float* weight_scales, int64_t rows, int bits, int64_t group,
                 int activation_bits, const float* bias, float* y, void* workspace,
                 size_t workspace_bytes, uint32_t flags);

/* Decoder::Impl::linear for a weight that has a calibrated `input_scale`
 * tensor (SmoothQuant, decoder.cpp:1008-1019): x[t][c] * input_scale[c]
 * (one float rounding) is what gets quantised (activation_bits 8, the
 * scaling fused into the quantiser) or multiplied (activation_bits 32).
 * input_scale NULL is leafq_linear.  workspace: at least
 * leafq_linear_smooth_workspace_bytes(tokens, cols, activation_bits) bytes,
 * 256-byte aligned. */
size_t leafq_linear_smooth_workspace_bytes(int64_t tokens, int64_t cols, int activation_bits);
/* y[t][c] = x[t][c] * col_scale[c]: the SmoothQuant scaling alone (for a
 * caller that quantises elsewhere, e.g. before a sharded linear). */
int leafq_scale_columns(void* stream, const float* x, int64_t tokens, int64_t cols, const float* col_scale,
                        float* y);
int leafq_linear_smooth(void* stream, const float* x, const float* input_scale, int64_t tokens, int64_t cols,
                        const void* weight, const float* weight_scales, int64_t rows, int bits, int64_t group,
                        int activation_bits, const float* bias, float* y, void* workspace,
                        size_t workspace_bytes, uint32_t flags);

/* Integer linear from codes already produced by leafq_quantize_act (or by
 * the reference's quantiser).  acc, when not NULL, receives every int32
 * group sum, layout [tokens, rows, cols / group]: the accumulator the
 * reference keeps in quant_dot_avx / quant_vnni_tile (decoder.cpp:536-570,
 * 661-702), exposed for bit-exact checking. */
int leafq_linear_int_q(void* stream, const int8_t* q, const float* scales, int64_t tokens,
                       int64_t cols, const void* weight, const float* weight_scales, int64_t rows,
                       int bits, int64_t group, const float* bias, float* y, int32_t* acc,
                       uint32_t flags);

/* Graph executor static INT8 activation quantiser (executor.cpp:220-230):
 * q = nearbyint(clamp(x / scale, -127, 127)).  The reference throws on a
 * non-finite value; here the kernel sets *error_flag (device int32, caller
 * clears it) to 1, and the call itself returns LEAFQ_ERR_INVALID for a
 * non-finite or non-positive scale. */
int leafq_graph_quantize(void* stream, const float* x, int64_t count, float scale, int8_t* q,
                         int32_t* error_flag);

/* Graph executor INT8 GEMM, leaf::kernels::gemm_i8_per_channel
 * (engine/include/leaf/kernels/gemm.h:24-28, kernels/gemm.cpp:99-166):
 * a int8 [m, k], b int8 [k, n] (n contiguous), out fp32 [m, n] =
 * (float(a . b) * input_scale) * weight_scales[n] (+ bias[n]), then ReLU
 * when activation == 1. */
int leafq_gemm_i8_per_channel(void* stream, const int8_t* a, const int8_t* b, const float* bias,
                              float input_scale, const float* weight_scales, float* out,
                              int64_t m, int64_t k, int64_t n, int activation);

/* A quantised Gemm / MatMul node of the graph executor, execute_quant_linear
 * (executor.cpp:524-614): a fp32 [m, k] ([k, m] with trans_a, Gemm only),
 * statically quantised with input_scale (as leafq_graph_quantize); weight
 * int8 [k, n] ([n, k] with trans_b); out fp32 [m, n] =
 * act(alpha * ((float(acc) * input_scale) * weight_scales[col]) + beta * C),
 * C NULL or c_kind 1 (one value), 2 ([n], per column) or 3 ([m, n]);
 * activation 0 none, 1 Relu, 2 Silu, 3 Gelu (tanh form, libm tanhf bits).
 * A MatMul node is alpha = 1, beta = 0, C = NULL.  workspace: at least
 * leafq_graph_linear_workspace_bytes(m, k) bytes for the codes; a non-finite
 * input sets *error_flag (device int32, caller clears it). */
size_t leafq_graph_linear_workspace_bytes(int64_t m, int64_t k);
int leafq_graph_linear(void* stream, const float* a, int64_t m, int64_t k, int trans_a, const int8_t* weight,
                       int64_t n, int trans_b, float input_scale, const float* weight_scales, float alpha,
                       float beta, const float* c, int c_kind, int activation, float* out, void* workspace,
                       size_t workspace_bytes, int32_t* error_flag);

/* ------------------------------------------------------------------------
 * Persistent decode step.  The reference's forward loop calls linear() for
 * q, k, v, o, up, gate, down of every layer and lm_head
 * (decoder.cpp:1321-1441), each on the previous call's output.  A plan
 * holds such a chain of per-row W8A8 linears (one token); one run executes
 * the whole chain in a single cooperative launch whose blocks stream every
 * weight continuously and hand activations to each other through tagged
 * words in plan-owned buffers.  Results are bit-identical to calling
 * leafq_linear op by op. */
typedef struct leafq_decode_op {
    const float* x;            /* fp32 [cols] ready at launch when wait == -1, else NULL */
    float* y;                  /* fp32 [rows] copy of the output for the caller, or NULL */
    const void* weight;        /* int8 [rows, cols], per-row scales */
    const float* weight_scales;/* fp32 [rows] */
    const float* bias;         /* fp32 [rows] or NULL */
    int64_t rows;
    int64_t cols;              /* multiple of 16, at most 8192 */
    int32_t wait;              /* earlier op whose output is this op's x, or -1 */
    int32_t x_offset;          /* first element of that output used as x (multiple of 4) */
} leafq_decode_op;

typedef struct leafq_decode_plan_t leafq_decode_plan_t;

/* Validates the ops, copies them to device memory of the current device and
 * allocates the buffers that carry outputs to later ops; set-up time only.
 * tokens must be 1, at most 160 ops. */
int leafq_decode_plan_create(const leafq_decode_op* ops, int nops, int tokens,
                             leafq_decode_plan_t** plan);
/* Runs the whole chain on `stream` as one cooperative launch (capturable in
 * a CUDA graph).  Runs of one plan must be ordered (one stream).  Waits are
 * bounded: a stuck hand-off ends the kernel and leafq_device_status()
 * reports it; destroy and recreate the plan after such an error. */
int leafq_decode_plan_run(void* stream, leafq_decode_plan_t* plan);
int leafq_decode_plan_destroy(leafq_decode_plan_t* plan);

/* Per-row W8A8 linear (INT8 weights, group == cols) that allocates nothing:
 * for callers that cannot allocate device memory -- a plugin whose host
 * runtime owns all device memory, a serving loop that may not touch the
 * allocator after start-up, an embedder with a fixed budget -- and so cannot
 * hand leafq_linear a workspace.  No counterpart in the reference (its CPU
 * decoder reuses host vectors).  It runs the kernels leafq_linear runs for
 * the same call (the decode GEMV for 1-8 tokens needs no scratch), so the
 * results are leafq_linear's bit for bit.  Its scratch is a library-owned
 * device array of 8 MiB of codes plus 16384 token scales, held on every GPU
 * that loads the library until exit: calls with tokens * cols > 8 MiB or
 * tokens > 16384 return LEAFQ_ERR_INVALID.  The first call in each CUDA
 * context looks up the array's address (make it before any stream capture;
 * after a device reset the next call looks it up again).  All calls share
 * the array: calls that overlap on the GPU race; calls ordered on one stream
 * do not. */
int leafq_linear_w8a8_static_scratch(void* stream, const float* x, int64_t tokens, int64_t cols,
                                     const int8_t* weight, const float* weight_scales,
                                     int64_t rows, const float* bias, float* y, uint32_t flags);

/* ------------------------------------------------------------------------
 * N-sharded linear across GPUs (one process per GPU).  Output rows are
 * independent (the reference splits them over its worker threads,
 * decoder.cpp:1109 / host_support.h:151-178), so rank g computes rows
 * [row_begin, row_begin + local_rows) of every linear and the rows are
 * gathered along N -- bit-identical to the unsharded leafq_linear.
 *
 * The gather runs over peer memory without NCCL: each rank's rows are
 * stored straight into every rank's receive buffer (CUDA IPC mapping over
 * NVLink) as flag-in-data words, by the GEMV epilogue itself on the decode
 * path.  The reference has no multi-GPU code; these replace the
 * all-gather step of its row partitioning. */
#define LEAFQ_IPC_HANDLE_BYTES 64

typedef struct leafq_allgather leafq_allgather_t;

/* Creates this rank's side (current device = this rank's GPU): a receive
 * buffer for up to max_elements gathered floats (2 x 8 bytes each) and a
 * scratch of max_elements floats.  Writes the buffer's CUDA IPC handle
 * (LEAFQ_IPC_HANDLE_BYTES) to ipc_handle; the caller exchanges the handles
 * of all ranks (any host collective) and passes them to _connect.
 * world 1..8. */
int leafq_allgather_init(int rank, int world, int64_t max_elements, leafq_allgather_t** ag,
                         void* ipc_handle);
/* Maps the other ranks' receive buffers.  handles: world x
 * LEAFQ_IPC_HANDLE_BYTES in rank order (this rank's entry is ignored). */
int leafq_allgather_connect(leafq_allgather_t* ag, const void* handles);
/* out[t, row_begin_g + j] = local_g[t, j] on every rank g, for t < tokens.
 * local: [tokens, local_rows] fp32; out: [tokens, rows] fp32.  Every rank
 * must make the same sequence of _run / _linear_allgather calls with the
 * same tokens and rows; a rank that stops leaves the others waiting 2 s,
 * after which their output is NaN and leafq_device_status reports
 * LEAFQ_ERR_TIMEOUT. */
int leafq_allgather_run(void* stream, leafq_allgather_t* ag, const float* local, int64_t tokens,
                        int64_t local_rows, int64_t row_begin, int64_t rows, float* out);
/* leafq_linear on this rank's weight rows (weight/weight_scales/bias hold
 * local_rows rows), gathered into out [tokens, rows] on every rank.  The
 * per-row INT8 decode GEMV (tokens <= 8) stores its rows into the peers
 * from its epilogue; other paths run the linear into the scratch first.
 * Workspace rules are those of leafq_linear for (tokens, cols). */
int leafq_linear_allgather(void* stream, leafq_allgather_t* ag, const float* x, int64_t tokens,
                           int64_t cols, const void* weight, const float* weight_scales,
                           int64_t local_rows, int64_t row_begin, int64_t rows, int bits,
                           int64_t group, int activation_bits, const float* bias, float* out,
                           void* workspace, size_t workspace_bytes, uint32_t flags);
/* Unmaps the peers and frees.  Every rank must have finished its last run
 * (a host barrier after a device synchronise) before any rank destroys. */
int leafq_allgather_destroy(leafq_allgather_t* ag);

/* ------------------------------------------------------------------------
 * Whole-model decode step.  One cooperative launch runs one token through
 * every layer of a Llama-family W8A8 decoder (per-row INT8 linears and
 * embedding; RMSNorm, RoPE, GQA attention over an fp32 KV cache, SiLU gate,
 * sequential residual, final norm, lm_head) and the greedy argmax:
 * Decoder::Impl::forward_into for one token (decoder.cpp:1282-1452) plus
 * main_decoder.cpp:101.  Bit-identical to the reference.  The launch reads
 * the token at *ids and the cache length at *position, appends to the
 * caches, writes the logits (if given), sets *ids to the argmax, writes it to
 * history[*position + 1] (if given) and increments *position -- so repeated
 * launches (or replays of one captured launch) generate greedily with no
 * host work.  Prefill (several tokens) uses the per-operator entry points,
 * which share the caches and position. */
typedef struct leafq_model_layer {
    const float* input_norm;     /* fp32 [hidden] */
    const float* post_norm;      /* fp32 [hidden] */
    const int8_t* qkv;           /* [(heads + 2 kv_heads) * head_dim][hidden]: q, k, v rows stacked */
    const float* qkv_scales;
    const int8_t* o;             /* [hidden][hidden] */
    const float* o_scales;
    const int8_t* gate_up;       /* [2 * intermediate][hidden]: gate / up rows interleaved */
    const float* gate_up_scales;
    const int8_t* down;          /* [hidden][intermediate] */
    const float* down_scales;
    float* k_cache;              /* fp32 [kv_heads][capacity][head_dim] */
    float* v_cache;
} leafq_model_layer;

typedef struct leafq_model_desc {
    int32_t layers, hidden, intermediate, heads, kv_heads, head_dim, vocab;
    int64_t capacity;            /* cache rows (<= 4096) */
    float epsilon;               /* RMSNorm epsilon */
    float embedding_scale;
    float attn_scale;            /* 1 / sqrt(sqrt(head_dim)), applied to q.k twice */
    const int8_t* embed;         /* [vocab][hidden], per-row scales */
    const float* embed_scales;
    const float* final_norm;
    const int8_t* lm_head;       /* [vocab][hidden], per-row scales */
    const float* lm_head_scales;
    const float* cos_table;      /* [capacity][head_dim / 2] from leafq_rope_tables */
    const float* sin_table;
    const leafq_model_layer* layer;  /* host array [layers] */
    int32_t* ids;                /* device [1] */
    int32_t* position;           /* device [1] */
    int32_t* history;            /* device [capacity] or NULL */
    float* logits;               /* device [vocab] or NULL */
} leafq_model_desc;

typedef struct leafq_model_plan_t leafq_model_plan_t;

/* Checks the geometry (hidden <= 4096, intermediate <= 6144, both multiples
 * of 16; wider models use the per-operator entry points), allocates the
 * plan's hand-off buffers on the current device and records the op list;
 * pointers in desc must stay valid. */
int leafq_model_plan_create(const leafq_model_desc* desc, leafq_model_plan_t** plan);
/* One decode step (one cooperative launch of one block per SM). */
int leafq_model_plan_run(void* stream, leafq_model_plan_t* plan);
int leafq_model_plan_destroy(leafq_model_plan_t* plan);

/* ------------------------------------------------------------------------
 * Decoder operators around the linears (Decoder::Impl::forward_into,
 * decoder.cpp:1282-1452), for a GPU port of the decode loop.  Device
 * pointers, fp32 activations, token-major rows.  `position` is a device
 * int32 holding the number of tokens already in the KV cache, so one CUDA
 * graph serves every decode step (leafq_advance_position moves it). */

/* out[t, c] = Weight::value(ids[t], c) * embedding_scale
 * (decoder.cpp:1293-1304, :241-250); table in artifact layout (bits 8/4
 * with group scales, or fp32).  Out-of-range ids set *error_flag (if
 * given) and read row 0. */
int leafq_embed(void* stream, const int32_t* ids, int64_t tokens, const void* table,
                const float* scales, int bits, int64_t group, int64_t vocab, int64_t hidden,
                float embedding_scale, float* out, int32_t* error_flag);
/* RMSNorm (norm(), decoder.cpp:706-727) of each token row, optionally after
 * the residual add hidden += delta (+ 0.0f first when add_zero, as
 * decoder.cpp:1434 does); hidden is updated in place.  Bit-identical to the
 * reference (sum of squares accumulated left to right). */
int leafq_rmsnorm(void* stream, float* hidden, const float* delta, int add_zero, int64_t tokens,
                  int64_t width, const float* weight, float epsilon, float* out);
/* leafq_rmsnorm, and the normalised rows quantised in the same pass to
 * per-token INT8 codes [tokens][width] and scales [tokens] exactly as
 * leafq_quantize_act quantises them (the input of a W8A8 linear, for
 * leafq_linear_int_q).  out may be NULL when only the codes are wanted.
 * Codes need width % 4 == 0, width <= 4096 and 16-byte aligned rows. */
int leafq_rmsnorm_quantize(void* stream, float* hidden, const float* delta, int add_zero, int64_t tokens,
                           int64_t width, const float* weight, float epsilon, float* out, int8_t* codes,
                           float* code_scales);
/* Host function: RoPE tables [positions][rotary_dim/2] with the reference's
 * float libm calls (frequencies decoder.cpp:929-933, angles :1248-1256). */
int leafq_rope_tables(float theta, int rotary_dim, int64_t positions, float* cos_out,
                      float* sin_out);
/* qkv [tokens][(heads + 2*kv_heads) * dim] (q | k | v): rotates q and k
 * (decoder.cpp:1259-1281), writes q as [heads][tokens][dim] and appends k,
 * v at rows position..position+tokens-1 of caches [kv_heads][capacity][dim]
 * (kv_cache.cpp:21-59). */
int leafq_rotary_append(void* stream, const float* qkv, int64_t tokens, int heads, int kv_heads,
                        int dim, int rotary_dim, const float* cos_table, const float* sin_table,
                        const int32_t* position, float* q_heads, float* k_cache, float* v_cache,
                        int64_t capacity);
/* Causal GQA attention of the chunk's tokens over the cache
 * (KVCache::attend, transformer.cpp:93-145): score = (q.k * scale) * scale,
 * softmax with libm's expf, probability-weighted V, every sum in the
 * reference's order; out [tokens][heads * dim], bit-identical to the
 * reference.  Keys 0..position+t for query t; (dim + capacity) * 4 bytes
 * must fit in shared memory. */
int leafq_attention(void* stream, const float* q_heads, const float* k_cache, const float* v_cache,
                    int64_t tokens, int heads, int kv_heads, int dim, const int32_t* position,
                    int64_t capacity, float scale, float* out);
/* Batches of independent sequences (several requests decoded together).
 * Sequence s owns rows s*tokens .. s*tokens+tokens-1 of qkv and out, the
 * start position positions[s] (device int32 array), and its own caches at
 * s * kv_heads * capacity * dim of k_cache / v_cache ([sequences][kv_heads]
 * [capacity][dim]); q_heads is [sequences][heads][tokens][dim].  Every
 * sequence's results equal the single-sequence calls' bit for bit.  A start
 * position with start + tokens past the cache (or past max_keys) is not
 * processed and leafq_device_status reports it. */
int leafq_rotary_append_batch(void* stream, const float* qkv, int sequences, int64_t tokens, int heads,
                              int kv_heads, int dim, int rotary_dim, const float* cos_table,
                              const float* sin_table, const int32_t* positions, float* q_heads,
                              float* k_cache, float* v_cache, int64_t capacity);
/* Device workspace (bytes) leafq_attention_batch needs for this geometry,
 * max_keys being a bound on positions[s] + tokens (0: none needed, the
 * per-query form runs).  Prompts (16 or more tokens per sequence, head size
 * 32 or 64) run a tiled form whose scores live in the workspace. */
int64_t leafq_attention_workspace_bytes(int sequences, int64_t tokens, int heads, int kv_heads, int dim,
                                        int64_t max_keys);
int leafq_attention_batch(void* stream, const float* q_heads, const float* k_cache, const float* v_cache,
                          int sequences, int64_t tokens, int heads, int kv_heads, int dim,
                          const int32_t* positions, int64_t capacity, int64_t max_keys, float scale,
                          float* out, void* workspace, int64_t workspace_bytes);
/* gate_up [tokens][2 * width] with gate and up interleaved (g0, u0, g1, u1,
 * ..., the output of one linear over interleaved gate / up rows) -> out
 * [tokens][width] = u * (g / (1 + expf(-g))) (decoder.cpp:982-988, 1414). */
int leafq_silu_gate(void* stream, const float* gate_up, int64_t tokens, int64_t width, float* out);
/* leafq_silu_gate with the per-token INT8 quantisation of the result fused
 * in: codes [tokens][width] and scales [tokens] exactly as
 * leafq_quantize_act quantises the activations (the input of the down
 * projection, for leafq_linear_int_q); act may be NULL.  width <= 6144. */
int leafq_silu_gate_quantize(void* stream, const float* gate_up, int64_t tokens, int64_t width, float* act,
                             int8_t* codes, float* code_scales);
/* ids[r] = first index of the largest value of logits row r
 * (std::max_element, main_decoder.cpp:101). */
int leafq_argmax(void* stream, const float* logits, int64_t rows, int64_t width, int32_t* ids);
/* y[i] = expf(x[i]) bit-identical to the system libm's expf (GNU C Library
 * 2.39), the exponential of the decoder's softmax and SiLU. */
int leafq_expf(void* stream, const float* x, int64_t n, float* y);
/* *position += count on the stream. */
int leafq_advance_position(void* stream, int32_t* position, int32_t count);
/* positions[s] += count for every s < sequences, on the stream. */
int leafq_advance_positions(void* stream, int32_t* positions, int sequences, int32_t count);

#ifdef __cplusplus
}
#endif
#endif /* LEAFQ_H */
