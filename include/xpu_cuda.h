/*
 * xpu_cuda.h - C ABI of libxpu_cuda.so, the B200 (sm_100a) implementation of
 * the xpu_playground decode hot path.
 *
 * Every entry point takes plain pointers, sizes and an opaque CUDA stream
 * (a cudaStream_t passed as void*, NULL = the legacy default stream) and
 * returns an int status (XPU_OK on success). No C++ exception crosses this
 * boundary; xpu_last_error() returns the calling thread's last message.
 * Device pointers must come from cudaMalloc (or any allocation on the
 * current device). Launches are asynchronous on `stream` unless a function
 * says otherwise.
 *
 * Each declaration cites the reference interface it replaces
 * (path:line inside the DanielSawczuk/xpu_playground tree).
 */
#ifndef XPU_CUDA_H
#define XPU_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define XPU_OK 0
#define XPU_ERR_INVALID 1     /* bad argument (null pointer, size, alignment) */
#define XPU_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define XPU_ERR_UNSUPPORTED 3 /* shape or device the kernels do not support */
#define XPU_ERR_TIMEOUT 4     /* a bounded device-side wait gave up */
#define XPU_ERR_NONFINITE 5   /* NaN/Inf logits (argmax sentinel 0xffffffff) */
#define XPU_ERR_NO_MEMORY 6   /* allocation refused or device memory too small */

/* Element types of the GEMV/GEMM entry points. */
#define XPU_BF16 0
#define XPU_FP16 1

/* Last error message of the calling thread ("" if none). */
const char *xpu_last_error(void);
/* ABI revision of this header; bumps on any incompatible change. */
int xpu_abi_version(void);

/* ------------------------------------------------------------------ GEMV --
 * y[m] = A[m,k] . x[k], A row-major, FP32 accumulation, output rounded to
 * dtype. Replaces gemv::Kernel<T>::run (gemv_kernel.hpp:21-63) as launched
 * by run<T> (gemv.cpp:78-153). Unlike the reference, m and k need no padding.
 */
int xpu_gemv(int dtype, const void *matrix, const void *vector, void *output, uint32_t m,
             uint32_t k, void *stream);

/* ------------------------------------------------------------------ GEMM --
 * C[m,n] = A[m,k] . B[k,n], all row-major, FP32 accumulation on the tensor
 * cores, output rounded to dtype. Replaces gemm::Kernel<T, LargeTile>
 * (gemm_kernel.hpp:25-143) as launched by run<T, LargeTile>
 * (gemm.cpp:73-131). Unlike the reference, m, n and k need no padding to the
 * tile sizes. n and k multiples of 8 with 16-byte aligned pointers take the
 * tensor-core path; other shapes run a CUDA-core kernel.
 */
int xpu_gemm(int dtype, const void *a, const void *b, void *c, uint32_t m, uint32_t n, uint32_t k,
             void *stream);
/* C[m,n] = A[m,k] . W^T with W row-major [n,k] (the layout of a Linear
 * weight), FP32 accumulation, on the same tcgen05 kernel as xpu_gemm with the
 * second operand read K-major. No counterpart in the reference (its gemm
 * takes B as [k,n]); the dense prefill's projections use it. n and k
 * multiples of 8, operands 16-byte aligned. */
int xpu_gemm_bt(int dtype, const void *a, const void *w, void *c, uint32_t m, uint32_t n, uint32_t k, void *stream);

/* Sticky device-side error word of this library's asynchronous kernels,
 * read and cleared (synchronises the device). Bit 0: a GEMM pipeline wait
 * timed out and its tile is incomplete; bit 1: a calibrator wait timed out. No reference counterpart (the
 * reference's kernels have no bounded waits). */
int xpu_device_status(uint32_t *flags);

/* ----------------------------------------------------------- Calibrators --
 * Roofline calibrators with the reference benchmarks' checksums.
 *
 * xpu_peak_mem_fill: surface[i] = 1 + (hash(i) & 0xffff) / 65536, the
 * irregular fill of peak_mem_2d.cpp:36-47 (defeats memory compression).
 * xpu_peak_mem_read: reads a row-major float surface 1024 wide and
 * surface_height rows (a multiple of 32) once; sink[u] (one per 2 KiB read
 * unit, surface_height * 2 units) = the FP32 sum of the unit's elements at
 * rows y, y+8, y+16, y+24 of column x, x = 16 (u % 64), y = 32 (u / 64).
 * Replaces peak_mem_2d_kernel (peak_mem_2d_kernel.cpp:16-52).
 * xpu_peak_compute: `ctas` CTAs each issue rounds x 8 tensor-core MMAs of
 * 128x256x16 bf16 (1,048,576 FLOP each) on 0.5-filled tiles; sink[cta] =
 * 1 + 32 * rounds. rounds <= 524287. Replaces peak_compute_dpas_kernel
 * (peak_compute_dpas_kernel.cpp:13-68).
 */
int xpu_peak_mem_fill(float *surface, uint64_t elements, void *stream);
int xpu_peak_mem_read(const float *surface, float *sink, uint32_t surface_height, void *stream);
int xpu_peak_compute(float *sink, uint32_t ctas, uint32_t rounds, void *stream);

/* ------------------------------------------------------- Qwen3 operators --
 * One entry per reference kernel entry (qwen3/kernels_entry.cpp:8-72), with
 * the same argument order. All tensors are bf16 (uint16_t bit patterns).
 * The reference passes the launch width as `work_items`
 * (qwen3/main.cpp:162-220); here it is an explicit argument.
 */

/* QwenEmbedding (kernels_entry.cpp:8-13, kernels.hpp:24-34):
 * output[i] = table[token*width + i], i < width. */
int xpu_qwen_embedding(const uint16_t *table, uint16_t *output, uint32_t token, uint32_t width,
                       void *stream);

/* QwenRmsNorm (kernels_entry.cpp:15-21, kernels.hpp:36-56):
 * output = bf16(input * weight * rsqrt(mean(input^2) + epsilon)). */
int xpu_qwen_rms_norm(const uint16_t *input, const uint16_t *weight, uint16_t *output,
                      uint32_t width, float epsilon, void *stream);

/* QwenGemv (kernels_entry.cpp:23-29): bf16 xpu_gemv. */
int xpu_qwen_gemv(const uint16_t *matrix, const uint16_t *vector, uint16_t *output,
                  uint32_t rows, uint32_t columns, void *stream);

/* QwenQkvRopeCache (kernels_entry.cpp:31-42, kernels.hpp:58-155): per-head
 * QK-RMSNorm (eps 1e-6), rotate-half RoPE from the bf16 tables at `position`,
 * K/V written to cache slot [(position*key_value_heads + h)*128]. query is
 * rewritten in place (normed + roped), key in place (normed), value copied.
 * Does nothing when position >= maximum_sequence (kernels.hpp:74-75).
 * head_dim is 128; query_heads must be a multiple of key_value_heads. */
int xpu_qwen_qkv_rope_cache(uint16_t *query, uint16_t *key, const uint16_t *value,
                            const uint16_t *query_norm, const uint16_t *key_norm,
                            const uint16_t *rope_cos, const uint16_t *rope_sin,
                            uint16_t *key_cache, uint16_t *value_cache, uint32_t position,
                            uint32_t maximum_sequence, uint32_t query_heads,
                            uint32_t key_value_heads, void *stream);

/* Bytes of FP32 workspace xpu_qwen_attention needs for positions
 * 0..maximum_positions-1. */
size_t xpu_qwen_attention_workspace_size(uint32_t query_heads, uint32_t maximum_positions);

/* QwenAttention (kernels_entry.cpp:44-51, kernels.hpp:157-192): GQA decode
 * attention over cache positions 0..position, FP32 softmax, scale 1/sqrt(128).
 * Head h reads KV head h / (query_heads / key_value_heads). The caller owns
 * `workspace` (at least xpu_qwen_attention_workspace_size(query_heads,
 * position + 1) bytes, 16-byte aligned). query_heads / key_value_heads must
 * be 1, 2, 4 or 8. */
int xpu_qwen_attention(const uint16_t *query, const uint16_t *key_cache,
                       const uint16_t *value_cache, uint16_t *output, uint32_t position,
                       uint32_t query_heads, uint32_t key_value_heads, void *workspace,
                       size_t workspace_bytes, void *stream);

/* Attention for callers that cannot allocate device memory (no counterpart in
 * the reference): same inputs, output and kernels as xpu_qwen_attention, but
 * the split-K scratch is a fixed 6 MiB array inside this library instead of a
 * caller-owned workspace, and nothing is allocated. For hosts whose allocator
 * owns the device, serving loops that may not call cudaMalloc/cudaFree (they
 * can synchronise the device), or plugin hosts that pass only inputs and
 * outputs. Limit: xpu_qwen_attention_workspace_size(query_heads, position + 1)
 * must be at most 6 MiB (32 query heads: every position up to 40,959);
 * larger requests return XPU_ERR_INVALID. The array costs 6 MiB on each device
 * where this code is loaded, until exit. The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture; after a cudaDeviceReset the next call looks it up
 * again. All calls share the one array: calls that can overlap on the GPU
 * (different streams, or different threads on one device) race on it and
 * must be ordered by the caller (the qwen3::LevelZeroRuntime class does this
 * for its attention launches with a per-device lock). */
int xpu_qwen_attention_noalloc(const uint16_t *query, const uint16_t *key_cache,
                               const uint16_t *value_cache, uint16_t *output, uint32_t position,
                               uint32_t query_heads, uint32_t key_value_heads, void *stream);

/* QwenAdd (kernels_entry.cpp:53-58, kernels.hpp:194-207): left = bf16(left + right). */
int xpu_qwen_add(uint16_t *left, const uint16_t *right, uint32_t width, void *stream);

/* QwenSiluMultiply (kernels_entry.cpp:60-65, kernels.hpp:209-223):
 * gate = bf16(gate / (1 + exp(-gate)) * up). */
int xpu_qwen_silu_multiply(uint16_t *gate, const uint16_t *up, uint32_t width, void *stream);

/* QwenArgmax (kernels_entry.cpp:67-72, kernels.hpp:225-246): *token = first
 * index of the maximum, 0xffffffff if any value is NaN or +-Inf. */
int xpu_qwen_argmax(const uint16_t *values, uint32_t *token, uint32_t width, void *stream);

/* ------------------------------------------------------- synthetic data --
 * Seeded, irregular inputs generated on the device (the reference generates
 * its benchmark inputs on the device too: gemv.cpp:156-167). Each element is
 * a pure function of (seed, tag, index); the CPU oracle reproduces it bit
 * for bit. */

/* out[i] = uniform[-1, 1) rounded to dtype (XPU_BF16 / XPU_FP16). */
int xpu_fill_uniform16(int dtype, void *out, uint64_t count, uint64_t seed, uint64_t tag,
                       void *stream);
/* out[i] ~ N(0, stddev^2) (Irwin-Hall sum of twelve 10-bit uniforms), bf16. */
int xpu_fill_normal_bf16(uint16_t *out, uint64_t count, uint64_t seed, uint64_t tag, float stddev,
                         void *stream);

/* ------------------------------------------------------ Qwen3 decoder --
 * The decode engine of qwen3/main.cpp:118-329 (Engine): weights in one
 * device arena, bf16 KV caches [layer][position][kv_head][128], RoPE tables,
 * and one decode step captured as a CUDA graph. Shape-generic (the
 * reference pins Qwen3-8B in qwen3/model.hpp:11-22): head_dim 128,
 * query/key-value head ratio 1, 2, 4 or 8, tied or untied lm_head.
 * tp_size > 1 builds rank tp_rank of a tensor-parallel group. */
typedef struct xpu_qwen3_engine xpu_qwen3_engine;

typedef struct {
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_hidden_layers;
  uint32_t num_attention_heads;
  uint32_t num_key_value_heads;
  uint32_t vocab_size;
  uint32_t tie_word_embeddings; /* 0 or 1 */
  float rms_norm_eps;
  double rope_theta;
} xpu_qwen3_shape;

typedef struct {
  uint64_t weight_bytes;     /* bytes of this rank's weight arena */
  uint32_t kernels_per_step; /* kernel launches in one decode step */
  uint32_t vocab_rows;       /* lm_head rows held by this rank */
  uint32_t vocab_offset;     /* first vocabulary id of this rank */
  void *stream;              /* the engine's CUDA stream */
} xpu_qwen3_info_t;

/* Engine ctor + Engine::reserve (qwen3/main.cpp:120-157): allocates the
 * weight arena, caches for maximum_sequence positions and the activations on
 * `device`. */
int xpu_qwen3_create(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                     uint32_t tp_rank, uint32_t tp_size, xpu_qwen3_engine **out);
int xpu_qwen3_destroy(xpu_qwen3_engine *engine);
/* ------------------------------------------------------- checkpoints --
 * Replace load_and_validate_config / load_and_validate_checkpoint
 * (qwen3/model.cpp:376-495) for any Qwen3 shape with head_dim 128, tied or
 * untied, sharded (model.safetensors.index.json) or single-file
 * (model.safetensors). Checks: model_type qwen3, silu, bfloat16, no
 * rope_scaling; BF16 tensors with exactly the shapes the config implies,
 * every expected tensor and nothing else, payloads inside their shard and
 * not overlapping, the index's total_size equal to the payload bytes.
 *
 * xpu_qwen3_read_config: <model_dir>/config.json -> *shape.
 * xpu_qwen3_validate_checkpoint: config + every tensor header, no GPU needed;
 *   *payload_bytes (optional) = total tensor bytes.
 * xpu_qwen3_load_checkpoint: validates against the engine's shape and streams
 *   this rank's part of every tensor to the GPU (pinned double buffering). */
int xpu_qwen3_read_config(const char *model_dir, xpu_qwen3_shape *shape);
int xpu_qwen3_validate_checkpoint(const char *model_dir, xpu_qwen3_shape *shape, uint64_t *payload_bytes);
int xpu_qwen3_load_checkpoint(xpu_qwen3_engine *engine, const char *model_dir);

/* Tensor-parallel rendezvous (tp_size > 1; ranks are processes, one GPU
 * each, on one NVLink/NVSwitch node). Each rank writes its exchange-region
 * handle (XPU_TP_HANDLE_BYTES bytes, a CUDA IPC handle) with
 * xpu_qwen3_tp_handle; the caller all-gathers the handles over its host
 * process group (the reference has no tensor parallelism; this replaces
 * nothing) and every rank calls xpu_qwen3_tp_connect with all tp_size handles
 * in rank order. Decoding before that fails with XPU_ERR_INVALID. Every rank
 * must then make the same decode/generate calls in the same order; an
 * exchange that times out (a rank stopped) returns XPU_ERR_TIMEOUT on the
 * waiting ranks and leaves the engines unusable (recreate them). */
#define XPU_TP_HANDLE_BYTES 64
int xpu_qwen3_tp_handle(xpu_qwen3_engine *engine, void *handle);
int xpu_qwen3_tp_connect(xpu_qwen3_engine *engine, const void *handles, uint32_t count);

/* Seeded synthetic checkpoint: norm weights 1, all other tensors N(0, stddev)
 * drawn per tensor (xpu_fill_normal_bf16 stream = tensor tag: 0 embed, 1 final
 * norm, 2 lm_head, 3 + 11*layer + index in the layer's tensor list). */
int xpu_qwen3_init_synthetic(xpu_qwen3_engine *engine, uint64_t seed, float stddev);
/* Engine::upload_weights (qwen3/main.cpp:265-298) for one tensor: `elements`
 * bf16 values of the full, unsharded checkpoint tensor `name` (safetensors
 * naming, qwen3/model.cpp:412-425) from host memory; this rank keeps its shard. */
int xpu_qwen3_set_tensor(xpu_qwen3_engine *engine, const char *name, const uint16_t *host_bf16,
                         uint64_t elements);
/* Engine::decode (qwen3/main.cpp:159-226): one synchronous step; returns the
 * greedy next token. XPU_ERR_NONFINITE (and 0xffffffff) on NaN/Inf logits. */
int xpu_qwen3_decode(xpu_qwen3_engine *engine, uint32_t token, uint32_t position,
                     uint32_t *next_token);
/* qwen3/main.cpp:342-352 on the device: the prompt fed token by token, then up
 * to max_new_tokens greedy tokens (stopping after EOS 151645 / 151643 when
 * stop_at_eos), with one host synchronisation. */
int xpu_qwen3_generate(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len,
                       uint32_t max_new_tokens, int stop_at_eos, uint32_t *out_tokens,
                       uint32_t *out_count);
/* Device-resident stepping: set the next step's input, enqueue steps without
 * synchronising (each step feeds its greedy token to the next), read back. */
int xpu_qwen3_set_state(xpu_qwen3_engine *engine, uint32_t token, uint32_t position,
                        uint32_t prompt_len);
int xpu_qwen3_enqueue_steps(xpu_qwen3_engine *engine, uint32_t steps, void *stream);
int xpu_qwen3_get_state(xpu_qwen3_engine *engine, uint32_t *last_token, uint32_t *next_position,
                        uint32_t *error);
int xpu_qwen3_synchronize(xpu_qwen3_engine *engine);
/* Decode-step implementation: 0 = one persistent cooperative kernel per
 * token (default), 1 = a CUDA graph of per-phase kernels. Identical results;
 * set before the first decode. */
int xpu_qwen3_set_mode(xpu_qwen3_engine *engine, int mode);
/* Step tracing (persistent mode, when the process runs with XPU_STEP_TRACE=1):
 * per-CTA globaltimer stamps (ns) of the last step's phase boundaries,
 * [cta][event]; *count = total stamps available (0 when tracing is off). */
int xpu_qwen3_trace(xpu_qwen3_engine *engine, uint64_t *host_ns, uint32_t capacity, uint32_t *count);
/* Greedy token of every step at positions [first_position, first_position +
 * count): entry p is the token the step at position p produced (the prompt's
 * last position holds the first generated token), as main.cpp:345-352 would
 * print them; written by every decode path (decode, generate, device-resident
 * steps, prefill). No counterpart call in the reference, whose engine returns
 * each token from decode(). */
int xpu_qwen3_token_log(xpu_qwen3_engine *engine, uint32_t first_position, uint32_t count,
                        uint32_t *host_out);
/* bf16 logits of the last step (this rank's vocab_rows rows). */
int xpu_qwen3_logits(xpu_qwen3_engine *engine, uint16_t *host_out, uint32_t count);
int xpu_qwen3_info(xpu_qwen3_engine *engine, xpu_qwen3_info_t *info);
/* Algorithmic HBM bytes of one decode step at `context` cached positions:
 * every weight streamed once (one embedding row) plus K/V reads. */
uint64_t xpu_qwen3_bytes_per_token(xpu_qwen3_engine *engine, uint32_t context);

/* ------------------------------------------------------ batched decode --
 * Up to XPU_MAX_BATCH sequences per step on one GPU (the reference decodes
 * one sequence per Engine; qwen3/main.cpp:159-226 per sequence). Each step
 * streams the weights once for every sequence (tcgen05 GEMMs with N = 16);
 * norms, RoPE, the KV cache, attention and argmax are per sequence with the
 * batch-1 arithmetic. xpu_qwen3_create_batched makes a single-GPU engine
 * whose KV cache holds max_batch sequences (sequence 0 is the one the
 * batch-1 calls above use); every engine accepts batch 1.
 * xpu_qwen3_create_batched_tp makes one rank of a tensor-parallel batched
 * engine (connect it with xpu_qwen3_tp_connect like the batch-1 engine;
 * every rank then makes the same batch calls): each rank streams its shard
 * of the weights, o_proj and down partials are summed across the ranks in
 * rank order through the exchange regions, the lm_head candidates of every
 * sequence meet the same way, and every rank returns the same tokens.
 * Unlike the batch-1 path the row-parallel sums are not in a fixed order
 * shared with one GPU, so logits match one GPU within rounding, not bit
 * for bit. xpu_qwen3_batch_logits then returns this rank's vocabulary
 * shard.
 *
 * xpu_qwen3_batch_decode: one synchronous step of sequences 0..batch-1,
 *   tokens[s] at positions[s] -> next_tokens[s]; XPU_ERR_NONFINITE if any
 *   sequence's logits held a NaN/Inf (its token is 0xffffffff).
 * xpu_qwen3_batch_generate: prompts (back to back, prompt_lens[s] tokens
 *   each) fed token by token, then up to max_new_tokens greedy tokens per
 *   sequence into out_tokens[s * max_new_tokens + i], out_counts[s] as
 *   xpu_qwen3_generate; all sequences advance together, one host sync.
 * xpu_qwen3_batch_set_state / _enqueue_steps / _get_state: device-resident
 *   stepping of the batch set up by the last batched call.
 * xpu_qwen3_batch_logits: bf16 logits of row `sequence` (< 16) of the last
 *   batched step: sequence s of a batch, or after xpu_qwen3_prefill the last
 *   chunk's positions, the last prompt position in row (prompt_len - 1) % 16. */
#define XPU_MAX_BATCH 16
/* Chunked prefill of the batch-1 sequence (replaces the token-by-token prompt
 * loop of qwen3/main.cpp:343-344): prompt[0..prompt_len) runs 16 positions
 * per step through the batched GEMMs, with causal attention inside each
 * chunk, writing the batch-1 KV cache; then the engine's state continues at
 * position prompt_len with *next_token (the greedy token after the prompt),
 * so xpu_qwen3_enqueue_steps / xpu_qwen3_decode carry on from there. One
 * GPU only. */
int xpu_qwen3_prefill(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len, uint32_t *next_token);
/* Dense prefill of the batch-1 sequence (no counterpart in the reference,
 * which feeds the prompt token by token, qwen3/main.cpp:343-344): every
 * prompt position goes through each layer together - the projections as
 * tcgen05 GEMMs over all positions against the stored weights (compute-bound),
 * causal attention over the cache - in segments of up to 2048 positions.
 * Same result contract as xpu_qwen3_prefill (greedy token after the prompt
 * returned, engine left at position prompt_len), with the last position's
 * logits (this rank's vocabulary shard) in xpu_qwen3_logits. Tensor parallel
 * engines (connected with xpu_qwen3_tp_connect) call it on every rank with
 * the same prompt; o_proj and down are summed over 8 fixed K chunks in a
 * fixed order, so every tp_size returns the same token and logits bits and
 * writes the same KV cache. A rank whose peers do not join within ~2 s
 * returns XPU_ERR_TIMEOUT and the engines must be recreated. */
int xpu_qwen3_prefill_dense(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len,
                            uint32_t *next_token);
int xpu_qwen3_create_batched(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                             uint32_t max_batch, xpu_qwen3_engine **out);
int xpu_qwen3_create_batched_tp(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                                uint32_t tp_rank, uint32_t tp_size, uint32_t max_batch, xpu_qwen3_engine **out);
int xpu_qwen3_batch_decode(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *tokens,
                           const uint32_t *positions, uint32_t *next_tokens);
int xpu_qwen3_batch_generate(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *prompts,
                             const uint32_t *prompt_lens, uint32_t max_new_tokens, int stop_at_eos,
                             uint32_t *out_tokens, uint32_t *out_counts);
int xpu_qwen3_batch_set_state(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *tokens,
                              const uint32_t *positions);
int xpu_qwen3_batch_enqueue_steps(xpu_qwen3_engine *engine, uint32_t steps, void *stream);
int xpu_qwen3_batch_get_state(xpu_qwen3_engine *engine, uint32_t batch, uint32_t *last_tokens,
                              uint32_t *next_positions, uint32_t *error);
int xpu_qwen3_batch_logits(xpu_qwen3_engine *engine, uint32_t sequence, uint16_t *host_out, uint32_t count);
/* Algorithmic HBM bytes of one batched step: the weights once plus every
 * sequence's K/V over `context` positions. */
uint64_t xpu_qwen3_batch_bytes_per_step(xpu_qwen3_engine *engine, uint32_t batch, uint32_t context);
uint32_t xpu_qwen3_batch_kernels_per_step(xpu_qwen3_engine *engine);
/* Batched-step tracing (when the process runs with XPU_BATCH_TRACE=1): per
 * kernel of the step, in launch order, 8 globaltimer values (ns): first CTA
 * start, last return from the wait on the previous kernel, last CTA end,
 * first return from that wait, last CTA start, and for the GEMMs the last
 * CTA's first landed stage, final accumulator and epilogue end; over all
 * steps since the previous call, which it resets. *count = values written
 * (0 when tracing is off). */
int xpu_qwen3_batch_trace(xpu_qwen3_engine *engine, uint64_t *host_ns, uint32_t capacity, uint32_t *count);

#ifdef __cplusplus
}
#endif

#endif /* XPU_CUDA_H */
