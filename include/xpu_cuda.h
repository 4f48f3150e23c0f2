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

/* QwenAdd (kernels_entry.cpp:53-58, kernels.hpp:194-207): left = bf16(left + right). */
int xpu_qwen_add(uint16_t *left, const uint16_t *right, uint32_t width, void *stream);

/* QwenSiluMultiply (kernels_entry.cpp:60-65, kernels.hpp:209-223):
 * gate = bf16(gate / (1 + exp(-gate)) * up). */
int xpu_qwen_silu_multiply(uint16_t *gate, const uint16_t *up, uint32_t width, void *stream);

/* QwenArgmax (kernels_entry.cpp:67-72, kernels.hpp:225-246): *token = first
 * index of the maximum, 0xffffffff if any value is NaN or +-Inf. */
int xpu_qwen_argmax(const uint16_t *values, uint32_t *token, uint32_t width, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* XPU_CUDA_H */
