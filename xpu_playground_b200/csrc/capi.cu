// extern "C" entry points of libxpu_cuda (declared in include/xpu_cuda.h).
// Each validates its arguments on the host, launches on the caller's stream
// and converts every failure into a status code plus a thread-local message.
#include <exception>
#include <string>

#include "xpu_internal.h"

namespace xpu {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string &message) { g_last_error = message; }

int fail(int status, const std::string &message) {
  g_last_error = message;
  return status;
}

int cuda_status(cudaError_t error, const char *what) {
  if (error == cudaSuccess) return XPU_OK;
  return fail(XPU_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(error) + " (" +
                                cudaGetErrorString(error) + ")");
}

}  // namespace xpu

using namespace xpu;

static inline cudaStream_t as_stream(void *stream) { return static_cast<cudaStream_t>(stream); }

#define XPU_REQUIRE(cond, msg) \
  do {                         \
    if (!(cond)) return fail(XPU_ERR_INVALID, msg); \
  } while (0)

// Wraps a body so that no C++ exception crosses the C boundary.
#define XPU_GUARD(body)                                               \
  try {                                                               \
    body                                                              \
  } catch (const std::exception &e) {                                 \
    return fail(XPU_ERR_INVALID, std::string("exception: ") + e.what()); \
  } catch (...) {                                                     \
    return fail(XPU_ERR_INVALID, "unknown exception");                \
  }

extern "C" {

const char *xpu_last_error(void) { return g_last_error.c_str(); }

int xpu_abi_version(void) { return 1; }

int xpu_gemv(int dtype, const void *matrix, const void *vector, void *output, uint32_t m,
             uint32_t k, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(matrix && vector && output, "xpu_gemv: null pointer");
    XPU_REQUIRE(m > 0 && k > 0, "xpu_gemv: m and k must be positive");
    cudaError_t e;
    if (dtype == XPU_BF16)
      e = gemv_launch(static_cast<const __nv_bfloat16 *>(matrix),
                      static_cast<const __nv_bfloat16 *>(vector),
                      static_cast<__nv_bfloat16 *>(output), m, k, as_stream(stream));
    else if (dtype == XPU_FP16)
      e = gemv_launch(static_cast<const __half *>(matrix), static_cast<const __half *>(vector),
                      static_cast<__half *>(output), m, k, as_stream(stream));
    else
      return fail(XPU_ERR_INVALID, "xpu_gemv: dtype must be XPU_BF16 or XPU_FP16");
    return cuda_status(e, "xpu_gemv");
  })
}

int xpu_gemm(int dtype, const void *a, const void *b, void *c, uint32_t m, uint32_t n, uint32_t k,
             void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(a && b && c, "xpu_gemm: null pointer");
    XPU_REQUIRE(m > 0 && n > 0 && k > 0, "xpu_gemm: m, n and k must be positive");
    if (dtype != XPU_BF16 && dtype != XPU_FP16)
      return fail(XPU_ERR_INVALID, "xpu_gemm: dtype must be XPU_BF16 or XPU_FP16");
    return cuda_status(gemm_launch(dtype == XPU_FP16, a, b, c, m, n, k, as_stream(stream)), "xpu_gemm");
  })
}

int xpu_gemm_bt(int dtype, const void *a, const void *w, void *c, uint32_t m, uint32_t n, uint32_t k, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(a && w && c, "xpu_gemm_bt: null pointer");
    XPU_REQUIRE(m > 0 && n > 0 && k > 0, "xpu_gemm_bt: m, n and k must be positive");
    XPU_REQUIRE(n % 8 == 0 && k % 8 == 0, "xpu_gemm_bt: n and k must be multiples of 8");
    XPU_REQUIRE(aligned16(a) && aligned16(w) && aligned16(c), "xpu_gemm_bt: operands must be 16-byte aligned");
    if (dtype != XPU_BF16 && dtype != XPU_FP16)
      return fail(XPU_ERR_INVALID, "xpu_gemm_bt: dtype must be XPU_BF16 or XPU_FP16");
    return cuda_status(gemm_launch_ex(dtype == XPU_FP16, true, a, w, c, m, n, k, as_stream(stream)), "xpu_gemm_bt");
  })
}

int xpu_device_status(uint32_t *flags) {
  XPU_GUARD({
    XPU_REQUIRE(flags, "xpu_device_status: null pointer");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_status(e, "xpu_device_status");
    *flags = take_device_error() | take_peak_error();
    return XPU_OK;
  })
}

int xpu_qwen_embedding(const uint16_t *table, uint16_t *output, uint32_t token, uint32_t width,
                       void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(table && output, "xpu_qwen_embedding: null pointer");
    if (width == 0) return XPU_OK;
    return cuda_status(qwen_embedding_launch(table, output, token, width, as_stream(stream)),
                       "xpu_qwen_embedding");
  })
}

int xpu_qwen_rms_norm(const uint16_t *input, const uint16_t *weight, uint16_t *output,
                      uint32_t width, float epsilon, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(input && weight && output, "xpu_qwen_rms_norm: null pointer");
    XPU_REQUIRE(width > 0, "xpu_qwen_rms_norm: width must be positive");
    return cuda_status(qwen_rms_norm_launch(input, weight, output, width, epsilon,
                                            as_stream(stream)),
                       "xpu_qwen_rms_norm");
  })
}

int xpu_qwen_gemv(const uint16_t *matrix, const uint16_t *vector, uint16_t *output,
                  uint32_t rows, uint32_t columns, void *stream) {
  return xpu_gemv(XPU_BF16, matrix, vector, output, rows, columns, stream);
}

int xpu_qwen_qkv_rope_cache(uint16_t *query, uint16_t *key, const uint16_t *value,
                            const uint16_t *query_norm, const uint16_t *key_norm,
                            const uint16_t *rope_cos, const uint16_t *rope_sin,
                            uint16_t *key_cache, uint16_t *value_cache, uint32_t position,
                            uint32_t maximum_sequence, uint32_t query_heads,
                            uint32_t key_value_heads, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(query && key && value && query_norm && key_norm && rope_cos && rope_sin &&
                    key_cache && value_cache,
                "xpu_qwen_qkv_rope_cache: null pointer");
    XPU_REQUIRE(key_value_heads > 0 && query_heads >= key_value_heads &&
                    query_heads % key_value_heads == 0,
                "xpu_qwen_qkv_rope_cache: query_heads must be a positive multiple of "
                "key_value_heads");
    return cuda_status(
        qwen_qkv_rope_cache_launch(query, key, value, query_norm, key_norm, rope_cos, rope_sin,
                                   key_cache, value_cache, position, maximum_sequence,
                                   query_heads, key_value_heads, as_stream(stream)),
        "xpu_qwen_qkv_rope_cache");
  })
}

size_t xpu_qwen_attention_workspace_size(uint32_t query_heads, uint32_t maximum_positions) {
  return qwen_attention_workspace(query_heads, maximum_positions);
}

int xpu_qwen_attention(const uint16_t *query, const uint16_t *key_cache,
                       const uint16_t *value_cache, uint16_t *output, uint32_t position,
                       uint32_t query_heads, uint32_t key_value_heads, void *workspace,
                       size_t workspace_bytes, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(query && key_cache && value_cache && output && workspace,
                "xpu_qwen_attention: null pointer");
    XPU_REQUIRE(aligned16(workspace), "xpu_qwen_attention: workspace must be 16-byte aligned");
    XPU_REQUIRE(key_value_heads > 0 && query_heads % key_value_heads == 0,
                "xpu_qwen_attention: query_heads must be a multiple of key_value_heads");
    const uint32_t group = query_heads / key_value_heads;
    if (group != 1 && group != 2 && group != 4 && group != 8)
      return fail(XPU_ERR_UNSUPPORTED, "xpu_qwen_attention: query_heads / key_value_heads must "
                                       "be 1, 2, 4 or 8");
    XPU_REQUIRE(position != UINT32_MAX, "xpu_qwen_attention: position out of range");
    const size_t need = qwen_attention_workspace(query_heads, position + 1);
    if (workspace_bytes < need)
      return fail(XPU_ERR_INVALID, "xpu_qwen_attention: workspace holds " +
                                       std::to_string(workspace_bytes) + " bytes, needs " +
                                       std::to_string(need));
    return cuda_status(qwen_attention_launch(query, key_cache, value_cache, output, position,
                                             query_heads, key_value_heads,
                                             static_cast<float *>(workspace), as_stream(stream)),
                       "xpu_qwen_attention");
  })
}

int xpu_qwen_add(uint16_t *left, const uint16_t *right, uint32_t width, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(left && right, "xpu_qwen_add: null pointer");
    if (width == 0) return XPU_OK;
    return cuda_status(qwen_add_launch(left, right, width, as_stream(stream)), "xpu_qwen_add");
  })
}

int xpu_qwen_silu_multiply(uint16_t *gate, const uint16_t *up, uint32_t width, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(gate && up, "xpu_qwen_silu_multiply: null pointer");
    if (width == 0) return XPU_OK;
    return cuda_status(qwen_silu_multiply_launch(gate, up, width, as_stream(stream)),
                       "xpu_qwen_silu_multiply");
  })
}

int xpu_qwen_argmax(const uint16_t *values, uint32_t *token, uint32_t width, void *stream) {
  XPU_GUARD({
    XPU_REQUIRE(values && token, "xpu_qwen_argmax: null pointer");
    return cuda_status(qwen_argmax_launch(values, token, width, as_stream(stream)),
                       "xpu_qwen_argmax");
  })
}

}  // extern "C"
