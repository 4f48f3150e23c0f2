// Internal declarations shared by the translation units of libxpu_cuda.
// Nothing here is part of the C ABI (include/xpu_cuda.h is).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/xpu_cuda.h"

namespace xpu {

// Largest vector (in bytes) the GEMV stages whole into shared memory.
constexpr size_t kMaxGemvVectorBytes = 200 * 1024;

__host__ __device__ inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Thread-local "last error" text behind xpu_last_error().
void set_error(const std::string &message);
int fail(int status, const std::string &message);
int cuda_status(cudaError_t error, const char *what);

// ---- TMA tensor maps (tmap.cu) ----
cudaError_t make_tmap_2d_u16(struct CUtensorMap_st *map, const void *base, uint64_t cols, uint64_t rows,
                             uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows);
cudaError_t make_tmap_2d_u16_swizzled(struct CUtensorMap_st *map, const void *base, uint64_t cols, uint64_t rows,
                                      uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows);

cudaError_t make_tmap_3d_u16_swizzled(struct CUtensorMap_st *map, const void *base, uint64_t d0, uint64_t d1,
                                      uint64_t d2, uint64_t stride1, uint64_t stride2, uint32_t box_cols,
                                      uint32_t box_rows);

// ---- GEMM (gemm.cu) ----
cudaError_t gemm_launch(bool fp16, const void *A, const void *B, void *C, uint32_t m, uint32_t n, uint32_t k,
                        cudaStream_t stream);
// C[M,N] = A[M,K] . B with B row-major [K,N], or (b_kmajor) C = A . B^T with
// B row-major [N,K] (tcgen05 path only: K and N multiples of 8, 16-byte
// aligned operands).
cudaError_t gemm_launch_ex(bool fp16, bool b_kmajor, const void *A, const void *B, void *C, uint32_t m, uint32_t n,
                           uint32_t k, cudaStream_t stream);
// Split GEMM for the row-parallel prefill projections: with A row-major
// [M, chunks x Kc] and W row-major [N, chunks x Kc], C[c] = A[:, chunk c] .
// W[:, chunk c]^T as FP32 [chunks][M][N], one accumulation per chunk (bf16
// in; Kc and N multiples of 8, 16-byte aligned operands).
cudaError_t gemm_chunks_launch(const void *A, const void *W, float *C, uint32_t M, uint32_t N, uint32_t Kc,
                               uint32_t chunks, cudaStream_t stream);
// Reads and clears the sticky device error word (bit 0: a GEMM wait timed out).
unsigned take_device_error();
// Same for the calibrator kernels (peak.cu; bit 1: a pipeline wait timed out).
unsigned take_peak_error();

// ---- dense prefill (prefill.cu): bf16 [M][width] row-major activations ----
cudaError_t prefill_embed(const uint16_t *embed, const uint32_t *tokens, uint16_t *x, uint32_t M, uint32_t H,
                          cudaStream_t s);
cudaError_t prefill_rms(const uint16_t *x, const uint16_t *w, uint16_t *xn, uint32_t M, uint32_t H, float eps,
                        cudaStream_t s);
cudaError_t prefill_heads(const uint16_t *qkv, const uint16_t *q_norm, const uint16_t *k_norm, const uint16_t *cos_t,
                          const uint16_t *sin_t, uint16_t *q, uint16_t *kc, uint16_t *vc, uint32_t p0, uint32_t M,
                          uint32_t QH, uint32_t KVH, float eps, cudaStream_t s);
cudaError_t prefill_attention(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, uint16_t *out, uint32_t p0,
                              uint32_t M, uint32_t QH, uint32_t KVH, cudaStream_t s);
cudaError_t prefill_swiglu(const uint16_t *gu, uint16_t *h, uint32_t M, uint32_t I, cudaStream_t s);

// ---- GEMV ----
template <typename T>
cudaError_t gemv_launch(const T *A, const T *x, T *y, uint32_t m, uint32_t k,
                        cudaStream_t stream);

// ---- Qwen3 operators with the reference kernels' semantics ----
cudaError_t qwen_embedding_launch(const uint16_t *table, uint16_t *out, uint32_t token,
                                  uint32_t width, cudaStream_t stream);
cudaError_t qwen_rms_norm_launch(const uint16_t *in, const uint16_t *w, uint16_t *out,
                                 uint32_t width, float eps, cudaStream_t stream);
cudaError_t qwen_qkv_rope_cache_launch(uint16_t *q, uint16_t *k, const uint16_t *v,
                                       const uint16_t *qn, const uint16_t *kn,
                                       const uint16_t *cos_table, const uint16_t *sin_table,
                                       uint16_t *kc, uint16_t *vc, uint32_t position,
                                       uint32_t max_seq, uint32_t q_heads, uint32_t kv_heads,
                                       cudaStream_t stream);
size_t qwen_attention_workspace(uint32_t q_heads, uint32_t max_positions);
cudaError_t qwen_attention_launch(const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                  uint16_t *out, uint32_t position, uint32_t q_heads,
                                  uint32_t kv_heads, float *workspace, cudaStream_t stream);
cudaError_t qwen_add_launch(uint16_t *left, const uint16_t *right, uint32_t width,
                            cudaStream_t stream);
cudaError_t qwen_silu_multiply_launch(uint16_t *gate, const uint16_t *up, uint32_t width,
                                      cudaStream_t stream);
cudaError_t qwen_argmax_launch(const uint16_t *values, uint32_t *token, uint32_t width,
                               cudaStream_t stream);

// ---- Qwen3 checkpoints (loader.cpp) ----
struct CkptTensor {
  std::string name, path;       // tensor name, shard file
  uint64_t offset = 0, bytes = 0;  // payload position in the file
  std::vector<uint64_t> shape;
};
// Reads <dir>/config.json into a shape (throws std::runtime_error on anything
// this engine cannot run).
void read_qwen3_config(const std::string &dir, xpu_qwen3_shape *out, uint32_t *eos_token_id);
// Every tensor the shape needs, located and validated in <dir>'s safetensors.
std::vector<CkptTensor> index_qwen3_checkpoint(const std::string &dir, const xpu_qwen3_shape &shape);
std::vector<std::string> qwen3_tensor_names(const xpu_qwen3_shape &s);
std::vector<uint64_t> qwen3_tensor_shape(const xpu_qwen3_shape &s, const std::string &name);

// Positional reads (pread) of one open file.
class FileReader {
 public:
  explicit FileReader(const std::string &path);
  ~FileReader();
  FileReader(const FileReader &) = delete;
  FileReader &operator=(const FileReader &) = delete;
  uint64_t size() const;
  void read(void *dst, uint64_t bytes, uint64_t offset) const;

 private:
  int fd_;
  std::string path_;
};

}  // namespace xpu
