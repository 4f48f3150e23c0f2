// Seeded synthetic data generated on the device.
//
// The benchmarks need inputs that are irregular (no compression artefacts,
// as peak_mem_2d.cpp:90-101 warns) and reproducible on the CPU for parity
// checks; a synthetic Qwen3 checkpoint is (shape, seed) rather than files.
// Every element is a pure function of (seed, tag, index), computed with a
// splitmix64 finaliser, so any window of a tensor can be generated on any
// rank and matches the CPU generator bit for bit:
//   uniform16: u = (int(h >> 40) - 2^23) * 2^-23 in [-1, 1), rounded to bf16/fp16
//   normal:    twelve 10-bit uniforms summed (Irwin-Hall), centred at 6138,
//              scaled by std/1024 in FP32, rounded to bf16
#include "common.cuh"
#include "xpu_internal.h"

namespace xpu {

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t stream_base(uint64_t seed, uint64_t tag) { return mix64(seed ^ (tag * 0xD1B54A32D192ED03ull)); }

__device__ __forceinline__ uint16_t normal_bits(uint64_t base, uint64_t i, float scale) {
  const uint64_t h1 = mix64(base + 2 * i), h2 = mix64(base + 2 * i + 1);
  int32_t sum = 0;
#pragma unroll
  for (int j = 0; j < 6; ++j)
    sum += static_cast<int32_t>((h1 >> (10 * j)) & 1023u) + static_cast<int32_t>((h2 >> (10 * j)) & 1023u);
  return float_to_bf16_bits(__fmul_rn(static_cast<float>(sum - 6138), scale));
}

__global__ void k_fill_uniform16(uint16_t *out, uint64_t n, uint64_t base, int fp16) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t h = mix64(base + i);
    const float u = __fmul_rn(static_cast<float>(static_cast<int32_t>(h >> 40) - 8388608), 1.0f / 8388608.0f);
    out[i] = fp16 ? __half_as_ushort(__float2half_rn(u)) : float_to_bf16_bits(u);
  }
}

// dst[(row_base + r * row_step) * dst_ld + c] = N(r0 + r, c0 + c) of a tensor
// whose rows are src_cols long, for r < nrows, c < ncols.
__global__ void k_fill_normal_window(uint16_t *dst, uint64_t dst_ld, uint32_t row_step,
                                     uint64_t nrows, uint64_t ncols, uint64_t src_cols, uint64_t r0,
                                     uint64_t c0, uint64_t base, float scale) {
  const uint64_t n = nrows * ncols;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t r = i / ncols, c = i - r * ncols;
    dst[r * row_step * dst_ld + c] = normal_bits(base, (r0 + r) * src_cols + (c0 + c), scale);
  }
}

__global__ void k_fill_value16(uint16_t *dst, uint64_t n, uint16_t bits) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    dst[i] = bits;
}

static unsigned fill_grid(uint64_t n) {
  const uint64_t blocks = (n + 255) / 256;
  return static_cast<unsigned>(blocks < 148ull * 64 ? (blocks ? blocks : 1) : 148ull * 64);
}

cudaError_t fill_uniform16(uint16_t *out, uint64_t n, uint64_t seed, uint64_t tag, int fp16,
                           cudaStream_t s) {
  k_fill_uniform16<<<fill_grid(n), 256, 0, s>>>(out, n, stream_base(seed, tag), fp16);
  return cudaGetLastError();
}

cudaError_t fill_normal_window(uint16_t *dst, uint64_t dst_ld, uint32_t row_step, uint64_t nrows,
                               uint64_t ncols, uint64_t src_cols, uint64_t r0, uint64_t c0,
                               uint64_t seed, uint64_t tag, float stddev, cudaStream_t s) {
  k_fill_normal_window<<<fill_grid(nrows * ncols), 256, 0, s>>>(
      dst, dst_ld, row_step, nrows, ncols, src_cols, r0, c0, stream_base(seed, tag),
      stddev * (1.0f / 1024.0f));
  return cudaGetLastError();
}

cudaError_t fill_value16(uint16_t *dst, uint64_t n, uint16_t bits, cudaStream_t s) {
  k_fill_value16<<<fill_grid(n), 256, 0, s>>>(dst, n, bits);
  return cudaGetLastError();
}

}  // namespace xpu

extern "C" {

int xpu_fill_uniform16(int dtype, void *out, uint64_t count, uint64_t seed, uint64_t tag,
                       void *stream) {
  if (!out) return xpu::fail(XPU_ERR_INVALID, "xpu_fill_uniform16: null pointer");
  if (dtype != XPU_BF16 && dtype != XPU_FP16)
    return xpu::fail(XPU_ERR_INVALID, "xpu_fill_uniform16: dtype must be XPU_BF16 or XPU_FP16");
  if (count == 0) return XPU_OK;
  return xpu::cuda_status(xpu::fill_uniform16(static_cast<uint16_t *>(out), count, seed, tag,
                                              dtype == XPU_FP16, static_cast<cudaStream_t>(stream)),
                          "xpu_fill_uniform16");
}

int xpu_fill_normal_bf16(uint16_t *out, uint64_t count, uint64_t seed, uint64_t tag, float stddev,
                         void *stream) {
  if (!out) return xpu::fail(XPU_ERR_INVALID, "xpu_fill_normal_bf16: null pointer");
  if (count == 0) return XPU_OK;
  return xpu::cuda_status(xpu::fill_normal_window(out, count, 1, 1, count, count, 0, 0, seed, tag,
                                                  stddev, static_cast<cudaStream_t>(stream)),
                          "xpu_fill_normal_bf16");
}

}  // extern "C"
