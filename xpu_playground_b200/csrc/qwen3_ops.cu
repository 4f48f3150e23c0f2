// Qwen3 per-token operators with the semantics of the reference's eSIMD
// kernels (qwen3/kernels.hpp), one CUDA kernel per reference entry point
// (qwen3/kernels_entry.cpp:9-72). These are the drop-in operator ABI; the
// decode engine uses the fused kernels in decode_kernels.cu instead.
//
// Shapes are generic where the reference hard-codes Qwen3-8B: the hidden
// width, the number of query and key/value heads and the cache length are
// arguments. head_dim is fixed at 128 (every Qwen3 checkpoint uses it).
#include "common.cuh"
#include "xpu_internal.h"

namespace xpu {

constexpr uint32_t kHeadDim = 128;
constexpr float kAttentionScale = 0.08838834764831845f;  // 1/sqrt(128), kernels.hpp:173
constexpr uint32_t kAttnChunk = 128;                      // positions per split-K chunk
constexpr uint32_t kAttnStride = kHeadDim + 2;            // (max, sum, acc[128]) per chunk

// ----------------------------------------------------------- embedding ----
// out[i] = table[token * width + i]  (kernels.hpp:24-34)
__global__ void embedding_vec_kernel(const uint4 *__restrict__ table, uint4 *__restrict__ out,
                                     uint32_t token, uint32_t chunks) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < chunks) out[i] = ld_ro16(table + static_cast<size_t>(token) * chunks + i);
}
__global__ void embedding_scalar_kernel(const uint16_t *__restrict__ table,
                                        uint16_t *__restrict__ out, uint32_t token,
                                        uint32_t width) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < width) out[i] = table[static_cast<size_t>(token) * width + i];
}

cudaError_t qwen_embedding_launch(const uint16_t *table, uint16_t *out, uint32_t token,
                                  uint32_t width, cudaStream_t stream) {
  if (width % 8 == 0 && aligned16(table) && aligned16(out)) {
    const uint32_t chunks = width / 8;
    embedding_vec_kernel<<<(chunks + 255) / 256, 256, 0, stream>>>(
        reinterpret_cast<const uint4 *>(table), reinterpret_cast<uint4 *>(out), token, chunks);
  } else {
    embedding_scalar_kernel<<<(width + 255) / 256, 256, 0, stream>>>(table, out, token, width);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------- RMSNorm ----
// out = bf16(x * w * rsqrt(sum(x^2)/width + eps))  (kernels.hpp:36-56).
// One CTA, like the reference's single work-item, but 256 threads wide.
__global__ void __launch_bounds__(256)
rms_norm_kernel(const uint16_t *__restrict__ in, const uint16_t *__restrict__ w,
                uint16_t *__restrict__ out, uint32_t width, float eps) {
  __shared__ float scratch[8];
  float sq = 0.f;
  for (uint32_t i = threadIdx.x; i < width; i += 256) {
    const float v = bf16_bits_to_float(in[i]);
    sq = fmaf(v, v, sq);
  }
  const float total = block_sum<8>(sq, scratch);
  const float scale = exact_rsqrt(total / static_cast<float>(width) + eps);
  for (uint32_t i = threadIdx.x; i < width; i += 256) {
    const float v = bf16_bits_to_float(in[i]);
    out[i] = float_to_bf16_bits(__fmul_rn(__fmul_rn(v, bf16_bits_to_float(w[i])), scale));
  }
}

cudaError_t qwen_rms_norm_launch(const uint16_t *in, const uint16_t *w, uint16_t *out,
                                 uint32_t width, float eps, cudaStream_t stream) {
  rms_norm_kernel<<<1, 256, 0, stream>>>(in, w, out, width, eps);
  return cudaGetLastError();
}

// -------------------------------------------------- QK-norm, RoPE, cache ----
// One warp per query head (kernels.hpp:58-155). Lane l owns dimensions
// l, l+32, l+64, l+96, so both rotate-half pairs (i, i+64) sit in one lane.
// Writes: query <- roped(norm(q)); key <- norm(k) (un-roped, as the
// reference does); key_cache[pos][h] <- roped(norm(k)); value_cache <- v.
__device__ __forceinline__ void head_norm(float (&v)[4], const uint16_t *norm_w, uint32_t lane) {
  float sq = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) sq = fmaf(v[j], v[j], sq);
  sq = warp_sum(sq);
  const float scale = exact_rsqrt(sq / static_cast<float>(kHeadDim) + 1.0e-6f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float wj = bf16_bits_to_float(norm_w[lane + 32 * j]);
    v[j] = round_bf16(__fmul_rn(__fmul_rn(v[j], wj), scale));
  }
}

__device__ __forceinline__ void head_rope(float (&v)[4], const uint16_t *cos_row,
                                          const uint16_t *sin_row, uint32_t lane) {
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const uint32_t i = lane + 32 * j;
    const float a = v[j], b = v[j + 2];
    const float ca = bf16_bits_to_float(cos_row[i]), sa = bf16_bits_to_float(sin_row[i]);
    const float cb = bf16_bits_to_float(cos_row[i + 64]), sb = bf16_bits_to_float(sin_row[i + 64]);
    v[j] = round_bf16(__fsub_rn(__fmul_rn(a, ca), __fmul_rn(b, sa)));
    v[j + 2] = round_bf16(__fadd_rn(__fmul_rn(b, cb), __fmul_rn(a, sb)));
  }
}

__global__ void __launch_bounds__(32)
qkv_rope_cache_kernel(uint16_t *__restrict__ query, uint16_t *__restrict__ key,
                      const uint16_t *__restrict__ value, const uint16_t *__restrict__ qn,
                      const uint16_t *__restrict__ kn, const uint16_t *__restrict__ cos_table,
                      const uint16_t *__restrict__ sin_table, uint16_t *__restrict__ key_cache,
                      uint16_t *__restrict__ value_cache, uint32_t position, uint32_t max_seq,
                      uint32_t kv_heads) {
  if (position >= max_seq) return;  // kernels.hpp:74-75
  const uint32_t head = blockIdx.x, lane = threadIdx.x;
  const uint16_t *cos_row = cos_table + static_cast<size_t>(position) * kHeadDim;
  const uint16_t *sin_row = sin_table + static_cast<size_t>(position) * kHeadDim;

  uint16_t *q = query + static_cast<size_t>(head) * kHeadDim;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = bf16_bits_to_float(q[lane + 32 * j]);
  head_norm(v, qn, lane);
  head_rope(v, cos_row, sin_row, lane);
#pragma unroll
  for (int j = 0; j < 4; ++j) q[lane + 32 * j] = float_to_bf16_bits(v[j]);

  if (head < kv_heads) {
    uint16_t *k = key + static_cast<size_t>(head) * kHeadDim;
    const size_t slot = (static_cast<size_t>(position) * kv_heads + head) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = bf16_bits_to_float(k[lane + 32 * j]);
    head_norm(v, kn, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) k[lane + 32 * j] = float_to_bf16_bits(v[j]);
    head_rope(v, cos_row, sin_row, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      key_cache[slot + lane + 32 * j] = float_to_bf16_bits(v[j]);
      value_cache[slot + lane + 32 * j] = value[static_cast<size_t>(head) * kHeadDim + lane + 32 * j];
    }
  }
}

cudaError_t qwen_qkv_rope_cache_launch(uint16_t *q, uint16_t *k, const uint16_t *v,
                                       const uint16_t *qn, const uint16_t *kn,
                                       const uint16_t *cos_table, const uint16_t *sin_table,
                                       uint16_t *kc, uint16_t *vc, uint32_t position,
                                       uint32_t max_seq, uint32_t q_heads, uint32_t kv_heads,
                                       cudaStream_t stream) {
  qkv_rope_cache_kernel<<<q_heads, 32, 0, stream>>>(q, k, v, qn, kn, cos_table, sin_table, kc, vc,
                                                    position, max_seq, kv_heads);
  return cudaGetLastError();
}

// ----------------------------------------------------------- attention ----
// GQA decode attention over cache positions 0..position with FP32 softmax
// (kernels.hpp:157-192). The reference walks positions serially per head;
// here the positions are split into 128-long chunks: one CTA per
// (kv head, chunk) runs an online softmax for the G query heads of its group
// and writes (max, sum, acc[128]) per head; a second kernel merges chunks.
template <int G>
__global__ void __launch_bounds__(128)
attention_chunk_kernel(const uint16_t *__restrict__ query, const uint16_t *__restrict__ key_cache,
                       const uint16_t *__restrict__ value_cache, float *__restrict__ workspace,
                       uint32_t position, uint32_t kv_heads, uint32_t chunks) {
  const uint32_t kvh = blockIdx.x, chunk = blockIdx.y;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ float s_m[4][G], s_l[4][G];
  __shared__ float s_acc[4][G][kHeadDim];

  float q[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint2 raw = *reinterpret_cast<const uint2 *>(
        query + (static_cast<size_t>(kvh) * G + g) * kHeadDim + lane * 4);
    q[g][0] = bf16_lo(raw.x); q[g][1] = bf16_hi(raw.x);
    q[g][2] = bf16_lo(raw.y); q[g][3] = bf16_hi(raw.y);
  }
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
  }
  const uint32_t begin = chunk * kAttnChunk;
  const uint32_t end = min(begin + kAttnChunk, position + 1);
  for (uint32_t p = begin + warp; p < end; p += 4) {
    const size_t off = (static_cast<size_t>(p) * kv_heads + kvh) * kHeadDim + lane * 4;
    const uint2 kr = *reinterpret_cast<const uint2 *>(key_cache + off);
    const uint2 vr = *reinterpret_cast<const uint2 *>(value_cache + off);
    const float k4[4] = {bf16_lo(kr.x), bf16_hi(kr.x), bf16_lo(kr.y), bf16_hi(kr.y)};
    const float v4[4] = {bf16_lo(vr.x), bf16_hi(vr.x), bf16_lo(vr.y), bf16_hi(vr.y)};
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) s = fmaf(q[g][j], k4[j], s);
      s = warp_sum(s) * kAttentionScale;
      const float m_new = fmaxf(m[g], s);
      const float alpha = expf(m[g] - m_new);
      const float pexp = expf(s - m_new);
      l[g] = l[g] * alpha + pexp;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = acc[g][j] * alpha + v4[j] * pexp;
      m[g] = m_new;
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) { s_m[warp][g] = m[g]; s_l[warp][g] = l[g]; }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_acc[warp][g][lane * 4 + j] = acc[g][j];
  }
  __syncthreads();
  // Merge the four warps; thread t owns dimension t of every head.
  const uint32_t d = threadIdx.x;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, s_m[w][g]);
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = (s_l[w][g] > 0.f) ? expf(s_m[w][g] - mm) : 0.f;
      ll += s_l[w][g] * f;
      aa += s_acc[w][g][d] * f;
    }
    float *slot = workspace + (static_cast<size_t>(kvh * G + g) * chunks + chunk) * kAttnStride;
    if (d == 0) { slot[0] = mm; slot[1] = ll; }
    slot[2 + d] = aa;
  }
}

__global__ void __launch_bounds__(128)
attention_merge_kernel(const float *__restrict__ workspace, uint16_t *__restrict__ out,
                       uint32_t chunks) {
  const uint32_t head = blockIdx.x, d = threadIdx.x;
  const float *base = workspace + static_cast<size_t>(head) * chunks * kAttnStride;
  float mm = -INFINITY;
  for (uint32_t c = 0; c < chunks; ++c) mm = fmaxf(mm, base[c * kAttnStride]);
  float ll = 0.f, aa = 0.f;
  for (uint32_t c = 0; c < chunks; ++c) {
    const float f = expf(base[c * kAttnStride] - mm);
    ll += base[c * kAttnStride + 1] * f;
    aa += base[c * kAttnStride + 2 + d] * f;
  }
  out[static_cast<size_t>(head) * kHeadDim + d] = float_to_bf16_bits(aa / ll);
}

size_t qwen_attention_workspace(uint32_t q_heads, uint32_t max_positions) {
  const size_t chunks = (static_cast<size_t>(max_positions) + kAttnChunk - 1) / kAttnChunk;
  return static_cast<size_t>(q_heads) * chunks * kAttnStride * sizeof(float);
}

cudaError_t qwen_attention_launch(const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                  uint16_t *out, uint32_t position, uint32_t q_heads,
                                  uint32_t kv_heads, float *workspace, cudaStream_t stream) {
  const uint32_t chunks = (position + kAttnChunk) / kAttnChunk;  // ceil((position + 1) / chunk)
  const dim3 grid(kv_heads, chunks);
  switch (q_heads / kv_heads) {
    case 1: attention_chunk_kernel<1><<<grid, 128, 0, stream>>>(q, kc, vc, workspace, position, kv_heads, chunks); break;
    case 2: attention_chunk_kernel<2><<<grid, 128, 0, stream>>>(q, kc, vc, workspace, position, kv_heads, chunks); break;
    case 4: attention_chunk_kernel<4><<<grid, 128, 0, stream>>>(q, kc, vc, workspace, position, kv_heads, chunks); break;
    case 8: attention_chunk_kernel<8><<<grid, 128, 0, stream>>>(q, kc, vc, workspace, position, kv_heads, chunks); break;
    default: return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attention_merge_kernel<<<q_heads, 128, 0, stream>>>(workspace, out, chunks);
  return cudaGetLastError();
}

// ---------------------------------------------------- add / SiLU-multiply ----
// left = bf16(left + right) (kernels.hpp:194-207) and
// gate = bf16(silu(gate) * up) (kernels.hpp:209-223), 8 elements per thread.
template <bool SILU>
__global__ void elementwise_kernel(uint16_t *__restrict__ a, const uint16_t *__restrict__ b,
                                   uint32_t width) {
  const uint32_t base = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (base >= width) return;
  if (base + 8 <= width && aligned16(a + base) && aligned16(b + base)) {
    uint4 va = *reinterpret_cast<const uint4 *>(a + base);
    const uint4 vb = *reinterpret_cast<const uint4 *>(b + base);
    uint32_t *pa = &va.x;
    const uint32_t *pb = &vb.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float lo, hi;
      if (SILU) {
        const float g0 = bf16_lo(pa[j]), g1 = bf16_hi(pa[j]);
        lo = __fmul_rn(__fdiv_rn(g0, 1.0f + expf(-g0)), bf16_lo(pb[j]));
        hi = __fmul_rn(__fdiv_rn(g1, 1.0f + expf(-g1)), bf16_hi(pb[j]));
      } else {
        lo = __fadd_rn(bf16_lo(pa[j]), bf16_lo(pb[j]));
        hi = __fadd_rn(bf16_hi(pa[j]), bf16_hi(pb[j]));
      }
      pa[j] = pack_bf16x2(lo, hi);
    }
    *reinterpret_cast<uint4 *>(a + base) = va;
    return;
  }
  for (uint32_t i = base; i < min(base + 8, width); ++i) {
    const float x = bf16_bits_to_float(a[i]), y = bf16_bits_to_float(b[i]);
    a[i] = float_to_bf16_bits(SILU ? __fmul_rn(__fdiv_rn(x, 1.0f + expf(-x)), y) : __fadd_rn(x, y));
  }
}

cudaError_t qwen_add_launch(uint16_t *left, const uint16_t *right, uint32_t width,
                            cudaStream_t stream) {
  const uint32_t threads = (width + 7) / 8;
  elementwise_kernel<false><<<(threads + 255) / 256, 256, 0, stream>>>(left, right, width);
  return cudaGetLastError();
}

cudaError_t qwen_silu_multiply_launch(uint16_t *gate, const uint16_t *up, uint32_t width,
                                      cudaStream_t stream) {
  const uint32_t threads = (width + 7) / 8;
  elementwise_kernel<true><<<(threads + 255) / 256, 256, 0, stream>>>(gate, up, width);
  return cudaGetLastError();
}

// -------------------------------------------------------------- argmax ----
// First index of the maximum; any NaN or +-Inf gives 0xffffffff
// (kernels.hpp:225-246). One 1024-thread CTA: strided scan, then a
// (value, lowest index) tree.
__global__ void __launch_bounds__(1024)
argmax_kernel(const uint16_t *__restrict__ values, uint32_t *__restrict__ token, uint32_t width) {
  __shared__ ArgBest s_best[32];
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  ArgBest best{-INFINITY, 0xffffffffu};
  bool bad = false;
  for (uint32_t i = threadIdx.x; i < width; i += 1024) {
    const float v = bf16_bits_to_float(values[i]);
    bad |= not_finite(v);
    if (v > best.value) best = ArgBest{v, i};  // strided indices rise, so ties keep the lowest
  }
  if (bad) s_bad = 1;
  best = warp_argbest(best);
  if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = warp_argbest(s_best[threadIdx.x]);
    // An empty row returns 0, like the reference's untouched best_index.
    if (threadIdx.x == 0) *token = width == 0 ? 0u : (s_bad ? 0xffffffffu : best.index);
  }
}

cudaError_t qwen_argmax_launch(const uint16_t *values, uint32_t *token, uint32_t width,
                               cudaStream_t stream) {
  argmax_kernel<<<1, 1024, 0, stream>>>(values, token, width);
  return cudaGetLastError();
}

}  // namespace xpu
