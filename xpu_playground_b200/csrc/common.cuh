// Shared device helpers for the sm_100a kernels of libxpu_cuda.
//
// Everything here is plain CUDA C++ plus a few lines of hand-written PTX for
// streaming loads. Nothing in the library is compiled with fast-math: the
// reciprocal square roots below must round like the host references
// (RN(1 / RN(sqrt(v))), the same double rounding torch's CPU rsqrt uses).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xpu {

constexpr unsigned kFullMask = 0xffffffffu;

// ---------------------------------------------------------------- loads ----

// 16-byte streaming load that bypasses L1 (weights are read exactly once per
// decode step, so they must not evict the activations staged in L1/smem).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}

// 16-byte read-only load through L1 (small vectors re-read by many CTAs).
__device__ __forceinline__ uint4 ld_ro16(const void *p) {
  return __ldg(reinterpret_cast<const uint4 *>(p));
}

// ------------------------------------------------------------ conversion ----

// bf16 is the top half of an fp32, so widening is a shift or a mask.
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Round-to-nearest-even fp32 -> bf16 bits (NaN stays NaN).
__device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&h);
}

// Round an fp32 value to the nearest bf16 and widen it back.
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_bits_to_float(float_to_bf16_bits(f));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(float_to_bf16_bits(lo)) |
         (static_cast<uint32_t>(float_to_bf16_bits(hi)) << 16);
}

// Element-type traits for the bf16 / fp16 GEMV and GEMM paths.
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float lo(uint32_t u) { return bf16_lo(u); }
  __device__ __forceinline__ static float hi(uint32_t u) { return bf16_hi(u); }
  __device__ __forceinline__ static float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<__half> {
  __device__ __forceinline__ static float lo(uint32_t u) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(u & 0xffffu)));
  }
  __device__ __forceinline__ static float hi(uint32_t u) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(u >> 16)));
  }
  __device__ __forceinline__ static float to_float(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_float(float v) { return __float2half_rn(v); }
};

// acc += dot(a[0..7], x[0..7]) in element order (a fixed order keeps every
// partial sum reproducible regardless of how the K range is split).
template <typename T>
__device__ __forceinline__ float dot8(const uint4 &a, const uint4 &x, float acc) {
  acc = fmaf(Elem<T>::lo(a.x), Elem<T>::lo(x.x), acc);
  acc = fmaf(Elem<T>::hi(a.x), Elem<T>::hi(x.x), acc);
  acc = fmaf(Elem<T>::lo(a.y), Elem<T>::lo(x.y), acc);
  acc = fmaf(Elem<T>::hi(a.y), Elem<T>::hi(x.y), acc);
  acc = fmaf(Elem<T>::lo(a.z), Elem<T>::lo(x.z), acc);
  acc = fmaf(Elem<T>::hi(a.z), Elem<T>::hi(x.z), acc);
  acc = fmaf(Elem<T>::lo(a.w), Elem<T>::lo(x.w), acc);
  acc = fmaf(Elem<T>::hi(a.w), Elem<T>::hi(x.w), acc);
  return acc;
}

// ------------------------------------------------------------ reductions ----

// Butterfly sum: every lane ends with the same, order-fixed value.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFullMask, v, o));
  return v;
}

// Block-wide sum for blockDim.x == 32 * W threads; the result is broadcast.
// `scratch` needs W floats. Order is fixed: lanes, then warps in index order.
template <int W>
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < W; ++i) total += scratch[i];
  return total;
}

// (value, index) argmax pair: larger value wins, lowest index on ties.
struct ArgBest {
  float value;
  uint32_t index;
};

__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
  if (b.value > a.value || (b.value == a.value && b.index < a.index)) return b;
  return a;
}

__device__ __forceinline__ ArgBest warp_argbest(ArgBest v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest other;
    other.value = __shfl_xor_sync(kFullMask, v.value, o);
    other.index = __shfl_xor_sync(kFullMask, v.index, o);
    v = arg_better(v, other);
  }
  return v;
}

// True for NaN and +-Inf.
__device__ __forceinline__ bool not_finite(float v) {
  return (__float_as_uint(v) & 0x7f800000u) == 0x7f800000u;
}

// Correctly rounded 1/sqrt(v) as RN(1 / RN(sqrt(v))).
__device__ __forceinline__ float exact_rsqrt(float v) { return 1.0f / sqrtf(v); }

}  // namespace xpu
