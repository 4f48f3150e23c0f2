// Row-major GEMV y = A.x with FP32 accumulation (bf16 or fp16 in and out).
//
// Replaces gemv::Kernel<T>::run (gemv_kernel.hpp:21-63), which gives one
// eSIMD work-item per row and walks K 32 columns at a time. Here:
//   * the vector x is staged once per CTA into shared memory (16-byte chunks);
//   * every warp owns ROWS rows and streams them with 16-byte
//     ld.global.nc.L1::no_allocate loads, UNROLL chunks in flight per row;
//   * lane l accumulates chunks l, l+32, l+64, ... in order, 8 products per
//     chunk, then a butterfly shuffle sum folds the 32 lanes (fixed order).
// Rows whose K is not a multiple of 8, or whose base is not 16-byte aligned,
// take the scalar kernel below (same FP32 math, one element per lane step).
// The vector kernel is launched with programmatic dependent launch: it lets
// the next launch start right away and waits for the previous one before
// its first global access, so back-to-back GEMVs overlap the next launch's
// CTA start-up with this one's tail (a 4096 x 4096 launch streams for only
// ~5 us) while every read still sees the previous kernel's writes.
#include "common.cuh"
#include "gemv_core.cuh"
#include "xpu_internal.h"

namespace xpu {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;

template <typename T, int ROWS, int UNROLL>
__global__ void __launch_bounds__(kGemvThreads)
gemv_vec_kernel(const T *__restrict__ A, const T *__restrict__ x, T *__restrict__ y,
                uint32_t m, uint32_t k) {
  extern __shared__ uint4 xs[];  // k / 8 chunks of x
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const uint32_t chunks = k >> 3;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row0 = (blockIdx.x * kGemvWarps + warp) * ROWS;
  // The rows' first batch is requested before x is staged, so the two
  // round trips overlap (a 4096 x 4096 launch is only a few microseconds).
  const uint4 *rows[ROWS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    const uint32_t row = min(row0 + r, m - 1);  // clamp: duplicate rows are dropped below
    rows[r] = reinterpret_cast<const uint4 *>(A + static_cast<size_t>(row) * k);
  }
  uint4 first[ROWS][UNROLL];
  warp_rows_load<ROWS, UNROLL>(rows, 0, row0 < m ? chunks : 0, lane, first);
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
  for (uint32_t i = threadIdx.x; i < chunks; i += kGemvThreads) xs[i] = ld_ro16(x4 + i);
  __syncthreads();
  if (row0 >= m) return;
  float acc[ROWS];
  warp_dot_rows<T, ROWS, UNROLL>(rows, xs, chunks, lane, first, acc);
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
      if (row0 + r < m) y[row0 + r] = Elem<T>::from_float(acc[r]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kGemvThreads)
gemv_scalar_kernel(const T *__restrict__ A, const T *__restrict__ x, T *__restrict__ y,
                   uint32_t m, uint32_t k) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row = blockIdx.x * kGemvWarps + warp;
  if (row >= m) return;
  const T *a = A + static_cast<size_t>(row) * k;
  float acc = 0.f;
  for (uint32_t c = lane; c < k; c += 32)
    acc = fmaf(Elem<T>::to_float(a[c]), Elem<T>::to_float(x[c]), acc);
  acc = warp_sum(acc);
  if (lane == 0) y[row] = Elem<T>::from_float(acc);
}

template <typename T, int ROWS, int UNROLL>
static cudaError_t launch_vec(const T *A, const T *x, T *y, uint32_t m, uint32_t k,
                              cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(k / 8) * sizeof(uint4);
  auto kernel = gemv_vec_kernel<T, ROWS, UNROLL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const uint32_t rows_per_cta = kGemvWarps * ROWS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((m + rows_per_cta - 1) / rows_per_cta);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, A, x, y, m, k);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <typename T>
cudaError_t gemv_launch(const T *A, const T *x, T *y, uint32_t m, uint32_t k,
                        cudaStream_t stream) {
  const bool vector_path = (k % 8 == 0) && aligned16(A) && aligned16(x) &&
                           static_cast<size_t>(k / 8) * sizeof(uint4) <= kMaxGemvVectorBytes;
  if (!vector_path) {
    const uint32_t grid = (m + kGemvWarps - 1) / kGemvWarps;
    gemv_scalar_kernel<T><<<grid, kGemvThreads, 0, stream>>>(A, x, y, m, k);
    return cudaGetLastError();
  }
  // Two rows per warp once there are enough rows to fill every SM several
  // times over; one row per warp keeps small matrices spread across SMs.
  if (m >= 8192) return launch_vec<T, 2, 4>(A, x, y, m, k, stream);
  return launch_vec<T, 1, 8>(A, x, y, m, k, stream);
}

template cudaError_t gemv_launch<__nv_bfloat16>(const __nv_bfloat16 *, const __nv_bfloat16 *,
                                                __nv_bfloat16 *, uint32_t, uint32_t, cudaStream_t);
template cudaError_t gemv_launch<__half>(const __half *, const __half *, __half *, uint32_t,
                                         uint32_t, cudaStream_t);

}  // namespace xpu
