// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled), reached
// through cudaGetDriverEntryPoint so the library does not link libcuda.
#include <cuda.h>

#include <mutex>
#include <string>

#include "xpu_internal.h"

namespace xpu {

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

namespace {
cudaError_t encode_2d_u16(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows, uint64_t pitch_elems,
                          uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (pitch_elems * 2) % 16 || (box_cols * 2) % 16 || box_cols > 256 ||
      box_rows > 256)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch_elems * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
}  // namespace

// Row-major [rows][cols] matrix of 16-bit elements with a row pitch of
// pitch_elems; box = box_rows rows x box_cols columns, no swizzle, rows past
// the end read as zero.
cudaError_t make_tmap_2d_u16(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                             uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows) {
  return encode_2d_u16(map, base, cols, rows, pitch_elems, box_cols, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Same, with the 128-byte swizzle the tensor-core shared-memory descriptors
// expect (box_cols x 2 bytes must then be at most 128). Elements outside the
// matrix (either dimension) read as zero.
cudaError_t make_tmap_2d_u16_swizzled(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                                      uint64_t pitch_elems, uint32_t box_cols, uint32_t box_rows) {
  if (box_cols * 2 > 128) return cudaErrorInvalidValue;
  return encode_2d_u16(map, base, cols, rows, pitch_elems, box_cols, box_rows, CU_TENSOR_MAP_SWIZZLE_128B);
}

// 3D view [d2][d1][d0] of 16-bit elements (strides in elements: dimension 1
// every stride1, dimension 2 every stride2), 128-byte swizzled boxes of
// box_rows x 1 x box_cols. The split GEMM reads a row-major [rows][chunks x
// Kc] matrix as (Kc, chunks, rows): a box that starts near the end of a chunk
// reads zeros past it, not the next chunk's columns.
cudaError_t make_tmap_3d_u16_swizzled(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                                      uint64_t stride1, uint64_t stride2, uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (stride1 * 2) % 16 || (stride2 * 2) % 16 || box_cols * 2 > 128 ||
      (box_cols * 2) % 16 || box_rows > 256)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1 * 2, stride2 * 2};
  const cuuint32_t box[3] = {box_cols, 1, box_rows};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void *>(base), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace xpu
