// Warp-level GEMV building block shared by the standalone GEMV and the fused
// decode kernels.
//
// A warp owns ROWS rows; their 16-byte chunks [0, n) (relative to each row
// pointer) are streamed with L1-bypassing loads, two batches of UNROLL
// chunks per row in flight; the matching chunks of x come from shared memory. Lane l folds
// chunks l, l+32, l+64, ... in order and a butterfly shuffle sums the lanes,
// so the result depends only on (row, x, n) - never on how many CTAs share a
// row or which rank of a tensor-parallel group computes it.
#pragma once

#include "common.cuh"

namespace xpu {

// One batch of a warp's row chunks: chunk base + lane + 32 u of each row
// (zero past n).
template <int ROWS, int UNROLL>
__device__ __forceinline__ void warp_rows_load(const uint4 *const (&rows)[ROWS], uint32_t base, uint32_t n,
                                               uint32_t lane, uint4 (&a)[ROWS][UNROLL]) {
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    const uint32_t c = base + lane + 32 * u;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) a[r][u] = c < n ? ld_stream16(rows[r] + c) : make_uint4(0, 0, 0, 0);
  }
}

// `first` holds the batch at base 0 (loaded by the caller, e.g. before it
// staged x); each later batch is requested before the previous one is
// folded, so two batches per row are in flight.
template <typename T, int ROWS, int UNROLL>
__device__ __forceinline__ void warp_dot_rows(const uint4 *const (&rows)[ROWS], const uint4 *xs, uint32_t n,
                                              uint32_t lane, const uint4 (&first)[ROWS][UNROLL], float (&acc)[ROWS]) {
#pragma unroll
  for (int r = 0; r < ROWS; ++r) acc[r] = 0.f;
  constexpr uint32_t kStep = 32 * UNROLL;
  uint4 cur[ROWS][UNROLL];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) cur[r][u] = first[r][u];
  for (uint32_t base = 0; base < n; base += kStep) {
    uint4 nxt[ROWS][UNROLL];
    warp_rows_load<ROWS, UNROLL>(rows, base + kStep, n, lane, nxt);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t c = base + lane + 32 * u;
      if (c < n) {
        const uint4 xv = xs[c];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) acc[r] = dot8<T>(cur[r][u], xv, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) cur[r][u] = nxt[r][u];
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) acc[r] = warp_sum(acc[r]);
}

}  // namespace xpu
