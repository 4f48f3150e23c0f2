// Row-major GEMM C[M,N] = A[M,K] . B[K,N] on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), FP32 accumulation, bf16 or fp16 in and
// out. Replaces gemm::Kernel<T, LargeTile> (gemm_kernel.hpp:25-143), whose
// work-items run 8x16x16 DPAS tiles out of registers.
//
// Persistent, two CTAs per cluster working as one pair (cta_group::2): a pair
// owns 256 x 256 output tiles, visited in groups of 8 tile-rows so that the
// pairs running at once share A and B panels in L2. Each CTA of the pair
// stages its half of the operands, A rows [128 r, 128 r + 128) and B columns
// [128 r, 128 r + 128) of the tile, and holds its 128 rows x 256 columns of
// the FP32 accumulator in its own TMEM; one thread of the even CTA issues
// the 256x256x16 MMAs that read both CTAs' shared memory. 320 threads:
//   warp 0     TMA producer: per 128-deep K stage, two 128 x 64 A boxes
//              and two 64(N) x 128(K) B boxes, 128-byte swizzled, into a
//              ring of 3 x 64 KB stages; both CTAs' copies complete on the
//              even CTA's full barrier (128-deep stages halve the barrier
//              and commit traffic per MMA against 64-deep ones);
//   warp 1     TMEM owner (2 x 256 columns: a double-buffered accumulator);
//              in the even CTA its elected lane issues the MMAs, releases
//              each stage to both CTAs' producers with tcgen05.commit and
//              signals both epilogues when a tile's accumulator is final;
//   warps 2-9  epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its
//              rows), columns [128 h, 128 h + 128) for h = (w - 2) / 4,
//              rounds to bf16/fp16 and stores with row/column predication,
//              then frees the accumulator buffer for the tile after next.
// A is K-major (row-major [M,K]); B is used MN-major straight from its
// row-major [K,N] layout (instruction descriptor b_major = MN) - or, for
// C = A . W^T with W row-major [N,K] (prefill projections against the
// stored weights), K-major like A - so neither operand is transposed or
// padded in memory: TMA zero-fills out-of-range
// rows/columns/K and the epilogue masks the edge tiles. No load uses
// multicast; the even CTA signals the odd CTA's barriers by their cluster
// addresses.
//
// Waits are bounded; a timeout sets a sticky device error word (read by
// xpu_device_status) and every role leaves its loop, so both CTAs still meet
// at the closing cluster barrier and free their TMEM.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "stream.cuh"
#include "tcgen05.cuh"
#include "xpu_internal.h"

namespace xpu {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr uint32_t kBM = 256, kBN = 256, kBK = 128;  // pair tile, K stage
constexpr uint32_t kHalfM = kBM / 2, kHalfN = kBN / 2;
constexpr uint32_t kStages = 3;
constexpr uint32_t kSwz = 64;                       // elements per 128-byte swizzled row
constexpr uint32_t kABoxBytes = kHalfM * kSwz * 2;  // 16 KB: 128 rows x 64 K
constexpr uint32_t kABytes = kHalfM * kBK * 2;      // 32 KB: two boxes along K
constexpr uint32_t kBBoxBytes = kSwz * kBK * 2;     // 16 KB: 64 (N) x 128 (K)
constexpr uint32_t kBBytes = kHalfN * kBK * 2;      // 32 KB: two boxes along N
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kAccCols = kBN;                 // FP32 columns of one accumulator
constexpr uint32_t kTmemCols = 2 * kAccCols;       // double buffered: all 512
constexpr uint32_t kGroupRows = 8;                 // tile-rows per L2 group
constexpr int kEpilogueWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpilogueWarps;
constexpr unsigned kErrGemmTimeout = 1u;

// Instruction descriptor, kind::f16: FP32 accumulator, A K-major, B MN-major
// (row-major [K,N]) or, with b_kmajor, K-major (row-major [N,K]: C = A . B^T).
__host__ __device__ constexpr uint32_t instr_desc(bool fp16, uint32_t m, uint32_t n, bool b_kmajor = false) {
  return (1u << 4) |                          // D format F32
         ((fp16 ? 0u : 1u) << 7) |            // A format: F16 = 0, BF16 = 1
         ((fp16 ? 0u : 1u) << 10) |           // B format
         (0u << 15) |                         // A K-major
         ((b_kmajor ? 0u : 1u) << 16) |       // B MN-major (1) or K-major (0)
         ((n >> 3) << 17) |                   // N / 8
         ((m >> 4) << 24);                    // M / 16
}

// 2D tiled TMA load into this CTA's shared memory, completing on an mbarrier
// that may belong to either CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_pair(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                              uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(cluster_bar)
      : "memory");
}

// 3D form (split GEMM: x = K inside a chunk, y = chunk, z = row).
__device__ __forceinline__ void tma_load_pair3(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                               uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrives once on `cluster_bar` when every MMA this thread issued so far has
// completed (on both CTAs of the pair).
__device__ __forceinline__ void mma_commit_pair(uint32_t cluster_bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <bool FP16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if (FP16) {
    const uint32_t l = __half_as_ushort(__float2half_rn(lo)), h = __half_as_ushort(__float2half_rn(hi));
    return l | (h << 16);
  }
  return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ bool has_failed(const int *flag) { return *reinterpret_cast<const volatile int *>(flag) != 0; }

struct TileCoord {
  uint32_t m, n;
};

// Tile t in group-of-rows order: kGroupRows tile-rows at a time, column by
// column inside the group.
__device__ __forceinline__ TileCoord tile_coord(uint32_t t, uint32_t tiles_m, uint32_t tiles_n) {
  const uint32_t per_group = kGroupRows * tiles_n;
  const uint32_t group = t / per_group, first = group * kGroupRows;
  const uint32_t rows = min(kGroupRows, tiles_m - first);
  const uint32_t local = t - group * per_group;
  return {first + local % rows, local / rows};
}

// BK: B is K-major (W[N,K] row-major, C = A . W^T); its per-CTA half of the
// tile (128 N rows x 128 K) is staged exactly like A's (two 128 x 64 boxes).
// SPLIT (with BK): K is cut into `chunks` chunks of K columns each and every
// chunk is its own accumulation, written as FP32 C[chunk][M][N]; the maps
// are 3D (K inside the chunk, chunk, row) so a chunk's last stage reads zeros
// past its end instead of the next chunk's columns.
template <bool FP16, bool BK, bool SPLIT>
__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, void *C,
          uint32_t M, uint32_t N, uint32_t K, uint32_t chunks) {
  static_assert(!SPLIT || BK, "split GEMM is the A . W^T form");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  // 1024-byte aligned stage ring (128-byte swizzle atoms); same offset in both CTAs.
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0 = the CTA that issues the MMAs
  const uint32_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const uint32_t tiles_m = (M + kBM - 1) / kBM, tiles_n = (N + kBN - 1) / kBN, tiles = tiles_m * tiles_n;
  const uint32_t work = SPLIT ? tiles * chunks : tiles;  // chunk-major: a chunk's tiles share its panels in L2
  const uint32_t nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);   // the even CTA's expect_tx; both CTAs' bytes
      mbar_init(&empty[i], 1);  // one commit per use
    }
    for (uint32_t i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * kEpilogueWarps);  // every epilogue warp of the pair
    }
    fence_mbar_init();
    failed = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = cluster_addr(&full[0], 0);
      uint32_t g = 0;
      for (uint32_t t = pair; t < work && !has_failed(&failed); t += pairs) {
        const uint32_t chunk = SPLIT ? t / tiles : 0;
        const TileCoord tc = tile_coord(t - chunk * tiles, tiles_m, tiles_n);
        const int32_t ya = static_cast<int32_t>(tc.m * kBM + rank * kHalfM);
        const int32_t xb = static_cast<int32_t>(tc.n * kBN + rank * kHalfN);
        for (uint32_t k = 0; k < nk; ++k, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) { failed = 1; break; }
          if (rank == 0) mbar_expect_tx(&full[s], 2 * kStageBytes);
          const uint32_t bar = full0 + s * 8u;
          uint8_t *st = ring + s * kStageBytes;
          const int32_t xk = static_cast<int32_t>(k * kBK);
          if (SPLIT) {
            const int32_t z = static_cast<int32_t>(chunk);
            tma_load_pair3(st, &map_a, xk, z, ya, bar);
            tma_load_pair3(st + kABoxBytes, &map_a, xk + static_cast<int32_t>(kSwz), z, ya, bar);
            tma_load_pair3(st + kABytes, &map_b, xk, z, xb, bar);
            tma_load_pair3(st + kABytes + kABoxBytes, &map_b, xk + static_cast<int32_t>(kSwz), z, xb, bar);
            continue;
          }
          tma_load_pair(st, &map_a, xk, ya, bar);
          tma_load_pair(st + kABoxBytes, &map_a, xk + static_cast<int32_t>(kSwz), ya, bar);
          if (BK) {
            tma_load_pair(st + kABytes, &map_b, xk, xb, bar);
            tma_load_pair(st + kABytes + kABoxBytes, &map_b, xk + static_cast<int32_t>(kSwz), xb, bar);
          } else {
            tma_load_pair(st + kABytes, &map_b, xb, xk, bar);
            tma_load_pair(st + kABytes + kBBoxBytes, &map_b, xb + static_cast<int32_t>(kSwz), xk, bar);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = instr_desc(FP16, kBM, kBN, BK);
      uint32_t g = 0, i = 0;
      for (uint32_t t = pair; t < work && !has_failed(&failed); t += pairs, ++i) {
        const uint32_t b = i & 1, use_b = i >> 1;
        if (use_b > 0 && !mbar_wait(&acc_empty[b], (use_b - 1) & 1)) { failed = 1; break; }
        tc_fence_after();
        const uint32_t d = tmem + b * kAccCols;
        for (uint32_t k = 0; k < nk; ++k, ++g) {
          const uint32_t s = g % kStages, use = g / kStages;
          if (!mbar_wait(&full[s], use & 1)) { failed = 1; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(ring + s * kStageBytes), sb = sa + kABytes;
          const uint64_t da = smem_desc(sa, 16, 1024), db = BK ? smem_desc(sb, 16, 1024) : smem_desc(sb, kBBoxBytes, 1024);
#pragma unroll
          for (uint32_t kk = 0; kk < kBK / 16; ++kk) {
            // K step of 16: +32 bytes inside A's 128-byte swizzled rows (the
            // next A box every 4 steps); B the same when K-major, else +2
            // eight-row groups of its MN-major boxes.
            const uint32_t a_off = (kk / 4) * kABoxBytes + (kk % 4) * 32u;
            const uint32_t b_off = BK ? a_off : kk * 2048u;
            mma_pair(d, da + (a_off >> 4), db + (b_off >> 4), idesc, (k | kk) != 0);
          }
          mma_commit_pair(cluster_addr(&empty[s], 0));
          mma_commit_pair(cluster_addr(&empty[s], 1));
        }
        if (has_failed(&failed)) break;
        mma_commit_pair(cluster_addr(&acc_full[b], 0));
        mma_commit_pair(cluster_addr(&acc_full[b], 1));
      }
    }
  } else {
    // Epilogue warps 2..9: TMEM lanes 32 (warp % 4) .. + 31 hold 32 rows of
    // this CTA's half; column half h = (warp - 2) / 4.
    const uint32_t quarter = warp & 3, h = (warp - 2) >> 2;
    const uint32_t release = cluster_addr(&acc_empty[0], 0);
    uint32_t i = 0;
    for (uint32_t t = pair; t < work; t += pairs, ++i) {
      const uint32_t b = i & 1;
      if (!mbar_wait(&acc_full[b], (i >> 1) & 1)) { failed = 1; break; }
      tc_fence_after();
      const uint32_t chunk = SPLIT ? t / tiles : 0;
      const TileCoord tc = tile_coord(t - chunk * tiles, tiles_m, tiles_n);
      const uint32_t row = tc.m * kBM + rank * kHalfM + quarter * 32 + lane;
#pragma unroll 1
      for (uint32_t c = h * 128; c < h * 128 + 128; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((quarter * 32u) << 16) + b * kAccCols + c, r);
        const uint32_t col = tc.n * kBN + c;
        if (SPLIT && row < M && col < N) {  // FP32 partial of this chunk, unrounded
          float *dst = static_cast<float *>(C) + (static_cast<size_t>(chunk) * M + row) * N + col;
#pragma unroll
          for (uint32_t q = 0; q < 8; ++q) {
            if (col + 4 * q >= N) break;
            *reinterpret_cast<uint4 *>(dst + 4 * q) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
        } else if (row < M && col < N) {
          uint16_t *dst = static_cast<uint16_t *>(C) + static_cast<size_t>(row) * N + col;
#pragma unroll
          for (uint32_t q = 0; q < 4; ++q) {
            if (col + 8 * q >= N) break;
            uint4 v;
            v.x = pack2<FP16>(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
            v.y = pack2<FP16>(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
            v.z = pack2<FP16>(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
            v.w = pack2<FP16>(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
            *reinterpret_cast<uint4 *>(dst + 8 * q) = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(release + b * 8u);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && failed) atomicOr(&g_device_error, kErrGemmTimeout);
  cluster_sync();  // no CTA of the pair touches the other's barriers or TMEM after this
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  cluster_sync();
}

// CUDA-core fallback for shapes the TMA path cannot describe (a row stride
// that is not a multiple of 16 bytes, or a misaligned base): 32 x 32 output
// tiles through shared memory, FP32 accumulation in K order.
template <typename T>
__global__ void __launch_bounds__(256) k_gemm_simple(const T *A, const T *B, T *C, uint32_t M, uint32_t N,
                                                      uint32_t K) {
  __shared__ float As[32][33], Bs[32][33];
  const uint32_t tx = threadIdx.x % 32, ty = threadIdx.x / 32;  // 32 x 8 threads, 4 rows each
  const uint32_t row0 = blockIdx.y * 32, col = blockIdx.x * 32 + tx;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (uint32_t k0 = 0; k0 < K; k0 += 32) {
    for (uint32_t i = ty; i < 32; i += 8) {
      const uint32_t r = row0 + i, ka = k0 + tx, kb = k0 + i;
      As[i][tx] = (r < M && ka < K) ? Elem<T>::to_float(A[static_cast<size_t>(r) * K + ka]) : 0.f;
      Bs[i][tx] = (kb < K && col < N) ? Elem<T>::to_float(B[static_cast<size_t>(kb) * N + col]) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (uint32_t kk = 0; kk < 32; ++kk)
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) acc[j] = fmaf(As[ty + 8 * j][kk], Bs[kk][tx], acc[j]);
    __syncthreads();
  }
  for (uint32_t j = 0; j < 4; ++j) {
    const uint32_t r = row0 + ty + 8 * j;
    if (r < M && col < N) C[static_cast<size_t>(r) * N + col] = Elem<T>::from_float(acc[j]);
  }
}

}  // namespace

size_t gemm_smem_bytes() { return kStages * kStageBytes + 1024; }

namespace {
using GemmKernel = void (*)(CUtensorMap, CUtensorMap, void *, uint32_t, uint32_t, uint32_t, uint32_t);

// Persistent 2-CTA launch: as many pairs as can be resident at once (the
// pairs do not wait on one another, so fewer resident pairs only cost time),
// cached per kernel kind and device.
cudaError_t launch_tc(GemmKernel kernel, int kind, const CUtensorMap &map_a, const CUtensorMap &map_b, void *C,
                      uint32_t M, uint32_t N, uint32_t K, uint32_t chunks, cudaStream_t stream) {
  const size_t smem = gemm_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  static std::mutex cache_mutex;
  static int resident_pairs[5][64] = {};
  int pairs = 0;
  {
    std::lock_guard<std::mutex> lock(cache_mutex);
    int &cached = resident_pairs[kind][device & 63];
    if (cached == 0) {
      cfg.gridDim = dim3(2);
      e = cudaOccupancyMaxActiveClusters(&cached, kernel, &cfg);
      if (e != cudaSuccess) return e;
      if (cached < 1) return cudaErrorLaunchOutOfResources;
    }
    pairs = cached;
  }
  const uint64_t work = static_cast<uint64_t>((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN) * chunks;
  cfg.gridDim = dim3(2 * static_cast<uint32_t>(std::min<uint64_t>(work, static_cast<uint64_t>(pairs))));
  e = cudaLaunchKernelEx(&cfg, kernel, map_a, map_b, C, M, N, K, chunks);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
}  // namespace

cudaError_t gemm_launch(bool fp16, const void *A, const void *B, void *C, uint32_t M, uint32_t N, uint32_t K,
                        cudaStream_t stream) {
  return gemm_launch_ex(fp16, false, A, B, C, M, N, K, stream);
}

cudaError_t gemm_launch_ex(bool fp16, bool b_kmajor, const void *A, const void *B, void *C, uint32_t M, uint32_t N,
                           uint32_t K, cudaStream_t stream) {
  const bool tma_ok = (K % 8 == 0) && (N % 8 == 0) && aligned16(A) && aligned16(B) && aligned16(C);
  if (!tma_ok) {
    if (b_kmajor) return cudaErrorInvalidValue;  // the A . B^T form needs the TMA path
    const dim3 grid((N + 31) / 32, (M + 31) / 32);
    if (fp16)
      k_gemm_simple<__half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(A), static_cast<const __half *>(B),
                                                     static_cast<__half *>(C), M, N, K);
    else
      k_gemm_simple<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(A),
                                                            static_cast<const __nv_bfloat16 *>(B),
                                                            static_cast<__nv_bfloat16 *>(C), M, N, K);
    return cudaGetLastError();
  }
  CUtensorMap map_a, map_b;
  cudaError_t e = make_tmap_2d_u16_swizzled(&map_a, A, K, M, K, kSwz, kHalfM);
  if (e != cudaSuccess) return e;
  e = b_kmajor ? make_tmap_2d_u16_swizzled(&map_b, B, K, N, K, kSwz, kHalfN)
               : make_tmap_2d_u16_swizzled(&map_b, B, N, K, N, kSwz, kBK);
  if (e != cudaSuccess) return e;
  auto kernel = fp16 ? (b_kmajor ? k_gemm_tc<true, true, false> : k_gemm_tc<true, false, false>)
                     : (b_kmajor ? k_gemm_tc<false, true, false> : k_gemm_tc<false, false, false>);
  return launch_tc(kernel, (fp16 ? 1 : 0) + (b_kmajor ? 2 : 0), map_a, map_b, C, M, N, K, 1, stream);
}

cudaError_t gemm_chunks_launch(const void *A, const void *W, float *C, uint32_t M, uint32_t N, uint32_t Kc,
                               uint32_t chunks, cudaStream_t stream) {
  if (M == 0 || N == 0 || Kc == 0 || chunks == 0) return cudaErrorInvalidValue;
  if (Kc % 8 || N % 8 || !aligned16(A) || !aligned16(W) || !aligned16(C)) return cudaErrorInvalidValue;
  CUtensorMap map_a, map_b;
  const uint64_t K = static_cast<uint64_t>(Kc) * chunks;
  cudaError_t e = make_tmap_3d_u16_swizzled(&map_a, A, Kc, chunks, M, Kc, K, kSwz, kHalfM);
  if (e != cudaSuccess) return e;
  e = make_tmap_3d_u16_swizzled(&map_b, W, Kc, chunks, N, Kc, K, kSwz, kHalfN);
  if (e != cudaSuccess) return e;
  return launch_tc(k_gemm_tc<false, true, true>, 4, map_a, map_b, C, M, N, Kc, chunks, stream);
}

unsigned take_device_error() {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
  if (v) cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  return v;
}

}  // namespace xpu
