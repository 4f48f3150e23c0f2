// Row-major GEMM C[M,N] = A[M,K] . B[K,N] on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM), FP32 accumulation, bf16 or fp16 in and
// out. Replaces gemm::Kernel<T, LargeTile> (gemm_kernel.hpp:25-143), whose
// work-items run 8x16x16 DPAS tiles out of registers.
//
// One CTA per 128 x 256 output tile; 192 threads in four roles:
//   warp 0     TMA producer: per 64-deep K stage, A as one 128 x 64 box and B
//              as four 64(N) x 64(K) boxes, 128-byte swizzled, into a ring of
//              4 x 48 KB shared-memory stages (full/empty mbarriers);
//   warp 1     allocates 256 TMEM columns (the FP32 128 x 256 accumulator)
//              and, from one elected lane, issues four 128x256x16
//              tcgen05.mma per stage; tcgen05.commit releases each stage and,
//              after the last, signals the epilogue;
//   warps 2-5  epilogue: tcgen05.ld 32 rows x 32 columns at a time (warp w
//              reads TMEM lanes 32 (w % 4) .. + 31 = output rows), round to
//              bf16/fp16 and store with row/column predication.
// A is K-major (row-major [M,K]); B is used MN-major straight from its
// row-major [K,N] layout (instruction descriptor b_major = MN), so neither
// operand is transposed or padded in memory: TMA zero-fills out-of-range
// rows/columns/K and the epilogue masks the edge tiles.
//
// Waits are bounded; a timeout sets a sticky device error word (reported by
// xpu_device_status) and the CTA still frees its TMEM before it exits.
#include <cuda.h>

#include "common.cuh"
#include "stream.cuh"
#include "xpu_internal.h"

namespace xpu {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr uint32_t kBM = 128, kBN = 256, kBK = 64;
constexpr uint32_t kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;        // 16 KB
constexpr uint32_t kBBoxBytes = 64 * kBK * 2;      // 8 KB: 64 (N) x 64 (K)
constexpr uint32_t kBBytes = kBN * kBK * 2;        // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 256;
constexpr int kGemmThreads = 192;
constexpr unsigned kErrGemmTimeout = 1u;

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: 128-byte swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // version
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: FP32 accumulator, A K-major, B MN-major.
__host__ __device__ constexpr uint32_t instr_desc(bool fp16) {
  return (1u << 4) |                          // D format F32
         ((fp16 ? 0u : 1u) << 7) |            // A format: F16 = 0, BF16 = 1
         ((fp16 ? 0u : 1u) << 10) |           // B format
         (0u << 15) |                         // A K-major
         (1u << 16) |                         // B MN-major
         ((kBN >> 3) << 17) |                 // N / 8
         ((kBM >> 4) << 24);                  // M / 16
}

__device__ __forceinline__ void tma_load_2d_plain(void *dst, const CUtensorMap *map, int32_t x, int32_t y,
                                                  uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
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

template <bool FP16>
__global__ void __launch_bounds__(kGemmThreads, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, uint16_t *C,
          uint32_t M, uint32_t N, uint32_t K) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], accum_full;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  // 1024-byte aligned stage ring (128-byte swizzle atoms).
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tiles_m = (M + kBM - 1) / kBM;
  const uint32_t tm = blockIdx.x % tiles_m, tn = blockIdx.x / tiles_m;
  const uint32_t nk = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&accum_full, 1);
    fence_mbar_init();
    failed = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      for (uint32_t k = 0; k < nk; ++k) {
        const uint32_t s = k % kStages, use = k / kStages;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) { failed = 1; break; }
        if (*reinterpret_cast<volatile int *>(&failed)) break;
        mbar_expect_tx(&full[s], kStageBytes);
        uint8_t *st = ring + s * kStageBytes;
        tma_load_2d_plain(st, &map_a, static_cast<int32_t>(k * kBK), static_cast<int32_t>(tm * kBM), &full[s]);
        for (uint32_t j = 0; j < kBN / 64; ++j)
          tma_load_2d_plain(st + kABytes + j * kBBoxBytes, &map_b, static_cast<int32_t>(tn * kBN + j * 64),
                            static_cast<int32_t>(k * kBK), &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(FP16);
      uint32_t k = 0;
      for (; k < nk; ++k) {
        const uint32_t s = k % kStages, use = k / kStages;
        if (!mbar_wait(&full[s], use & 1)) { failed = 1; break; }
        tc_fence_after();
        const uint32_t sa = smem_addr(ring + s * kStageBytes), sb = sa + kABytes;
        const uint64_t da = smem_desc(sa, 16, 1024), db = smem_desc(sb, kBBoxBytes, 1024);
#pragma unroll
        for (uint32_t kk = 0; kk < kBK / 16; ++kk)
          // K step of 16: +32 bytes inside A's 128-byte swizzled rows, +2 eight-row groups of B.
          mma_bf16(tmem, da + ((kk * 32u) >> 4), db + ((kk * 2048u) >> 4), idesc, (k | kk) != 0);
        mma_commit(&empty[s]);
      }
      mma_commit(&accum_full);  // fires once every issued MMA has completed
    }
  } else {
    // Epilogue warps 2..5: TMEM lanes 32 (warp % 4) .. + 31 hold rows of the tile.
    const uint32_t quarter = warp & 3;
    const bool ok = mbar_wait(&accum_full, 0);
    tc_fence_after();
    const uint32_t row = tm * kBM + quarter * 32 + lane;
    if (!ok) {
      failed = 1;
    } else {
      for (uint32_t c = 0; c < kBN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((quarter * 32u) << 16) + c, r);
        const uint32_t col = tn * kBN + c;
        if (row < M && col < N) {
          uint16_t *dst = C + static_cast<size_t>(row) * N + col;
#pragma unroll
          for (uint32_t g = 0; g < 4; ++g) {
            if (col + 8 * g >= N) break;
            uint4 v;
            v.x = pack2<FP16>(__uint_as_float(r[8 * g + 0]), __uint_as_float(r[8 * g + 1]));
            v.y = pack2<FP16>(__uint_as_float(r[8 * g + 2]), __uint_as_float(r[8 * g + 3]));
            v.z = pack2<FP16>(__uint_as_float(r[8 * g + 4]), __uint_as_float(r[8 * g + 5]));
            v.w = pack2<FP16>(__uint_as_float(r[8 * g + 6]), __uint_as_float(r[8 * g + 7]));
            *reinterpret_cast<uint4 *>(dst + 8 * g) = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && failed) atomicOr(&g_device_error, kErrGemmTimeout);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
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

cudaError_t gemm_launch(bool fp16, const void *A, const void *B, void *C, uint32_t M, uint32_t N, uint32_t K,
                        cudaStream_t stream) {
  const bool tma_ok = (K % 8 == 0) && (N % 8 == 0) && aligned16(A) && aligned16(B) && aligned16(C);
  if (!tma_ok) {
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
  cudaError_t e = make_tmap_2d_u16_swizzled(&map_a, A, K, M, K, kBK, kBM);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_u16_swizzled(&map_b, B, N, K, N, 64, kBK);
  if (e != cudaSuccess) return e;
  const size_t smem = gemm_smem_bytes();
  auto kernel = fp16 ? k_gemm_tc<true> : k_gemm_tc<false>;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const uint32_t tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  kernel<<<tiles, kGemmThreads, smem, stream>>>(map_a, map_b, static_cast<uint16_t *>(C), M, N, K);
  return cudaGetLastError();
}

unsigned take_device_error() {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return 0;
  if (v) cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  return v;
}

}  // namespace xpu
