// Roofline calibrators: a DRAM read-bandwidth kernel and a tensor-core
// throughput kernel, with the reference benchmarks' checksums.
//
// Read calibrator (replaces peak_mem_2d_kernel, peak_mem_2d_kernel.cpp:16-52).
// The surface is a row-major float matrix 1024 wide; a read unit is 16
// columns x 32 rows (2 KiB) at x = 16 (u % 64), y = 32 (u / 64), and its
// checksum is the FP32 sum, in order, of the unit's elements at (x, y),
// (x, y + 8), (x, y + 16), (x, y + 24) (the first element of each 16 x 8
// block the reference reads). Units sharing a band of 32 rows are contiguous
// in memory, so each CTA streams whole 8-row slabs (32 KiB, one bulk TMA copy
// each) through a shared-memory ring and 64 threads pick the checksum values
// out of the first row of each slab. Every byte of the surface crosses HBM
// once per launch.
//
// Compute calibrator (replaces peak_compute_dpas_kernel,
// peak_compute_dpas_kernel.cpp:13-68). One CTA per SM holds 0.5-filled bf16
// operand tiles in shared memory and issues `rounds` x 8 tcgen05.mma
// (128 x 256 x 16, FP32 accumulators in TMEM), alternating between two
// 256-column accumulators. Every MMA adds 16 x 0.25 = 4 to each accumulator
// element, so sink[cta] = (0 + acc0[0][0]) + (1 + acc1[0][0]) = 1 + 32 rounds.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "stream.cuh"
#include "xpu_internal.h"

namespace xpu {

// Sticky error word of this file's kernels (read by xpu_device_status).
__device__ unsigned int g_peak_error = 0;

namespace {

// ------------------------------------------------------------- read ----
constexpr uint32_t kSurfaceWidth = 1024;           // floats per row
constexpr uint32_t kUnitWidth = 16, kUnitRows = 32, kSlabRows = 8;
constexpr uint32_t kUnitsPerBand = kSurfaceWidth / kUnitWidth;  // 64
constexpr uint32_t kSlabBytes = kSlabRows * kSurfaceWidth * 4;  // 32 KiB
constexpr uint32_t kReadStages = 6;
constexpr int kReadThreads = 96;  // warp 0: producer; warps 1-2: checksum lanes
constexpr unsigned kErrPeakTimeout = 2u;

__device__ __forceinline__ uint32_t hash_u32(uint32_t bits) {
  bits ^= bits >> 16;
  bits *= 0x7feb352du;
  bits ^= bits >> 15;
  bits *= 0x846ca68bu;
  bits ^= bits >> 16;
  return bits;
}

// peak_mem_2d.cpp:36-47: 1 + (hash(index) & 0xffff) / 65536.
__global__ void k_peak_fill(float *surface, uint64_t elements) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < elements;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    surface[i] = 1.0f + static_cast<float>(hash_u32(static_cast<uint32_t>(i)) & 0xffffu) * (1.0f / 65536.0f);
}

__global__ void __launch_bounds__(kReadThreads, 1)
k_peak_read(const float *surface, float *sink, uint32_t bands) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kReadStages], empty[kReadStages];
  __shared__ int failed;
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 127u) / 128u * 128u - a0);
  const uint32_t warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kReadStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 2);  // the two checksum warps
    }
    fence_mbar_init();
    failed = 0;
  }
  __syncthreads();
  const uint64_t policy = evict_first_policy();
  // Slab j of this CTA: band = blockIdx.x + (j / 4) * gridDim.x, slab j % 4.
  const uint32_t my_bands = bands > blockIdx.x ? (bands - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const uint32_t slabs = my_bands * (kUnitRows / kSlabRows);
  if (warp == 0) {
    if (threadIdx.x == 0) {
      for (uint32_t j = 0; j < slabs; ++j) {
        const uint32_t s = j % kReadStages, use = j / kReadStages;
        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) { failed = 1; break; }
        const uint64_t band = blockIdx.x + static_cast<uint64_t>(j / 4) * gridDim.x;
        const float *src = surface + (band * kUnitRows + (j % 4) * kSlabRows) * kSurfaceWidth;
        mbar_expect_tx(&full[s], kSlabBytes);
        bulk_load(ring + s * kSlabBytes, src, kSlabBytes, &full[s], policy);
      }
    }
  } else {
    const uint32_t u = threadIdx.x - 32;  // unit within the band, 0..63
    float sum = 0.0f;
    for (uint32_t j = 0; j < slabs; ++j) {
      const uint32_t s = j % kReadStages, use = j / kReadStages;
      if (!mbar_wait(&full[s], use & 1)) { failed = 1; break; }
      sum += reinterpret_cast<const float *>(ring + s * kSlabBytes)[u * kUnitWidth];
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[s]);
      if (j % 4 == 3) {
        const uint64_t band = blockIdx.x + static_cast<uint64_t>(j / 4) * gridDim.x;
        sink[band * kUnitsPerBand + u] = sum;
        sum = 0.0f;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && failed) atomicOr(&g_peak_error, kErrPeakTimeout);
}

// ---------------------------------------------------------- compute ----
constexpr uint32_t kMmaM = 128, kMmaN = 256;  // K = 16 per instruction
constexpr uint32_t kMmasPerRound = 8;
constexpr uint32_t kPeakABytes = 16 * 1024;  // 16 eight-row groups x 1024 B (128-byte swizzle)
constexpr uint32_t kPeakBBytes = 32 * 1024;  // 4 atoms of 64 columns x 8 KB
constexpr int kComputeThreads = 128;
constexpr uint32_t kMaxPeakRounds = 524287;  // 1 + 32 rounds stays exact in FP32
// Dynamic shared memory of the compute CTA: the tiles need 48 KB; asking for
// 120 KB keeps one CTA per SM, so no CTA waits for another's TMEM columns.
constexpr size_t kComputeSmem = 120 * 1024;

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

__global__ void __launch_bounds__(kComputeThreads, 1) k_peak_compute(float *sink, uint32_t rounds, long long limit) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *tiles = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 0.5 in bf16 everywhere: the swizzled layout then cannot change a product.
  uint4 *t4 = reinterpret_cast<uint4 *>(tiles);
  for (uint32_t i = threadIdx.x; i < (kPeakABytes + kPeakBBytes) / 16; i += blockDim.x)
    t4[i] = make_uint4(0x3F003F00u, 0x3F003F00u, 0x3F003F00u, 0x3F003F00u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_base)),
                 "r"(512u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t sa = smem_addr(tiles), sb = sa + kPeakABytes;
    const uint64_t da = desc_sw128(sa, 16, 1024), db = desc_sw128(sb, 8192, 1024);
    // kind::f16, D = F32, A = B = BF16, A K-major, B MN-major, N = 256, M = 128.
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((kMmaN >> 3) << 17) | ((kMmaM >> 4) << 24);
    for (uint32_t r = 0; r < rounds; ++r) {
#pragma unroll
      for (uint32_t j = 0; j < kMmasPerRound; ++j) {
        const uint32_t acc = (r > 0 || j >= 2) ? 1u : 0u;
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem + (j & 1) * 256u),
            "l"(da), "l"(db), "r"(idesc), "r"(acc)
            : "memory");
      }
    }
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(&done))
                 : "memory");
  }
  __syncwarp();
  // Every thread waits for the MMAs (bounded by the host's estimate).
  bool ok = mbar_try_wait(&done, 0);
  if (!ok) {
    const long long start = clock64();
    while (!(ok = mbar_try_wait(&done, 0)))
      if (clock64() - start > limit) break;
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok && warp == 0) {
    uint32_t v0, v1;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v0) : "r"(tmem));
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(v1) : "r"(tmem + 256u));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    if (lane == 0) sink[blockIdx.x] = (0.0f + __uint_as_float(v0)) + (1.0f + __uint_as_float(v1));
  }
  if (!ok && threadIdx.x == 0) atomicOr(&g_peak_error, kErrPeakTimeout);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
  }
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

}  // namespace

unsigned take_peak_error() {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_peak_error, sizeof(v)) != cudaSuccess) return 0;
  if (v) cudaMemcpyToSymbol(g_peak_error, &zero, sizeof(zero));
  return v;
}

}  // namespace xpu

using namespace xpu;

extern "C" int xpu_peak_mem_fill(float *surface, uint64_t elements, void *stream) {
  if (!surface) return fail(XPU_ERR_INVALID, "xpu_peak_mem_fill: null pointer");
  if (elements == 0) return XPU_OK;
  const int sms = sm_count();
  if (sms <= 0) return cuda_status(cudaGetLastError(), "xpu_peak_mem_fill: device query");
  k_peak_fill<<<sms * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(surface, elements);
  return cuda_status(cudaGetLastError(), "xpu_peak_mem_fill");
}

extern "C" int xpu_peak_mem_read(const float *surface, float *sink, uint32_t surface_height, void *stream) {
  if (!surface || !sink) return fail(XPU_ERR_INVALID, "xpu_peak_mem_read: null pointer");
  if (surface_height == 0 || surface_height % kUnitRows)
    return fail(XPU_ERR_INVALID, "xpu_peak_mem_read: surface_height must be a positive multiple of 32");
  if (!aligned16(surface)) return fail(XPU_ERR_INVALID, "xpu_peak_mem_read: surface must be 16-byte aligned");
  const uint32_t bands = surface_height / kUnitRows;
  const int sms = sm_count();
  if (sms <= 0) return cuda_status(cudaGetLastError(), "xpu_peak_mem_read: device query");
  const size_t smem = kReadStages * kSlabBytes + 128;
  cudaError_t e = cudaFuncSetAttribute(k_peak_read, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "xpu_peak_mem_read");
  const uint32_t grid = std::min<uint32_t>(bands, static_cast<uint32_t>(sms));
  k_peak_read<<<grid, kReadThreads, smem, static_cast<cudaStream_t>(stream)>>>(surface, sink, bands);
  return cuda_status(cudaGetLastError(), "xpu_peak_mem_read");
}

extern "C" int xpu_peak_compute(float *sink, uint32_t ctas, uint32_t rounds, void *stream) {
  if (!sink) return fail(XPU_ERR_INVALID, "xpu_peak_compute: null pointer");
  if (ctas == 0 || rounds == 0) return fail(XPU_ERR_INVALID, "xpu_peak_compute: ctas and rounds must be positive");
  if (rounds > kMaxPeakRounds)
    return fail(XPU_ERR_INVALID, "xpu_peak_compute: rounds must be at most 524287 (FP32-exact checksum)");
  const size_t smem = kComputeSmem;
  cudaError_t e =
      cudaFuncSetAttribute(k_peak_compute, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return cuda_status(e, "xpu_peak_compute");
  // Wait bound: 2 s of clocks plus 1024 cycles per MMA (8x the issue time at full rate).
  const long long limit = 4000000000ll + static_cast<long long>(rounds) * kMmasPerRound * 1024;
  k_peak_compute<<<ctas, kComputeThreads, smem, static_cast<cudaStream_t>(stream)>>>(sink, rounds, limit);
  return cuda_status(cudaGetLastError(), "xpu_peak_compute");
}
