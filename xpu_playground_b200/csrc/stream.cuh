// TMA-fed weight streaming for the GEMV family (standalone GEMV and the
// fused decode kernels).
//
// A CTA is one producer warp plus kConsumerWarps consumer warps. The
// producer's elected lane walks the CTA's work list and, per stage
// (32 rows x ks columns, up to 32 KB), issues ks/box 2D TMA loads
// (cp.async.bulk.tensor, box = 32 rows x up to 256 columns) into a ring of
// shared-memory slots guarded by full/empty mbarriers. Consumer warp w owns
// rows 4w..4w+3 of every stage: it reads them (and the matching slice of the
// vector staged once in shared memory) with 16-byte shared loads, lane l
// folding chunks l, l+32, ... of each stage in order, and releases the slot.
// 32-row stages halve the per-stage barrier traffic of 16-row ones, which is
// what lets one CTA per SM stream at ~7 TB/s.
// Weight loads never wait on the math, so the copy engine keeps every SM's
// share of HBM bandwidth busy across tiles, epilogues and arrival fences.
//
// Waits are bounded (about two seconds of clock64): on a timeout the thread
// records an error code and gives up instead of hanging the GPU.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace xpu {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = 32 * kConsumerWarps;
constexpr int kStreamThreads = kConsumerThreads + 32;  // + one producer warp
constexpr uint32_t kRowsPerWarp = 4;
constexpr uint32_t kStageRows = kRowsPerWarp * kConsumerWarps;  // 32 rows per stage
constexpr long long kWaitCycles = 4000000000ll;        // ~2 s at 1.9 GHz
constexpr uint32_t kErrPipelineTimeout = 4;

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase of `bar` with the given parity; false after kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - start > kWaitCycles) return false;
  return true;
}

// Global -> shared bulk copy completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 2D tiled TMA load of box (x = column, y = row), completing on `bar`. No
// multicast: the source is this GPU's own memory and nothing else.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, uint64_t *bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Weights are read once per decode step: evict them from L2 first so the
// activations, partial sums and the KV cache stay resident.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Barrier among the consumer warps only (the producer never joins it).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}

// Programmatic dependent launch: let the next kernel's CTAs start (they only
// prefetch weights until they wait), and wait for the previous kernel.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Sum over the consumer threads (ctid = threadIdx.x - 32), fixed order.
__device__ __forceinline__ float consumer_sum(float v, float *scratch) {
  const int lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 1;
  v = warp_sum(v);
  consumer_sync();
  if (lane == 0) scratch[cw] = v;
  consumer_sync();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) total += scratch[i];
  return total;
}

// Geometry of one streamed weight matrix. Work item i covers row tile
// i / kparts (kStageRows rows) and K part i % kparts (kt columns starting at
// col0 + part * kt); an item is kt / ks stages of kStageRows x ks.
struct StreamGeom {
  const void *W;
  uint64_t pitch;   // row pitch in elements
  uint64_t col0;
  uint32_t rows;
  uint32_t kt, ks, kparts;
  uint32_t box;     // columns per TMA box (ks is a multiple)
  uint32_t stages;  // ring slots
  uint32_t slot;    // bytes per ring slot (>= one stage)
  __host__ __device__ uint32_t items() const { return ((rows + kStageRows - 1) / kStageRows) * kparts; }
};

// Shared-memory carve-up: [ring][x vector][full barriers][empty barriers].
struct StreamSmem {
  uint8_t *ring;
  uint4 *xs;
  uint64_t *full, *empty;
  float *scratch;  // kConsumerWarps floats
};

__host__ __device__ inline uint32_t stage_bytes(const StreamGeom &g) { return kStageRows * g.ks * 2; }

// TMA writes its boxes to 128-byte aligned shared memory; the ring start is
// rounded up to kRingAlign inside the dynamic allocation (which begins after
// the kernel's static shared variables, at any 16-byte boundary).
constexpr uint32_t kRingAlign = 1024;

__host__ __device__ inline size_t stream_smem_bytes(const StreamGeom &g, uint32_t x_elems) {
  return kRingAlign + static_cast<size_t>(g.stages) * g.slot + ((x_elems * 2 + 15) / 16) * 16 +
         2 * g.stages * sizeof(uint64_t) + kConsumerWarps * sizeof(float) + 16;
}

__device__ inline StreamSmem stream_smem(uint8_t *base, const StreamGeom &g, uint32_t x_elems) {
  StreamSmem s;
  const uint32_t a = smem_addr(base);
  s.ring = base + ((a + kRingAlign - 1) / kRingAlign * kRingAlign - a);
  s.xs = reinterpret_cast<uint4 *>(s.ring + static_cast<size_t>(g.stages) * g.slot);
  uint8_t *after_x = reinterpret_cast<uint8_t *>(s.xs) + ((x_elems * 2 + 15) / 16) * 16;
  s.full = reinterpret_cast<uint64_t *>(after_x);
  s.empty = s.full + g.stages;
  s.scratch = reinterpret_cast<float *>(s.empty + g.stages);
  return s;
}

// Called by every thread at kernel start: barrier init by thread 0. Returns
// false (in every thread) if the ring is not 128-byte aligned, in which case
// no TMA copy may be issued.
__device__ inline bool stream_init(const StreamSmem &s, const StreamGeom &g) {
  if (smem_addr(s.ring) & 127u) return false;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < g.stages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  return true;
}

// Producer: lane 0 of warp 0 issues every stage of this CTA's items. A
// stage slot holds ks / box boxes, each 16 rows x box columns, row-major.
// Rows past the end of the matrix are zero-filled by the TMA unit.
// Returns false on a timeout.
__device__ inline bool stream_produce(const StreamSmem &s, const StreamGeom &g, const CUtensorMap *map, uint32_t &it) {
  const uint32_t nst = g.kt / g.ks, sbytes = stage_bytes(g), nbox = g.ks / g.box;
  const uint32_t bbytes = kStageRows * g.box * 2;
  const uint64_t policy = evict_first_policy();
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    const uint32_t tile = item / g.kparts, part = item % g.kparts;
    const int32_t y = static_cast<int32_t>(tile * kStageRows);
    const uint32_t x0 = static_cast<uint32_t>(g.col0) + part * g.kt;
    for (uint32_t st = 0; st < nst; ++st, ++it) {
      const uint32_t slot = it % g.stages, use = it / g.stages;
      if (use > 0 && !mbar_wait(&s.empty[slot], (use - 1) & 1)) return false;
      mbar_expect_tx(&s.full[slot], sbytes);
      uint8_t *dst = s.ring + static_cast<size_t>(slot) * g.slot;
      for (uint32_t bx = 0; bx < nbox; ++bx)
        tma_load_2d(dst + bx * bbytes, map, static_cast<int32_t>(x0 + st * g.ks + bx * g.box), y, &s.full[slot], policy);
    }
  }
  return true;
}

// Consumer side of one item: accumulate rows 2cw and 2cw+1 of every stage.
// `xs` points at the x chunk of the item's first column. `it` is the running
// stage counter of this CTA. Returns false on a timeout.
template <typename T>
__device__ __forceinline__ bool stream_consume_item(const StreamSmem &s, const StreamGeom &g, const uint4 *xs,
                                                    uint32_t &it, float (&acc)[kRowsPerWarp]) {
  const uint32_t lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) - 1;
  const uint32_t nst = g.kt / g.ks, nck = g.ks / 8, bck = g.box / 8;
#pragma unroll
  for (uint32_t r = 0; r < kRowsPerWarp; ++r) acc[r] = 0.f;
  for (uint32_t st = 0; st < nst; ++st, ++it) {
    const uint32_t slot = it % g.stages, use = it / g.stages;
    if (!mbar_wait(&s.full[slot], use & 1)) return false;
    const uint4 *stage = reinterpret_cast<const uint4 *>(s.ring + static_cast<size_t>(slot) * g.slot);
    const uint4 *xv = xs + st * nck;
    for (uint32_t c = lane; c < nck; c += 32) {
      // chunk c of row r sits in box c / bck at row r, column chunk c % bck
      const uint32_t bx = c / bck, cc = c - bx * bck;
      const uint4 *a = stage + (bx * kStageRows + kRowsPerWarp * cw) * bck + cc;
      const uint4 x = xv[c];
#pragma unroll
      for (uint32_t r = 0; r < kRowsPerWarp; ++r) acc[r] = dot8<T>(a[r * bck], x, acc[r]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.empty[slot]);
  }
#pragma unroll
  for (uint32_t r = 0; r < kRowsPerWarp; ++r) acc[r] = warp_sum(acc[r]);
  return true;
}

// Largest multiple of 8 that divides kt and is at most 512.
__host__ inline uint32_t pick_stage_cols(uint32_t kt) {
  for (uint32_t ks = 512; ks >= 8; ks -= 8)
    if (kt % ks == 0) return ks;
  return 8;
}

__host__ inline StreamGeom make_geom(const void *W, uint64_t pitch, uint64_t col0, uint32_t rows, uint32_t kt,
                                     uint32_t kparts) {
  StreamGeom g;
  g.W = W;
  g.pitch = pitch;
  g.col0 = col0;
  g.rows = rows;
  g.kt = kt;
  g.ks = pick_stage_cols(kt);
  g.box = g.ks <= 256 ? g.ks : 256;
  while (g.ks % g.box) g.box -= 8;
  g.kparts = kparts;
  const uint32_t sb = kStageRows * g.ks * 2;
  uint32_t stages = (128u * 1024u) / sb;
  g.stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
  g.slot = sb;
  return g;
}

}  // namespace xpu
