// Kernels and graph recording of the batched decode step (batch.cuh).
//
// The projections are one kernel, k_bgemm: a persistent skinny GEMM
// Y[16 x rows] = X[16 x K] . W^T on tcgen05 with the weights W ([rows][K]
// row-major, as the checkpoint stores them) as the 128-row A operand and the
// 16 sequences' activations as the N = 16 B operand, both K-major and
// 128-byte swizzled straight from their row-major layouts by TMA.
//
// Work split (stream-K): the (128-row tile, 64-column K block) grid of a
// GEMM is one list of tiles * K/64 blocks in tile-major order, cut into
// `grid` equal contiguous ranges, one per CTA (one CTA per SM). Every SM thus
// streams the same number of weight bytes to within one 16 KB block, where
// a fixed split-K would leave up to 13% of the SMs idle. A CTA's range
// covers whole tiles, whose accumulators go straight to the epilogue, and at
// most two partial tiles at its ends, whose FP32 accumulators it publishes
// to gemm_part (slot 0: its first tile, slot 1: its last); the CTA that
// completes a partial tile's arrivals sums the tile's slots in CTA order
// (results do not depend on arrival order) and runs the epilogue.
//
// 192 threads per CTA:
//   warp 0     TMA producer: a stage is up to 4 consecutive K blocks of one
//              tile (split at tile and range ends), i.e. per block a 128 x 64
//              weight box (16 KB) and a 16 x 64 activation box (2 KB), into
//              a 3-stage ring of 72 KB stages. The 4 boxes of a stage cover
//              512 contiguous bytes of each weight row, requested back to
//              back (one-box stages, 128 bytes per row at a time, left HBM at
//              two thirds of its copy bandwidth). Weights do not depend on
//              the previous kernel: the first ring's worth is requested
//              before griddepcontrol.wait, so it streams while the previous
//              kernel drains.
//   warp 1     TMEM owner (2 x 4 x 16 columns: a double-buffered set of 4
//              accumulators); its elected lane issues 4 MMAs (M128 N16 K16)
//              per K block, the j-th into accumulator j, so consecutive MMAs
//              never wait on each other's accumulation (at N = 16 one MMA's
//              math is a few cycles; a chain through one accumulator would
//              be bound by the accumulate latency), and commits the stage
//              back to the producer and each finished segment to the
//              epilogue.
//   warps 2-5  epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, i.e.
//              weight rows, and all 16 sequence columns of the 4
//              accumulators, summed in accumulator order.
//   warps 6-7  (normalising GEMMs: QKV of layers > 0, gate/up, lm_head)
//              RMSNorm of the activation operand in place: the operand is
//              the raw residual x; per sequence r = 1/sqrt(mean(x^2) + eps)
//              from the per-tile sums of squares the residual GEMM epilogue
//              published (tiles in order), and every landed activation box
//              becomes bf16(w * bf16(x * r)) (the transformers rounding)
//              in its swizzled shared-memory place before the MMA warp may
//              read it. This replaces a separate norm kernel per GEMM.
//
// Waits are bounded; a timeout sets bit 4 of the batch error word and every
// role leaves its loop, waiting (bounded) for its own copies and MMAs.
#include <cuda.h>

#include <algorithm>
#include <cmath>

#include "batch.cuh"
#include "decode_device.cuh"
#include "tcgen05.cuh"
#include "xpu_internal.h"

namespace xpu {

namespace {

using dec::AttnShared;
using dec::pv_item;
using dec::scores_item;

constexpr uint32_t kTileM = 128;                       // weight rows per tile (MMA M, TMEM lanes)
constexpr uint32_t kSeqN = kMaxBatch;                  // MMA N
constexpr uint32_t kKb = 64;                           // K per block: one 128-byte swizzled row
constexpr uint32_t kWBytes = kTileM * kKb * 2;         // 16 KB
constexpr uint32_t kXBytes = kSeqN * kKb * 2;          // 2 KB
constexpr uint32_t kBoxes = 4;                         // K blocks per stage (at most)
constexpr uint32_t kStageW = kBoxes * kWBytes;          // 64 KB
constexpr uint32_t kStageBytes = kStageW + kBoxes * kXBytes;  // 72 KB (1024-byte multiple)
constexpr uint32_t kRing = 3;
constexpr uint32_t kGemmThreads = 256;
constexpr uint32_t kAccs = kKb / 16;                   // accumulators per buffer: one per MMA of a K block
constexpr uint32_t kAccCols = kSeqN;                   // TMEM columns of one accumulator
constexpr uint32_t kBufCols = kAccs * kAccCols;        // 64 columns per buffer
constexpr uint32_t kTmemCols = 2 * kBufCols;           // double buffered: 128 columns
// kind::f16 instruction descriptor: FP32 D, BF16 A and B, both K-major, N, M.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kSeqN >> 3) << 17) | ((kTileM >> 4) << 24);

static_assert(kStageBytes % 1024 == 0, "swizzled stages stay 1024-byte aligned");

enum Epi : int { kEpiQkv = 0, kEpiResid = 1, kEpiGateUp = 2, kEpiLm = 3, kEpiPart = 4 };

struct BGemm {
  uint32_t rows, nk, tiles, total;  // weight rows, K blocks per tile, tiles, tiles * nk
  BatchDims d;
  BatchBuffers b;
  bf16 *out;                    // residual x (kEpiResid), h (kEpiGateUp) or raw qkv (kEpiQkv)
  float *part;                  // kEpiPart: this rank's FP32 partial [16][rows] (tensor parallel)
  uint32_t xwhich, xk;          // kEpiPart: exchange slot (0 o_proj, 1 down) and number in the step
  const bf16 *norm_w;           // normalising GEMMs: the RMSNorm weight of the operand
};

struct EpiShared {
  float ssq[2][4][kSeqN];  // residual epilogue, alternating per tile
  ArgBest best[4][kSeqN];  // lm_head epilogue
  uint32_t bad[4][kSeqN];
};

__host__ __device__ inline uint32_t range_start(uint32_t c, uint32_t total, uint32_t grid) {
  return static_cast<uint32_t>(static_cast<uint64_t>(c) * total / grid);
}
// The CTA whose range holds K block kb (the largest c with range_start(c) <= kb).
__host__ __device__ inline uint32_t range_owner(uint32_t kb, uint32_t total, uint32_t grid) {
  return static_cast<uint32_t>((static_cast<uint64_t>(kb + 1) * grid + total - 1) / total) - 1;
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

// Step tracing, per launch [slot][8] globaltimer ns: 0 first CTA start,
// 1 last wait return, 2 last CTA end, 3 first wait return, 4 last CTA start,
// 5 last first-stage arrival, 6 last final accumulator, 7 last epilogue end.
// what: 0 start, 1 wait returned, 2 end, 5, 6, 7 as above (max over CTAs).
__device__ __forceinline__ void trace_mark(const BatchDims &d, const BatchBuffers &b, int what) {
  if (!b.trace) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  unsigned long long *slot = b.trace + static_cast<size_t>(d.trace_slot) * kBatchTraceValues;
  if (what == 0) { atomicMin(slot, t); atomicMax(slot + 4, t); }
  if (what == 1) { atomicMax(slot + 1, t); atomicMin(slot + 3, t); }
  if (what == 2 || what >= 5) atomicMax(slot + what, t);
}

__device__ __forceinline__ float bfv(const bf16 *p, size_t i) {
  return bf16_bits_to_float(reinterpret_cast<const uint16_t *>(p)[i]);
}
__device__ __forceinline__ void putv(bf16 *p, size_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = float_to_bf16_bits(v);
}

// Transpose reduction: lane l holds V partial sums; afterwards lane l
// holds the warp-wide sums of values [l V / 32, (l + 1) V / 32) in val[0..]
// (for V < 32 lanes that share a value hold identical sums).
template <int V>
__device__ __forceinline__ void warp_transpose_sum(float (&val)[V], uint32_t lane) {
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    const int o = 16 >> k, half = V >> (k + 1);
    if (half >= 1) {
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? val[i] : val[i + half];
        const float keep = upper ? val[i + half] : val[i];
        val[i] = keep + __shfl_xor_sync(kFullMask, send, o);
      }
    } else {
      val[0] += __shfl_xor_sync(kFullMask, val[0], o);
    }
  }
}

// ---- epilogues: thread = weight row r of tile t, v[s] = FP32 sum for sequence s ----

// Raw q/k/v: qkv[s][row] = bf16(sum); the per-head RMSNorm, RoPE and
// cache writes run in the attention kernel, whose CTA owns the head group.
__device__ inline void epi_qkv(const BGemm &p, uint32_t row, const float (&v)[kSeqN]) {
  if (row >= p.rows) return;
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s)
    if (s < p.d.batch) putv(p.out, static_cast<size_t>(s) * p.rows + row, v[s]);
}

// Tensor parallel o_proj / down: this rank's unrounded partial sums.
__device__ inline void epi_part(const BGemm &p, uint32_t row, const float (&v)[kSeqN]) {
  if (row >= p.rows) return;
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s)
    if (s < p.d.batch) p.part[static_cast<size_t>(s) * p.rows + row] = v[s];
}

// x[s][row] = bf16(x[s][row] + bf16(sum)) with x[s][row] preloaded in xr;
// the tile's sum of x^2 per sequence (lanes by a transpose reduction, then
// quarters in order) goes to ssq[tile][s] for the next normalising GEMM.
// `par` alternates per call so one barrier suffices.
__device__ inline void epi_resid(const BGemm &p, uint32_t t, uint32_t row, const float (&v)[kSeqN],
                                 const float (&xr)[kSeqN], EpiShared &es, uint32_t par) {
  const uint32_t lane = threadIdx.x & 31, quarter = (threadIdx.x >> 5) & 3, et = threadIdx.x - 64;
  const bool ok = row < p.rows;
  float sq[kSeqN];
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) {
    const float xn = round_bf16(__fadd_rn(xr[s], round_bf16(v[s])));
    if (ok && s < p.d.batch) putv(p.out, static_cast<size_t>(s) * p.rows + row, xn);
    sq[s] = ok ? __fmul_rn(xn, xn) : 0.f;
  }
  warp_transpose_sum<kSeqN>(sq, lane);  // lanes 2s, 2s + 1: the warp's sum for sequence s
  if ((lane & 1) == 0) es.ssq[par][quarter][lane / 2] = sq[0];
  epi_sync();
  if (et < kSeqN)
    p.b.ssq[t * kSeqN + et] = ((es.ssq[par][0][et] + es.ssq[par][1][et]) + es.ssq[par][2][et]) + es.ssq[par][3][et];
}

// Rows 2i, 2i + 1 are gate and up of unit i (adjacent lanes of one warp):
// h[s][i] = bf16(bf16(silu(bf16 g)) * bf16 u).
__device__ inline void epi_gateup(const BGemm &p, uint32_t row, const float (&v)[kSeqN]) {
  const uint32_t lane = threadIdx.x & 31, units = p.rows / 2;
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) {
    const float gv = round_bf16(v[s]);
    const float uv = __shfl_down_sync(kFullMask, gv, 1);
    if (!(lane & 1) && s < p.d.batch && row < p.rows) {
      const float act = round_bf16(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))));
      putv(p.out, static_cast<size_t>(s) * units + row / 2, __fmul_rn(act, uv));
    }
  }
}

// bf16 logits and the tile's (max, lowest index) candidate per sequence;
// NaN/Inf logits mark the tile bad.
__device__ inline void epi_lm(const BGemm &p, uint32_t t, uint32_t row, const float (&v)[kSeqN], EpiShared &es) {
  const uint32_t lane = threadIdx.x & 31, quarter = (threadIdx.x >> 5) & 3, et = threadIdx.x - 64;
  const bool ok = row < p.rows;
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) {
    const float lv = round_bf16(v[s]);
    if (ok && s < p.d.batch) p.b.logits[static_cast<size_t>(s) * p.rows + row] = float_to_bf16_bits(lv);
    const bool bad = ok && not_finite(lv);
    ArgBest cb = (ok && !bad) ? ArgBest{lv, p.d.v_offset + row} : ArgBest{-INFINITY, 0xffffffffu};
    cb = warp_argbest(cb);
    const uint32_t anybad = __any_sync(kFullMask, bad) ? 1u : 0u;
    if (lane == 0) { es.best[quarter][s] = cb; es.bad[quarter][s] = anybad; }
  }
  epi_sync();
  if (et < p.d.batch) {
    ArgBest cb = es.best[0][et];
    uint32_t bad = es.bad[0][et];
    for (uint32_t qq = 1; qq < 4; ++qq) { cb = arg_better(cb, es.best[qq][et]); bad |= es.bad[qq][et]; }
    p.b.cand[static_cast<size_t>(et) * p.tiles + t] = cb;
    p.b.cand_bad[static_cast<size_t>(et) * p.tiles + t] = bad;
  }
  epi_sync();
}

template <int EPI>
__device__ __forceinline__ void run_epilogue(const BGemm &p, uint32_t t, uint32_t r, const float (&v)[kSeqN],
                                             const float (&xr)[kSeqN], EpiShared &es, uint32_t par) {
  const uint32_t row = t * kTileM + r;
  if (EPI == kEpiQkv) epi_qkv(p, row, v);
  if (EPI == kEpiResid) epi_resid(p, t, row, v, xr, es, par);
  if (EPI == kEpiGateUp) epi_gateup(p, row, v);
  if (EPI == kEpiLm) epi_lm(p, t, row, v, es);
  if (EPI == kEpiPart) epi_part(p, row, v);
}

__device__ __forceinline__ bool failed_now(const int *f) { return *reinterpret_cast<const volatile int *>(f) != 0; }

// End of the stage that starts at K block kb: up to kBoxes blocks, not past
// the tile or the CTA's range. A CTA's first stage (kb == kb0) is one block:
// it is the one the pipeline waits for after the previous kernel, and a
// 16 KB weight box lands well before a 64 KB stage would when every SM
// starts at once.
__device__ __forceinline__ uint32_t stage_end(uint32_t kb, uint32_t kb0, uint32_t kb1, uint32_t nk) {
  const uint32_t tile_end = (kb / nk + 1) * nk;
  return min(min(kb + (kb == kb0 ? 1u : kBoxes), kb1), tile_end);
}

// Round two floats to bf16 (RNE) and pack them: lo in the low half.
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// bf16(w * bf16(x * r)) for the two bf16 of x and w in one word each.
__device__ __forceinline__ uint32_t norm_word(uint32_t x, uint32_t w, float r) {
  const uint32_t t = pack2_rn(__fmul_rn(bf16_lo(x), r), __fmul_rn(bf16_hi(x), r));
  return pack2_rn(__fmul_rn(bf16_lo(w), bf16_lo(t)), __fmul_rn(bf16_hi(w), bf16_hi(t)));
}

// RMSNorm of the activation boxes of one stage in place (transform warps,
// 64 threads): thread u owns logical 16-byte chunk u % 8 of rows 2 (u / 8)
// and 2 (u / 8) + 1 of each box; the 128-byte swizzle stores chunk j of row
// s at chunk j ^ (s % 8). Every load of the stage is issued before any math.
__device__ inline void norm_stage(uint8_t *xs, uint32_t kb, uint32_t e, uint32_t nk, const bf16 *w, const float *rs,
                                  uint32_t u) {
  const uint32_t j = u % 8, s0 = 2 * (u / 8), nb = e - kb;
  uint4 wv[kBoxes], xv[kBoxes][2];
#pragma unroll
  for (uint32_t b = 0; b < kBoxes; ++b)
    if (b < nb) {
      wv[b] = ld_ro16(w + ((kb + b) % nk) * kKb + j * 8);
#pragma unroll
      for (uint32_t q = 0; q < 2; ++q)
        xv[b][q] = *reinterpret_cast<const uint4 *>(xs + b * kXBytes + (s0 + q) * 128 + ((j ^ ((s0 + q) & 7)) * 16));
    }
  const float r0 = rs[s0], r1 = rs[s0 + 1];
#pragma unroll
  for (uint32_t b = 0; b < kBoxes; ++b)
    if (b < nb)
#pragma unroll
      for (uint32_t q = 0; q < 2; ++q) {
        const float r = q ? r1 : r0;
        const uint4 x = xv[b][q], wq = wv[b];
        *reinterpret_cast<uint4 *>(xs + b * kXBytes + (s0 + q) * 128 + ((j ^ ((s0 + q) & 7)) * 16)) =
            make_uint4(norm_word(x.x, wq.x, r), norm_word(x.y, wq.y, r), norm_word(x.z, wq.z, r),
                       norm_word(x.w, wq.w, r));
      }
}

// Tensor parallel partial GEMM: the last CTA to finish publishes exchange
// xk's epoch to the peers, once every CTA's partial sums are written (each
// CTA fences its writes before counting itself done).
__device__ __forceinline__ void part_published(const BGemm &p) {
  const unsigned prev = atomicAdd(p.b.xdone, 1u);
  if (prev == gridDim.x - 1) {
    __threadfence();
    *p.b.xdone = 0;  // for the next partial GEMM, which runs after this one
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.b.xflag[p.d.rank] + p.xwhich),
                 "l"(*p.b.xepoch + p.xk)
                 : "memory");
  }
}

template <int EPI, bool NORM>
__global__ void __launch_bounds__(kGemmThreads, 1)
k_bgemm(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x, const BGemm p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kRing], empty[kRing], xready[kRing], acc_full[2], acc_empty[2], mma_done;
  __shared__ float s_rs[kSeqN];
  __shared__ uint32_t tmem_base, consumed, issued_count;
  __shared__ int failed, last_flag;
  __shared__ EpiShared es;
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t G = gridDim.x, c = blockIdx.x, nk = p.nk;
  const uint32_t kb0 = range_start(c, p.total, G), kb1 = range_start(c + 1, p.total, G);

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kRing; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&xready[i], 2);  // one arrival per transform warp
    }
    for (uint32_t i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
    failed = 0;
    consumed = 0;
    issued_count = 0;
  }
  if (warp == 1) tmem_alloc1(&tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  grid_dep_launch();
  if (threadIdx.x == 0) trace_mark(p.d, p.b, 0);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      uint32_t issued = 0, kb = kb0;
      // Weights first (independent of the previous kernel), then, once it
      // has finished, the activations of those stages and the rest.
      uint32_t pre_end[kRing];
      for (; issued < kRing && kb < kb1; ++issued) {
        const uint32_t e = stage_end(kb, kb0, kb1, nk);
        uint8_t *st = ring + issued * kStageBytes;
        mbar_expect_tx(&full[issued], (e - kb) * (kWBytes + kXBytes));
        for (uint32_t j = 0; j < e - kb; ++j)
          tma_load_2d(st + j * kWBytes, &map_w, static_cast<int32_t>(((kb + j) % nk) * kKb),
                      static_cast<int32_t>((kb / nk) * kTileM), &full[issued], pol);
        pre_end[issued] = e;
        kb = e;
      }
      grid_dep_wait();
      for (uint32_t i = 0, b = kb0; i < issued; b = pre_end[i], ++i)
        for (uint32_t j = 0; j < pre_end[i] - b; ++j)
          tma_load_2d_plain(ring + i * kStageBytes + kStageW + j * kXBytes, &map_x,
                            static_cast<int32_t>(((b + j) % nk) * kKb), 0, &full[i]);
      for (uint32_t i = issued; kb < kb1; ++i) {
        const uint32_t s = i % kRing, use = i / kRing;
        if (failed_now(&failed) || !mbar_wait(&empty[s], (use - 1) & 1)) { failed = 1; break; }
        const uint32_t e = stage_end(kb, kb0, kb1, nk);
        uint8_t *st = ring + s * kStageBytes;
        mbar_expect_tx(&full[s], (e - kb) * (kWBytes + kXBytes));
        for (uint32_t j = 0; j < e - kb; ++j)
          tma_load_2d(st + j * kWBytes, &map_w, static_cast<int32_t>(((kb + j) % nk) * kKb),
                      static_cast<int32_t>((kb / nk) * kTileM), &full[s], pol);
        for (uint32_t j = 0; j < e - kb; ++j)
          tma_load_2d_plain(st + kStageW + j * kXBytes, &map_x, static_cast<int32_t>(((kb + j) % nk) * kKb), 0,
                            &full[s]);
        issued = i + 1;
        kb = e;
      }
      issued_count = issued;  // copies not consumed by the MMAs are drained at exit
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t seg = 0, i = 0;
      for (uint32_t kb = kb0; kb < kb1; ++i) {
        const uint32_t e = stage_end(kb, kb0, kb1, nk);
        const bool first = kb == kb0 || kb % nk == 0, last = e == kb1 || e % nk == 0;
        const uint32_t buf = seg & 1;
        if (first && seg >= 2) {
          if (!mbar_wait(&acc_empty[buf], ((seg >> 1) - 1) & 1)) { failed = 1; break; }
          tc_fence_after();
        }
        const uint32_t s = i % kRing;
        if (failed_now(&failed) || !mbar_wait(NORM ? &xready[s] : &full[s], (i / kRing) & 1)) { failed = 1; break; }
        if (i == 0) trace_mark(p.d, p.b, 5);
        tc_fence_after();
        const uint32_t sa = smem_addr(ring + s * kStageBytes), sx = sa + kStageW;
        for (uint32_t j = 0; j < e - kb; ++j)
#pragma unroll
          for (uint32_t k16 = 0; k16 < kAccs; ++k16)
            mma1_f16(tmem + buf * kBufCols + k16 * kAccCols, smem_desc(sa + j * kWBytes + 32 * k16, 16, 1024),
                     smem_desc(sx + j * kXBytes + 32 * k16, 16, 1024), kIdesc, (first && j == 0) ? 0u : 1u);
        mma1_commit(&empty[s]);
        if (last) {
          mma1_commit(&acc_full[buf]);
          ++seg;
        }
        kb = e;
      }
      consumed = i;
      // Every MMA this thread issued has completed before TMEM is freed.
      mma1_commit(&mma_done);
      if (!mbar_wait(&mma_done, 0)) failed = 1;
    }
  } else if (warp >= 6) {
    if (NORM) {
      // Transform warps: r per sequence from the residual GEMM's tile sums,
      // then every stage's activation boxes normalised in place.
      grid_dep_wait();
      const uint32_t u = threadIdx.x - 192;
      {
        // Sequence u / 4: thread u % 4 sums tiles [q0, q0 + per) in order
        // (all loads in flight at once), the four partials are added in
        // quarter order: a fixed order for every H.
        const uint32_t T = p.d.H / kTileM, per = (T + 3) / 4, s = u / 4, q0 = (u % 4) * per;
        float part = 0.f;
        if (per <= 16) {
          float x[16];
#pragma unroll
          for (uint32_t k = 0; k < 16; ++k) x[k] = (k < per && q0 + k < T) ? __ldcg(p.b.ssq + (q0 + k) * kSeqN + s) : 0.f;
#pragma unroll
          for (uint32_t k = 0; k < 16; ++k) part += x[k];
        } else {
          for (uint32_t k = 0; k < per && q0 + k < T; ++k) part += __ldcg(p.b.ssq + (q0 + k) * kSeqN + s);
        }
        const float p1 = __shfl_down_sync(kFullMask, part, 1), p2 = __shfl_down_sync(kFullMask, part, 2),
                    p3 = __shfl_down_sync(kFullMask, part, 3);
        if (u % 4 == 0) s_rs[s] = 1.0f / sqrtf(((part + p1) + p2 + p3) / static_cast<float>(p.d.H) + p.d.eps);
      }
      asm volatile("bar.sync 3, 64;" ::: "memory");
      bool dead = false;
      uint32_t i = 0;
      for (uint32_t kb = kb0; kb < kb1; ++i) {
        const uint32_t e = stage_end(kb, kb0, kb1, nk), s = i % kRing;
        if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&full[s], (i / kRing) & 1));
        if (dead) { failed = 1; break; }
        norm_stage(ring + s * kStageBytes + kStageW, kb, e, nk, p.norm_w, s_rs, u);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&xready[s]);
        kb = e;
      }
    }
  } else {
    // Epilogue warps: inputs of the epilogue (residual, positions, caches)
    // come from earlier kernels.
    grid_dep_wait();
    if (threadIdx.x == 64) trace_mark(p.d, p.b, 1);
    const uint32_t quarter = warp & 3, r = quarter * 32 + lane, et = threadIdx.x - 64;
    uint32_t par = 0;
    // A warp that gives up waiting stays in the loop (every epilogue warp
    // must reach the same named barriers) and computes on zeros from then on.
    bool dead = false;
    uint32_t seg = 0;
    for (uint32_t kb = kb0; kb < kb1; ++seg) {
      const uint32_t t = kb / nk, end = min(kb1, (t + 1) * nk);
      const bool whole = kb == t * nk && end == (t + 1) * nk;
      const uint32_t buf = seg & 1;
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&acc_full[buf], (seg >> 1) & 1));
      if (dead) failed = 1;
      if (threadIdx.x == 64 && end == kb1) trace_mark(p.d, p.b, 6);
      float v[kSeqN];
#pragma unroll
      for (uint32_t s = 0; s < kSeqN; ++s) v[s] = 0.f;
      if (!dead) {
        tc_fence_after();
        uint32_t a[kAccs][kSeqN];
        const uint32_t base = tmem + ((quarter * 32u) << 16) + buf * kBufCols;
#pragma unroll
        for (uint32_t j = 0; j < kAccs; ++j) tmem_ld16_nowait(base + j * kAccCols, a[j]);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t s = 0; s < kSeqN; ++s) {
          float sum = __uint_as_float(a[0][s]);
#pragma unroll
          for (uint32_t j = 1; j < kAccs; ++j) sum += __uint_as_float(a[j][s]);
          v[s] = sum;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      // Residual epilogue input, loaded before the arrival round trips.
      float xr[kSeqN];
#pragma unroll
      for (uint32_t s = 0; s < kSeqN; ++s)
        xr[s] = (EPI == kEpiResid && t * kTileM + r < p.rows && s < p.d.batch)
                    ? dec::bfcg(p.out, static_cast<size_t>(s) * p.rows + t * kTileM + r)
                    : 0.f;
      bool run = true;
      if (!whole) {
        const uint32_t slot = t == kb0 / nk ? 0u : 1u;
        float *dst = p.b.gemm_part + (static_cast<size_t>(c) * 2 + slot) * (kSeqN * kTileM) + r;
#pragma unroll
        for (uint32_t s = 0; s < kSeqN; ++s) dst[s * kTileM] = v[s];
        const uint32_t c0 = range_owner(t * nk, p.total, G), c1 = range_owner((t + 1) * nk - 1, p.total, G);
        epi_sync();  // the tile's partial is complete in this CTA; one thread fences for all
        if (et == 0) {
          // Release (cumulative over the barrier: every epilogue thread's
          // partial) and acquire (the other CTAs' partials) in one atomic.
          uint32_t old;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.b.cnt_tile + t) : "memory");
          last_flag = old == c1 - c0;
        }
        epi_sync();
        run = last_flag != 0;
        if (run) {
          float w[kSeqN];
#pragma unroll
          for (uint32_t s = 0; s < kSeqN; ++s) w[s] = 0.f;
          // Slots in CTA order, four at a time with all their loads in flight.
          for (uint32_t c4 = c0; c4 <= c1; c4 += 4) {
            float x[4][kSeqN];
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) {
              const uint32_t cc = c4 + j;
              if (cc > c1) break;
              const uint32_t sl = t == range_start(cc, p.total, G) / nk ? 0u : 1u;
              const float *src = p.b.gemm_part + (static_cast<size_t>(cc) * 2 + sl) * (kSeqN * kTileM) + r;
#pragma unroll
              for (uint32_t s = 0; s < kSeqN; ++s) x[j][s] = __ldcg(src + s * kTileM);
            }
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) {
              if (c4 + j > c1) break;
#pragma unroll
              for (uint32_t s = 0; s < kSeqN; ++s) w[s] += x[j][s];
            }
          }
#pragma unroll
          for (uint32_t s = 0; s < kSeqN; ++s) v[s] = w[s];
          if (et == 0) p.b.cnt_tile[t] = 0;
        }
      }
      if (run) {
        run_epilogue<EPI>(p, t, r, v, xr, es, par);
        par ^= 1u;
      }
      if (threadIdx.x == 64 && end == kb1) trace_mark(p.d, p.b, 7);
      kb = end;
    }
  }
  if (EPI == kEpiPart) __threadfence();  // this thread's partial sums, before the CTA counts itself done
  __syncthreads();
  if (threadIdx.x == 0) {
    // Copies still in flight after a failure: wait (bounded) for each issued
    // stage that the MMA thread did not consume.
    for (uint32_t i = consumed; i < issued_count; ++i)
      if (!mbar_wait(&full[i % kRing], (i / kRing) & 1)) break;
    if (failed) atomicOr(p.b.error, kErrPipelineTimeout);
    if (EPI == kEpiPart) part_published(p);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc1(tmem, kTmemCols);
  }
  if (threadIdx.x == 0) trace_mark(p.d, p.b, 2);
}

// ---------------------------------------------------------------- norms ----
// xn[s] = RMSNorm(x[s]) * w (transformers rounding, the batch-1 arithmetic
// and summation order); with `embed`, x[s] = embed[token s] first.
__global__ void __launch_bounds__(256) k_bnorm(BatchDims d, BatchBuffers b, const bf16 *w, int embed) {
  __shared__ float scratch[8];
  grid_dep_launch();
  if (threadIdx.x == 0) trace_mark(d, b, 0);
  grid_dep_wait();
  if (threadIdx.x == 0) trace_mark(d, b, 1);
  const uint32_t s = blockIdx.x, t = threadIdx.x, H = d.H;
  uint4 *x4 = reinterpret_cast<uint4 *>(b.x + static_cast<size_t>(s) * H);
  uint4 *xn4 = reinterpret_cast<uint4 *>(b.xn + static_cast<size_t>(s) * H);
  const uint4 *src = x4;
  if (embed) {
    const SeqState st = b.seq[s];
    uint32_t tok = st.position < st.prompt_len ? b.prompt[static_cast<size_t>(s) * d.max_seq + st.position] : st.token;
    if (tok >= d.tokens) {  // a NaN step's sentinel or a bad id: read row 0, flag the batch
      if (t == 0) atomicOr(b.error, 1u);
      tok = 0;
    }
    src = reinterpret_cast<const uint4 *>(b.embed) + static_cast<size_t>(tok) * (H / 8);
  }
  float ss = 0.f;
  for (uint32_t c = t; c < H / 8; c += 256) {
    const uint4 v = src[c];
    if (embed) x4[c] = v;
    ss = dec::sq8(v, ss);
  }
  ss = block_sum<8>(ss, scratch);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + d.eps);
  const uint4 *w4 = reinterpret_cast<const uint4 *>(w);
  for (uint32_t c = t; c < H / 8; c += 256) {
    const uint4 xv = src[c], wv = w4[c];
    const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = round_bf16(__fmul_rn(bf16_lo(wa[j]), round_bf16(__fmul_rn(bf16_lo(xa[j]), r))));
      const float hi = round_bf16(__fmul_rn(bf16_hi(wa[j]), round_bf16(__fmul_rn(bf16_hi(xa[j]), r))));
      o[j] = pack_bf16x2(lo, hi);
    }
    xn4[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) trace_mark(d, b, 2);
}

// ------------------------------------------------------------ attention ----
// Per (position chunk, kv head, sequence): the batch-1 scores and p.v items
// on sequence s's views of q, the caches and the attention scratch.
__device__ inline void seq_views(const BatchDims &bd, const BatchBuffers &bb, const LayerWeights &w, uint32_t s,
                                 DecodeDims &d, DecodeBuffers &b, LayerWeights &ws) {
  d = DecodeDims{};
  d.H = bd.H;
  d.QH_l = bd.QH;
  d.KVH_l = bd.KVH;
  d.max_seq = bd.max_seq;
  b = DecodeBuffers{};
  const size_t qs = static_cast<size_t>(s) * bd.QH;
  b.q = bb.q + qs * kHD;
  b.attn = bb.attn + qs * kHD;
  b.scores = bb.scores + qs * bd.max_seq;
  b.stats = bb.stats + qs * bd.nchunks * 2;
  b.attn_part = bb.attn_part + qs * bd.nchunks * kHD;
  b.cnt_attn = bb.cnt_attn + static_cast<size_t>(s) * bd.KVH;
  ws = w;
  ws.kcache = w.kcache + s * bb.kv_seq_stride;
  ws.vcache = w.vcache + s * bb.kv_seq_stride;
}

template <int G>
__global__ void __launch_bounds__(kStreamThreads) k_bscores(BatchDims bd, BatchBuffers bb, LayerWeights w) {
  __shared__ AttnShared<G> as;
  grid_dep_launch();
  grid_dep_wait();
  if (threadIdx.x < 32) return;
  const uint32_t s = blockIdx.z, n = bb.seq[s].position + 1;
  if (blockIdx.x * kPosChunk >= n) return;
  DecodeDims d;
  DecodeBuffers b;
  LayerWeights ws;
  seq_views(bd, bb, w, s, d, b, ws);
  scores_item<G>(d, b, ws, blockIdx.y, blockIdx.x, bd.nchunks, n, as);
}

template <int G>
__global__ void __launch_bounds__(kStreamThreads) k_bpv(BatchDims bd, BatchBuffers bb, LayerWeights w) {
  __shared__ AttnShared<G> as;
  grid_dep_launch();
  grid_dep_wait();
  if (threadIdx.x < 32) return;
  const uint32_t s = blockIdx.z, n = bb.seq[s].position + 1;
  if (blockIdx.x * kPosChunk >= n) return;
  DecodeDims d;
  DecodeBuffers b;
  LayerWeights ws;
  seq_views(bd, bb, w, s, d, b, ws);
  pv_item<G>(d, b, ws, blockIdx.y, blockIdx.x, bd.nchunks, n, as);
}

// ------------------------------------------------------ head epilogues ----
// One warp finishes head `col` of sequence s's raw [q; k; v] (the QKV
// GEMM's bf16 output) at position pos with the batch-1 arithmetic (lane l
// owns dimensions l + 32 j, so both rotate-half partners sit in one lane):
// q/k: RMSNorm with the head norm weight, then RoPE; v: unchanged. Returns
// the lane's four finished values (dims l, l + 32, l + 64, l + 96).
// The step-invariant inputs of one head epilogue (norm weight, RoPE row):
// they can be loaded before waiting for the QKV GEMM.
struct HeadConst {
  float nw[4], c[4], s[4];
};

__device__ inline HeadConst head_const(const BatchDims &bd, const BatchBuffers &bb, const LayerWeights &w, uint32_t col,
                                       uint32_t pos) {
  const uint32_t lane = threadIdx.x & 31;
  const bool is_v = col >= bd.QH + bd.KVH, is_q = col < bd.QH;
  HeadConst k;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    k.nw[j] = is_v ? 0.f : bfv(is_q ? w.q_norm : w.k_norm, lane + 32 * j);
    k.c[j] = is_v ? 0.f : bfv(bb.cos_t, static_cast<size_t>(pos) * kHD + lane + 32 * j);
    k.s[j] = is_v ? 0.f : bfv(bb.sin_t, static_cast<size_t>(pos) * kHD + lane + 32 * j);
  }
  return k;
}

// The lane's four raw values of head `col` of sequence s (QKV GEMM output).
__device__ inline void head_raw(const BatchDims &bd, const BatchBuffers &bb, uint32_t s, uint32_t col, float (&v)[4]) {
  const uint32_t lane = threadIdx.x & 31, rows = (bd.QH + 2 * bd.KVH) * kHD;
  const bf16 *raw = bb.qkv + static_cast<size_t>(s) * rows + static_cast<size_t>(col) * kHD;
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = bfv(raw, lane + 32 * j);
}

__device__ inline void head_math(const BatchDims &bd, uint32_t col, const float (&v)[4], const HeadConst &k,
                                 float (&out)[4]) {
  const bool is_v = col >= bd.QH + bd.KVH;
  const float(&nwv)[4] = k.nw;
  const float(&cv)[4] = k.c;
  const float(&sv)[4] = k.s;
  if (is_v) {
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = v[j];
    return;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(kHD) + bd.eps);
  float nv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) nv[j] = round_bf16(__fmul_rn(nwv[j], round_bf16(__fmul_rn(v[j], r))));
#pragma unroll
  for (int j = 0; j < 2; ++j) {  // pairs (i, i + 64): rotate_half
    const float a = nv[j], c = nv[j + 2];
    out[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(a, cv[j])), round_bf16(__fmul_rn(-c, sv[j]))));
    out[j + 2] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(c, cv[j + 2])), round_bf16(__fmul_rn(a, sv[j + 2]))));
  }
}

__device__ inline void head_finish(const BatchDims &bd, const BatchBuffers &bb, const LayerWeights &w, uint32_t s,
                                   uint32_t col, uint32_t pos, float (&out)[4]) {
  const HeadConst k = head_const(bd, bb, w, col, pos);
  float v[4];
  head_raw(bd, bb, s, col, v);
  head_math(bd, col, v, k, out);
}

// Chunked-attention path: the head epilogues of (kv head blockIdx.x,
// sequence blockIdx.y) into q and the caches (one warp per head).
__global__ void __launch_bounds__(256) k_bheads(BatchDims bd, BatchBuffers bb, LayerWeights w) {
  grid_dep_launch();
  grid_dep_wait();
  const uint32_t h = blockIdx.x, s = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t G = bd.QH / bd.KVH, pos = bb.seq[s].position;
  for (uint32_t k = warp; k < G + 2; k += 8) {
    const uint32_t col = k < G ? h * G + k : (k == G ? bd.QH + h : bd.QH + bd.KVH + h);
    float out[4];
    head_finish(bd, bb, w, s, col, pos, out);
    bf16 *dst = k < G ? bb.q + (static_cast<size_t>(s) * bd.QH + col) * kHD
                      : (k == G ? w.kcache : w.vcache) + s * bb.kv_seq_stride + (static_cast<size_t>(pos) * bd.KVH + h) * kHD;
#pragma unroll
    for (int j = 0; j < 4; ++j) putv(dst, lane + 32 * j, out[j]);
  }
}

// ------------------------------------------------- fused attention (one CTA) ----
// One CTA per (kv head h, sequence s) runs the whole decode attention of the
// head group over positions [0, n): pass 1 streams K (TMA, 64-position
// stages of the head's 256-byte rows) and stores s = bf16(bf16(q.k) * scale)
// for the group's G query heads in shared memory - exactly, as bf16; then
// per head M = max s, S = sum exp(s - M) (fixed order) and the scores become
// p = bf16(exp(s - M) * (1 / S)) in place (the rounding points of the
// batch-1 path); pass 2 streams V and accumulates p * v, and the CTA writes
// the bf16 output of its G heads. Nothing crosses CTAs, so there is no
// score scratch, statistics exchange or chunk combine in global memory.
// Attention leaves HBM bandwidth unused, so the producer warp's other lanes
// also prefetch a slice of the next GEMM's weights (o_proj, 33.5 MB on the
// 8B shape, a quarter of L2) into L2 with an evict-last hint, while the K/V
// stream is marked evict-first: the o_proj GEMM then streams from L2.
// Warp 0 is the TMA producer; the 16 consumer warps take 4 positions each
// of every stage, lane l dimensions 4l .. 4l + 3 (16 warps rather than 8:
// a stage's dot products and reductions are short dependent chains, and
// twice the warps hide their latency behind the stream). K stages that hold only
// positions below n - 1 (rows written by earlier steps) are requested before
// griddepcontrol.wait; the newest row comes from the previous kernel.
constexpr uint32_t kAttnPos = 64;                       // positions per stage
constexpr uint32_t kAttnStageBytes = kAttnPos * kHD * 2;  // 16 KB
constexpr uint32_t kAttnStages = 6;
constexpr uint32_t kAttnWarps = 16;                             // consumer warps
constexpr uint32_t kAttnThreads = 32 * (kAttnWarps + 1);
constexpr uint32_t kAttnPosPerWarp = kAttnPos / kAttnWarps;     // 4

__device__ __forceinline__ void attn_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kAttnWarps) : "memory"); }

__host__ __device__ inline size_t attn_scores_bytes(uint32_t G, uint32_t max_seq) {
  return (static_cast<size_t>(G) * max_seq * 2 + 15) / 16 * 16;
}
__host__ __device__ inline size_t attn_smem_bytes(uint32_t G, uint32_t max_seq) {
  return 1024 + static_cast<size_t>(kAttnStages) * kAttnStageBytes + attn_scores_bytes(G, max_seq);
}

template <int G>
__global__ void __launch_bounds__(kAttnThreads, 1)
k_battn(BatchDims bd, BatchBuffers bb, LayerWeights w, const __grid_constant__ CUtensorMap map_k,
        const __grid_constant__ CUtensorMap map_v, const uint8_t *prefetch, uint64_t prefetch_bytes) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kAttnStages], empty[kAttnStages];
  __shared__ float red_m[kAttnWarps][G], red_s[kAttnWarps][G];
  __shared__ float sM[G], sInv[G];
  __shared__ float q_s[G][kHD];                            // finished q of the group
  __shared__ __align__(16) uint16_t knew[kHD], vnew[kHD];  // finished k, v of the newest position
  __shared__ int failed;
  __shared__ uint32_t issued_n;
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  uint16_t *sc = reinterpret_cast<uint16_t *>(ring + kAttnStages * kAttnStageBytes);  // [G][max_seq] bf16
  const uint32_t h = blockIdx.x, s = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ms = bd.max_seq;
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < kAttnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kAttnWarps);
    }
    fence_mbar_init();
    failed = 0;
    issued_n = 0;
  }
  __syncthreads();
  grid_dep_launch();
  if (threadIdx.x == 0) trace_mark(bd, bb, 0);
  // The position comes from the step state, which no kernel of the step
  // writes before the argmax, so it is read before waiting.
  const uint32_t n = bb.seq[s].position + 1;
  const uint32_t nst = (n + kAttnPos - 1) / kAttnPos;  // stages per pass
  const int32_t y0 = static_cast<int32_t>(s * ms), xh = static_cast<int32_t>(h * kHD);

  if (warp == 0 && lane != 0) {
    if (prefetch) {
      // This CTA's slice of the next GEMM's weights, 32 KB per request.
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
      const uint64_t ctas = static_cast<uint64_t>(gridDim.x) * gridDim.y, c = blockIdx.y * gridDim.x + blockIdx.x;
      const uint64_t b0 = (prefetch_bytes * c / ctas) & ~uint64_t(15), b1 = (prefetch_bytes * (c + 1) / ctas) & ~uint64_t(15);
      for (uint64_t off = b0 + (lane - 1) * 32768ull; off < b1; off += 31 * 32768ull) {
        const uint32_t len = static_cast<uint32_t>(b1 - off < 32768ull ? b1 - off : 32768ull);
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(prefetch + off), "r"(len),
                     "l"(pol)
                     : "memory");
      }
    }
  } else if (warp == 0) {
    {
      const uint64_t kv_pol = evict_first_policy();
      // The cache rows below the newest were written by earlier steps, and
      // the newest row is taken from shared memory (this CTA computes it):
      // the first ring's worth of K stages is fetched before the wait.
      uint32_t early = nst < kAttnStages ? nst : kAttnStages;
      for (uint32_t i = 0; i < early; ++i) {
        mbar_expect_tx(&full[i], kAttnStageBytes);
        tma_load_2d(ring + i * kAttnStageBytes, &map_k, xh, y0 + static_cast<int32_t>(i * kAttnPos), &full[i], kv_pol);
      }
      grid_dep_wait();
      uint32_t i = early;
      for (; i < 2 * nst; ++i) {
        const uint32_t slot = i % kAttnStages, use = i / kAttnStages;
        if (use > 0 && (failed_now(&failed) || !mbar_wait(&empty[slot], (use - 1) & 1))) { failed = 1; break; }
        mbar_expect_tx(&full[slot], kAttnStageBytes);
        const bool is_v = i >= nst;
        const int32_t y = y0 + static_cast<int32_t>((is_v ? i - nst : i) * kAttnPos);
        tma_load_2d(ring + slot * kAttnStageBytes, is_v ? &map_v : &map_k, xh, y, &full[slot], kv_pol);
      }
      issued_n = i;
    }
  } else {
    grid_dep_wait();
    if (threadIdx.x == 32) trace_mark(bd, bb, 1);
    const uint32_t cw = warp - 1, t = threadIdx.x - 32;
    bool dead = false;
    // Head epilogues of the group (warp g < G: q head h G + g; G: k; G + 1: v)
    // at the newest position; k and v also go to the caches for later steps.
    const uint32_t pos_new = n - 1;
    if (cw < static_cast<uint32_t>(G) + 2) {
      const uint32_t col = cw < G ? h * G + cw : (cw == G ? bd.QH + h : bd.QH + bd.KVH + h);
      float out[4];
      head_finish(bd, bb, w, s, col, pos_new, out);
      if (cw < G) {
#pragma unroll
        for (int j = 0; j < 4; ++j) q_s[cw][lane + 32 * j] = out[j];
      } else {
        bf16 *cache = (cw == G ? w.kcache : w.vcache) + s * bb.kv_seq_stride +
                      (static_cast<size_t>(pos_new) * bd.KVH + h) * kHD;
        uint16_t *row = cw == G ? knew : vnew;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          row[lane + 32 * j] = float_to_bf16_bits(out[j]);
          putv(cache, lane + 32 * j, out[j]);
        }
      }
    }
    attn_sync();
    // q of the group's heads, this lane's 4 dimensions 4l .. 4l + 3
    float q[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) q[g][j] = q_s[g][lane * 4 + j];
    // ---- pass 1: scores
    for (uint32_t i = 0; i < nst; ++i) {
      const uint32_t slot = i % kAttnStages;
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&full[slot], (i / kAttnStages) & 1));
      const uint8_t *st = ring + slot * kAttnStageBytes;
      float val[kAttnPosPerWarp * G];
#pragma unroll
      for (uint32_t pp = 0; pp < kAttnPosPerWarp; ++pp) {
        const uint32_t pos = i * kAttnPos + cw * kAttnPosPerWarp + pp;
        const uint2 kr = dead ? make_uint2(0, 0)
                         : pos == pos_new ? *reinterpret_cast<const uint2 *>(knew + lane * 4)
                                          : *reinterpret_cast<const uint2 *>(st + (cw * kAttnPosPerWarp + pp) * (kHD * 2) + lane * 8);
        const float k4[4] = {bf16_lo(kr.x), bf16_hi(kr.x), bf16_lo(kr.y), bf16_hi(kr.y)};
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float a = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) a = fmaf(q[g][j], k4[j], a);
          val[pp * G + g] = a;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      warp_transpose_sum<kAttnPosPerWarp * G>(val, lane);
      constexpr uint32_t kVals = kAttnPosPerWarp * G;               // sums per warp and stage
      constexpr uint32_t kPer = kVals >= 32 ? kVals / 32 : 1;         // sums held per lane
      constexpr uint32_t kShare = kVals >= 32 ? 1 : 32 / kVals;       // lanes holding the same sum
#pragma unroll
      for (uint32_t k = 0; k < kPer; ++k) {
        const uint32_t idx = lane / kShare * kPer + k;
        const uint32_t pp = idx / G, g = idx % G, pos = i * kAttnPos + cw * kAttnPosPerWarp + pp;
        if (lane % kShare == 0 && pos < n)
          sc[g * ms + pos] = float_to_bf16_bits(round_bf16(__fmul_rn(round_bf16(val[k]), kAttnScale)));
      }
    }
    attn_sync();
    // ---- per head: max, sum of exp, then probabilities in place
    float m[G];
#pragma unroll
    for (int g = 0; g < G; ++g) m[g] = -INFINITY;
    for (uint32_t pos = t; pos < n; pos += 32 * kAttnWarps)
#pragma unroll
      for (int g = 0; g < G; ++g) m[g] = fmaxf(m[g], bf16_bits_to_float(sc[g * ms + pos]));
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float wm = warp_max(m[g]);
      if (lane == 0) red_m[cw][g] = wm;
    }
    attn_sync();
    if (t < static_cast<uint32_t>(G)) {
      float mm = red_m[0][t];
      for (uint32_t w = 1; w < kAttnWarps; ++w) mm = fmaxf(mm, red_m[w][t]);
      sM[t] = mm;
    }
    attn_sync();
    float l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) l[g] = 0.f;
    for (uint32_t pos = t; pos < n; pos += 32 * kAttnWarps)
#pragma unroll
      for (int g = 0; g < G; ++g) l[g] += expf(bf16_bits_to_float(sc[g * ms + pos]) - sM[g]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ws = warp_sum(l[g]);
      if (lane == 0) red_s[cw][g] = ws;
    }
    attn_sync();
    if (t < static_cast<uint32_t>(G)) {
      float ss = 0.f;
      for (uint32_t w = 0; w < kAttnWarps; ++w) ss += red_s[w][t];
      sInv[t] = 1.0f / ss;
    }
    attn_sync();
    for (uint32_t pos = t; pos < n; pos += 32 * kAttnWarps)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float sv = bf16_bits_to_float(sc[g * ms + pos]);
        sc[g * ms + pos] = float_to_bf16_bits(__fmul_rn(expf(sv - sM[g]), sInv[g]));
      }
    attn_sync();
    // ---- pass 2: p . v
    float acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
    for (uint32_t i = 0; i < nst; ++i) {
      const uint32_t gi = nst + i, slot = gi % kAttnStages;
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&full[slot], (gi / kAttnStages) & 1));
      const uint8_t *st = ring + slot * kAttnStageBytes;
#pragma unroll
      for (uint32_t pp = 0; pp < kAttnPosPerWarp; ++pp) {
        const uint32_t pos = i * kAttnPos + cw * kAttnPosPerWarp + pp;
        if (pos >= n || dead) continue;
        const uint2 vr = pos == pos_new ? *reinterpret_cast<const uint2 *>(vnew + lane * 4)
                                        : *reinterpret_cast<const uint2 *>(st + (cw * kAttnPosPerWarp + pp) * (kHD * 2) + lane * 8);
        const float v4[4] = {bf16_lo(vr.x), bf16_hi(vr.x), bf16_lo(vr.y), bf16_hi(vr.y)};
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pr = bf16_bits_to_float(sc[g * ms + pos]);
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[g][j] = fmaf(pr, v4[j], acc[g][j]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (dead) failed = 1;
    attn_sync();  // every stage consumed: the ring is free for the warp partials
    float *part = reinterpret_cast<float *>(ring);  // [16 warps][G][128]
#pragma unroll
    for (int g = 0; g < G; ++g)
      *reinterpret_cast<float4 *>(part + (cw * G + g) * kHD + lane * 4) =
          make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    attn_sync();
    for (uint32_t e = t; e < G * kHD; e += 32 * kAttnWarps) {
      float o = 0.f;
#pragma unroll
      for (uint32_t w = 0; w < kAttnWarps; ++w) o += part[w * G * kHD + e];
      const uint32_t g = e / kHD, dd = e % kHD;
      putv(bb.attn, (static_cast<size_t>(s) * bd.QH + h * G + g) * kHD + dd, o);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && failed) {
    // After a failure copies may still be in flight: wait (bounded) for the
    // last ring's worth that was issued.
    const uint32_t from = issued_n > kAttnStages ? issued_n - kAttnStages : 0;
    for (uint32_t i = from; i < issued_n; ++i)
      if (!mbar_wait(&full[i % kAttnStages], (i / kAttnStages) & 1)) break;
    atomicOr(bb.error, kErrPipelineTimeout);
  }
  if (threadIdx.x == 0) trace_mark(bd, bb, 2);
}

// ------------------------------------ tensor-core attention (2-CTA cluster) ----
// The (kv head h, sequence s) attention of k_battn with both products on
// tcgen05 (M = 128, N = 16 head slots, G of them used), split over a
// cluster of two CTAs that take the first and second half of the
// context's 128-position stages:
//   pass 1  S = K . Q^T per stage: A = the K stage (positions x 128 dims, two
//           64-dim TMA boxes, K-major, 128-byte swizzle), B = the group's
//           finished q (16 rows x 128 dims, same layout), D = 128 positions
//           x 16 slots in TMEM (4 buffers); the compute warps read one
//           position per thread and store s = bf16(bf16(S) * scale) into P
//           (bf16, rows = head slots, K-major, 128-byte swizzle, 64
//           positions per 2 KB atom);
//   softmax the two CTAs exchange their maxima and then their sums of
//           exp(s - M) through distributed shared memory (stores into the
//           peer plus a remote mbarrier arrival): M = max, S = sum in CTA
//           order, identical in both; then P = bf16(exp(s - M) * (1 / S)) in
//           place, 0 past the context;
//   pass 2  O^T = V^T . P^T over the CTA's V stages: A = the V stage read
//           MN-major (dims contiguous: cache rows as TMA lands them), B = P;
//           D = 128 dims x 16 slots in TMEM; the second CTA stores its O^T
//           into the first's shared memory, which adds the halves in order
//           and writes the bf16 output.
// The CTA holding the newest position finishes that position's k and v and
// writes them to the caches (with a proxy fence) before its producer
// fetches the stages that hold them; its last V stage's rows past the
// context are zeroed in shared memory (a stale row must not meet a zero
// probability as 0 * NaN). Both CTAs finish the group's q.
// Warp 0: TMA producer (lane 0) and the L2 prefetch of the next GEMM's
// weights (lanes 1-31); warp 1: TMEM owner and MMA issuer; warps 2-5:
// compute. Two clusters share an SM (their rings are sized for that).
constexpr uint32_t kTcPos = 128;                   // positions per stage
constexpr uint32_t kTcBox = 128 * 64 * 2;          // one 64-dim box of a stage: 16 KB
constexpr uint32_t kTcStage = 2 * kTcBox;          // 32 KB
constexpr uint32_t kTcMaxStages = 6;               // ring slots: as many as fit (>= 2)
constexpr uint32_t kTcThreads = 192;
constexpr uint32_t kTcN = 16;                      // MMA N: head slots
constexpr uint32_t kPAtom = 16 * 128;              // 16 rows x 64 bf16: 2 KB
constexpr uint32_t kTcSBufs = 4;                   // TMEM score buffers (MMA runs up to 4 stages ahead)
constexpr uint32_t kTcTmemCols = 128;              // S[4] (4 x 16) + O (16)
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((kTcN >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescO = kIdescS | (1u << 15);  // A MN-major

// Dynamic shared memory of one CTA: ring + q + P for half the stages of max_seq.
__host__ __device__ inline size_t tc_attn_smem_bytes(uint32_t max_seq, uint32_t stages) {
  const size_t half = ((static_cast<size_t>(max_seq) + kTcPos - 1) / kTcPos + 1) / 2;
  return 1024 + static_cast<size_t>(stages) * kTcStage + 2 * kPAtom + half * 2 * kPAtom;
}

// Byte offset of element (row r, column c < 64) inside a 128-byte swizzled
// atom block of 128-byte rows.
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
  return r * 128 + ((((c >> 3) ^ (r & 7)) << 4) | ((c & 7) << 1));
}

__device__ __forceinline__ void tc_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// HEADS: the cluster finishes its group's heads (decode); otherwise q, k and
// v are finished and cached by k_bheads first (prefill).
template <int G, bool HEADS>
__global__ void __launch_bounds__(kTcThreads, 2)
k_battn_tc(BatchDims bd, BatchBuffers bb, LayerWeights w, const __grid_constant__ CUtensorMap map_k,
           const __grid_constant__ CUtensorMap map_v, const uint8_t *prefetch, uint64_t prefetch_bytes,
           uint32_t stages) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kTcMaxStages], empty[kTcMaxStages], s_full[kTcSBufs], s_empty[kTcSBufs], hd_ready, p_ready,
      last_landed, v_patched, o_full, mma_done, x_max, x_sum, x_out;
  __shared__ uint32_t tmem_base, issued_n, consumed_n;
  __shared__ float red[4][G], sM[G], sInv[G];
  __shared__ float xm[2][G], xl[2][G];  // the two CTAs' maxima / sums (written by both)
  __shared__ float xo[G][kHD];           // second CTA's O^T (in the first CTA)
  __shared__ int failed;
  const uint32_t a0 = smem_addr(smem_raw);
  uint8_t *ring = smem_raw + ((a0 + 1023u) / 1024u * 1024u - a0);
  uint8_t *qs = ring + stages * kTcStage;  // 2 atoms: dims 0-63, 64-127
  uint8_t *ps = qs + 2 * kPAtom;           // P atoms, 64 positions each
  const uint32_t rank = cluster_rank(), peer = rank ^ 1u;
  const uint32_t h = blockIdx.x >> 1, s = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t n = bb.seq[s].position + 1, pos_new = n - 1;
  const uint32_t nst = (n + kTcPos - 1) / kTcPos, nh = (nst + 1) / 2;
  const uint32_t st0 = rank ? nh : 0, my = (rank ? nst : nh) - st0;  // this CTA's stages [st0, st0 + my)
  const bool owner = my > 0 && st0 + my == nst;                      // holds the newest position
  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (uint32_t i = 0; i < kTcSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
    }
    mbar_init(&hd_ready, 4);
    mbar_init(&p_ready, 4);
    mbar_init(&last_landed, 1);
    mbar_init(&v_patched, 4);
    mbar_init(&o_full, 1);
    mbar_init(&mma_done, 1);
    mbar_init(&x_max, G);    // the peer's G maximum writers
    mbar_init(&x_sum, G);    // the peer's G sum writers
    mbar_init(&x_out, 128);  // the second CTA's 128 output threads
    fence_mbar_init();
    failed = 0;
    issued_n = 0;
    consumed_n = 0;
  }
  if (warp == 1) tmem_alloc1(&tmem_base, kTcTmemCols);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  grid_dep_launch();
  if (threadIdx.x == 0) trace_mark(bd, bb, 0);
  const int32_t y0 = static_cast<int32_t>(s * bd.seq_rows), xh = static_cast<int32_t>(h * kHD);

  if (warp == 0 && lane != 0) {
    if (prefetch) {
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
      const uint64_t ctas = static_cast<uint64_t>(gridDim.x) * gridDim.y, c = blockIdx.y * gridDim.x + blockIdx.x;
      const uint64_t b0 = (prefetch_bytes * c / ctas) & ~uint64_t(15), b1 = (prefetch_bytes * (c + 1) / ctas) & ~uint64_t(15);
      for (uint64_t off = b0 + (lane - 1) * 32768ull; off < b1; off += 31 * 32768ull) {
        const uint32_t len = static_cast<uint32_t>(b1 - off < 32768ull ? b1 - off : 32768ull);
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(prefetch + off), "r"(len),
                     "l"(pol)
                     : "memory");
      }
    }
  } else if (warp == 0) {
    // Producer: local stages 0 .. my-1 are K, my .. 2 my - 1 are V (global
    // stage st0 + local). Stages without the newest row may go before the
    // wait (decode); the owner's last K and V stages wait until the newest
    // row is cached (hd_ready). Prefill: every row was cached before.
    const uint64_t kv_pol = evict_first_policy();
    auto issue = [&](uint32_t i, uint32_t slot) {
      const bool is_v = i >= my;
      const int32_t y = y0 + static_cast<int32_t>((st0 + (is_v ? i - my : i)) * kTcPos);
      const CUtensorMap *m = is_v ? &map_v : &map_k;
      mbar_expect_tx(&full[slot], kTcStage);
      tma_load_2d(ring + slot * kTcStage, m, xh, y, &full[slot], kv_pol);
      tma_load_2d(ring + slot * kTcStage + kTcBox, m, xh + 64, y, &full[slot], kv_pol);
    };
    uint32_t i = 0;
    if (HEADS)
      for (; i < stages && i < my && st0 + i + 1 < nst; ++i) issue(i, i);  // K stages below the newest row
    grid_dep_wait();
    bool have_row = !HEADS || !owner;
    for (; i < 2 * my; ++i) {
      const uint32_t slot = i % stages, use = i / stages;
      if (use > 0 && (failed_now(&failed) || !mbar_wait(&empty[slot], (use - 1) & 1))) { failed = 1; break; }
      if (!have_row && (i == my - 1 || i == 2 * my - 1)) {
        if (!mbar_wait(&hd_ready, 0)) { failed = 1; break; }
        have_row = true;
      }
      issue(i, slot);
    }
    issued_n = i;
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t i = 0;
      bool ok = my == 0 || mbar_wait(&hd_ready, 0);  // q in shared memory
      tc_fence_after();
      // pass 1: scores
      for (; ok && i < my; ++i) {
        const uint32_t slot = i % stages, b = i % kTcSBufs;
        if (i >= kTcSBufs && !mbar_wait(&s_empty[b], ((i / kTcSBufs) - 1) & 1)) { ok = false; break; }
        if (!mbar_wait(&full[slot], (i / stages) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = smem_addr(ring + slot * kTcStage), sq = smem_addr(qs);
#pragma unroll
        for (uint32_t kk = 0; kk < 8; ++kk)
          mma1_f16(tmem + b * kTcN, smem_desc(sa + (kk / 4) * kTcBox + 32 * (kk % 4), 16, 1024),
                   smem_desc(sq + (kk / 4) * kPAtom + 32 * (kk % 4), 16, 1024), kIdescS, kk ? 1u : 0u);
        mma1_commit(&empty[slot]);
        mma1_commit(&s_full[b]);
      }
      // pass 2: p . v
      if (ok && my) ok = mbar_wait(&p_ready, 0);
      tc_fence_after();
      for (uint32_t j = 0; ok && j < my; ++j, ++i) {
        const uint32_t slot = i % stages;
        if (!mbar_wait(&full[slot], (i / stages) & 1)) { ok = false; break; }
        if (owner && j + 1 == my) {
          // The last V stage has landed: the compute warps zero its rows
          // past the context before it is read (they learn of the landing
          // from this thread, which observes the ring's phases in order).
          mbar_arrive(&last_landed);
          if (!mbar_wait(&v_patched, 0)) { ok = false; break; }
        }
        tc_fence_after();
        const uint32_t sa = smem_addr(ring + slot * kTcStage), sp = smem_addr(ps) + j * 2 * kPAtom;
#pragma unroll
        for (uint32_t kk = 0; kk < 8; ++kk)
          mma1_f16(tmem + kTcSBufs * kTcN, smem_desc(sa + kk * 2048, kTcBox, 1024),
                   smem_desc(sp + (kk / 4) * kPAtom + 32 * (kk % 4), 16, 1024), kIdescO, (j | kk) ? 1u : 0u);
        mma1_commit(&empty[slot]);
      }
      if (ok && my) mma1_commit(&o_full);
      if (!ok) failed = 1;
      consumed_n = i;
      mma1_commit(&mma_done);
      if (!mbar_wait(&mma_done, 0)) failed = 1;
    }
  } else {
    // Compute warps 2-5: thread et; TMEM lane quarter (warp % 4).
    const uint32_t et = threadIdx.x - 64, quarter = warp & 3, cw = warp - 2;
    bool dead = false;
    // Padding rows G..15 of q are zero (those of P after the heads).
    for (uint32_t k = et; k < 2 * (kTcN - G) * 8; k += 128) {
      const uint32_t atom = k / ((kTcN - G) * 8), rem = k % ((kTcN - G) * 8);
      *reinterpret_cast<uint4 *>(qs + atom * kPAtom + (G + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
    }
    // This warp's heads (cw and cw + 4 of q 0..G-1, then k, v for the owner):
    // their norm weights and RoPE rows do not depend on the previous kernel.
    const uint32_t nheads = owner ? G + 2 : G;
    uint32_t hcol[2] = {0, 0};
    HeadConst hk[2];
#pragma unroll
    for (uint32_t t2 = 0; t2 < 2; ++t2) {
      const uint32_t k = cw + 4 * t2;
      if (HEADS && k < nheads) {
        hcol[t2] = k < G ? h * G + k : (k == G ? bd.QH + h : bd.QH + bd.KVH + h);
        hk[t2] = head_const(bd, bb, w, hcol[t2], pos_new);
      }
    }
    grid_dep_wait();
    if (threadIdx.x == 64) trace_mark(bd, bb, 1);
    // Head epilogues at the newest position: q into shared memory (both
    // CTAs), k and v into the caches (the owner; prefill: all from k_bheads).
    if (!HEADS)
      for (uint32_t k = et; k < G * kHD; k += 128) {
        const uint32_t g = k / kHD, d = k % kHD;
        *reinterpret_cast<uint16_t *>(qs + (d / 64) * kPAtom + swz(g, d % 64)) =
            reinterpret_cast<const uint16_t *>(bb.q)[(static_cast<size_t>(s) * bd.QH + h * G + g) * kHD + d];
      }
    float hraw[2][4];
#pragma unroll
    for (uint32_t t2 = 0; t2 < 2; ++t2)
      if (HEADS && cw + 4 * t2 < nheads) head_raw(bd, bb, s, hcol[t2], hraw[t2]);  // both heads' loads in flight
#pragma unroll
    for (uint32_t t2 = 0; t2 < 2; ++t2) {
      const uint32_t k = cw + 4 * t2;
      if (!HEADS || k >= nheads) continue;
      float out[4];
      head_math(bd, hcol[t2], hraw[t2], hk[t2], out);
      if (k < G) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t d = lane + 32 * j;
          *reinterpret_cast<uint16_t *>(qs + (d / 64) * kPAtom + swz(k, d % 64)) = float_to_bf16_bits(out[j]);
        }
      } else {
        bf16 *cache = (k == G ? w.kcache : w.vcache) + s * bb.kv_seq_stride +
                      (static_cast<size_t>(pos_new) * bd.KVH + h) * kHD;
#pragma unroll
        for (int j = 0; j < 4; ++j) putv(cache, lane + 32 * j, out[j]);
      }
    }
    // Shared writes -> tensor-core reads; global cache writes -> TMA reads.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&hd_ready);
    if (et == 0) trace_mark(bd, bb, 5);  // heads finished
    for (uint32_t k = et; k < 2 * my * (kTcN - G) * 8; k += 128) {
      const uint32_t atom = k / ((kTcN - G) * 8), rem = k % ((kTcN - G) * 8);
      *reinterpret_cast<uint4 *>(ps + atom * kPAtom + (G + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
    }
    // pass 1: scores of position p = 128 (st0 + i) + 32 quarter + lane
    float m[G];
#pragma unroll
    for (int g = 0; g < G; ++g) m[g] = -INFINITY;
    for (uint32_t i = 0; i < my; ++i) {
      const uint32_t b = i % kTcSBufs;
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&s_full[b], (i / kTcSBufs) & 1));
      float acc[16];
#pragma unroll
      for (int g = 0; g < 16; ++g) acc[g] = 0.f;
      if (!dead) {
        tc_fence_after();
        tmem_ld16(tmem + ((quarter * 32u) << 16) + b * kTcN, acc);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[b]);
      const uint32_t pl = i * kTcPos + quarter * 32 + lane, p = st0 * kTcPos + pl;
      if (p < n) {
        uint8_t *atom = ps + (pl / 64) * kPAtom;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float sv = round_bf16(__fmul_rn(round_bf16(acc[g]), kAttnScale));
          *reinterpret_cast<uint16_t *>(atom + swz(g, pl % 64)) = float_to_bf16_bits(sv);
          m[g] = fmaxf(m[g], sv);
        }
      }
    }
    // softmax statistics: this CTA's per head (quarters in order), then both
    // CTAs' through distributed shared memory (same values in both CTAs).
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float wm = warp_max(m[g]);
      if (lane == 0) red[quarter][g] = wm;
    }
    tc_sync();
    if (et < static_cast<uint32_t>(G)) {
      const float cm = fmaxf(fmaxf(red[0][et], red[1][et]), fmaxf(red[2][et], red[3][et]));
      xm[rank][et] = cm;
      st_cluster_f32(cluster_addr(&xm[rank][et], peer), cm);
      remote_arrive(cluster_addr(&x_max, peer));
    }
    if (!dead) dead = !__all_sync(kFullMask, mbar_wait_cluster(&x_max, 0));
    if (et < static_cast<uint32_t>(G)) sM[et] = fmaxf(xm[0][et], xm[1][et]);
    tc_sync();
    float l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) l[g] = 0.f;
    for (uint32_t pl = et; pl < my * kTcPos && st0 * kTcPos + pl < n; pl += 128) {
      const uint8_t *atom = ps + (pl / 64) * kPAtom;
#pragma unroll
      for (int g = 0; g < G; ++g)
        l[g] += expf(bf16_bits_to_float(*reinterpret_cast<const uint16_t *>(atom + swz(g, pl % 64))) - sM[g]);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ws = warp_sum(l[g]);
      if (lane == 0) red[quarter][g] = ws;
    }
    tc_sync();
    if (et < static_cast<uint32_t>(G)) {
      const float cl = ((red[0][et] + red[1][et]) + red[2][et]) + red[3][et];
      xl[rank][et] = cl;
      st_cluster_f32(cluster_addr(&xl[rank][et], peer), cl);
      remote_arrive(cluster_addr(&x_sum, peer));
    }
    if (!dead) dead = !__all_sync(kFullMask, mbar_wait_cluster(&x_sum, 0));
    if (et < static_cast<uint32_t>(G)) sInv[et] = 1.0f / (xl[0][et] + xl[1][et]);
    tc_sync();
    for (uint32_t pl = et; pl < my * kTcPos; pl += 128) {
      uint8_t *atom = ps + (pl / 64) * kPAtom;
      const bool valid = st0 * kTcPos + pl < n;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        uint16_t *e = reinterpret_cast<uint16_t *>(atom + swz(g, pl % 64));
        *e = valid ? float_to_bf16_bits(__fmul_rn(expf(bf16_bits_to_float(*e) - sM[g]), sInv[g])) : 0;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&p_ready);
    if (et == 0) trace_mark(bd, bb, 6);  // probabilities ready
    // The owner zeroes its last V stage's rows past the context once landed.
    if (owner) {
      const uint32_t slot = (2 * my - 1) % stages;
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait(&last_landed, 0));
      const uint32_t valid = n - (nst - 1) * kTcPos;
      if (!dead)
        for (uint32_t k = valid * 8 + et; k < kTcPos * 8; k += 128) {  // 16-byte pieces of rows valid..127
          const uint32_t row = k / 8, piece = k % 8;
          uint8_t *st = ring + slot * kTcStage;
          *reinterpret_cast<uint4 *>(st + row * 128 + piece * 16) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4 *>(st + kTcBox + row * 128 + piece * 16) = make_uint4(0, 0, 0, 0);
        }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&v_patched);
    }
    // output: dim d = 32 quarter + lane of the group's heads
    if (!dead && my) dead = !__all_sync(kFullMask, mbar_wait(&o_full, 0));
    if (et == 0) trace_mark(bd, bb, 7);  // output accumulated
    float o[16];
#pragma unroll
    for (int g = 0; g < 16; ++g) o[g] = 0.f;
    if (!dead && my) {
      tc_fence_after();
      tmem_ld16(tmem + ((quarter * 32u) << 16) + kTcSBufs * kTcN, o);
    }
    const uint32_t d = quarter * 32 + lane;
    if (rank == 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) st_cluster_f32(cluster_addr(&xo[g][d], 0), o[g]);
      remote_arrive(cluster_addr(&x_out, 0));
    } else {
      if (!dead) dead = !__all_sync(kFullMask, mbar_wait_cluster(&x_out, 0));
#pragma unroll
      for (int g = 0; g < G; ++g)
        putv(bb.attn, (static_cast<size_t>(s) * bd.QH + h * G + g) * kHD + d, o[g] + xo[g][d]);
    }
    if (dead) failed = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (failed) {
      const uint32_t from = consumed_n > issued_n ? issued_n : consumed_n;
      for (uint32_t i = from; i < issued_n; ++i)
        if (!mbar_wait(&full[i % stages], (i / stages) & 1)) break;
      atomicOr(bb.error, kErrPipelineTimeout);
    }
    trace_mark(bd, bb, 2);
  }
  cluster_sync();  // neither CTA leaves while the other may still address its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc1(tmem, kTcTmemCols);
  }
}

// --------------------------------------------------------------- argmax ----
// Per sequence: the lm tiles' candidates in tile order -> greedy token
// (lowest index on ties; 0xffffffff when any logit was NaN/Inf), then the
// state advances one position.
// ---------------------------------------------- tensor-parallel exchange
constexpr long long kBxWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

__device__ __forceinline__ unsigned long long bx_ld_acquire(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void bx_st_release(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void bx_st_relaxed(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// One thread: bounded wait until *flag(q) >= epoch for q < n (flags `stride`
// 64-bit words apart from base[q]); false on a timeout.
__device__ bool bx_wait(const unsigned long long *const *base, uint32_t offset, uint32_t n, unsigned long long epoch) {
  const long long start = clock64();
  for (uint32_t q = 0; q < n; ++q)
    while (bx_ld_acquire(base[q] + offset) < epoch) {
      if (clock64() - start > kBxWaitCycles) return false;
      __nanosleep(64);
    }
  return true;
}

// Tile blockIdx.x of H (128 rows, one thread each): once every rank's
// partial of exchange k is published, x = bf16(x + bf16(partials summed in
// rank order)) and the tile's sums of x^2 per sequence, as the residual
// epilogue leaves them.
// Launched with programmatic dependent launch: it lets the next GEMM start
// (and prefetch its weights) at once, and needs no wait on the partial GEMM
// before it - this rank's own flag is among those it waits for, and that
// flag is published only when the partial GEMM, and so everything before
// it, has completed.
__global__ void __launch_bounds__(kTileM) k_bxchg(BatchDims d, BatchBuffers b, uint32_t which, uint32_t k) {
  __shared__ int ok;
  __shared__ float part_ssq[4][kSeqN];
  const uint32_t t = blockIdx.x, r = threadIdx.x, row = t * kTileM + r, lane = r & 31, quarter = r >> 5;
  grid_dep_launch();
  if (r == 0) {
    ok = bx_wait(b.xflag, which, d.tp, *b.xepoch + k) ? 1 : 0;
    if (!ok) atomicOr(b.error, 4u);
  }
  __syncthreads();
  if (!ok) return;
  const size_t slot = static_cast<size_t>(which) * kMaxBatch * d.H + row;
  // Every sequence's value of one rank is requested before any is used (one
  // NVLink round trip per rank, not one per sequence), the ranks summed in
  // order, and only then is x read and written.
  float v[kSeqN], sq[kSeqN];
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) v[s] = s < d.batch ? __ldcg(b.xpart[0] + slot + s * d.H) : 0.f;
  for (uint32_t q = 1; q < d.tp; ++q) {
    float w[kSeqN];
#pragma unroll
    for (uint32_t s = 0; s < kSeqN; ++s) w[s] = s < d.batch ? __ldcg(b.xpart[q] + slot + s * d.H) : 0.f;
#pragma unroll
    for (uint32_t s = 0; s < kSeqN; ++s) v[s] = __fadd_rn(v[s], w[s]);
  }
  float xr[kSeqN];
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) xr[s] = s < d.batch ? bfv(b.x, static_cast<size_t>(s) * d.H + row) : 0.f;
#pragma unroll
  for (uint32_t s = 0; s < kSeqN; ++s) {
    sq[s] = 0.f;
    if (s < d.batch) {
      const float xn = round_bf16(__fadd_rn(xr[s], round_bf16(v[s])));
      putv(b.x, static_cast<size_t>(s) * d.H + row, xn);
      sq[s] = __fmul_rn(xn, xn);
    }
  }
  warp_transpose_sum<kSeqN>(sq, lane);  // lanes 2s, 2s + 1: the warp's sum for sequence s
  if ((lane & 1) == 0) part_ssq[quarter][lane / 2] = sq[0];
  __syncthreads();
  if (r < kSeqN)
    b.ssq[t * kSeqN + r] = ((part_ssq[0][r] + part_ssq[1][r]) + part_ssq[2][r]) + part_ssq[3][r];
}

// Sequence s's greedy candidate across the ranks' vocabulary shards: each
// rank writes its candidate into slot [rank][s] of every rank's region,
// then combines slot [q][s] of its own for every q (global indices, lowest
// on ties). One thread; false on a timeout.
__device__ bool bx_pick(const BatchDims &d, const BatchBuffers &b, uint32_t s, ArgBest &best, uint32_t &bad) {
  const unsigned long long epoch = *b.xepoch + 2ull * d.layers + 1;
  for (uint32_t q = 0; q < d.tp; ++q) {
    LmSlot *slot = b.xlm[q] + d.rank * kMaxBatch + s;
    slot->value = best.value;
    slot->index = best.index;
    slot->bad = bad;
  }
  __threadfence_system();
  for (uint32_t q = 0; q < d.tp; ++q) bx_st_relaxed(&(b.xlm[q] + d.rank * kMaxBatch + s)->epoch, epoch);
  const LmSlot *own = b.xlm[d.rank];
  const long long start = clock64();
  for (uint32_t q = 0; q < d.tp; ++q)
    while (bx_ld_acquire(&own[q * kMaxBatch + s].epoch) < epoch) {
      if (clock64() - start > kBxWaitCycles) return false;
      __nanosleep(64);
    }
  best = ArgBest{-INFINITY, 0xffffffffu};
  bad = 0;
  for (uint32_t q = 0; q < d.tp; ++q) {
    best = arg_better(best, ArgBest{__ldcg(&own[q * kMaxBatch + s].value), __ldcg(&own[q * kMaxBatch + s].index)});
    bad |= __ldcg(&own[q * kMaxBatch + s].bad);
  }
  return true;
}

// After the step's argmax: the step's exchanges are done.
__global__ void k_bepoch(BatchBuffers b, uint32_t exchanges) { *b.xepoch += exchanges; }

__global__ void __launch_bounds__(256) k_bargmax(BatchDims d, BatchBuffers b, uint32_t tiles) {
  __shared__ ArgBest wb[8];
  __shared__ uint32_t wbad[8];
  grid_dep_launch();
  if (threadIdx.x == 0) trace_mark(d, b, 0);
  grid_dep_wait();
  if (threadIdx.x == 0) trace_mark(d, b, 1);
  const uint32_t s = blockIdx.x, t = threadIdx.x;
  ArgBest best{-INFINITY, 0xffffffffu};
  uint32_t bad = 0;
  for (uint32_t i = t; i < tiles; i += 256) {
    best = arg_better(best, b.cand[static_cast<size_t>(s) * tiles + i]);
    bad |= b.cand_bad[static_cast<size_t>(s) * tiles + i];
  }
  best = warp_argbest(best);
  bad = __reduce_or_sync(kFullMask, bad);
  if ((t & 31) == 0) { wb[t >> 5] = best; wbad[t >> 5] = bad; }
  __syncthreads();
  if (t == 0) {
    ArgBest fb = wb[0];
    uint32_t fbad = wbad[0];
    for (int i = 1; i < 8; ++i) { fb = arg_better(fb, wb[i]); fbad |= wbad[i]; }
    if (d.tp > 1 && !bx_pick(d, b, s, fb, fbad)) atomicOr(b.error, 4u);
    const uint32_t next = (fbad || fb.index == 0xffffffffu) ? 0xffffffffu : fb.index;
    if (next == 0xffffffffu) atomicOr(b.error, 1u);
    SeqState &st = b.seq[s];
    const uint32_t pos = st.position;
    st.next = next;
    st.token = next;
    if (pos < d.max_seq) b.log[static_cast<size_t>(s) * d.max_seq + pos] = next;
    st.position = pos + 1;
    trace_mark(d, b, 2);
  }
}

// ------------------------------------------------------------- launches ----
uint32_t sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
      count = 148;
  }
  return static_cast<uint32_t>(count);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr size_t kGemmSmem = static_cast<size_t>(kRing) * kStageBytes + 1024;

// Y = X . W^T for W [rows][K] and X [16][K] (K a multiple of 64, both 16-byte
// aligned with 16-byte row pitches), with epilogue EPI.
// NORM: X is the raw residual, RMS-normalised with p.norm_w inside the GEMM.
template <int EPI, bool NORM = false>
cudaError_t launch_bgemm(const bf16 *W, uint32_t rows, uint32_t K, const bf16 *X, BGemm p, cudaStream_t s) {
  if (K % kKb) return cudaErrorInvalidValue;
  CUtensorMap mw, mx;
  cudaError_t e = make_tmap_2d_u16_swizzled(&mw, W, K, rows, K, kKb, kTileM);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_u16_swizzled(&mx, X, K, kSeqN, K, kKb, kSeqN);
  if (e != cudaSuccess) return e;
  p.rows = rows;
  p.nk = K / kKb;
  p.tiles = (rows + kTileM - 1) / kTileM;
  p.total = p.tiles * p.nk;
  const uint32_t grid = std::min(sm_count(), p.total);
  return launch_pdl(k_bgemm<EPI, NORM>, dim3(grid), dim3(kGemmThreads), kGemmSmem, s, mw, mx, p);
}

int smem_optin() {
  static int bytes = 0;
  if (bytes == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&bytes, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || bytes <= 0)
      bytes = 227 * 1024;
  }
  return bytes;
}

// Fused one-CTA-per-(head, sequence) attention when the group's scores for
// max_seq positions fit in shared memory next to the K/V ring and the cache
// spans at least one stage; otherwise the batch-1 chunked kernels
// (scores, then p.v with a last-CTA combine) per (chunk, head, sequence).
// Launch with a 2-CTA cluster and programmatic dependent launch.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_pair(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args... args) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Attention path: the tensor-core cluster kernel when half the stages' P
// and a ring of >= 2 stages fit in half an SM's shared memory (two clusters
// per SM) and the cache spans a stage; else the CUDA-core fused kernel
// (decode) or the batch-1 chunked kernels (scores, then p.v with a last-CTA
// combine) per (chunk, head, sequence).
template <int G>
cudaError_t launch_battention(const BatchDims &d, const BatchBuffers &b, const LayerWeights &w, cudaStream_t s,
                              bool prefill) {
  const uint64_t rows = prefill ? d.max_seq : static_cast<uint64_t>(d.batch) * d.max_seq;
  const uint64_t o_bytes = static_cast<uint64_t>(d.H) * d.QH * kHD * 2;
  const size_t half_sm = static_cast<size_t>(smem_optin()) / 2;
  uint32_t stages = kTcMaxStages;
  while (stages > 2 && tc_attn_smem_bytes(d.max_seq, stages) + 2048 > half_sm) --stages;
  const size_t tc_smem = tc_attn_smem_bytes(d.max_seq, stages);
  if (tc_smem + 2048 <= half_sm && rows >= kTcPos) {
    CUtensorMap mk, mv;
    cudaError_t e = make_tmap_2d_u16_swizzled(&mk, w.kcache, static_cast<uint64_t>(d.KVH) * kHD, rows,
                                              static_cast<uint64_t>(d.KVH) * kHD, 64, kTcPos);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u16_swizzled(&mv, w.vcache, static_cast<uint64_t>(d.KVH) * kHD, rows,
                                  static_cast<uint64_t>(d.KVH) * kHD, 64, kTcPos);
    if (e != cudaSuccess) return e;
    if (prefill) {
      e = launch_pdl(k_bheads, dim3(d.KVH, d.batch), dim3(256), 0, s, d, b, w);
      if (e != cudaSuccess) return e;
      return launch_pdl_pair(k_battn_tc<G, false>, dim3(2 * d.KVH, d.batch), dim3(kTcThreads), tc_smem, s, d, b, w,
                             mk, mv, reinterpret_cast<const uint8_t *>(w.wo), o_bytes, stages);
    }
    return launch_pdl_pair(k_battn_tc<G, true>, dim3(2 * d.KVH, d.batch), dim3(kTcThreads), tc_smem, s, d, b, w, mk,
                           mv, reinterpret_cast<const uint8_t *>(w.wo), o_bytes, stages);
  }
  const size_t smem = attn_smem_bytes(G, d.max_seq);
  if (!prefill && smem + 4096 <= static_cast<size_t>(smem_optin()) && rows >= kAttnPos) {
    CUtensorMap mk, mv;
    cudaError_t e = make_tmap_2d_u16(&mk, w.kcache, static_cast<uint64_t>(d.KVH) * kHD, rows,
                                     static_cast<uint64_t>(d.KVH) * kHD, kHD, kAttnPos);
    if (e != cudaSuccess) return e;
    e = make_tmap_2d_u16(&mv, w.vcache, static_cast<uint64_t>(d.KVH) * kHD, rows, static_cast<uint64_t>(d.KVH) * kHD,
                         kHD, kAttnPos);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_battn<G>, dim3(d.KVH, d.batch), dim3(kAttnThreads), smem, s, d, b, w, mk, mv,
                      reinterpret_cast<const uint8_t *>(w.wo),
                      static_cast<uint64_t>(d.H) * d.QH * kHD * 2);
  }
  cudaError_t e = launch_pdl(k_bheads, dim3(d.KVH, d.batch), dim3(256), 0, s, d, b, w);
  if (e != cudaSuccess) return e;
  const dim3 grid(d.nchunks, d.KVH, d.batch), block(kStreamThreads);
  e = launch_pdl(k_bscores<G>, grid, block, 0, s, d, b, w);
  return e != cudaSuccess ? e : launch_pdl(k_bpv<G>, grid, block, 0, s, d, b, w);
}

}  // namespace

uint32_t batch_gemm_grid() { return sm_count(); }

uint32_t batch_max_tiles(const BatchDims &d) {
  const uint32_t qkv = d.QH + 2 * d.KVH, o = (d.H + kTileM - 1) / kTileM, gu = (2 * d.I + kTileM - 1) / kTileM;
  return std::max({qkv, o, gu, batch_lm_tiles(d.vocab)});
}

cudaError_t record_batch_step(const BatchDims &d0, const BatchBuffers &b, const LayerWeights *layers,
                              uint32_t n_layers, cudaStream_t s, bool prefill) {
  if (d0.batch < 1 || d0.batch > kMaxBatch) return cudaErrorInvalidValue;
  BatchDims d = d0;
  uint32_t slot = 0;
  // Each launch gets the next trace slot.
  auto at = [&](BGemm g) {
    d.trace_slot = slot++;
    g.d = d;
    g.b = b;
    return g;
  };
  auto next = [&]() {
    d.trace_slot = slot++;
    return d;
  };
  const uint32_t G = d.QH / d.KVH;
  if (d.tp > 1 && (prefill || d.H % kTileM)) return cudaErrorInvalidValue;
  // Tensor parallel o_proj / down: the partial GEMM into this rank's region
  // (its last CTA publishes the epoch), then every rank's partials applied to x.
  auto exchange = [&](uint32_t which, uint32_t k, const bf16 *W, uint32_t K, const bf16 *X) -> cudaError_t {
    BGemm pp{};
    pp.part = b.xpart[d.rank] + static_cast<size_t>(which) * kMaxBatch * d.H;
    pp.xwhich = which;
    pp.xk = k;
    const cudaError_t e = launch_bgemm<kEpiPart>(W, d.H, K, X, at(pp), s);
    if (e != cudaSuccess) return e;
    return launch_pdl(k_bxchg, dim3(d.H / kTileM), dim3(kTileM), 0, s, next(), b, which, k);
  };
#define XPU_TRY(expr)                        \
  do {                                       \
    const cudaError_t e_ = (expr);           \
    if (e_ != cudaSuccess) return e_;        \
  } while (0)
  XPU_TRY(launch_pdl(k_bnorm, dim3(d.batch), dim3(256), 0, s, next(), b, layers[0].in_norm, 1));
  for (uint32_t l = 0; l < n_layers; ++l) {
    const LayerWeights &w = layers[l];
    BGemm pq{};
    pq.out = b.qkv;
    pq.norm_w = w.in_norm;
    if (l == 0)  // the embedding kernel normalised layer 0's input
      XPU_TRY(launch_bgemm<kEpiQkv>(w.wqkv, (d.QH + 2 * d.KVH) * kHD, d.H, b.xn, at(pq), s));
    else
      XPU_TRY((launch_bgemm<kEpiQkv, true>(w.wqkv, (d.QH + 2 * d.KVH) * kHD, d.H, b.x, at(pq), s)));
    const BatchDims da = next();
    switch (G) {
      case 1: XPU_TRY(launch_battention<1>(da, b, w, s, prefill)); break;
      case 2: XPU_TRY(launch_battention<2>(da, b, w, s, prefill)); break;
      case 4: XPU_TRY(launch_battention<4>(da, b, w, s, prefill)); break;
      case 8: XPU_TRY(launch_battention<8>(da, b, w, s, prefill)); break;
      default: return cudaErrorInvalidValue;
    }
    BGemm po{};
    po.out = b.x;
    if (d.tp > 1)
      XPU_TRY(exchange(0, 2 * l + 1, w.wo, d.QH * kHD, b.attn));
    else
      XPU_TRY(launch_bgemm<kEpiResid>(w.wo, d.H, d.QH * kHD, b.attn, at(po), s));
    BGemm pg{};
    pg.out = b.h;
    pg.norm_w = w.post_norm;
    XPU_TRY((launch_bgemm<kEpiGateUp, true>(w.wgu, 2 * d.I, d.H, b.x, at(pg), s)));
    BGemm pd{};
    pd.out = b.x;
    if (d.tp > 1)
      XPU_TRY(exchange(1, 2 * l + 2, w.wd, d.I, b.h));
    else
      XPU_TRY(launch_bgemm<kEpiResid>(w.wd, d.H, d.I, b.h, at(pd), s));
  }
  BGemm pl{};
  pl.norm_w = b.final_norm;
  XPU_TRY((launch_bgemm<kEpiLm, true>(b.lm_head, d.vocab, d.H, b.x, at(pl), s)));
  XPU_TRY(launch_pdl(k_bargmax, dim3(d.batch), dim3(256), 0, s, next(), b, batch_lm_tiles(d.vocab)));
  if (d.tp > 1) {
    next();
    k_bepoch<<<1, 1, 0, s>>>(b, 2 * n_layers + 1);
    XPU_TRY(cudaGetLastError());
  }
#undef XPU_TRY
  return cudaSuccess;
}

}  // namespace xpu
