// Device-side building blocks of the Qwen3 decode step, shared by the
// multi-kernel CUDA-graph path (decode_kernels.cu) and the persistent
// single-kernel path (decode_step.cu), so that both compute bit-identical
// results.
//
// Thread conventions: a CTA is the producer warp (warp 0, see stream.cuh)
// plus kConsumerWarps consumer warps; everything here runs on the consumer
// warps (ctid() = threadIdx.x - 32) and synchronises with consumer_sync().
// Data written by other CTAs during the same step (activations, partial
// sums, the new KV-cache row) is read through L2 with ld.global.cg.
#pragma once

#include "decode.cuh"
#include "stream.cuh"

namespace xpu {
namespace dec {

__device__ __forceinline__ uint32_t ctid() { return threadIdx.x - 32; }
__device__ __forceinline__ uint32_t cwarp() { return (threadIdx.x >> 5) - 1; }
__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ uint4 ldcg16(const void *p) { return __ldcg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ uint2 ldcg8(const void *p) { return __ldcg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ float bfcg(const bf16 *p, size_t i) {
  return bf16_bits_to_float(__ldcg(reinterpret_cast<const unsigned short *>(p) + i));
}
// Constant-per-step data (norm weights, RoPE tables).
__device__ __forceinline__ float bf(const bf16 *p, size_t i) {
  return bf16_bits_to_float(reinterpret_cast<const uint16_t *>(p)[i]);
}
__device__ __forceinline__ void put(bf16 *p, size_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = float_to_bf16_bits(v);
}

__device__ __forceinline__ float sq8(const uint4 &v, float ss) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = bf16_lo(w[j]), b = bf16_hi(w[j]);
    ss = __fadd_rn(ss, __fmul_rn(a, a));
    ss = __fadd_rn(ss, __fmul_rn(b, b));
  }
  return ss;
}

// transformers Qwen3RMSNorm into shared memory:
// xs = bf16(w * bf16(x * RN(1/RN(sqrt(mean(x^2) + eps))))), over [0, H).
// x is read from L2 once into xs; the sum of squares and the normalisation
// then work on the shared copy.
__device__ inline void stage_rms(const bf16 *x, const bf16 *w, uint32_t H, float eps, uint4 *xs, float *scratch) {
  const uint32_t t = ctid();
  float ss = 0.f;
  for (uint32_t c = t; c < H / 8; c += kConsumerThreads) {
    const uint4 v = ldcg16(x + 8 * c);
    xs[c] = v;
    ss = sq8(v, ss);
  }
  ss = consumer_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
  const uint4 *w4 = reinterpret_cast<const uint4 *>(w);
  for (uint32_t c = t; c < H / 8; c += kConsumerThreads) {
    const uint4 xv = xs[c], wv = w4[c];
    const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = round_bf16(__fmul_rn(bf16_lo(wa[j]), round_bf16(__fmul_rn(bf16_lo(xa[j]), r))));
      const float hi = round_bf16(__fmul_rn(bf16_hi(wa[j]), round_bf16(__fmul_rn(bf16_hi(xa[j]), r))));
      o[j] = pack_bf16x2(lo, hi);
    }
    xs[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  consumer_sync();
}

__device__ inline void stage_copy(const bf16 *x, uint32_t n, uint4 *xs) {
  for (uint32_t c = ctid(); c < n / 8; c += kConsumerThreads) xs[c] = ldcg16(x + 8 * c);
  consumer_sync();
}

// Deferred arrivals of this CTA's items (blockIdx.x + j * gridDim.x, j < mine)
// on counters[item / per_counter]; s_last[j] = this CTA completed the counter.
constexpr uint32_t kMaxLocalItems = 64;

__device__ inline uint32_t arrive_items(unsigned *counters, uint32_t items, uint32_t per_counter, unsigned total,
                                        uint8_t *s_last) {
  const uint32_t mine = items > blockIdx.x ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const uint32_t n = mine < kMaxLocalItems ? mine : kMaxLocalItems;
  // The consumer barrier orders every consumer's stores before the arriving
  // threads, whose fences (release before, acquire after the atomic) are
  // cumulative over them; the second barrier hands the acquire to everyone.
  consumer_sync();
  for (uint32_t j = ctid(); j < n; j += kConsumerThreads) {
    const uint32_t item = blockIdx.x + j * gridDim.x;
    __threadfence();
    s_last[j] = atomicAdd(counters + item / per_counter, 1u) == total - 1u;
    __threadfence();
  }
  consumer_sync();
  return n;
}

// Whole-CTA (consumer warps) publish-then-count on one counter.
__device__ inline bool arrive_one(unsigned *counter, unsigned total, int *flag) {
  consumer_sync();  // as arrive_items: one arriving thread fences for the CTA
  if (ctid() == 0) {
    __threadfence();
    *flag = (atomicAdd(counter, 1u) == total - 1u);
    __threadfence();
  }
  consumer_sync();
  return *flag != 0;
}

__device__ __forceinline__ void flag_error(DecodeState *st, uint32_t bits) { atomicOr(&st->error, bits); }

// Cross-GPU exchange flags: published with relaxed system-scope stores after
// one system-scope fence, polled with relaxed system-scope loads and followed
// by one acquire fence (a release/acquire pattern per flag without a fence in
// every store and every poll).
__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// ------------------------------------------------------------------ QKV ----
// Items: (tile, split) of [Wq; Wk; Wv]; partial sums to part_qkv[split][row].
__device__ inline bool qkv_items(const DecodeDims &d, const DecodeBuffers &b, const StreamSmem &sm,
                                 const StreamGeom &g, uint32_t &it) {
  const uint32_t lane = lane_id(), cw = cwarp();
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    const uint32_t tile = item / g.kparts, part = item % g.kparts;
    float acc[kRowsPerWarp];
    if (!stream_consume_item<bf16>(sm, g, sm.xs + part * (g.kt / 8), it, acc)) return false;
    const uint32_t row = tile * kStageRows + kRowsPerWarp * cw;
    if (lane == 0)
#pragma unroll
      for (uint32_t r = 0; r < kRowsPerWarp; ++r) b.part_qkv[static_cast<size_t>(part) * g.rows + row + r] = acc[r];
  }
  return true;
}

// Finish head `head` of the QKV output with one warp (lane l owns dimensions
// l, l+32, l+64, l+96, so both rotate-half pairs sit in one lane): sum the
// splits, then q/k RMSNorm + RoPE (transformers rounding) into the q buffer /
// key cache, or v into the value cache, at `pos`.
constexpr uint32_t kMaxQkvSplits = 4;  // split partials held in registers by the head epilogue

__device__ inline void qkv_head_warp(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                                     uint32_t head, uint32_t pos, bf16 *q_dst = nullptr) {
  const uint32_t lane = lane_id();
  const uint32_t rows_total = (d.QH_l + 2 * d.KVH_l) * kHD;
  const bool is_v = head >= d.QH_l + d.KVH_l, is_q = head < d.QH_l;
  // Every input of the epilogue is loaded before any is used (one memory
  // round trip): the split partials, and for q/k the norm weight and the
  // RoPE table entries of this lane's four dimensions l + 32 j.
  float part[kMaxQkvSplits][4];
  const uint32_t splits = d.qkv_splits < kMaxQkvSplits ? d.qkv_splits : kMaxQkvSplits;
#pragma unroll
  for (uint32_t s = 0; s < kMaxQkvSplits; ++s)
    if (s < splits)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        part[s][j] = __ldcg(b.part_qkv + static_cast<size_t>(s) * rows_total + head * kHD + lane + 32 * j);
  float nwv[4] = {0.f, 0.f, 0.f, 0.f}, cv[4] = {0.f, 0.f, 0.f, 0.f}, sv[4] = {0.f, 0.f, 0.f, 0.f};
  if (!is_v) {
    const bf16 *nw = is_q ? w.q_norm : w.k_norm;
    const bf16 *cr = b.cos_t + static_cast<size_t>(pos) * kHD, *sr = b.sin_t + static_cast<size_t>(pos) * kHD;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      nwv[j] = bf(nw, lane + 32 * j);
      cv[j] = bf(cr, lane + 32 * j);
      sv[j] = bf(sr, lane + 32 * j);
    }
  }
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float y = 0.f;
#pragma unroll
    for (uint32_t s = 0; s < kMaxQkvSplits; ++s)
      if (s < splits) y += part[s][j];
    for (uint32_t s = kMaxQkvSplits; s < d.qkv_splits; ++s)
      y += __ldcg(b.part_qkv + static_cast<size_t>(s) * rows_total + head * kHD + lane + 32 * j);
    v[j] = round_bf16(y);
  }
  if (is_v) {  // value head: straight into the cache
    const size_t slot = (static_cast<size_t>(pos) * d.KVH_l + (head - d.QH_l - d.KVH_l)) * kHD;
#pragma unroll
    for (int j = 0; j < 4; ++j) put(w.vcache, slot + lane + 32 * j, v[j]);
    return;
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(kHD) + d.eps);
  float nv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) nv[j] = round_bf16(__fmul_rn(nwv[j], round_bf16(__fmul_rn(v[j], r))));
  float out[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {  // pairs (i, i + 64): rotate_half
    const float a = nv[j], c = nv[j + 2];
    out[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(a, cv[j])), round_bf16(__fmul_rn(-c, sv[j]))));
    out[j + 2] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(c, cv[j + 2])), round_bf16(__fmul_rn(a, sv[j + 2]))));
  }
  bf16 *dst = is_q ? (q_dst ? q_dst : b.q + static_cast<size_t>(head) * kHD)
                   : w.kcache + (static_cast<size_t>(pos) * d.KVH_l + (head - d.QH_l)) * kHD;
#pragma unroll
  for (int j = 0; j < 4; ++j) put(dst, lane + 32 * j, out[j]);
}

// Deferred arrivals of this CTA's QKV items; every head it completed is
// Persistent step: the head epilogues of one attention item's kv group, run
// by the item's CTA itself (so no separate finishing phase): the group's q
// heads, and for the item holding the newest position also its k and v
// heads (into the cache at pos). Every CTA of the group computes the same q
// bits, so their duplicate stores to b.q are harmless. With q_shared the q
// heads go to shared memory ([G][128]) instead, for this CTA alone.
__device__ inline void attn_group_heads(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                                        uint32_t kvh, bool newest, uint32_t pos, bf16 *q_shared = nullptr) {
  const uint32_t G = d.QH_l / d.KVH_l, n = G + (newest ? 2 : 0);
  for (uint32_t h = cwarp(); h < n; h += kConsumerWarps) {
    const uint32_t head = h < G ? kvh * G + h : (h == G ? d.QH_l + kvh : d.QH_l + d.KVH_l + kvh);
    qkv_head_warp(d, b, w, head, pos, q_shared && h < G ? q_shared + h * kHD : nullptr);
  }
  consumer_sync();
}

// finished by one warp (heads spread over the 8 consumer warps).
__device__ inline void qkv_finish(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                                  const StreamGeom &g, uint32_t pos, uint8_t *s_last) {
  const uint32_t per_head = g.kparts * (kHD / kStageRows);
  const uint32_t n = arrive_items(b.cnt_qkv, g.items(), per_head, per_head, s_last);
  uint32_t k = 0;
  for (uint32_t j = 0; j < n; ++j) {
    if (!s_last[j]) continue;
    if (k++ % kConsumerWarps != cwarp()) continue;
    const uint32_t head = (blockIdx.x + j * gridDim.x) / per_head;
    qkv_head_warp(d, b, w, head, pos);
    if (lane_id() == 0) b.cnt_qkv[head] = 0;
  }
  consumer_sync();
}

// ---------------------------------------------------- row-parallel (o, down) ----
// Items: (tile, local chunk j) of W [H][K_l]; partials to part[chunk0 + j][row].
__device__ inline bool rowpar_items(const DecodeDims &d, const DecodeBuffers &b, const StreamSmem &sm,
                                    const StreamGeom &g, uint32_t &it) {
  const uint32_t lane = lane_id(), cw = cwarp();
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    const uint32_t tile = item / g.kparts, part = item % g.kparts, chunk = d.chunk0 + part;
    float acc[kRowsPerWarp];
    if (!stream_consume_item<bf16>(sm, g, sm.xs + part * (g.kt / 8), it, acc)) return false;
    const uint32_t row = tile * kStageRows + kRowsPerWarp * cw;
    if (lane == 0)
#pragma unroll
      for (uint32_t r = 0; r < kRowsPerWarp; ++r) b.part[static_cast<size_t>(chunk) * d.H + row + r] = acc[r];
  }
  return true;
}

// Tensor-parallel variant: this rank's canonical-chunk partials go to every
// rank's exchange region (slot `which`: 0 o_proj, 1 down), each value as a
// 64-bit word (epoch << 32 | FP32 bits) so that it carries its own
// readiness; lane q of a warp writes the warp's 4 rows to rank q. The
// residual is applied by stage_residual_rms once all words have arrived.
__device__ __forceinline__ void st_relaxed_sys_v2(unsigned long long *p, unsigned long long a, unsigned long long b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ unsigned long long tagged(float v, uint32_t epoch) {
  return (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
}

__device__ inline bool rowpar_items_tp(const DecodeDims &d, const DecodeBuffers &b, const StreamSmem &sm,
                                       const StreamGeom &g, uint32_t &it, uint32_t which, uint32_t epoch) {
  const uint32_t lane = lane_id(), cw = cwarp();
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    const uint32_t tile = item / g.kparts, part = item % g.kparts, chunk = d.chunk0 + part;
    float acc[kRowsPerWarp];
    if (!stream_consume_item<bf16>(sm, g, sm.xs + part * (g.kt / 8), it, acc)) return false;
    const uint32_t row = tile * kStageRows + kRowsPerWarp * cw;
    if (lane < d.tp_size) {
      unsigned long long *dst = b.tp.part[lane] + (static_cast<size_t>(which) * kCanonChunks + chunk) * d.H + row;
      st_relaxed_sys_v2(dst, tagged(acc[0], epoch), tagged(acc[1], epoch));
      st_relaxed_sys_v2(dst + 2, tagged(acc[2], epoch), tagged(acc[3], epoch));
    }
  }
  return true;
}

__device__ __forceinline__ void ld_relaxed_sys_v2(const unsigned long long *p, unsigned long long &a,
                                                  unsigned long long &b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Waits (bounded) until chunks [k0, k0 + 4) of rows [8c, 8c + 8) in exchange
// slot `slot` carry `epoch` (all 32 words requested before the first
// check), and adds them to y in chunk order. False on a timeout (error bit
// 4 set) or when another waiter failed.
__device__ __forceinline__ bool take_chunks(const DecodeBuffers &b, const unsigned long long *slot, uint32_t H,
                                            uint32_t c, uint32_t k0, uint32_t epoch, float (&y)[8]) {
  unsigned long long v[4][8];
  const long long start = clock64();
  while (true) {
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k)
#pragma unroll
      for (uint32_t j = 0; j < 8; j += 2)
        ld_relaxed_sys_v2(slot + static_cast<size_t>(k0 + k) * H + 8 * c + j, v[k][j], v[k][j + 1]);
    bool ready = true;
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k)
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j) ready &= static_cast<uint32_t>(v[k][j] >> 32) == epoch;
    if (ready) break;
    if (*reinterpret_cast<volatile uint32_t *>(&b.state->error) & kErrPipelineTimeout) return false;
    if (clock64() - start > kWaitCycles) {
      flag_error(b.state, kErrPipelineTimeout);
      return false;
    }
  }
#pragma unroll
  for (uint32_t k = 0; k < 4; ++k)
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) y[j] = __fadd_rn(y[j], __uint_as_float(static_cast<uint32_t>(v[k][j])));
  return true;
}

// Tensor parallel, after a row-parallel exchange: as every rank's words of
// exchange `epoch` arrive, x_new = bf16(x_old + bf16(sum of the 8 canonical
// chunks of slot `which`, in chunk order)) - the arithmetic of the
// single-GPU residual epilogue (rowpar_finish) - staged into xs and
// RMS-normalised with w exactly as stage_rms does; CTA 0 also stores x_new
// to x_out for the next residual. Every CTA reads every word itself: a
// second, local round (one CTA per row range publishing its sums) measured
// slower, since it queues a dependent round trip behind the NVLink arrival.
// False (in every thread of the CTA) on a timeout.
__device__ inline bool stage_residual_rms(const DecodeDims &d, const DecodeBuffers &b, uint32_t which, uint32_t epoch,
                                          const bf16 *x_old, bf16 *x_out, const bf16 *w, uint4 *xs, float *scratch,
                                          int *s_fail) {
  const uint32_t t = ctid(), lane = lane_id(), cw = cwarp(), H = d.H;
  const unsigned long long *slot = b.tp.part[d.tp_rank] + static_cast<size_t>(which) * kCanonChunks * H;
  float ss = 0.f;
  bool ok = true;  // after a timeout this thread stops waiting but still joins every barrier
  for (uint32_t c = t; c < H / 8; c += kConsumerThreads) {
    const uint4 xv = ldcg16(x_old + 8 * c);
    float y[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    ok = ok && take_chunks(b, slot, H, c, 0, epoch, y) && take_chunks(b, slot, H, c, 4, epoch, y);
    const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2(__fadd_rn(bf16_lo(xa[j]), round_bf16(y[2 * j])), __fadd_rn(bf16_hi(xa[j]), round_bf16(y[2 * j + 1])));
    const uint4 nv = make_uint4(o[0], o[1], o[2], o[3]);
    xs[c] = nv;
    if (blockIdx.x == 0) reinterpret_cast<uint4 *>(x_out)[c] = nv;
    ss = sq8(nv, ss);
  }
  // consumer_sum's tree, with every warp's "gave up" carried along, so the
  // CTA agrees on failure without another memory round trip
  ss = warp_sum(ss);
  const bool bad = __any_sync(kFullMask, !ok);
  consumer_sync();
  if (lane == 0) {
    scratch[cw] = ss;
    s_fail[cw] = bad;
  }
  consumer_sync();
  ss = 0.f;
  int failed = 0;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) {
    ss += scratch[i];
    failed |= s_fail[i];
  }
  const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + d.eps);
  const uint4 *w4 = reinterpret_cast<const uint4 *>(w);
  for (uint32_t c = t; c < H / 8; c += kConsumerThreads) {
    const uint4 xv = xs[c], wv = w4[c];
    const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = round_bf16(__fmul_rn(bf16_lo(wa[j]), round_bf16(__fmul_rn(bf16_lo(xa[j]), r))));
      const float hi = round_bf16(__fmul_rn(bf16_hi(wa[j]), round_bf16(__fmul_rn(bf16_hi(xa[j]), r))));
      o[j] = pack_bf16x2(lo, hi);
    }
    xs[c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  consumer_sync();
  return !failed;
}

// Residual epilogue of every row tile this CTA completed:
// x = bf16(x + bf16(sum of the 8 canonical chunks, in chunk order)).
__device__ inline void rowpar_finish(const DecodeDims &d, const DecodeBuffers &b, const StreamGeom &g,
                                     uint8_t *s_last) {
  const uint32_t n = arrive_items(b.cnt_tile, g.items(), g.kparts, g.kparts, s_last);
  const uint32_t t = ctid();
  for (uint32_t j0 = 0; j0 < n; j0 += kConsumerThreads / kStageRows) {
    const uint32_t j = j0 + t / kStageRows;
    if (j < n && s_last[j]) {
      const uint32_t tile = (blockIdx.x + j * gridDim.x) / g.kparts;
      const uint32_t r = tile * kStageRows + t % kStageRows;
      float v[kCanonChunks];  // every chunk's partial in flight before the in-order sum
#pragma unroll
      for (uint32_t c = 0; c < kCanonChunks; ++c) v[c] = __ldcg(b.part + static_cast<size_t>(c) * d.H + r);
      const float xr = bfcg(b.x, r);
      float y = 0.f;
#pragma unroll
      for (uint32_t c = 0; c < kCanonChunks; ++c) y += v[c];
      put(b.x, r, __fadd_rn(xr, round_bf16(y)));
      if (t % kStageRows == 0) b.cnt_tile[tile] = 0;
    }
  }
  consumer_sync();
}

// ------------------------------------------------------------- gate / up ----
// Rows 2i, 2i+1 of Wgu are gate and up of unit i; warp cw of tile t holds
// units i = 16t + 2cw and 16t + 2cw + 1: h = bf16(bf16(silu(bf16 g)) * bf16 u).
__device__ inline bool gateup_items(const DecodeDims &d, const DecodeBuffers &b, const StreamSmem &sm,
                                    const StreamGeom &g, uint32_t &it) {
  const uint32_t lane = lane_id(), cw = cwarp();
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    float acc[kRowsPerWarp];
    if (!stream_consume_item<bf16>(sm, g, sm.xs, it, acc)) return false;
    if (lane == 0)
#pragma unroll
      for (uint32_t u = 0; u < kRowsPerWarp / 2; ++u) {
        const uint32_t i = item * (kStageRows / 2) + (kRowsPerWarp / 2) * cw + u;
        if (i >= d.I_l) break;
        const float gv = round_bf16(acc[2 * u]), uv = round_bf16(acc[2 * u + 1]);
        const float act = round_bf16(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))));
        put(b.h, i, __fmul_rn(act, uv));
      }
  }
  consumer_sync();
  return true;
}

// --------------------------------------------------------------- lm_head ----
struct LmShared {
  ArgBest wbest[kConsumerWarps];
  uint32_t wbad[kConsumerWarps];
  int flag;
};

// Logits of this CTA's rows, then the CTA's (max, lowest index) candidate;
// the last CTA reduces all candidates (fixed order) into the greedy token
// and advances the step state. Returns false on a timeout.
__device__ inline bool lm_items_and_argmax(const DecodeDims &d, const DecodeBuffers &b, const StreamSmem &sm,
                                           const StreamGeom &g, uint32_t &it, LmShared &ls, uint32_t pos,
                                           uint64_t bar_advance, uint64_t lm_epoch = 0, uint64_t x_advance = 0) {
  const uint32_t lane = lane_id(), cw = cwarp(), t = ctid();
  ArgBest best{-INFINITY, 0xffffffffu};
  uint32_t bad = 0;
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    float acc[kRowsPerWarp];
    if (!stream_consume_item<bf16>(sm, g, sm.xs, it, acc)) return false;
    if (lane == 0) {
#pragma unroll
      for (uint32_t rr = 0; rr < kRowsPerWarp; ++rr) {
        const uint32_t row = item * kStageRows + kRowsPerWarp * cw + rr;
        if (row >= d.V_l) break;
        const float v = round_bf16(acc[rr]);
        b.logits[row] = float_to_bf16_bits(v);
        bad |= not_finite(v) ? 1u : 0u;
        best = arg_better(best, ArgBest{v, d.v_offset + row});
      }
    }
  }
  if (lane == 0) { ls.wbest[cw] = best; ls.wbad[cw] = bad; }
  consumer_sync();
  if (t == 0) {
    ArgBest cb = ls.wbest[0];
    uint32_t cbad = ls.wbad[0];
    for (int i = 1; i < kConsumerWarps; ++i) { cb = arg_better(cb, ls.wbest[i]); cbad |= ls.wbad[i]; }
    b.lm_best[blockIdx.x] = cb;
    b.lm_bad[blockIdx.x] = cbad;
  }
  if (arrive_one(b.cnt_lm, gridDim.x, &ls.flag)) {
    ArgBest tb{-INFINITY, 0xffffffffu};
    uint32_t tbad = 0;
    for (uint32_t i = t; i < gridDim.x; i += kConsumerThreads) {
      ArgBest e;
      e.value = __ldcg(&b.lm_best[i].value);
      e.index = __ldcg(&b.lm_best[i].index);
      tb = arg_better(tb, e);
      tbad |= __ldcg(b.lm_bad + i);
    }
    tb = warp_argbest(tb);
    tbad = __reduce_or_sync(kFullMask, tbad);
    consumer_sync();
    if (lane == 0) { ls.wbest[cw] = tb; ls.wbad[cw] = tbad; }
    consumer_sync();
    if (t == 0) {
      ArgBest fb = ls.wbest[0];
      uint32_t fbad = ls.wbad[0];
      for (int i = 1; i < kConsumerWarps; ++i) { fb = arg_better(fb, ls.wbest[i]); fbad |= ls.wbad[i]; }
      DecodeState *st = b.state;
      if (d.tp_size > 1) {
        // Publish this rank's candidate to every rank, then combine all
        // ranks' candidates (global indices; lowest index on ties).
        for (uint32_t q = 0; q < d.tp_size; ++q) {
          LmSlot *slot = b.tp.lm[q] + d.tp_rank;
          slot->value = fb.value;
          slot->index = fb.index;
          slot->bad = fbad;
        }
        __threadfence_system();
        for (uint32_t q = 0; q < d.tp_size; ++q) st_relaxed_sys(&(b.tp.lm[q] + d.tp_rank)->epoch, lm_epoch);
        const LmSlot *own = b.tp.lm[d.tp_rank];
        bool ok = true;
        const long long start = clock64();
        for (uint32_t q = 0; ok && q < d.tp_size; ++q)
          while (ld_relaxed_sys(&own[q].epoch) < lm_epoch) {
            if (clock64() - start > kWaitCycles) { ok = false; break; }
          }
        fence_acq_rel_sys();
        if (!ok) {
          flag_error(st, kErrPipelineTimeout);
        } else {
          fb = ArgBest{-INFINITY, 0xffffffffu};
          fbad = 0;
          for (uint32_t q = 0; q < d.tp_size; ++q) {
            const ArgBest e{__ldcg(&own[q].value), __ldcg(&own[q].index)};
            fb = arg_better(fb, e);
            fbad |= __ldcg(&own[q].bad);
          }
        }
      }
      st->x_base += x_advance;
      const uint32_t next = (fbad || fb.index == 0xffffffffu) ? 0xffffffffu : fb.index;
      if (next == 0xffffffffu) st->error |= 1u;
      st->next = next;
      st->token = next;
      if (pos < d.max_seq) b.log[pos] = next;
      st->bar_base += bar_advance;
      st->steps += 1;
      __threadfence();
      st->position = pos + 1;
      *b.cnt_lm = 0;
    }
  }
  return true;
}

// ------------------------------------------------------------- attention ----
// Item (kv head, 128-position chunk): 8 consumer warps x 16 positions; each
// warp issues its 16 cache-row loads before using any.
constexpr uint32_t kPosPerWarp = kPosChunk / kConsumerWarps;  // 16

template <int G>
struct AttnShared {
  float sc[G][kPosChunk];
  float sM[G], sInv[G];
  float sacc[kConsumerWarps][G][kHD];
  int flag;
};

// This warp's 16 cache rows of the chunk (one 8-byte slice per lane), zero
// past the context; the row at position `skip` is left out (its head
// epilogue has not written it yet) and loaded by reload_row afterwards.
__device__ __forceinline__ void load_rows(const bf16 *cache, const DecodeDims &d, uint32_t kvh, uint32_t pw,
                                          uint32_t p1, uint32_t skip, uint2 (&r)[kPosPerWarp]) {
  const uint32_t lane = lane_id();
#pragma unroll
  for (uint32_t i = 0; i < kPosPerWarp; ++i) {
    const uint32_t p = pw + i;
    r[i] = p < p1 && p != skip ? ldcg8(cache + (static_cast<size_t>(p) * d.KVH_l + kvh) * kHD + lane * 4)
                               : make_uint2(0, 0);
  }
}

__device__ __forceinline__ void reload_row(const bf16 *cache, const DecodeDims &d, uint32_t kvh, uint32_t pw,
                                           uint32_t p, uint2 (&r)[kPosPerWarp]) {
  if (p >= pw && p < pw + kPosPerWarp)
#pragma unroll
    for (uint32_t i = 0; i < kPosPerWarp; ++i)
      if (pw + i == p) r[i] = ldcg8(cache + (static_cast<size_t>(p) * d.KVH_l + kvh) * kHD + lane_id() * 4);
}

// Warp sums of N (16 or 32) per-lane values at once, by recursive halving:
// at offset o (16, 8, 4, 2, 1) each lane keeps half of its values, adds the
// partner lane's (lane ^ o) copies of them, and hands over the other half;
// once one value is left the remaining offsets add like warp_sum. Every total
// is thus warp_sum's addition tree over the same lane pairs (bit-identical)
// at N - 1 shuffles instead of 5 N. Returns the total of value `lane` (N =
// 32) or `lane >> 1` (N = 16).
template <int N>
__device__ __forceinline__ float warp_sum_transposed(float (&v)[N]) {
  static_assert(N == 16 || N == 32, "16 or 32 values per lane");
  const uint32_t lane = lane_id();
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int o = 16 >> step, n = N >> step;
    if (n >= 2) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int k = 0; k < n / 2; ++k) {
        const float send = up ? v[k] : v[k + n / 2];
        const float keep = up ? v[k + n / 2] : v[k];
        v[k] = keep + __shfl_xor_sync(kFullMask, send, o);
      }
    } else {
      v[0] += __shfl_xor_sync(kFullMask, v[0], o);
    }
  }
  return v[0];
}

// s = bf16(bf16(q.k) * scale) for the chunk's positions into sc (and
// b.scores when store_scores); chunk max and sum of exp(s - max) into stats.
// q comes from q_shared ([G][128], this CTA's head epilogue) or b.q.
template <int G>
__device__ inline void chunk_scores(const DecodeDims &d, const DecodeBuffers &b, uint32_t kvh, uint32_t chunk,
                                    uint32_t nchunks, uint32_t p0, uint32_t p1, const uint2 (&kr)[kPosPerWarp],
                                    float (&sc)[G][kPosChunk], bool store_scores,
                                    const bf16 *q_shared = nullptr) {
  const uint32_t lane = lane_id(), cw = cwarp();
  float q[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint2 raw = q_shared ? *reinterpret_cast<const uint2 *>(q_shared + g * kHD + lane * 4)
                               : ldcg8(b.q + (static_cast<size_t>(kvh) * G + g) * kHD + lane * 4);
    q[g][0] = bf16_lo(raw.x); q[g][1] = bf16_hi(raw.x);
    q[g][2] = bf16_lo(raw.y); q[g][3] = bf16_hi(raw.y);
  }
  // Positions in batches whose G x batch per-lane dot-product partials (16
  // or 32 values) are summed over the warp together.
  constexpr int kBatch = G >= 2 ? 32 / G : 16;
  constexpr int kVals = kBatch * G;
#pragma unroll
  for (int bt = 0; bt < static_cast<int>(kPosPerWarp) / kBatch; ++bt) {
    float v[kVals];
#pragma unroll
    for (int ii = 0; ii < kBatch; ++ii) {
      const uint2 k = kr[bt * kBatch + ii];
      const float k4[4] = {bf16_lo(k.x), bf16_hi(k.x), bf16_lo(k.y), bf16_hi(k.y)};
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) s = fmaf(q[g][j], k4[j], s);
        v[ii * G + g] = s;
      }
    }
    const float tot = warp_sum_transposed<kVals>(v);
    const uint32_t idx = kVals == 32 ? lane : lane >> 1;
    if (kVals == 32 || (lane & 1) == 0)
      sc[idx % G][cw * kPosPerWarp + bt * kBatch + idx / G] = round_bf16(__fmul_rn(round_bf16(tot), kAttnScale));
  }
  consumer_sync();
  for (uint32_t g = cw; g < static_cast<uint32_t>(G); g += kConsumerWarps) {
    float m = -INFINITY;
    for (uint32_t i = lane; i < p1 - p0; i += 32) m = fmaxf(m, sc[g][i]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t i = lane; i < p1 - p0; i += 32) l += expf(sc[g][i] - m);
    l = warp_sum(l);
    const uint32_t h = kvh * G + g;
    if (store_scores)
      for (uint32_t i = lane; i < p1 - p0; i += 32) b.scores[static_cast<size_t>(h) * d.max_seq + p0 + i] = sc[g][i];
    if (lane == 0) {
      b.stats[(static_cast<size_t>(h) * nchunks + chunk) * 2] = m;
      b.stats[(static_cast<size_t>(h) * nchunks + chunk) * 2 + 1] = l;
    }
  }
  consumer_sync();
}

// Softmax statistics over all `nch` chunks of every head of the group:
// sM = global max M, sInv = 1 / S with S = sum of l_c exp(m_c - M) (each
// lane its chunks lane, lane + 32, ..., then a warp sum).
template <int G>
__device__ inline void group_stats(const DecodeBuffers &b, uint32_t kvh, uint32_t nchunks, uint32_t nch,
                                   float (&sM)[G], float (&sInv)[G]) {
  const uint32_t lane = lane_id(), cw = cwarp();
  for (uint32_t g = cw; g < static_cast<uint32_t>(G); g += kConsumerWarps) {
    const float *st = b.stats + static_cast<size_t>(kvh * G + g) * nchunks * 2;
    // this lane's first chunk statistics, read once (up to 32 chunks, 4096
    // positions, without a second read)
    const float cm = lane < nch ? __ldcg(st + 2 * lane) : -INFINITY;
    const float cl = lane < nch ? __ldcg(st + 2 * lane + 1) : 0.f;
    float m = cm;
    for (uint32_t c = lane + 32; c < nch; c += 32) m = fmaxf(m, __ldcg(st + 2 * c));
    m = warp_max(m);
    float sum = lane < nch ? cl * expf(cm - m) : 0.f;
    for (uint32_t c = lane + 32; c < nch; c += 32) sum += __ldcg(st + 2 * c + 1) * expf(__ldcg(st + 2 * c) - m);
    sum = warp_sum(sum);
    if (lane == 0) { sM[g] = m; sInv[g] = 1.0f / sum; }
  }
  consumer_sync();
}

// The chunk's partial sum of p * v (probabilities in sc) into
// attn_part[head][chunk] (warps' partials added in warp order).
template <int G>
__device__ inline void chunk_pv(const DecodeBuffers &b, uint32_t kvh, uint32_t chunk, uint32_t nchunks,
                                const uint2 (&vr)[kPosPerWarp], const float (&sc)[G][kPosChunk],
                                float (&sacc)[kConsumerWarps][G][kHD]) {
  const uint32_t lane = lane_id(), cw = cwarp(), t = ctid();
  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[g][j] = 0.f;
#pragma unroll
  for (uint32_t i = 0; i < kPosPerWarp; ++i) {
    const float v4[4] = {bf16_lo(vr[i].x), bf16_hi(vr[i].x), bf16_lo(vr[i].y), bf16_hi(vr[i].y)};
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float prob = sc[g][cw * kPosPerWarp + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = fmaf(prob, v4[j], acc[g][j]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) sacc[cw][g][lane * 4 + j] = acc[g][j];
  consumer_sync();
  for (uint32_t e = t; e < G * kHD; e += kConsumerThreads) {
    const uint32_t g = e / kHD, dd = e % kHD;
    float tot = 0.f;
#pragma unroll
    for (uint32_t ww = 0; ww < static_cast<uint32_t>(kConsumerWarps); ++ww) tot += sacc[ww][g][dd];
    b.attn_part[(static_cast<size_t>(kvh * G + g) * nchunks + chunk) * kHD + dd] = tot;
  }
}

// Scores of one item (kv head, chunk) of the multi-kernel paths, whose head
// epilogues ran before (the persistent step runs them inside attn_item).
template <int G>
__device__ inline void scores_item(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, uint32_t kvh,
                                   uint32_t chunk, uint32_t nchunks, uint32_t n, AttnShared<G> &as) {
  const uint32_t p0 = chunk * kPosChunk, p1 = min(p0 + kPosChunk, n);
  const uint32_t pw = p0 + cwarp() * kPosPerWarp;
  uint2 kr[kPosPerWarp];
  load_rows(w.kcache, d, kvh, pw, p1, 0xffffffffu, kr);
  chunk_scores<G>(d, b, kvh, chunk, nchunks, p0, p1, kr, as.sc, true);
}

// Probabilities bf16(exp(s - M) * (1 / S)) over all chunks' statistics, the
// chunk's partial sum of p * v, and (last CTA of the kv head) the sum over
// chunks into the attention output.
template <int G>
__device__ inline void pv_item(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, uint32_t kvh,
                               uint32_t chunk, uint32_t nchunks, uint32_t n, AttnShared<G> &as) {
  const uint32_t t = ctid();
  const uint32_t nch = (n + kPosChunk - 1) / kPosChunk;
  const uint32_t p0 = chunk * kPosChunk, p1 = min(p0 + kPosChunk, n);
  const uint32_t pw = p0 + cwarp() * kPosPerWarp;
  uint2 vr[kPosPerWarp];
  load_rows(w.vcache, d, kvh, pw, p1, 0xffffffffu, vr);
  // This thread's scores of the chunk, loaded now with the V rows (they do
  // not depend on the softmax statistics).
  constexpr uint32_t kScPerThread = (G * kPosChunk + kConsumerThreads - 1) / kConsumerThreads;
  float sreg[kScPerThread];
#pragma unroll
  for (uint32_t k = 0; k < kScPerThread; ++k) {
    const uint32_t i = t + k * kConsumerThreads, g = i / kPosChunk, p = p0 + i % kPosChunk;
    sreg[k] = (i < G * kPosChunk && p < p1) ? __ldcg(b.scores + static_cast<size_t>(kvh * G + g) * d.max_seq + p) : 0.f;
  }
  group_stats<G>(b, kvh, nchunks, nch, as.sM, as.sInv);
#pragma unroll
  for (uint32_t k = 0; k < kScPerThread; ++k) {
    const uint32_t i = t + k * kConsumerThreads;
    if (i < G * kPosChunk) {
      const uint32_t g = i / kPosChunk, j = i % kPosChunk;
      as.sc[g][j] = p0 + j < p1 ? round_bf16(__fmul_rn(expf(sreg[k] - as.sM[g]), as.sInv[g])) : 0.f;
    }
  }
  consumer_sync();
  chunk_pv<G>(b, kvh, chunk, nchunks, vr, as.sc, as.sacc);
  if (arrive_one(b.cnt_attn + kvh, nch, &as.flag)) {
    for (uint32_t e = t; e < G * kHD; e += kConsumerThreads) {
      const uint32_t g = e / kHD, dd = e % kHD;
      const float *src = b.attn_part + static_cast<size_t>(kvh * G + g) * nchunks * kHD + dd;
      float o = 0.f;
      for (uint32_t c = 0; c < nch; ++c) o += __ldcg(src + static_cast<size_t>(c) * kHD);
      put(b.attn, static_cast<size_t>(kvh * G + g) * kHD + dd, o);
    }
    if (t == 0) b.cnt_attn[kvh] = 0;
  }
  consumer_sync();
}

// Attention staging of the persistent step: the scores of up to
// kMaxItemChunks chunks of one item, the group's softmax statistics and the
// warps' p.v partials.
constexpr uint32_t kMaxItemChunks = 3;  // 40960 positions over >= 107 CTAs

template <int G>
struct StepAttnShared {
  float sc[kMaxItemChunks][G][kPosChunk];
  alignas(16) bf16 q[G][kHD];  // the group's q heads (head epilogue -> scores)
  float sM[G], sInv[G];
  float sacc[kConsumerWarps][G][kHD];
};

// Persistent step, one pass per item: chunks [c0, c1) of kv head kvh. The
// head epilogues (q heads into shared memory) and scores of scores_item for
// each chunk, then - once every
// item of the kv head has published its chunk statistics - the probabilities
// and partial p.v of pv_item (combine deferred to the o_proj staging). The
// first chunk's V rows are in flight during the wait.
// `wait()` arrives on the kv head's counter and waits (bounded) for the
// layer's full count: false on a timeout or another waiter's failure. The
// arithmetic per chunk is that of scores_item + pv_item, so the bits are the
// same. No CTA may hold two items of one kv head (it would wait for itself).
template <int G, typename Wait>
__device__ inline bool attn_item(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, uint32_t kvh,
                                 uint32_t c0, uint32_t c1, uint32_t nchunks, uint32_t n, StepAttnShared<G> &as,
                                 Wait wait) {
  const uint32_t t = ctid(), cw = cwarp();
  const uint32_t nch = (n + kPosChunk - 1) / kPosChunk;
  const uint32_t newest = n - 1, newest_chunk = newest / kPosChunk;
  uint2 vr[kPosPerWarp];
  for (uint32_t c = c0; c < c1; ++c) {
    const uint32_t p0 = c * kPosChunk, p1 = min(p0 + kPosChunk, n);
    const uint32_t pw = p0 + cw * kPosPerWarp;
    uint2 kr[kPosPerWarp];
    load_rows(w.kcache, d, kvh, pw, p1, c == c0 ? newest : 0xffffffffu, kr);
    if (c == c0) {
      attn_group_heads(d, b, w, kvh, newest_chunk >= c0 && newest_chunk < c1, newest, &as.q[0][0]);
      reload_row(w.kcache, d, kvh, pw, newest, kr);
    }
    chunk_scores<G>(d, b, kvh, c, nchunks, p0, p1, kr, as.sc[c - c0], false, &as.q[0][0]);
  }
  // the first chunk's V rows, in flight during the wait
  load_rows(w.vcache, d, kvh, c0 * kPosChunk + cw * kPosPerWarp, min(c0 * kPosChunk + kPosChunk, n), 0xffffffffu, vr);
  if (!wait()) return false;
  group_stats<G>(b, kvh, nchunks, nch, as.sM, as.sInv);
  constexpr uint32_t kScPerThread = (G * kPosChunk + kConsumerThreads - 1) / kConsumerThreads;
  for (uint32_t c = c0; c < c1; ++c) {
    const uint32_t p0 = c * kPosChunk, p1 = min(p0 + kPosChunk, n);
    if (c != c0) load_rows(w.vcache, d, kvh, p0 + cw * kPosPerWarp, p1, 0xffffffffu, vr);
    float (&sc)[G][kPosChunk] = as.sc[c - c0];
#pragma unroll
    for (uint32_t k = 0; k < kScPerThread; ++k) {
      const uint32_t i = t + k * kConsumerThreads;
      if (i < G * kPosChunk) {
        const uint32_t g = i / kPosChunk, j = i % kPosChunk;
        sc[g][j] = p0 + j < p1 ? round_bf16(__fmul_rn(expf(sc[g][j] - as.sM[g]), as.sInv[g])) : 0.f;
      }
    }
    consumer_sync();
    chunk_pv<G>(b, kvh, c, nchunks, vr, sc, as.sacc);
    consumer_sync();
  }
  return true;
}

// Persistent step, o_proj input: for each K part that this CTA's o_proj
// items use, the attention output of those dimensions, combined here from
// the position-chunk partials (chunks in order, then bf16: the arithmetic of
// pv_item's combine) and staged into xs at the part's offset.
__device__ inline void stage_attn_parts(const DecodeDims &d, const DecodeBuffers &b, const StreamGeom &g,
                                        uint32_t nchunks, uint32_t n, uint4 *xs) {
  constexpr uint32_t kHeld = 24;  // chunk partials loaded before the in-order sum (3072 positions)
  const uint32_t nch = (n + kPosChunk - 1) / kPosChunk;
  uint32_t list[8], nparts = 0;
  uint32_t seen = 0;
  for (uint32_t item = blockIdx.x; item < g.items(); item += gridDim.x) {
    const uint32_t part = item % g.kparts;
    if (!((seen >> part) & 1u) && nparts < 8) { seen |= 1u << part; list[nparts++] = part; }
  }
  const uint32_t quads = g.kt / 4;  // 4 dimensions per thread and pass
  for (uint32_t q = ctid(); q < nparts * quads; q += kConsumerThreads) {
    const uint32_t e0 = list[q / quads] * g.kt + 4 * (q % quads);
    const uint32_t h = e0 / kHD, dd = e0 % kHD;
    const float *src = b.attn_part + static_cast<size_t>(h) * nchunks * kHD + dd;
    float4 v[kHeld];
#pragma unroll
    for (uint32_t c = 0; c < kHeld; ++c)
      v[c] = c < nch ? __ldcg(reinterpret_cast<const float4 *>(src + static_cast<size_t>(c) * kHD))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
    for (uint32_t c = 0; c < kHeld; ++c)
      if (c < nch) { o0 += v[c].x; o1 += v[c].y; o2 += v[c].z; o3 += v[c].w; }
    for (uint32_t c = kHeld; c < nch; ++c) {
      const float4 x = __ldcg(reinterpret_cast<const float4 *>(src + static_cast<size_t>(c) * kHD));
      o0 += x.x; o1 += x.y; o2 += x.z; o3 += x.w;
    }
    reinterpret_cast<uint2 *>(xs)[e0 / 4] = make_uint2(pack_bf16x2(o0, o1), pack_bf16x2(o2, o3));
  }
  consumer_sync();
}

}  // namespace dec
}  // namespace xpu
