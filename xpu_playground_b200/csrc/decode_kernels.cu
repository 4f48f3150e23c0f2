// Fused kernels of the Qwen3 decode step (launch order and rounding points
// are described in decode.cuh). Every GEMV here streams its weight rows with
// warp_dot_rows; CTAs loop over row tiles (grid-stride) so that the vector
// they stage in shared memory is reused across many tiles.
//
// Cross-CTA reductions (split-K partial sums, attention chunks, argmax) use
// the "last CTA finishes" pattern: each CTA publishes its partial results,
// fences, and bumps an arrival counter; the CTA that sees the final count
// reads every partial in a fixed order (so results never depend on arrival
// order), runs the epilogue and resets the counter for the next replay.
// Nothing in these kernels waits on another CTA.
#include "decode.cuh"
#include "gemv_core.cuh"

namespace xpu {

namespace {

constexpr uint32_t kWarps = kDecThreads / 32;

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

// transformers Qwen3RMSNorm scale: RN(1/RN(sqrt(mean(x^2) + eps))).
__device__ float rms_scale(const bf16 *x, uint32_t H, float eps, float *red) {
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x);
  float ss = 0.f;
  for (uint32_t c = threadIdx.x; c < H / 8; c += kDecThreads) ss = sq8(x4[c], ss);
  ss = block_sum<kWarps>(ss, red);
  return 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
}

// Stage chunks [c0, c0 + n) of bf16(w * bf16(x * r)) into shared memory.
__device__ void stage_rms(const bf16 *x, const bf16 *w, float r, uint32_t c0, uint32_t n,
                          uint4 *xs) {
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x) + c0;
  const uint4 *w4 = reinterpret_cast<const uint4 *>(w) + c0;
  for (uint32_t c = threadIdx.x; c < n; c += kDecThreads) {
    const uint4 xv = x4[c], wv = w4[c];
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
}

__device__ void stage_copy(const bf16 *x, uint32_t c0, uint32_t n, uint4 *xs) {
  const uint4 *x4 = reinterpret_cast<const uint4 *>(x) + c0;
  for (uint32_t c = threadIdx.x; c < n; c += kDecThreads) xs[c] = x4[c];
}

// Publish-then-count: returns true in every thread of the CTA that arrived
// last. Partial results must already be stored by the calling threads.
__device__ bool arrive_last(unsigned *counter, unsigned total, int *flag) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *flag = (atomicAdd(counter, 1u) == total - 1u);
  __syncthreads();
  const bool last = *flag != 0;
  if (last) __threadfence();
  return last;
}

__device__ __forceinline__ float bf(const bf16 *p, size_t i) {
  return bf16_bits_to_float(reinterpret_cast<const uint16_t *>(p)[i]);
}
__device__ __forceinline__ void put(bf16 *p, size_t i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = float_to_bf16_bits(v);
}

// ------------------------------------------------------------ embedding ----
__global__ void __launch_bounds__(kDecThreads) k_embed(DecodeDims d, DecodeBuffers b, uint32_t vocab) {
  const DecodeState *st = b.state;
  const uint32_t pos = st->position;
  uint32_t tok = pos < st->prompt_len ? b.prompt[pos] : st->token;
  if (tok >= vocab) {  // a NaN step's sentinel or a bad id: read row 0, flag the state
    if (blockIdx.x == 0 && threadIdx.x == 0) b.state->error |= 1u;
    tok = 0;
  }
  const uint32_t c = blockIdx.x * kDecThreads + threadIdx.x;
  if (c < d.H / 8)
    reinterpret_cast<uint4 *>(b.x)[c] =
        reinterpret_cast<const uint4 *>(b.embed)[static_cast<size_t>(tok) * (d.H / 8) + c];
}

// ---------------------------------------------------------------- QKV ----
__device__ void qkv_head_epilogue(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                                  uint32_t head, float *ep, float *red) {
  const uint32_t t = threadIdx.x;
  const uint32_t heads = d.QH_l + 2 * d.KVH_l, rows_total = heads * kHD;
  const uint32_t pos = b.state->position;
  float y = 0.f;
  if (t < kHD) {
    for (uint32_t s = 0; s < d.qkv_splits; ++s)
      y += __ldcg(b.part_qkv + static_cast<size_t>(s) * rows_total + head * kHD + t);
    y = round_bf16(y);
  }
  if (head >= d.QH_l + d.KVH_l) {  // value head: straight into the cache
    const uint32_t j = head - d.QH_l - d.KVH_l;
    if (t < kHD) put(w.vcache, (static_cast<size_t>(pos) * d.KVH_l + j) * kHD + t, y);
    return;
  }
  const bool is_q = head < d.QH_l;
  const float ss = block_sum<kWarps>(t < kHD ? __fmul_rn(y, y) : 0.f, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(kHD) + d.eps);
  float nv = 0.f;
  if (t < kHD) {
    const float wt = bf(is_q ? w.q_norm : w.k_norm, t);
    nv = round_bf16(__fmul_rn(wt, round_bf16(__fmul_rn(y, r))));
    ep[t] = nv;
  }
  __syncthreads();
  if (t < kHD) {
    const float c = bf(b.cos_t, static_cast<size_t>(pos) * kHD + t);
    const float s = bf(b.sin_t, static_cast<size_t>(pos) * kHD + t);
    const float rot = t < kHD / 2 ? -ep[t + kHD / 2] : ep[t - kHD / 2];  // rotate_half
    const float out = round_bf16(__fadd_rn(round_bf16(__fmul_rn(nv, c)), round_bf16(__fmul_rn(rot, s))));
    if (is_q) put(b.q, static_cast<size_t>(head) * kHD + t, out);
    else put(w.kcache, (static_cast<size_t>(pos) * d.KVH_l + (head - d.QH_l)) * kHD + t, out);
  }
}

__global__ void __launch_bounds__(kDecThreads) k_qkv(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  extern __shared__ uint4 xs[];
  __shared__ float red[kWarps];
  __shared__ float ep[kHD];
  __shared__ int flag;
  const uint32_t H = d.H, split = blockIdx.y, Ks = H / d.qkv_splits, nck = Ks / 8;
  const uint32_t heads = d.QH_l + 2 * d.KVH_l, rows_total = heads * kHD;
  const uint32_t ntiles = rows_total / kTileRows, tiles_per_head = kHD / kTileRows;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float r = rms_scale(b.x, H, d.eps, red);
  stage_rms(b.x, w.in_norm, r, split * nck, nck, xs);
  __syncthreads();
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const uint32_t row0 = tile * kTileRows + warp * 2;
    const uint4 *rows[2] = {
        reinterpret_cast<const uint4 *>(w.wqkv + static_cast<size_t>(row0) * H + split * Ks),
        reinterpret_cast<const uint4 *>(w.wqkv + static_cast<size_t>(row0 + 1) * H + split * Ks)};
    float acc[2];
    warp_dot_rows<bf16, 2, 4>(rows, xs, nck, lane, acc);
    if (lane == 0) {
      b.part_qkv[static_cast<size_t>(split) * rows_total + row0] = acc[0];
      b.part_qkv[static_cast<size_t>(split) * rows_total + row0 + 1] = acc[1];
    }
    const uint32_t head = tile / tiles_per_head;
    if (arrive_last(b.cnt_qkv + head, tiles_per_head * d.qkv_splits, &flag)) {
      qkv_head_epilogue(d, b, w, head, ep, red);
      if (threadIdx.x == 0) b.cnt_qkv[head] = 0;
      __syncthreads();
    }
  }
}

// ----------------------------------------------------------- attention ----
// One CTA per (kv head, 128-position chunk), 8 warps x 16 positions. Each
// warp issues the loads of all its 16 cache rows before using any (one memory
// round trip per warp); lane l holds dimensions 4l..4l+3 of each row.
constexpr uint32_t kAttnThreads = 256;
constexpr uint32_t kAttnWarps = kAttnThreads / 32;
constexpr uint32_t kPosPerWarp = kPosChunk / kAttnWarps;  // 16

template <int G>
__global__ void __launch_bounds__(kAttnThreads) k_scores(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  __shared__ float sc[G][kPosChunk];
  const uint32_t kvh = blockIdx.x, chunk = blockIdx.y, nchunks = gridDim.y;
  const uint32_t n = b.state->position + 1, p0 = chunk * kPosChunk;
  if (p0 >= n) return;
  const uint32_t p1 = min(p0 + kPosChunk, n);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t pw = p0 + warp * kPosPerWarp;
  uint2 kr[kPosPerWarp];
#pragma unroll
  for (uint32_t i = 0; i < kPosPerWarp; ++i) {
    const uint32_t p = pw + i;
    kr[i] = p < p1 ? *reinterpret_cast<const uint2 *>(w.kcache + (static_cast<size_t>(p) * d.KVH_l + kvh) * kHD + lane * 4)
                   : make_uint2(0, 0);
  }
  float q[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const uint2 raw = *reinterpret_cast<const uint2 *>(b.q + (static_cast<size_t>(kvh) * G + g) * kHD + lane * 4);
    q[g][0] = bf16_lo(raw.x); q[g][1] = bf16_hi(raw.x);
    q[g][2] = bf16_lo(raw.y); q[g][3] = bf16_hi(raw.y);
  }
#pragma unroll
  for (uint32_t i = 0; i < kPosPerWarp; ++i) {
    const float k4[4] = {bf16_lo(kr[i].x), bf16_hi(kr[i].x), bf16_lo(kr[i].y), bf16_hi(kr[i].y)};
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) s = fmaf(q[g][j], k4[j], s);
      s = warp_sum(s);
      if (lane == 0) sc[g][warp * kPosPerWarp + i] = round_bf16(__fmul_rn(round_bf16(s), kAttnScale));
    }
  }
  __syncthreads();
  for (uint32_t g = warp; g < static_cast<uint32_t>(G); g += kAttnWarps) {
    float m = -INFINITY;
    for (uint32_t i = lane; i < p1 - p0; i += 32) m = fmaxf(m, sc[g][i]);
    m = warp_max(m);
    float l = 0.f;
    for (uint32_t i = lane; i < p1 - p0; i += 32) l += expf(sc[g][i] - m);
    l = warp_sum(l);
    const uint32_t h = kvh * G + g;
    for (uint32_t i = lane; i < p1 - p0; i += 32) b.scores[static_cast<size_t>(h) * d.max_seq + p0 + i] = sc[g][i];
    if (lane == 0) {
      b.stats[(static_cast<size_t>(h) * nchunks + chunk) * 2] = m;
      b.stats[(static_cast<size_t>(h) * nchunks + chunk) * 2 + 1] = l;
    }
  }
}

template <int G>
__global__ void __launch_bounds__(kAttnThreads) k_pv(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  __shared__ float sM[G], sInv[G];
  __shared__ float sp[G][kPosChunk];
  __shared__ float sacc[kAttnWarps][G][kHD];
  __shared__ int flag;
  const uint32_t kvh = blockIdx.x, chunk = blockIdx.y, nchunks = gridDim.y;
  const uint32_t n = b.state->position + 1, nch = (n + kPosChunk - 1) / kPosChunk;
  if (chunk >= nch) return;
  const uint32_t p0 = chunk * kPosChunk, p1 = min(p0 + kPosChunk, n);
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t pw = p0 + warp * kPosPerWarp;
  uint2 vr[kPosPerWarp];
#pragma unroll
  for (uint32_t i = 0; i < kPosPerWarp; ++i) {
    const uint32_t p = pw + i;
    vr[i] = p < p1 ? *reinterpret_cast<const uint2 *>(w.vcache + (static_cast<size_t>(p) * d.KVH_l + kvh) * kHD + lane * 4)
                   : make_uint2(0, 0);
  }
  // Softmax statistics over all chunks: M = max, S = sum exp(s - M).
  for (uint32_t g = warp; g < static_cast<uint32_t>(G); g += kAttnWarps) {
    const float *st = b.stats + static_cast<size_t>(kvh * G + g) * nchunks * 2;
    float m = -INFINITY;
    for (uint32_t c = lane; c < nch; c += 32) m = fmaxf(m, st[2 * c]);
    m = warp_max(m);
    float sum = 0.f;
    for (uint32_t c = lane; c < nch; c += 32) sum += st[2 * c + 1] * expf(st[2 * c] - m);
    sum = warp_sum(sum);
    if (lane == 0) { sM[g] = m; sInv[g] = 1.0f / sum; }
  }
  __syncthreads();
  // Probabilities of this chunk, rounded to bf16 as transformers does.
  for (uint32_t i = threadIdx.x; i < G * kPosChunk; i += kAttnThreads) {
    const uint32_t g = i / kPosChunk, j = i % kPosChunk;
    const uint32_t p = p0 + j;
    sp[g][j] = p < p1 ? round_bf16(__fmul_rn(expf(b.scores[static_cast<size_t>(kvh * G + g) * d.max_seq + p] - sM[g]), sInv[g]))
                      : 0.f;
  }
  __syncthreads();
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
      const float prob = sp[g][warp * kPosPerWarp + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = fmaf(prob, v4[j], acc[g][j]);
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < 4; ++j) sacc[warp][g][lane * 4 + j] = acc[g][j];
  __syncthreads();
  const uint32_t t = threadIdx.x;
  for (uint32_t e = t; e < G * kHD; e += kAttnThreads) {
    const uint32_t g = e / kHD, dd = e % kHD;
    float tot = 0.f;
#pragma unroll
    for (uint32_t ww = 0; ww < kAttnWarps; ++ww) tot += sacc[ww][g][dd];
    b.attn_part[(static_cast<size_t>(kvh * G + g) * nchunks + chunk) * kHD + dd] = tot;
  }
  if (arrive_last(b.cnt_attn + kvh, nch, &flag)) {
    for (uint32_t e = t; e < G * kHD; e += kAttnThreads) {
      const uint32_t g = e / kHD, dd = e % kHD;
      const float *src = b.attn_part + static_cast<size_t>(kvh * G + g) * nchunks * kHD + dd;
      float o = 0.f;
      for (uint32_t c = 0; c < nch; ++c) o += __ldcg(src + static_cast<size_t>(c) * kHD);
      put(b.attn, static_cast<size_t>(kvh * G + g) * kHD + dd, o);
    }
    if (t == 0) b.cnt_attn[kvh] = 0;
  }
}

// --------------------------------------------- row-parallel (o, down) ----
// W is [H][K_l]; CTA column j covers canonical chunk chunk0 + j. The last
// CTA of a row tile sums all 8 canonical chunks in order and adds the
// residual: x = bf16(x + bf16(sum)).
__global__ void __launch_bounds__(kDecThreads)
k_rowpar(DecodeDims d, DecodeBuffers b, const bf16 *W, uint32_t K_l, const bf16 *xin) {
  extern __shared__ uint4 xs[];
  __shared__ int flag;
  const uint32_t H = d.H, j = blockIdx.y, kc = K_l / d.chunks_l, nck = kc / 8;
  const uint32_t ntiles = H / kTileRows, g = d.chunk0 + j;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  stage_copy(xin, j * nck, nck, xs);
  __syncthreads();
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const uint32_t row0 = tile * kTileRows + warp * 2;
    const uint4 *rows[2] = {
        reinterpret_cast<const uint4 *>(W + static_cast<size_t>(row0) * K_l + j * kc),
        reinterpret_cast<const uint4 *>(W + static_cast<size_t>(row0 + 1) * K_l + j * kc)};
    float acc[2];
    warp_dot_rows<bf16, 2, 4>(rows, xs, nck, lane, acc);
    if (lane == 0) {
      b.part[static_cast<size_t>(g) * H + row0] = acc[0];
      b.part[static_cast<size_t>(g) * H + row0 + 1] = acc[1];
    }
    if (arrive_last(b.cnt_tile + tile, d.chunks_l, &flag)) {
      if (threadIdx.x < kTileRows) {
        const uint32_t row = tile * kTileRows + threadIdx.x;
        float y = 0.f;
        for (uint32_t c = 0; c < kCanonChunks; ++c) y += __ldcg(b.part + static_cast<size_t>(c) * H + row);
        put(b.x, row, __fadd_rn(bf(b.x, row), round_bf16(y)));
      }
      if (threadIdx.x == 0) b.cnt_tile[tile] = 0;
      __syncthreads();
    }
  }
}

// -------------------------------------------------------------- gate/up ----
__global__ void __launch_bounds__(kDecThreads) k_gateup(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  extern __shared__ uint4 xs[];
  __shared__ float red[kWarps];
  const uint32_t H = d.H, nck = H / 8, ntiles = (d.I_l + kWarps - 1) / kWarps;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float r = rms_scale(b.x, H, d.eps, red);
  stage_rms(b.x, w.post_norm, r, 0, nck, xs);
  __syncthreads();
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const uint32_t i = tile * kWarps + warp;
    if (i >= d.I_l) continue;
    const uint4 *rows[2] = {reinterpret_cast<const uint4 *>(w.wgu + static_cast<size_t>(2 * i) * H),
                            reinterpret_cast<const uint4 *>(w.wgu + static_cast<size_t>(2 * i + 1) * H)};
    float acc[2];
    warp_dot_rows<bf16, 2, 4>(rows, xs, nck, lane, acc);
    if (lane == 0) {
      const float gv = round_bf16(acc[0]), uv = round_bf16(acc[1]);
      const float act = round_bf16(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))));
      put(b.h, i, __fmul_rn(act, uv));
    }
  }
}

// -------------------------------------------------------------- lm_head ----
__global__ void __launch_bounds__(kDecThreads) k_lmhead(DecodeDims d, DecodeBuffers b) {
  extern __shared__ uint4 xs[];
  __shared__ float red[kWarps];
  __shared__ ArgBest wbest[kWarps];
  __shared__ uint32_t wbad[kWarps];
  __shared__ int flag;
  const uint32_t H = d.H, nck = H / 8, ntiles = (d.V_l + kTileRows - 1) / kTileRows;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float r = rms_scale(b.x, H, d.eps, red);
  stage_rms(b.x, b.final_norm, r, 0, nck, xs);
  __syncthreads();
  ArgBest best{-INFINITY, 0xffffffffu};
  uint32_t bad = 0;
  for (uint32_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const uint32_t row0 = tile * kTileRows + warp * 2;
    if (row0 >= d.V_l) continue;
    const uint32_t row1 = min(row0 + 1, d.V_l - 1);
    const uint4 *rows[2] = {reinterpret_cast<const uint4 *>(b.lm_head + static_cast<size_t>(row0) * H),
                            reinterpret_cast<const uint4 *>(b.lm_head + static_cast<size_t>(row1) * H)};
    float acc[2];
    warp_dot_rows<bf16, 2, 4>(rows, xs, nck, lane, acc);
    if (lane == 0) {
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const uint32_t row = row0 + rr;
        if (row >= d.V_l) break;
        const float v = round_bf16(acc[rr]);
        b.logits[row] = float_to_bf16_bits(v);
        bad |= not_finite(v) ? 1u : 0u;
        best = arg_better(best, ArgBest{v, d.v_offset + row});
      }
    }
  }
  if (lane == 0) { wbest[warp] = best; wbad[warp] = bad; }
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgBest cb = wbest[0];
    uint32_t cbad = wbad[0];
    for (uint32_t i = 1; i < kWarps; ++i) { cb = arg_better(cb, wbest[i]); cbad |= wbad[i]; }
    b.lm_best[blockIdx.x] = cb;
    b.lm_bad[blockIdx.x] = cbad;
  }
  if (arrive_last(b.cnt_lm, gridDim.x, &flag)) {
    ArgBest tb{-INFINITY, 0xffffffffu};
    uint32_t tbad = 0;
    for (uint32_t i = threadIdx.x; i < gridDim.x; i += kDecThreads) {
      ArgBest e;
      e.value = __ldcg(&b.lm_best[i].value);
      e.index = __ldcg(&b.lm_best[i].index);
      tb = arg_better(tb, e);
      tbad |= __ldcg(b.lm_bad + i);
    }
    tb = warp_argbest(tb);
    tbad = __reduce_or_sync(kFullMask, tbad);
    if (lane == 0) { wbest[warp] = tb; wbad[warp] = tbad; }
    __syncthreads();
    if (threadIdx.x == 0) {
      ArgBest fb = wbest[0];
      uint32_t fbad = wbad[0];
      for (uint32_t i = 1; i < kWarps; ++i) { fb = arg_better(fb, wbest[i]); fbad |= wbad[i]; }
      DecodeState *st = b.state;
      const uint32_t pos = st->position;
      const uint32_t next = (fbad || fb.index == 0xffffffffu) ? 0xffffffffu : fb.index;
      if (next == 0xffffffffu) st->error |= 1u;
      st->next = next;
      st->token = next;
      if (pos < d.max_seq) b.log[pos] = next;
      st->position = pos + 1;
      st->steps += 1;
      *b.cnt_lm = 0;
    }
  }
}

uint32_t decode_grid(uint32_t tiles, uint32_t splits) {
  // Four 256-thread CTAs per SM on a 148-SM B200, shared among the splits.
  const uint32_t target = (4u * 148u + splits - 1) / splits;
  return tiles < target ? tiles : target;
}

}  // namespace

uint32_t pos_chunks(uint32_t max_seq) { return (max_seq + kPosChunk - 1) / kPosChunk; }

uint32_t lmhead_ctas(const DecodeDims &d) {
  return decode_grid((d.V_l + kTileRows - 1) / kTileRows, 1);
}

static cudaError_t smem_attr(const void *kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
}

cudaError_t launch_embed(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s) {
  const uint32_t grid = (d.H / 8 + kDecThreads - 1) / kDecThreads;
  k_embed<<<grid, kDecThreads, 0, s>>>(d, b, d.vocab);
  return cudaGetLastError();
}

cudaError_t launch_qkv(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                       cudaStream_t s) {
  const uint32_t ntiles = (d.QH_l + 2 * d.KVH_l) * kHD / kTileRows;
  const size_t smem = static_cast<size_t>(d.H / d.qkv_splits) * 2;
  cudaError_t e = smem_attr(reinterpret_cast<const void *>(k_qkv), smem);
  if (e != cudaSuccess) return e;
  k_qkv<<<dim3(decode_grid(ntiles, d.qkv_splits), d.qkv_splits), kDecThreads, smem, s>>>(d, b, w);
  return cudaGetLastError();
}

cudaError_t launch_attention(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                             cudaStream_t s) {
  const dim3 grid(d.KVH_l, pos_chunks(d.max_seq));
  switch (d.QH_l / d.KVH_l) {
    case 1: k_scores<1><<<grid, kAttnThreads, 0, s>>>(d, b, w); k_pv<1><<<grid, kAttnThreads, 0, s>>>(d, b, w); break;
    case 2: k_scores<2><<<grid, kAttnThreads, 0, s>>>(d, b, w); k_pv<2><<<grid, kAttnThreads, 0, s>>>(d, b, w); break;
    case 4: k_scores<4><<<grid, kAttnThreads, 0, s>>>(d, b, w); k_pv<4><<<grid, kAttnThreads, 0, s>>>(d, b, w); break;
    case 8: k_scores<8><<<grid, kAttnThreads, 0, s>>>(d, b, w); k_pv<8><<<grid, kAttnThreads, 0, s>>>(d, b, w); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static cudaError_t launch_rowpar(const DecodeDims &d, const DecodeBuffers &b, const bf16 *W,
                                 uint32_t K_l, const bf16 *xin, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(K_l / d.chunks_l) * 2;
  cudaError_t e = smem_attr(reinterpret_cast<const void *>(k_rowpar), smem);
  if (e != cudaSuccess) return e;
  k_rowpar<<<dim3(decode_grid(d.H / kTileRows, d.chunks_l), d.chunks_l), kDecThreads, smem, s>>>(
      d, b, W, K_l, xin);
  return cudaGetLastError();
}

cudaError_t launch_oproj(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                         cudaStream_t s) {
  return launch_rowpar(d, b, w.wo, d.QH_l * kHD, b.attn, s);
}

cudaError_t launch_down(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                        cudaStream_t s) {
  return launch_rowpar(d, b, w.wd, d.I_l, b.h, s);
}

cudaError_t launch_gateup(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                          cudaStream_t s) {
  const size_t smem = static_cast<size_t>(d.H) * 2;
  cudaError_t e = smem_attr(reinterpret_cast<const void *>(k_gateup), smem);
  if (e != cudaSuccess) return e;
  k_gateup<<<decode_grid((d.I_l + kWarps - 1) / kWarps, 1), kDecThreads, smem, s>>>(d, b, w);
  return cudaGetLastError();
}

cudaError_t launch_lmhead(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(d.H) * 2;
  cudaError_t e = smem_attr(reinterpret_cast<const void *>(k_lmhead), smem);
  if (e != cudaSuccess) return e;
  k_lmhead<<<lmhead_ctas(d), kDecThreads, smem, s>>>(d, b);
  return cudaGetLastError();
}

}  // namespace xpu
