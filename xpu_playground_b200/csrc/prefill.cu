// Dense prefill: the prompt's positions go through each layer together, so
// every projection is a tcgen05 GEMM over all of them (C = X . W^T against
// the stored weights, gemm_launch_ex) - compute-bound, each weight read once
// per segment of up to kPrefillSegment positions - instead of the decode
// step's weight streaming per position. Around the GEMMs, the small kernels
// here apply the same rounding points as the decode step (those of the
// transformers Qwen3 bf16 eager forward):
//   k_pf_embed      x[m] = embed[token[m]]
//   k_pf_rms        xn[m] = bf16(w * bf16(x * RN(1/RN(sqrt(mean(x^2) + eps)))))
//   k_pf_heads      per (position, head) of the raw q/k/v rows: q/k RMSNorm
//                   + RoPE into q / the key cache, v into the value cache
//   k_pf_attention  causal GQA attention over the cache for the segment's
//                   queries: s = bf16(bf16(q.k) * scale), exact softmax over
//                   the whole context (two passes: statistics, then
//                   probabilities bf16(exp(s - M) * (1 / S)) and p.v in FP32)
//   k_pf_add_rms    x = bf16(x + y), then xn = RMSNorm(x) with the next norm
//   k_pf_swiglu     h = bf16(bf16(silu(g)) * u) from the interleaved gate/up
// The attention is CUDA-core FP32 (one CTA per kv head and block of 16
// queries; the group's heads share every K/V tile staged in shared memory).
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "xpu_internal.h"

namespace xpu {
namespace {

__device__ __forceinline__ float bfv(const uint16_t *p, size_t i) { return bf16_bits_to_float(p[i]); }
__device__ __forceinline__ uint16_t bfb(float v) { return float_to_bf16_bits(v); }

__global__ void k_pf_embed(const uint16_t *embed, const uint32_t *tokens, uint16_t *x, uint32_t H) {
  const uint32_t m = blockIdx.x;
  const uint4 *src = reinterpret_cast<const uint4 *>(embed + static_cast<size_t>(tokens[m]) * H);
  uint4 *dst = reinterpret_cast<uint4 *>(x + static_cast<size_t>(m) * H);
  for (uint32_t c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

// Block-wide FP32 sum (fixed order: warp butterflies, then warps in order).
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (uint32_t i = 0; i < warps; ++i) t += scratch[i];
  return t;
}

__device__ __forceinline__ void rms_row(const uint16_t *x, const uint16_t *w, uint16_t *xn, uint32_t H, float eps,
                                        float *scratch) {
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = bfv(x, i);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  ss = block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(H) + eps);
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x)
    xn[i] = bfb(__fmul_rn(bfv(w, i), round_bf16(__fmul_rn(bfv(x, i), r))));
}

__global__ void k_pf_rms(const uint16_t *x, const uint16_t *w, uint16_t *xn, uint32_t H, float eps) {
  __shared__ float scratch[32];
  const size_t m = blockIdx.x;
  rms_row(x + m * H, w, xn + m * H, H, eps, scratch);
}

// x = bf16(x + y) for row m, then xn = RMSNorm(x) with w.
__global__ void k_pf_add_rms(uint16_t *x, const uint16_t *y, const uint16_t *w, uint16_t *xn, uint32_t H, float eps) {
  __shared__ float scratch[32];
  const size_t m = blockIdx.x;
  uint16_t *xr = x + m * H;
  const uint16_t *yr = y + m * H;
  for (uint32_t i = threadIdx.x; i < H; i += blockDim.x) xr[i] = bfb(__fadd_rn(bfv(xr, i), bfv(yr, i)));
  __syncthreads();
  rms_row(xr, w, xn + m * H, H, eps, scratch);
}

// One warp per (position, head) of the raw [q heads; k heads; v heads] row
// (bf16 GEMM outputs): lane l owns dimensions l, l + 32, l + 64, l + 96, so
// both rotate-half pairs sit in one lane - the decode step's head epilogue.
__global__ void k_pf_heads(const uint16_t *qkv, uint32_t rows_qkv, const uint16_t *q_norm, const uint16_t *k_norm,
                           const uint16_t *cos_t, const uint16_t *sin_t, uint16_t *q, uint16_t *kc, uint16_t *vc,
                           uint32_t p0, uint32_t M, uint32_t QH, uint32_t KVH, float eps) {
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const uint32_t heads = QH + 2 * KVH;
  if (warp >= M * heads) return;
  const uint32_t m = warp / heads, head = warp % heads, pos = p0 + m;
  const uint16_t *src = qkv + static_cast<size_t>(m) * rows_qkv + head * kHD;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = bfv(src, lane + 32 * j);
  if (head >= QH + KVH) {
    uint16_t *dst = vc + (static_cast<size_t>(pos) * KVH + (head - QH - KVH)) * kHD;
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = bfb(v[j]);
    return;
  }
  const bool is_q = head < QH;
  const uint16_t *nw = is_q ? q_norm : k_norm;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(kHD) + eps);
  float nv[4], cv[4], sv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    nv[j] = round_bf16(__fmul_rn(bfv(nw, lane + 32 * j), round_bf16(__fmul_rn(v[j], r))));
    cv[j] = bfv(cos_t, static_cast<size_t>(pos) * kHD + lane + 32 * j);
    sv[j] = bfv(sin_t, static_cast<size_t>(pos) * kHD + lane + 32 * j);
  }
  float out[4];
#pragma unroll
  for (int j = 0; j < 2; ++j) {  // pairs (i, i + 64): rotate_half
    const float a = nv[j], c = nv[j + 2];
    out[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(a, cv[j])), round_bf16(__fmul_rn(-c, sv[j]))));
    out[j + 2] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(c, cv[j + 2])), round_bf16(__fmul_rn(a, sv[j + 2]))));
  }
  uint16_t *dst = is_q ? q + (static_cast<size_t>(m) * QH + head) * kHD
                       : kc + (static_cast<size_t>(pos) * KVH + (head - QH)) * kHD;
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[lane + 32 * j] = bfb(out[j]);
}

// ---------------------------------------------------------------- attention
constexpr uint32_t kPfQ = 16;        // queries per CTA
constexpr uint32_t kPfKeys = 64;     // keys per staged tile
constexpr uint32_t kPfThreads = 256;

template <int G>
struct PfAttnSmem {
  float qt[kHD][G * kPfQ];        // q, transposed: [dim][row]
  float kt[kHD][kPfKeys];         // k tile, transposed: [dim][key]
  float vt[kPfKeys][kHD];         // v tile: [key][dim]
  float p[kPfKeys][G * kPfQ];     // scores, then probabilities: [key][row]
  float rmax[G * kPfQ], rsum[G * kPfQ];
};

// Rows r = g * kPfQ + i: head kvh * G + g, query position p0 + q0 + i.
template <int G>
__global__ void __launch_bounds__(kPfThreads) k_pf_attention(const uint16_t *q, const uint16_t *kc, const uint16_t *vc,
                                                             uint16_t *out, uint32_t p0, uint32_t M, uint32_t QH,
                                                             uint32_t KVH) {
  constexpr uint32_t R = G * kPfQ;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PfAttnSmem<G> &s = *reinterpret_cast<PfAttnSmem<G> *>(smem_raw);
  const uint32_t kvh = blockIdx.y, q0 = blockIdx.x * kPfQ, t = threadIdx.x;
  const uint32_t nq = min(kPfQ, M - q0);
  const uint32_t last = p0 + q0 + nq - 1;  // last key any row of this CTA sees
  for (uint32_t e = t; e < R * kHD; e += kPfThreads) {
    const uint32_t r = e / kHD, dd = e % kHD, g = r / kPfQ, i = r % kPfQ;
    s.qt[dd][r] = i < nq ? bfv(q, (static_cast<size_t>(q0 + i) * QH + kvh * G + g) * kHD + dd) : 0.f;
  }
  // Score micro-tile of this thread: rows rr..rr+RT-1, keys kk..kk+3.
  constexpr uint32_t RT = R / 16;  // 16 row groups x 16 key groups of 4 keys
  const uint32_t rr = (t / 16) * RT, kk = (t % 16) * 4;
  auto tile_scores = [&](uint32_t key0) {
    float acc[RT][4];
#pragma unroll
    for (uint32_t a = 0; a < RT; ++a)
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b) acc[a][b] = 0.f;
    for (uint32_t dd = 0; dd < kHD; ++dd) {
      float qv[RT], kv[4];
#pragma unroll
      for (uint32_t a = 0; a < RT; ++a) qv[a] = s.qt[dd][rr + a];
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b) kv[b] = s.kt[dd][kk + b];
#pragma unroll
      for (uint32_t a = 0; a < RT; ++a)
#pragma unroll
        for (uint32_t b = 0; b < 4; ++b) acc[a][b] = fmaf(qv[a], kv[b], acc[a][b]);
    }
#pragma unroll
    for (uint32_t a = 0; a < RT; ++a) {
      const uint32_t qpos = p0 + q0 + (rr + a) % kPfQ;
#pragma unroll
      for (uint32_t b = 0; b < 4; ++b) {
        const uint32_t key = key0 + kk + b;
        s.p[kk + b][rr + a] = key <= qpos ? round_bf16(__fmul_rn(round_bf16(acc[a][b]), kAttnScale)) : -INFINITY;
      }
    }
  };
  auto load_k = [&](uint32_t key0) {
    for (uint32_t e = t; e < kPfKeys * kHD; e += kPfThreads) {
      const uint32_t key = e / kHD, dd = e % kHD, pos = key0 + key;
      s.kt[dd][key] = pos <= last ? bfv(kc, (static_cast<size_t>(pos) * KVH + kvh) * kHD + dd) : 0.f;
    }
  };
  // pass 1: per-row max and sum of exp over the whole causal context
  if (t < R) {
    s.rmax[t] = -INFINITY;
    s.rsum[t] = 0.f;
  }
  for (uint32_t key0 = 0; key0 <= last; key0 += kPfKeys) {
    __syncthreads();
    load_k(key0);
    __syncthreads();
    tile_scores(key0);
    __syncthreads();
    if (t < R) {  // one thread per row: fold the tile into (max, sum)
      float m = s.rmax[t];
      for (uint32_t key = 0; key < kPfKeys; ++key) m = fmaxf(m, s.p[key][t]);
      float l = s.rsum[t] * (s.rmax[t] == -INFINITY ? 0.f : expf(s.rmax[t] - m));
      for (uint32_t key = 0; key < kPfKeys; ++key) l += s.p[key][t] == -INFINITY ? 0.f : expf(s.p[key][t] - m);
      s.rmax[t] = m;
      s.rsum[t] = l;
    }
  }
  __syncthreads();
  if (t < R) s.rsum[t] = 1.0f / s.rsum[t];
  // pass 2: probabilities and p.v; thread output tile: rows ro..ro+RT-1 (as
  // above), dims od..od+7
  const uint32_t ro = (t / 16) * RT, od = (t % 16) * 8;
  float o[RT][8];
#pragma unroll
  for (uint32_t a = 0; a < RT; ++a)
#pragma unroll
    for (uint32_t b = 0; b < 8; ++b) o[a][b] = 0.f;
  for (uint32_t key0 = 0; key0 <= last; key0 += kPfKeys) {
    __syncthreads();
    load_k(key0);
    for (uint32_t e = t; e < kPfKeys * kHD; e += kPfThreads) {
      const uint32_t key = e / kHD, dd = e % kHD, pos = key0 + key;
      s.vt[key][dd] = pos <= last ? bfv(vc, (static_cast<size_t>(pos) * KVH + kvh) * kHD + dd) : 0.f;
    }
    __syncthreads();
    tile_scores(key0);
    __syncthreads();
    for (uint32_t e = t; e < kPfKeys * R; e += kPfThreads) {
      const uint32_t key = e / R, r = e % R;
      const float sc = s.p[key][r];
      s.p[key][r] = sc == -INFINITY ? 0.f : round_bf16(__fmul_rn(expf(sc - s.rmax[r]), s.rsum[r]));
    }
    __syncthreads();
    for (uint32_t key = 0; key < kPfKeys; ++key) {
      float pv[RT], vv[8];
#pragma unroll
      for (uint32_t a = 0; a < RT; ++a) pv[a] = s.p[key][ro + a];
#pragma unroll
      for (uint32_t b = 0; b < 8; ++b) vv[b] = s.vt[key][od + b];
#pragma unroll
      for (uint32_t a = 0; a < RT; ++a)
#pragma unroll
        for (uint32_t b = 0; b < 8; ++b) o[a][b] = fmaf(pv[a], vv[b], o[a][b]);
    }
  }
#pragma unroll
  for (uint32_t a = 0; a < RT; ++a) {
    const uint32_t r = ro + a, g = r / kPfQ, i = r % kPfQ;
    if (i >= nq) continue;
    uint16_t *dst = out + (static_cast<size_t>(q0 + i) * QH + kvh * G + g) * kHD + od;
    uint4 pk;
    pk.x = pack_bf16x2(o[a][0], o[a][1]);
    pk.y = pack_bf16x2(o[a][2], o[a][3]);
    pk.z = pack_bf16x2(o[a][4], o[a][5]);
    pk.w = pack_bf16x2(o[a][6], o[a][7]);
    *reinterpret_cast<uint4 *>(dst) = pk;
  }
}

// ---------------------------------------------- attention on tensor cores
// The same causal attention with the two products on the tensor cores
// (mma.sync m16n8k16, bf16 in, FP32 accumulation): per warp 16 rows (one
// head, 16 queries), S = Q K^T for 64 keys at a time, the scores rounded as
// above, exact two-pass softmax (row statistics over the whole context,
// then bf16 probabilities that feed P V straight from the S accumulators).
constexpr uint32_t kTcKeys = 64;
constexpr uint32_t kTcPad = 8;  // bf16 padding per smem row: conflict-free fragment loads

template <int G>
struct TcAttn {
  static constexpr uint32_t QB = G >= 4 ? 16 : 64 / G;  // queries per CTA
  static constexpr uint32_t ROWS = G * QB;              // 64 or 128
  static constexpr uint32_t WARPS = ROWS / 16;
  static constexpr uint32_t THREADS = 32 * WARPS;
};

template <int G>
struct TcAttnSmem {
  uint16_t q[TcAttn<G>::ROWS][kHD + kTcPad];
  uint16_t k[kTcKeys][kHD + kTcPad];
  uint16_t vt[kHD][kTcKeys + kTcPad];  // v tile transposed: [dim][key]
};

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(const uint16_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

template <int G>
__global__ void __launch_bounds__(TcAttn<G>::THREADS) k_pf_attention_tc(const uint16_t *q, const uint16_t *kc,
                                                                        const uint16_t *vc, uint16_t *out, uint32_t p0,
                                                                        uint32_t M, uint32_t QH, uint32_t KVH) {
  using C = TcAttn<G>;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  TcAttnSmem<G> &s = *reinterpret_cast<TcAttnSmem<G> *>(smem_raw);
  const uint32_t kvh = blockIdx.y, q0 = blockIdx.x * C::QB, tid = threadIdx.x;
  const uint32_t warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const uint32_t nq = min(C::QB, M - q0);
  const uint32_t last = p0 + q0 + nq - 1;
  // q rows: r = g * QB + i (head kvh G + g, query q0 + i); rows past nq are zero
  for (uint32_t e = tid; e < C::ROWS * (kHD / 8); e += C::THREADS) {
    const uint32_t r = e / (kHD / 8), c8 = e % (kHD / 8), g = r / C::QB, i = r % C::QB;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < nq) v = *reinterpret_cast<const uint4 *>(q + (static_cast<size_t>(q0 + i) * QH + kvh * G + g) * kHD + 8 * c8);
    *reinterpret_cast<uint4 *>(&s.q[r][8 * c8]) = v;
  }
  __syncthreads();
  // this warp's rows: row0 .. row0 + 15; the thread holds rows gq and gq + 8
  const uint32_t row0 = warp * 16;
  uint32_t qa[kHD / 16][4];
#pragma unroll
  for (uint32_t kk = 0; kk < kHD / 16; ++kk) {
    qa[kk][0] = lds32(&s.q[row0 + gq][16 * kk + 2 * tq]);
    qa[kk][1] = lds32(&s.q[row0 + gq + 8][16 * kk + 2 * tq]);
    qa[kk][2] = lds32(&s.q[row0 + gq][16 * kk + 8 + 2 * tq]);
    qa[kk][3] = lds32(&s.q[row0 + gq + 8][16 * kk + 8 + 2 * tq]);
  }
  const uint32_t qpos[2] = {p0 + q0 + (row0 + gq) % C::QB, p0 + q0 + (row0 + gq + 8) % C::QB};

  auto stage = [&](uint32_t key0, bool with_v) {
    for (uint32_t e = tid; e < kTcKeys * (kHD / 8); e += C::THREADS) {
      const uint32_t key = e / (kHD / 8), c8 = e % (kHD / 8), pos = key0 + key;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (pos <= last) {
        const size_t off = (static_cast<size_t>(pos) * KVH + kvh) * kHD + 8 * c8;
        kv = *reinterpret_cast<const uint4 *>(kc + off);
        if (with_v) vv = *reinterpret_cast<const uint4 *>(vc + off);
      }
      *reinterpret_cast<uint4 *>(&s.k[key][8 * c8]) = kv;
      if (with_v) {
        const uint16_t *vh = reinterpret_cast<const uint16_t *>(&vv);
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) s.vt[8 * c8 + j][key] = vh[j];
      }
    }
  };
  // scores of this warp's 16 rows x 64 keys: sc[n][c] = n-tile n (keys 8n..),
  // c0/c1 row gq keys 2tq, 2tq + 1; c2/c3 row gq + 8
  auto scores = [&](uint32_t key0, float (&sc)[kTcKeys / 8][4]) {
#pragma unroll
    for (uint32_t n = 0; n < kTcKeys / 8; ++n) {
      sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (uint32_t kk = 0; kk < kHD / 16; ++kk)
        mma_bf16(sc[n], qa[kk], lds32(&s.k[8 * n + gq][16 * kk + 2 * tq]), lds32(&s.k[8 * n + gq][16 * kk + 8 + 2 * tq]));
#pragma unroll
      for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t key = key0 + 8 * n + 2 * tq + (c & 1);
        sc[n][c] = key <= qpos[c >> 1] ? round_bf16(__fmul_rn(round_bf16(sc[n][c]), kAttnScale)) : -INFINITY;
      }
    }
  };
  // pass 1: row max and sum of exp over the whole causal context
  float rm[2] = {-INFINITY, -INFINITY}, rl[2] = {0.f, 0.f};
  for (uint32_t key0 = 0; key0 <= last; key0 += kTcKeys) {
    __syncthreads();
    stage(key0, false);
    __syncthreads();
    float sc[kTcKeys / 8][4];
    scores(key0, sc);
#pragma unroll
    for (uint32_t h = 0; h < 2; ++h) {
      float m = -INFINITY;
#pragma unroll
      for (uint32_t n = 0; n < kTcKeys / 8; ++n) m = fmaxf(m, fmaxf(sc[n][2 * h], sc[n][2 * h + 1]));
      m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 1));
      m = fmaxf(m, __shfl_xor_sync(kFullMask, m, 2));
      const float mn = fmaxf(rm[h], m);
      float l = 0.f;
      if (mn != -INFINITY) {
#pragma unroll
        for (uint32_t n = 0; n < kTcKeys / 8; ++n)
#pragma unroll
          for (uint32_t c = 2 * h; c < 2 * h + 2; ++c) l += sc[n][c] == -INFINITY ? 0.f : expf(sc[n][c] - mn);
      }
      l += __shfl_xor_sync(kFullMask, l, 1);
      l += __shfl_xor_sync(kFullMask, l, 2);
      rl[h] = (rm[h] == -INFINITY ? 0.f : rl[h] * expf(rm[h] - mn)) + l;
      rm[h] = mn;
    }
  }
  const float inv[2] = {1.0f / rl[0], 1.0f / rl[1]};
  // pass 2: probabilities and p.v
  float o[kHD / 8][4];
#pragma unroll
  for (uint32_t n = 0; n < kHD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  for (uint32_t key0 = 0; key0 <= last; key0 += kTcKeys) {
    __syncthreads();
    stage(key0, true);
    __syncthreads();
    float sc[kTcKeys / 8][4];
    scores(key0, sc);
#pragma unroll
    for (uint32_t n = 0; n < kTcKeys / 8; ++n)
#pragma unroll
      for (uint32_t c = 0; c < 4; ++c)
        sc[n][c] = sc[n][c] == -INFINITY ? 0.f : round_bf16(__fmul_rn(expf(sc[n][c] - rm[c >> 1]), inv[c >> 1]));
#pragma unroll
    for (uint32_t kk = 0; kk < kTcKeys / 16; ++kk) {
      const uint32_t pa[4] = {pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]), pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]),
                              pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                              pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3])};
#pragma unroll
      for (uint32_t n = 0; n < kHD / 8; ++n)
        mma_bf16(o[n], pa, lds32(&s.vt[8 * n + gq][16 * kk + 2 * tq]), lds32(&s.vt[8 * n + gq][16 * kk + 8 + 2 * tq]));
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < 2; ++h) {
    const uint32_t r = row0 + gq + 8 * h, g = r / C::QB, i = r % C::QB;
    if (i >= nq) continue;
    uint16_t *dst = out + (static_cast<size_t>(q0 + i) * QH + kvh * G + g) * kHD;
#pragma unroll
    for (uint32_t n = 0; n < kHD / 8; ++n)
      *reinterpret_cast<uint32_t *>(dst + 8 * n + 2 * tq) = pack_bf16x2(o[n][2 * h], o[n][2 * h + 1]);
  }
}

template <int G>
cudaError_t launch_attn_tc(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, uint16_t *out, uint32_t p0,
                           uint32_t M, uint32_t QH, uint32_t KVH, cudaStream_t s) {
  using C = TcAttn<G>;
  const size_t smem = sizeof(TcAttnSmem<G>);
  cudaError_t e =
      cudaFuncSetAttribute(k_pf_attention_tc<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  k_pf_attention_tc<G><<<dim3((M + C::QB - 1) / C::QB, KVH), C::THREADS, smem, s>>>(q, kc, vc, out, p0, M, QH, KVH);
  return cudaGetLastError();
}

__global__ void k_pf_swiglu(const uint16_t *gu, uint16_t *h, uint32_t I, uint64_t total) {
  for (uint64_t e = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t m = e / I, i = e % I;
    const float g = bfv(gu, m * 2 * I + 2 * i), u = bfv(gu, m * 2 * I + 2 * i + 1);
    const float act = round_bf16(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
    h[e] = bfb(__fmul_rn(act, u));
  }
}

template <int G>
cudaError_t launch_attn(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, uint16_t *out, uint32_t p0,
                        uint32_t M, uint32_t QH, uint32_t KVH, cudaStream_t s) {
  const size_t smem = sizeof(PfAttnSmem<G>);
  cudaError_t e = cudaFuncSetAttribute(k_pf_attention<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  k_pf_attention<G><<<dim3((M + kPfQ - 1) / kPfQ, KVH), kPfThreads, smem, s>>>(q, kc, vc, out, p0, M, QH, KVH);
  return cudaGetLastError();
}

}  // namespace

cudaError_t prefill_embed(const uint16_t *embed, const uint32_t *tokens, uint16_t *x, uint32_t M, uint32_t H,
                          cudaStream_t s) {
  k_pf_embed<<<M, 128, 0, s>>>(embed, tokens, x, H);
  return cudaGetLastError();
}

cudaError_t prefill_rms(const uint16_t *x, const uint16_t *w, uint16_t *xn, uint32_t M, uint32_t H, float eps,
                        cudaStream_t s) {
  k_pf_rms<<<M, 256, 0, s>>>(x, w, xn, H, eps);
  return cudaGetLastError();
}

cudaError_t prefill_add_rms(uint16_t *x, const uint16_t *y, const uint16_t *w, uint16_t *xn, uint32_t M, uint32_t H,
                            float eps, cudaStream_t s) {
  k_pf_add_rms<<<M, 256, 0, s>>>(x, y, w, xn, H, eps);
  return cudaGetLastError();
}

cudaError_t prefill_heads(const uint16_t *qkv, const uint16_t *q_norm, const uint16_t *k_norm, const uint16_t *cos_t,
                          const uint16_t *sin_t, uint16_t *q, uint16_t *kc, uint16_t *vc, uint32_t p0, uint32_t M,
                          uint32_t QH, uint32_t KVH, float eps, cudaStream_t s) {
  const uint64_t warps = static_cast<uint64_t>(M) * (QH + 2 * KVH);
  k_pf_heads<<<static_cast<uint32_t>((warps + 7) / 8), 256, 0, s>>>(qkv, (QH + 2 * KVH) * kHD, q_norm, k_norm, cos_t,
                                                                    sin_t, q, kc, vc, p0, M, QH, KVH, eps);
  return cudaGetLastError();
}

cudaError_t prefill_attention(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, uint16_t *out, uint32_t p0,
                              uint32_t M, uint32_t QH, uint32_t KVH, cudaStream_t s, bool tensor_cores) {
  if (tensor_cores) switch (QH / KVH) {
      case 1: return launch_attn_tc<1>(q, kc, vc, out, p0, M, QH, KVH, s);
      case 2: return launch_attn_tc<2>(q, kc, vc, out, p0, M, QH, KVH, s);
      case 4: return launch_attn_tc<4>(q, kc, vc, out, p0, M, QH, KVH, s);
      case 8: return launch_attn_tc<8>(q, kc, vc, out, p0, M, QH, KVH, s);
      default: return cudaErrorInvalidValue;
    }
  switch (QH / KVH) {
    case 1: return launch_attn<1>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 2: return launch_attn<2>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 4: return launch_attn<4>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 8: return launch_attn<8>(q, kc, vc, out, p0, M, QH, KVH, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prefill_swiglu(const uint16_t *gu, uint16_t *h, uint32_t M, uint32_t I, cudaStream_t s) {
  const uint64_t total = static_cast<uint64_t>(M) * I;
  k_pf_swiglu<<<static_cast<uint32_t>(std::min<uint64_t>((total + 255) / 256, 148 * 16)), 256, 0, s>>>(gu, h, I, total);
  return cudaGetLastError();
}

}  // namespace xpu
