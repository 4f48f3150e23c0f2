// Dense prefill: the prompt's positions go through each layer together, so
// every projection is a tcgen05 GEMM over all of them (C = X . W^T against
// the stored weights) - compute-bound, each weight read once per segment of
// up to kPrefillSegment positions - instead of the decode step's weight
// streaming per position. Around the GEMMs, the small kernels here apply the
// same rounding points as the decode step (those of the transformers Qwen3
// bf16 eager forward):
//   k_pf_embed        x[m] = embed[token[m]]
//   k_pf_rms          xn[m] = bf16(w * bf16(x * RN(1/RN(sqrt(mean(x^2) + eps)))))
//   k_pf_heads        per (position, head) of the raw q/k/v rows: q/k RMSNorm
//                     + RoPE into q / the key cache, v into the value cache
//   k_pf_attention_tc causal GQA attention over the cache for the segment's
//                     queries (mma.sync bf16 products, FP32 accumulation):
//                     s = bf16(bf16(q.k) * scale), exact softmax over the whole
//                     context (two passes: statistics, then probabilities
//                     bf16(exp(s - M) * (1 / S)) and p.v)
//   k_pf_swiglu       h = bf16(bf16(silu(g)) * u) from the interleaved gate/up
// and the row-parallel exchange of o_proj and down (canonical K chunks from
// gemm_chunks_launch, summed in the fixed tree of decode.cuh):
//   k_pf_presum       a rank's own chunks -> its subtree sum (tp 2, 4)
//   k_pf_signal       publishes an epoch after the kernels before it
//   k_pf_reduce_rms   rows this rank owns: x = bf16(x + bf16(tree sum of the
//                     ranks' subtrees, read over NVLink)), xn = RMSNorm(x)
//   k_pf_gather       the other ranks' xn rows, copied in over NVLink
//   k_pf_pick         greedy token of the last position across the ranks'
//                     vocabulary shards
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

// ---------------------------------------------- attention on tensor cores
// Causal GQA attention with the two products on the tensor cores (mma.sync
// m16n8k16, bf16 in, FP32 accumulation): per warp 16 rows (one head, 16
// queries), S = Q K^T for 64 keys at a time, the scores rounded as above,
// exact two-pass softmax (row statistics over the whole context, then bf16
// probabilities that feed P V straight from the S accumulators). K and V
// tiles stay row-major [key][dim] in shared memory, double buffered with
// cp.async (rows past the context zero-filled); fragments come from
// ldmatrix (V's transposed). The heaviest query blocks (most keys) start
// first.
constexpr uint32_t kTcKeys = 64;
constexpr uint32_t kTcRow = kHD + 8;  // bf16 per smem row: 272 bytes, conflict-free ldmatrix rows

template <int G>
struct TcAttn {
  static constexpr uint32_t QB = G >= 4 ? 16 : 64 / G;  // queries per CTA
  static constexpr uint32_t ROWS = G * QB;              // 64 or 128
  static constexpr uint32_t WARPS = ROWS / 16;
  static constexpr uint32_t THREADS = 32 * WARPS;
};

template <int G>
struct TcAttnSmem {
  uint16_t k[2][kTcKeys][kTcRow];
  union {
    uint16_t q[TcAttn<G>::ROWS][kTcRow];  // until the fragments are in registers
    uint16_t v[2][kTcKeys][kTcRow];
  };
};

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t sh_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(sh_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(sh_addr(p)));
}
// 16 bytes global -> shared, or 16 zero bytes when !valid.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sh_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int G>
__global__ void __launch_bounds__(TcAttn<G>::THREADS) k_pf_attention_tc(const uint16_t *q, const uint16_t *kc,
                                                                        const uint16_t *vc, uint16_t *out, uint32_t p0,
                                                                        uint32_t M, uint32_t QH, uint32_t KVH) {
  using C = TcAttn<G>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  TcAttnSmem<G> &s = *reinterpret_cast<TcAttnSmem<G> *>(smem_raw);
  const uint32_t kvh = blockIdx.y, q0 = (gridDim.x - 1 - blockIdx.x) * C::QB, tid = threadIdx.x;
  const uint32_t warp = tid >> 5, lane = tid & 31, gq = lane >> 2, tq = lane & 3;
  const uint32_t nq = min(C::QB, M - q0);
  const uint32_t last = p0 + q0 + nq - 1, tiles = last / kTcKeys + 1;
  // q rows: r = g * QB + i (head kvh G + g, query q0 + i); rows past nq are zero
  for (uint32_t e = tid; e < C::ROWS * (kHD / 8); e += C::THREADS) {
    const uint32_t r = e / (kHD / 8), c8 = e % (kHD / 8), g = r / C::QB, i = r % C::QB;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < nq) v = *reinterpret_cast<const uint4 *>(q + (static_cast<size_t>(q0 + i) * QH + kvh * G + g) * kHD + 8 * c8);
    *reinterpret_cast<uint4 *>(&s.q[r][8 * c8]) = v;
  }
  // K (and V) tile t into buffer t & 1
  auto issue = [&](uint32_t t, bool with_v) {
    const uint32_t key0 = t * kTcKeys, b = t & 1;
    for (uint32_t e = tid; e < kTcKeys * (kHD / 8); e += C::THREADS) {
      const uint32_t key = e / (kHD / 8), c8 = e % (kHD / 8), pos = key0 + key;
      const size_t off = (static_cast<size_t>(pos <= last ? pos : 0) * KVH + kvh) * kHD + 8 * c8;
      cp_async16(&s.k[b][key][8 * c8], kc + off, pos <= last);
      if (with_v) cp_async16(&s.v[b][key][8 * c8], vc + off, pos <= last);
    }
    cp_async_commit();
  };
  issue(0, false);  // pass 1 needs no V: its buffers still hold q
  __syncthreads();
  // this warp's rows: row0 .. row0 + 15; the thread holds rows gq and gq + 8
  const uint32_t row0 = warp * 16;
  uint32_t qa[kHD / 16][4];
#pragma unroll
  for (uint32_t kk = 0; kk < kHD / 16; ++kk)
    ldsm_x4(qa[kk], &s.q[row0 + 8 * ((lane >> 3) & 1) + (lane & 7)][16 * kk + 8 * (lane >> 4)]);
  const uint32_t qpos[2] = {p0 + q0 + (row0 + gq) % C::QB, p0 + q0 + (row0 + gq + 8) % C::QB};
  // ldmatrix row addresses of this lane inside a K / V tile
  const uint32_t k_row = 8 * (lane >> 4) + (lane & 7), k_col = 8 * ((lane >> 3) & 1);
  const uint32_t v_row = 8 * ((lane >> 3) & 1) + (lane & 7), v_col = 8 * (lane >> 4);

  // scores of this warp's 16 rows x 64 keys: sc[n][c] = n-tile n (keys 8n..),
  // c0/c1 row gq keys 2tq, 2tq + 1; c2/c3 row gq + 8
  auto scores = [&](uint32_t t, float (&sc)[kTcKeys / 8][4]) {
    const uint32_t key0 = t * kTcKeys, b = t & 1;
#pragma unroll
    for (uint32_t n = 0; n < kTcKeys / 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (uint32_t kk = 0; kk < kHD / 16; ++kk)
#pragma unroll
      for (uint32_t n = 0; n < kTcKeys / 8; n += 2) {
        uint32_t kb[4];  // b0/b1 of n-tiles n and n + 1
        ldsm_x4(kb, &s.k[b][8 * n + k_row][16 * kk + k_col]);
        mma_bf16(sc[n], qa[kk], kb[0], kb[1]);
        mma_bf16(sc[n + 1], qa[kk], kb[2], kb[3]);
      }
#pragma unroll
    for (uint32_t n = 0; n < kTcKeys / 8; ++n)
#pragma unroll
      for (uint32_t c = 0; c < 4; ++c) {
        const uint32_t key = key0 + 8 * n + 2 * tq + (c & 1);
        sc[n][c] = key <= qpos[c >> 1] ? round_bf16(__fmul_rn(round_bf16(sc[n][c]), kAttnScale)) : -INFINITY;
      }
  };
  // pass 1: row max and sum of exp over the whole causal context
  float rm[2] = {-INFINITY, -INFINITY}, rl[2] = {0.f, 0.f};
  for (uint32_t t = 0; t < tiles; ++t) {
    if (t + 1 < tiles) {
      issue(t + 1, false);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float sc[kTcKeys / 8][4];
    scores(t, sc);
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
    __syncthreads();  // buffer t & 1 is refilled by the next issue
  }
  const float inv[2] = {1.0f / rl[0], 1.0f / rl[1]};
  // pass 2: probabilities and p.v
  float o[kHD / 8][4];
#pragma unroll
  for (uint32_t n = 0; n < kHD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  issue(0, true);
  for (uint32_t t = 0; t < tiles; ++t) {
    if (t + 1 < tiles) {
      issue(t + 1, true);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float sc[kTcKeys / 8][4];
    scores(t, sc);
#pragma unroll
    for (uint32_t n = 0; n < kTcKeys / 8; ++n)
#pragma unroll
      for (uint32_t c = 0; c < 4; ++c)
        sc[n][c] = sc[n][c] == -INFINITY ? 0.f : round_bf16(__fmul_rn(expf(sc[n][c] - rm[c >> 1]), inv[c >> 1]));
    const uint32_t b = t & 1;
#pragma unroll
    for (uint32_t kk = 0; kk < kTcKeys / 16; ++kk) {
      const uint32_t pa[4] = {pack_bf16x2(sc[2 * kk][0], sc[2 * kk][1]), pack_bf16x2(sc[2 * kk][2], sc[2 * kk][3]),
                              pack_bf16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]),
                              pack_bf16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3])};
#pragma unroll
      for (uint32_t n = 0; n < kHD / 8; n += 2) {
        uint32_t vb[4];  // b0/b1 of dim tiles n and n + 1
        ldsm_x4_t(vb, &s.v[b][16 * kk + v_row][8 * n + v_col]);
        mma_bf16(o[n], pa, vb[0], vb[1]);
        mma_bf16(o[n + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();
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

// Row blockIdx.y, outputs 8 v .. 8 v + 7 for v = blockIdx.x * blockDim.x +
// threadIdx.x: two 16-byte loads of interleaved gate/up, one 16-byte store.
__global__ void k_pf_swiglu(const uint16_t *gu, uint16_t *h, uint32_t I) {
  const uint32_t v = blockIdx.x * blockDim.x + threadIdx.x;
  if (8 * v >= I) return;
  const size_t m = blockIdx.y;
  const uint4 *src = reinterpret_cast<const uint4 *>(gu + m * 2 * I + 16 * static_cast<size_t>(v));
  const uint4 w[2] = {src[0], src[1]};
  const uint32_t *p = reinterpret_cast<const uint32_t *>(w);
  uint32_t r[4];
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    float y[2];
#pragma unroll
    for (uint32_t e = 0; e < 2; ++e) {
      const uint32_t pair = p[2 * j + e];  // (gate, up) of output 2 j + e
      const float g = bf16_bits_to_float(pair & 0xffffu), u = bf16_bits_to_float(pair >> 16);
      const float act = round_bf16(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
      y[e] = __fmul_rn(act, u);
    }
    r[j] = pack_bf16x2(y[0], y[1]);
  }
  *reinterpret_cast<uint4 *>(h + m * I + 8 * static_cast<size_t>(v)) = make_uint4(r[0], r[1], r[2], r[3]);
}

// ------------------------------------------------ row-parallel exchange
constexpr long long kPfWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Thread 0: waits until every flag of w reaches w.epoch (bounded); false on
// a timeout, after recording it in *w.err.
__device__ bool wait_all(const PfWait &w) {
  const long long start = clock64();
  for (uint32_t q = 0; q < w.count; ++q)
    while (ld_acquire_sys(w.flag[q]) < w.epoch) {
      if (clock64() - start > kPfWaitCycles) {
        atomicOr(w.err, 1u);
        return false;
      }
      __nanosleep(64);
    }
  return true;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// Bottom-up pairwise tree over t.in[0..n) at element offset off (n a power
// of two up to 8): for 8, ((0 + 1) + (2 + 3)) + ((4 + 5) + (6 + 7)).
__device__ __forceinline__ float4 tree4(const PfTree &t, size_t off) {
  float4 v[kCanonChunks];
#pragma unroll
  for (uint32_t i = 0; i < kCanonChunks; ++i)
    if (i < t.n) v[i] = __ldcg(reinterpret_cast<const float4 *>(t.in[i] + off));
#pragma unroll
  for (uint32_t w = 1; w < kCanonChunks; w <<= 1)
#pragma unroll
    for (uint32_t i = 0; i < kCanonChunks; i += 2 * w)
      if (i + w < t.n) v[i] = add4(v[i], v[i + w]);
  return v[0];
}

__global__ void k_pf_presum(const __grid_constant__ PfTree t, float *out, uint64_t vecs) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < vecs;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    reinterpret_cast<float4 *>(out)[i] = tree4(t, 4 * i);
}

// This rank's writes before this kernel (stream order) become visible to the
// peers that see the flag.
__global__ void k_pf_signal(unsigned long long *flag, unsigned long long epoch) {
  __threadfence_system();
  st_release_sys(flag, epoch);
}

__global__ void k_pf_wait(const __grid_constant__ PfWait w) { wait_all(w); }

// Row row0 + blockIdx.x: o = bf16(tree sum of the inputs' row), x = bf16(x +
// o), xn = RMSNorm(x) with norm.
__global__ void __launch_bounds__(256) k_pf_reduce_rms(const __grid_constant__ PfTree t, const __grid_constant__ PfWait w,
                                                       uint16_t *x, const uint16_t *norm, uint16_t *xn, uint32_t row0,
                                                       uint32_t H, float eps) {
  __shared__ float scratch[32];
  __shared__ int ok;
  if (threadIdx.x == 0) ok = w.count ? wait_all(w) : 1;
  __syncthreads();
  if (!ok) return;
  const size_t m = row0 + blockIdx.x;
  uint16_t *xr = x + m * H;
  for (uint32_t i = 4 * threadIdx.x; i < H; i += 4 * blockDim.x) {
    const float4 o = tree4(t, m * H + i);
    const uint2 xv = *reinterpret_cast<const uint2 *>(xr + i);
    uint2 r;
    r.x = pack_bf16x2(__fadd_rn(bf16_bits_to_float(xv.x & 0xffffu), round_bf16(o.x)),
                      __fadd_rn(bf16_bits_to_float(xv.x >> 16), round_bf16(o.y)));
    r.y = pack_bf16x2(__fadd_rn(bf16_bits_to_float(xv.y & 0xffffu), round_bf16(o.z)),
                      __fadd_rn(bf16_bits_to_float(xv.y >> 16), round_bf16(o.w)));
    *reinterpret_cast<uint2 *>(xr + i) = r;
  }
  __syncthreads();
  rms_row(xr, norm, xn + m * H, H, eps, scratch);
}

// Row blockIdx.x of xn, unless this rank owns it: copied from its owner once
// the owner has published it.
__global__ void __launch_bounds__(128) k_pf_gather(const __grid_constant__ PfGather g, uint16_t *xn, uint32_t H) {
  const uint32_t m = blockIdx.x, q = m / g.rows_per;
  if (q == g.rank || q >= g.tp) return;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const PfWait w{{g.flag[q]}, 1, g.epoch, g.err};
    ok = wait_all(w);
  }
  __syncthreads();
  if (!ok) return;
  const uint4 *src = reinterpret_cast<const uint4 *>(g.src[q] + static_cast<size_t>(m) * H);
  uint4 *dst = reinterpret_cast<uint4 *>(xn + static_cast<size_t>(m) * H);
  for (uint32_t c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = __ldcg(src + c);
}

// One CTA: argmax of this rank's logit row, then (tp > 1) every rank's
// candidate through the lm slots: each rank writes its candidate into slot
// `rank` of every region, then reads all slots of its own.
constexpr uint32_t kPickThreads = 1024;
__global__ void __launch_bounds__(kPickThreads) k_pf_pick(const uint16_t *logits, uint32_t V_l,
                                                          const __grid_constant__ PfPick p, uint32_t *out) {
  __shared__ ArgBest wb[kPickThreads / 32];
  __shared__ uint32_t wbad[kPickThreads / 32];
  ArgBest best{-INFINITY, 0xffffffffu};
  uint32_t bad = 0;
  for (uint32_t i = threadIdx.x; i < V_l; i += kPickThreads) {
    const float v = bf16_bits_to_float(logits[i]);
    bad |= not_finite(v) ? 1u : 0u;
    best = arg_better(best, ArgBest{v, p.v_offset + i});
  }
  best = warp_argbest(best);
  bad = __reduce_or_sync(kFullMask, bad);
  if ((threadIdx.x & 31) == 0) {
    wb[threadIdx.x >> 5] = best;
    wbad[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  best = wb[0];
  for (uint32_t i = 1; i < kPickThreads / 32; ++i) {
    best = arg_better(best, wb[i]);
    bad |= wbad[i];
  }
  if (p.tp > 1) {
    for (uint32_t q = 0; q < p.tp; ++q) {
      LmSlot *slot = p.slots[q] + p.rank;
      slot->value = best.value;
      slot->index = best.index;
      slot->bad = bad;
    }
    __threadfence_system();
    for (uint32_t q = 0; q < p.tp; ++q) st_relaxed_sys64(&(p.slots[q] + p.rank)->epoch, p.epoch);
    const LmSlot *own = p.slots[p.rank];
    PfWait w{};
    for (uint32_t q = 0; q < p.tp; ++q) w.flag[q] = &own[q].epoch;
    w.count = p.tp;
    w.epoch = p.epoch;
    w.err = p.err;
    if (!wait_all(w)) {
      *out = 0xffffffffu;
      return;
    }
    best = ArgBest{-INFINITY, 0xffffffffu};
    bad = 0;
    for (uint32_t q = 0; q < p.tp; ++q) {
      best = arg_better(best, ArgBest{__ldcg(&own[q].value), __ldcg(&own[q].index)});
      bad |= __ldcg(&own[q].bad);
    }
  }
  *out = (bad || best.index == 0xffffffffu) ? 0xffffffffu : best.index;
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

cudaError_t prefill_heads(const uint16_t *qkv, const uint16_t *q_norm, const uint16_t *k_norm, const uint16_t *cos_t,
                          const uint16_t *sin_t, uint16_t *q, uint16_t *kc, uint16_t *vc, uint32_t p0, uint32_t M,
                          uint32_t QH, uint32_t KVH, float eps, cudaStream_t s) {
  const uint64_t warps = static_cast<uint64_t>(M) * (QH + 2 * KVH);
  k_pf_heads<<<static_cast<uint32_t>((warps + 7) / 8), 256, 0, s>>>(qkv, (QH + 2 * KVH) * kHD, q_norm, k_norm, cos_t,
                                                                    sin_t, q, kc, vc, p0, M, QH, KVH, eps);
  return cudaGetLastError();
}

cudaError_t prefill_attention(const uint16_t *q, const uint16_t *kc, const uint16_t *vc, uint16_t *out, uint32_t p0,
                              uint32_t M, uint32_t QH, uint32_t KVH, cudaStream_t s) {
  switch (QH / KVH) {
    case 1: return launch_attn_tc<1>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 2: return launch_attn_tc<2>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 4: return launch_attn_tc<4>(q, kc, vc, out, p0, M, QH, KVH, s);
    case 8: return launch_attn_tc<8>(q, kc, vc, out, p0, M, QH, KVH, s);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prefill_swiglu(const uint16_t *gu, uint16_t *h, uint32_t M, uint32_t I, cudaStream_t s) {
  if (I % 8 || !aligned16(gu) || !aligned16(h)) return cudaErrorInvalidValue;
  k_pf_swiglu<<<dim3((I / 8 + 255) / 256, M), 256, 0, s>>>(gu, h, I);
  return cudaGetLastError();
}

cudaError_t prefill_presum(const PfTree &t, float *out, uint64_t elems, cudaStream_t s) {
  if (elems % 4 || !aligned16(out)) return cudaErrorInvalidValue;
  const uint64_t vecs = elems / 4;
  k_pf_presum<<<static_cast<uint32_t>(std::min<uint64_t>((vecs + 255) / 256, 148 * 8)), 256, 0, s>>>(t, out, vecs);
  return cudaGetLastError();
}

cudaError_t prefill_signal(unsigned long long *flag, unsigned long long epoch, cudaStream_t s) {
  k_pf_signal<<<1, 1, 0, s>>>(flag, epoch);
  return cudaGetLastError();
}

cudaError_t prefill_wait(const PfWait &w, cudaStream_t s) {
  k_pf_wait<<<1, 1, 0, s>>>(w);
  return cudaGetLastError();
}

cudaError_t prefill_reduce_rms(const PfTree &t, const PfWait &w, uint16_t *x, const uint16_t *norm, uint16_t *xn,
                               uint32_t row0, uint32_t rows, uint32_t H, float eps, cudaStream_t s) {
  if (H % 8) return cudaErrorInvalidValue;
  if (rows == 0) return cudaSuccess;
  k_pf_reduce_rms<<<rows, 256, 0, s>>>(t, w, x, norm, xn, row0, H, eps);
  return cudaGetLastError();
}

cudaError_t prefill_gather(const PfGather &g, uint16_t *xn, uint32_t M, uint32_t H, cudaStream_t s) {
  if (H % 8 || g.rows_per == 0) return cudaErrorInvalidValue;
  k_pf_gather<<<M, 128, 0, s>>>(g, xn, H);
  return cudaGetLastError();
}

cudaError_t prefill_pick(const uint16_t *logits, uint32_t V_l, const PfPick &p, uint32_t *out, cudaStream_t s) {
  k_pf_pick<<<1, kPickThreads, 0, s>>>(logits, V_l, p, out);
  return cudaGetLastError();
}

}  // namespace xpu
