// Data layout and kernel interface of the fused Qwen3 decode step.
//
// One decode step of one tensor-parallel rank is this launch sequence
// (captured once into a CUDA graph and replayed per token):
//   embed                      x = embed[token]
//   per layer:
//     qkv      RMSNorm(x) -> [Wq;Wk;Wv] GEMV (split-K), last CTA per head:
//              q/k RMSNorm + RoPE, q -> q buffer, k/v -> cache[position]
//     scores   per (kv head, 128-position chunk): s = bf16(bf16(q.k) * scale),
//              chunk max and sum of exp
//     pv       softmax probabilities bf16(exp(s - M) / S), partial sum p*v per
//              chunk, last CTA per kv head sums the chunks -> attn buffer
//     oproj    Wo GEMV over canonical K chunks, last CTA per row tile:
//              x = bf16(x + bf16(sum of chunks))        [TP: exchange first]
//     gateup   RMSNorm(x) -> [gate;up] GEMV, h = bf16(bf16(silu(g)) * u)
//     down     Wd GEMV over canonical K chunks, residual add as oproj
//   lmhead     RMSNorm(x) -> lm_head GEMV, bf16 logits, argmax (lowest index
//              on ties, NaN/Inf -> 0xffffffff), state update
// The rounding points are those of the transformers Qwen3 eager/bf16 forward
// that qwen3/reference.py runs.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace xpu {

constexpr uint32_t kHD = 128;            // head_dim
constexpr uint32_t kCanonChunks = 8;     // K chunks of the row-parallel GEMVs
constexpr uint32_t kPosChunk = 128;      // positions per attention chunk
constexpr uint32_t kDecThreads = 256;    // threads per decode-GEMV CTA
constexpr uint32_t kTileRows = 32;       // rows per streamed row tile (8 warps x 4)
constexpr float kAttnScale = 0.08838834764831845f;  // 1/sqrt(128)

typedef __nv_bfloat16 bf16;

// Device-resident step state. Host writes it for synchronous decode calls;
// the lm_head kernel advances it for device-resident generation.
struct DecodeState {
  uint32_t token;       // input token of the next step (unless position < prompt_len)
  uint32_t position;    // position of the next step
  uint32_t prompt_len;  // positions below this read their token from prompt[]
  uint32_t next;        // greedy token of the last step (0xffffffff on NaN/Inf)
  uint32_t error;       // sticky: 1 = NaN/Inf logits, 2 = exchange timeout
  uint32_t steps;       // completed steps since the last reset
  uint64_t bar_base;    // grid-barrier arrivals before this step (persistent path)
  uint64_t x_base;      // cross-rank exchange epochs before this step (tensor parallel)
};

// ---- tensor-parallel exchange (persistent path, tp_size > 1) ----
// Every rank owns one exchange region in its device memory; every rank
// writes into every region (its own and its peers', the latter over NVLink
// through CUDA IPC mappings):
//   part[2][8][H]   canonical-chunk partials of o_proj (0) and down (1), one
//                   64-bit word per value: the FP32 bits in the low half and
//                   the epoch of the exchange that wrote it in the high half;
//                   rank r writes chunks [8 r / tp, 8 (r + 1) / tp)
//   lm[kMaxTp]      lm[r] = rank r's lm_head candidate for the current step
// Exchange k (1-based) of a step has epoch x_base + k; a step makes
// 2 * layers + 1 of them, so epochs only grow and never need clearing. A
// value and its epoch travel in one aligned 64-bit store, which reaches the
// reader whole (single-copy atomic), so a reader that sees the epoch it
// expects has the value too: no fence, flag or barrier is needed between
// the partial stores and their use. A slot is rewritten only after every
// rank has read it: the next write of slot 0 (1) follows the other slot's
// exchange, whose data every rank produces only after all of its CTAs have
// passed the grid barrier that follows their reads of slot 0 (1).
constexpr uint32_t kMaxTp = 8;

struct LmSlot {
  float value;
  uint32_t index;
  uint32_t bad;
  uint32_t pad;
  unsigned long long epoch;
};

struct TpLinks {
  unsigned long long *part[kMaxTp];   // region base of rank q ([2][8][H] words)
  LmSlot *lm[kMaxTp];                 // lm slots of rank q
};

__host__ __device__ inline size_t tp_region_part_bytes(uint32_t H) { return static_cast<size_t>(2) * 8 * H * 8; }
__host__ __device__ inline size_t tp_region_lm_offset(uint32_t H) { return tp_region_part_bytes(H); }
__host__ __device__ inline size_t tp_region_bytes(uint32_t H) { return tp_region_lm_offset(H) + sizeof(LmSlot) * kMaxTp; }

// ---- dense prefill exchange (prefill.cu) ----
// The row-parallel prefill projections (o_proj, down) are the 8 canonical K
// chunks, each its own FP32 accumulation, summed in one fixed tree
// ((c0 + c1) + (c2 + c3)) + ((c4 + c5) + (c6 + c7)): a rank sums the subtree
// of the chunks it holds, then the owner of each row sums the ranks'
// subtrees, so every tensor-parallel size (1, 2, 4, 8) yields the same bits.
// Tensor parallel: behind the decode exchange, every rank's region holds
//   flag[5]          epochs: subtree sums published (o_proj 0, down 1),
//                    normalised rows published (o_proj 2, down 3), the
//                    other ranks' rows of a segment copied in (4)
//   lm[kMaxTp]       lm_head candidates of the last prompt position
//   part[2][cap][H]  FP32 subtree sums of this rank (o_proj, down)
//   xn[cap][H]       bf16 normalised rows: the owner of a row writes it, the
//                    other ranks copy it in before their next GEMM
// Rows are owned in contiguous runs of ceil(M / tp). Flags only grow (one
// epoch per exchange, the same sequence on every rank), so nothing is cleared.
constexpr uint32_t kPfFlags = 5;
constexpr size_t kPfHeaderBytes = 4096;
constexpr size_t kPfLmOffset = 256;
__host__ __device__ inline size_t pf_region_offset(uint32_t H) { return (tp_region_bytes(H) + 4095) / 4096 * 4096; }
__host__ __device__ inline size_t pf_part_offset(uint32_t H) { return pf_region_offset(H) + kPfHeaderBytes; }
__host__ __device__ inline size_t pf_xn_offset(uint32_t H, uint32_t cap) {
  return pf_part_offset(H) + 2ull * cap * H * sizeof(float);
}
__host__ __device__ inline size_t pf_region_end(uint32_t H, uint32_t cap) {
  return pf_xn_offset(H, cap) + static_cast<size_t>(cap) * H * 2;
}

// Inputs of one tree sum: n (1, 2, 4 or 8) FP32 arrays of the same shape,
// summed as the bottom-up pairwise tree over them in index order.
struct PfTree {
  const float *in[kCanonChunks];
  uint32_t n;
};

// Flags that must reach `epoch` before the data behind them is read (a
// bounded wait; a timeout sets bit 0 of *err and the reader skips its rows).
struct PfWait {
  const unsigned long long *flag[kMaxTp];
  uint32_t count;
  unsigned long long epoch;
  uint32_t *err;
};

// Copy of the other ranks' normalised rows into this rank's xn.
struct PfGather {
  const uint16_t *src[kMaxTp];             // xn of rank q
  const unsigned long long *flag[kMaxTp];  // rank q's "rows published" flag
  unsigned long long epoch;
  uint32_t tp, rank, rows_per;
  uint32_t *err;
};

// Cross-rank greedy pick of the last prompt position.
struct PfPick {
  LmSlot *slots[kMaxTp];  // lm slot array of rank q
  unsigned long long epoch;
  uint32_t tp, rank, v_offset;
  uint32_t *err;
};

struct DecodeDims {
  uint32_t H;           // hidden size
  uint32_t I_l;         // intermediate rows held by this rank
  uint32_t QH_l, KVH_l; // heads held by this rank
  uint32_t vocab;       // full vocabulary (embedding rows)
  uint32_t V_l;         // vocabulary rows held by this rank
  uint32_t v_offset;    // first global vocabulary row of this rank
  uint32_t max_seq;
  uint32_t qkv_splits;  // K splits of the QKV GEMV (fixed per shape)
  uint32_t chunks_l;    // canonical chunks held by this rank (8 / tp_size)
  uint32_t chunk0;      // first canonical chunk of this rank
  uint32_t tp_size, tp_rank;
  float eps;
};

struct LayerWeights {
  const bf16 *in_norm, *post_norm, *q_norm, *k_norm;
  const bf16 *wqkv;  // [(QH_l + 2 KVH_l) * 128][H]
  const bf16 *wo;    // [H][QH_l * 128]
  const bf16 *wgu;   // [2 I_l][H], row 2i = gate i, 2i+1 = up i
  const bf16 *wd;    // [H][I_l]
  bf16 *kcache, *vcache;  // [max_seq][KVH_l][128]
};

struct DecodeBuffers {
  bf16 *x;           // residual stream [H]
  bf16 *x2;          // second residual buffer (tensor parallel: x and x2 alternate)
  bf16 *q;           // [QH_l * 128]
  bf16 *attn;        // attention output [QH_l * 128]
  bf16 *h;           // SwiGLU output [I_l]
  float *part_qkv;   // [qkv_splits][rows_qkv]
  float *part;       // [8][H] canonical-chunk partials (oproj and down share it)
  float *scores;     // [QH_l][max_seq]
  float *stats;      // [QH_l][n_pos_chunks][2]
  float *attn_part;  // [QH_l][n_pos_chunks][128]
  ArgBest *lm_best;  // [lm CTAs]
  uint32_t *lm_bad;  // [lm CTAs]
  uint16_t *logits;  // [V_l] bf16 bits
  unsigned *cnt_qkv; // [heads_qkv]
  unsigned *cnt_attn;// [KVH_l]
  unsigned *cnt_tile;// [H / 32]
  unsigned *cnt_lm;  // [1]
  DecodeState *state;
  const uint32_t *prompt;  // [max_seq]
  uint32_t *log;           // [max_seq] greedy token per position
  const bf16 *cos_t, *sin_t;  // [max_seq][128]
  const bf16 *embed;       // [vocab][H]
  const bf16 *final_norm;
  const bf16 *lm_head;     // [V_l][H]
  TpLinks tp;              // tensor-parallel exchange regions (tp_size > 1)
};

__host__ __device__ inline uint32_t pos_chunks_dev(uint32_t max_seq) { return (max_seq + kPosChunk - 1) / kPosChunk; }

// Launchers (decode_kernels.cu). Each returns the launch error.
cudaError_t launch_embed(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s);
cudaError_t launch_qkv(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                       cudaStream_t s);
cudaError_t launch_attention(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                             cudaStream_t s);
cudaError_t launch_oproj(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                         cudaStream_t s);
cudaError_t launch_gateup(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                          cudaStream_t s);
cudaError_t launch_down(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w,
                        cudaStream_t s);
cudaError_t launch_lmhead(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s);

// Number of CTAs the lm_head kernel launches (sizes lm_best / lm_bad).
uint32_t lmhead_ctas(const DecodeDims &d);

// Persistent single-kernel decode step (decode_step.cu): one cooperative
// CTA per SM runs every layer, with grid barriers between phases.
struct StepPlan;
cudaError_t step_plan_create(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights *layers, uint32_t n_layers,
                             StepPlan **plan);
void step_plan_destroy(StepPlan *plan);
cudaError_t launch_step(const StepPlan *plan, cudaStream_t s);
uint32_t step_grid(const StepPlan *plan);
// Phase timestamps of the last step (XPU_STEP_TRACE=1): returns the count.
uint32_t step_trace(const StepPlan *plan, uint64_t *host, uint32_t capacity);
// Re-arms the grid barrier (after a failed step or on reset).
cudaError_t step_reset(const StepPlan *plan, cudaStream_t s);
uint32_t pos_chunks(uint32_t max_seq);

// Dense prefill exchange kernels (prefill.cu).
cudaError_t prefill_presum(const PfTree &t, float *out, uint64_t elems, cudaStream_t s);
cudaError_t prefill_signal(unsigned long long *flag, unsigned long long epoch, cudaStream_t s);
// Holds the stream until every flag of w reaches its epoch (bounded).
cudaError_t prefill_wait(const PfWait &w, cudaStream_t s);
// Rows [row0, row0 + rows): o = bf16(tree sum), x = bf16(x + o), xn = RMSNorm(x).
cudaError_t prefill_reduce_rms(const PfTree &t, const PfWait &w, uint16_t *x, const uint16_t *norm, uint16_t *xn,
                               uint32_t row0, uint32_t rows, uint32_t H, float eps, cudaStream_t s);
cudaError_t prefill_gather(const PfGather &g, uint16_t *xn, uint32_t M, uint32_t H, cudaStream_t s);
// Greedy token of one logit row (this rank's vocabulary shard), combined
// across ranks when tp > 1: lowest index on ties, 0xffffffff on NaN/Inf.
cudaError_t prefill_pick(const uint16_t *logits, uint32_t V_l, const PfPick &p, uint32_t *out, cudaStream_t s);

}  // namespace xpu
