// Batched Qwen3 decode: up to 16 sequences advance one position per step.
//
// The reference engine decodes one sequence (qwen3/main.cpp:159-226); at
// batch 1 every weight byte feeds one multiply-add, at batch B it feeds B.
// A step streams the weights once for all sequences: each projection is a
// skinny GEMM Y[16 x rows] = X[16 x K] . W^T on the tensor cores
// (tcgen05.mma, M = 128 weight rows, N = 16 sequences, accumulators in
// TMEM), so 16 sequences cost little more HBM time than one. Everything
// that is per sequence (norms, RoPE, the KV cache, attention, argmax) runs
// per sequence with the batch-1 arithmetic.
//
// One step is this CUDA graph (programmatic dependent launch between
// kernels; the GEMMs prefetch weights before waiting on their input):
//   embed_norm                 x[s] = embed[token s], xn[s] = RMSNorm(x[s])
//   per layer:
//     gemm qkv                 operand RMSNorm(x) with input_layernorm (inside
//                              the GEMM for l > 0) -> raw bf16 q/k/v
//     attention                per (kv head, sequence): the group's q/k
//                              RMSNorm + RoPE at the sequence's position, k/v
//                              into the caches, scores, softmax, p.v
//     gemm o_proj              x = bf16(x + bf16(attn . Wo^T)), per-tile sums of x^2
//     gemm gate/up             operand RMSNorm(x) with post_attention_layernorm;
//                              h = bf16(bf16(silu(bf16 g)) * bf16 u)
//     gemm down                x = bf16(x + bf16(h . Wd^T)), per-tile sums of x^2
//   gemm lm_head               operand RMSNorm(x) with the final norm; bf16
//                              logits, per-tile (max, lowest index)
//   argmax                     per sequence: greedy token, state update
//
// HBM layout: weights are the batch-1 engine's (one arena). Activations are
// [16][n] row-major bf16 (row s = sequence s; rows >= batch are never
// written and their GEMM columns never read). The KV cache of layer l is
// [batch capacity][max_seq][kv heads][128]: sequence s at s * max_seq *
// kv_heads * 128 elements from the layer's base, sequence 0 being the
// batch-1 engine's cache.
#pragma once

#include <stdint.h>

#include "decode.cuh"

namespace xpu {

constexpr uint32_t kMaxBatch = 16;  // sequences per step: the N of one tcgen05 MMA

// Per-sequence step state (host writes it for synchronous calls; the argmax
// kernel advances it for device-resident generation).
struct SeqState {
  uint32_t token;       // input token of the next step (unless position < prompt_len)
  uint32_t position;    // position of the next step
  uint32_t prompt_len;  // positions below this read their token from prompt[s][]
  uint32_t next;        // greedy token of the last step (0xffffffff on NaN/Inf)
};

struct BatchDims {
  uint32_t H, I, QH, KVH;  // hidden, intermediate, query heads, kv heads
  uint32_t vocab;           // lm_head rows of this rank (the whole vocabulary on one GPU)
  uint32_t max_seq;
  uint32_t nchunks;        // attention position chunks of max_seq
  uint32_t batch;          // active sequences (1..16)
  float eps;
  uint32_t trace_slot;     // this launch's slot in BatchBuffers::trace
  uint32_t seq_rows;       // cache rows between two sequences: max_seq, or 0 when
                           // every sequence is a position of one prompt (prefill)
  uint32_t tp, rank;       // tensor parallel size and this rank (1, 0 on one GPU)
  uint32_t v_offset;       // first vocabulary row of this rank's lm_head shard
  uint32_t tokens;         // the whole vocabulary (valid token ids)
  uint32_t layers;         // decoder layers (exchanges per step: 2 layers + 1)
};

// Tensor-parallel batched step (tp > 1): QKV, gate/up and the lm_head rows
// are split over the ranks like the batch-1 engine's, o_proj and down over
// their K. Each rank's o_proj / down GEMM writes its FP32 partial Y_r[16][H]
// into its exchange region; once every rank has published the exchange's
// epoch, each rank sums the ranks' partials in rank order and applies the
// residual (x = bf16(x + bf16(sum))) and the per-tile sums of x^2 itself
// (the partial GEMM's last CTA publishes the epoch, the exchange kernel
// starts early under programmatic dependent launch and waits on it). The
// lm_head candidates of every sequence meet the same way. Exchange k (1-based)
// of a step has epoch *xepoch + k; a kernel after the step's argmax adds
// 2 layers + 1, so epochs only grow. Region layout behind the dense prefill
// exchange (decode.cuh): flag[2] (o_proj, down), lm[kMaxTp][16] LmSlot at
// kBatchLmOffset, part[2][16][H] FP32 at kBatchPartOffset.
constexpr size_t kBatchLmOffset = 256;
constexpr size_t kBatchPartOffset = 8192;
inline size_t batch_region_offset(uint32_t H, uint32_t prefill_cap) {
  return (pf_region_end(H, prefill_cap) + 4095) / 4096 * 4096;
}
inline size_t batch_region_end(uint32_t H, uint32_t prefill_cap) {
  return batch_region_offset(H, prefill_cap) + kBatchPartOffset + 2ull * kMaxBatch * H * sizeof(float);
}

struct BatchBuffers {
  bf16 *x;              // [16][H] residual stream
  bf16 *xn;             // [16][H] normalised activations (GEMM operand)
  bf16 *qkv;            // [16][(QH + 2 KVH) * 128] raw q/k/v (QKV GEMM output)
  bf16 *q;              // [16][QH * 128] finished q (chunked-attention path)
  bf16 *attn;           // [16][QH * 128] attention output (GEMM operand)
  bf16 *h;              // [16][I] SwiGLU output (GEMM operand)
  uint16_t *logits;     // [16][vocab] bf16 bits
  float *scores;        // [16][QH][max_seq]
  float *stats;         // [16][QH][nchunks][2]
  float *attn_part;     // [16][QH][nchunks][128]
  float *gemm_part;     // [grid][2][16][128] split-tile partial sums
  float *ssq;           // [H / 128][16] per-tile sums of x^2 of the residual (RMSNorm input)
  unsigned *cnt_tile;   // [max tiles] split-tile arrival counters
  unsigned *cnt_attn;   // [16][KVH] attention chunk arrivals
  ArgBest *cand;        // [16][lm tiles] per-tile argmax candidates
  uint32_t *cand_bad;   // [16][lm tiles] NaN/Inf seen in the tile
  SeqState *seq;        // [16]
  uint32_t *error;      // sticky: 1 = NaN/Inf logits or bad token, 4 = wait timeout
  const uint32_t *prompt;  // [16][max_seq]
  uint32_t *log;           // [16][max_seq] greedy token per position
  const bf16 *cos_t, *sin_t;  // [max_seq][128]
  const bf16 *embed;       // [vocab][H]
  const bf16 *final_norm;  // [H]
  const bf16 *lm_head;     // [vocab][H]
  uint64_t kv_seq_stride;  // elements between two sequences' caches of one layer
  // Step tracing (XPU_BATCH_TRACE=1, else null): per kernel of the step
  // [slot][8] globaltimer ns (see trace_mark in batch_step.cu).
  unsigned long long *trace;
  // tensor parallel (tp > 1): rank q's exchange region parts
  float *xpart[kMaxTp];               // [2][16][H] FP32 partials (o_proj, down)
  unsigned long long *xflag[kMaxTp];  // [2] published epochs
  LmSlot *xlm[kMaxTp];                // [kMaxTp][16] lm_head candidates (slot [rank][sequence])
  unsigned long long *xepoch;         // this rank's exchanges before the current step
  unsigned *xdone;                    // CTAs of the running partial GEMM that have finished
};

constexpr uint32_t kBatchTraceSlots = 512;
constexpr uint32_t kBatchTraceValues = 8;

// Number of 128-row tiles of the lm_head GEMM (sizes cand / cand_bad).
inline uint32_t batch_lm_tiles(uint32_t vocab) { return (vocab + 127) / 128; }
// Most tiles of any GEMM of the step (sizes cnt_tile).
uint32_t batch_max_tiles(const BatchDims &d);
// CTAs of the GEMMs (sizes gemm_part: grid * 2 * 16 * 128 floats).
uint32_t batch_gemm_grid();

// Records one batched step (d.batch sequences) on `s` (graph capture).
// prefill: the d.batch "sequences" are consecutive positions of one prompt
// sharing one cache (d.seq_rows = 0, b.kv_seq_stride = 0); every position's
// k and v are finished and cached before attention reads them.
cudaError_t record_batch_step(const BatchDims &d, const BatchBuffers &b, const LayerWeights *layers,
                              uint32_t n_layers, cudaStream_t s, bool prefill = false);

}  // namespace xpu
