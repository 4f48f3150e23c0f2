// Persistent single-kernel Qwen3 decode step.
//
// One cooperative launch per token: exactly one CTA per SM (co-residency is
// what makes the grid barriers below safe), each CTA = the TMA producer warp
// plus 8 consumer warps. The producer streams this CTA's share of every
// weight matrix of every layer - QKV, o_proj, gate/up, down, ..., lm_head -
// through one shared-memory ring, in the order the consumers will need them,
// without ever waiting for the consumers' phases: while the consumers sit in
// a grid barrier or run attention (which reads no weights), the ring keeps
// filling with the next matrix, so HBM never idles between phases and no
// kernel launch, prologue or tail separates them.
//
// Phases per layer (grid barrier after each): qkv (split-K partials),
// attention (per item = kv head x a run of 128-position chunks, one run per
// CTA and kv head at most: the group's q/k norm + RoPE and the cache write,
// scores, then - once every item of the kv head has published its softmax
// statistics, counted on a per-kv-head arrival counter instead of a grid
// barrier - probabilities and partial p.v), o_proj (+ chunk combine in its
// staging, residual by the last CTA of each row tile), gate/up + SwiGLU, down
// (+ residual); then lm_head + argmax. The per-item math is the same code as
// the multi-kernel path (decode_device.cuh), so both give identical bits.
//
// Grid barrier: a monotonic 64-bit arrival counter; barrier k of a step
// completes at bar_base + k * gridDim.x arrivals, where bar_base (in the step
// state) is advanced by the CTA that finishes the step. Waits are bounded
// (kWaitCycles); a timeout sets error bit 4, every other waiter sees it and
// leaves, and the host re-arms the barrier.
//
// Tensor parallelism (tp_size > 1): o_proj and down write this rank's
// canonical-chunk partials into every rank's exchange region (NVLink stores
// through CUDA IPC mappings), each value in a 64-bit word tagged with the
// exchange's epoch, and no barrier follows: each CTA stages the next
// RMSNorm input (stage_residual_rms) waiting word by word until every
// rank's partials have arrived, summing the 8 chunks in canonical order
// with the arithmetic of the single-GPU residual epilogue and staging, so
// every tp_size yields identical bits. (On one GPU the finish-and-barrier
// form above is faster: there the word protocol's extra memory round trips
// cost as much as the barrier they replace.) The lm_head
// candidates are exchanged once per step through epoch-flagged slots and
// combined with the lowest index winning ties.
#include <cstdlib>
#include <vector>

#include "decode_device.cuh"
#include "xpu_internal.h"

namespace xpu {

struct StepGeoms {
  StreamGeom qkv, o, gu, down, lm;
};

struct StepParams {
  DecodeDims d;
  DecodeBuffers b;
  const LayerWeights *layers;  // [n_layers] (device)
  const CUtensorMap *maps;     // [4 * n_layers + 1] (device): qkv, o, gate/up, down per layer; lm_head
  StepGeoms g;
  unsigned long long *bar;     // grid-barrier arrival counter (device)
  unsigned long long *acnt;    // [KVH_l] attention arrival counters (device, monotonic)
  uint32_t n_layers;
  uint32_t x_elems;            // capacity (bf16 elements) of the staging/attention region
  uint64_t *trace;             // optional: [gridDim.x][trace_events] globaltimer stamps
  uint32_t trace_events;
};

struct StepPlan {
  StepParams p;
  LayerWeights *d_layers = nullptr;
  CUtensorMap *d_maps = nullptr;
  unsigned long long *d_bar = nullptr;
  unsigned long long *d_acnt = nullptr;
  uint32_t grid = 0;
  size_t smem = 0;
  int group = 0;
};

namespace {

using namespace dec;

constexpr uint32_t kMaxStepKvHeads = 16;  // kv heads per rank (attention arrival counters)

// XPU_STEP_TRACE=1 records per-CTA phase timestamps (read with xpu_qwen3_trace).
bool trace_enabled() {
  const char *v = getenv("XPU_STEP_TRACE");
  return v && v[0] == '1';
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// The consumer barrier orders every consumer thread's earlier writes before
// the arriving thread, whose fence is cumulative over them: one fence per CTA
// instead of one per thread.
__device__ bool grid_barrier(unsigned long long *counter, unsigned long long target, DecodeState *st, int *flag) {
  consumer_sync();
  if (ctid() == 0) {
    __threadfence();
    atomicAdd(counter, 1ull);
    bool ok = false;
    const long long start = clock64();
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
      if (v >= target) { ok = true; break; }
      if (*reinterpret_cast<volatile uint32_t *>(&st->error) & kErrPipelineTimeout) break;
      if (clock64() - start > kWaitCycles) { atomicOr(&st->error, kErrPipelineTimeout); break; }
    }
    *flag = ok;
  }
  consumer_sync();
  return *flag != 0;
}

template <int G>
__global__ void __launch_bounds__(kStreamThreads, 1) k_step(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint8_t s_last[kMaxLocalItems];
  __shared__ LmShared ls;
  __shared__ int bflag;
  __shared__ int s_fail[kConsumerWarps];
  const DecodeDims &d = p.d;
  const DecodeBuffers &b = p.b;
  DecodeState *st = b.state;
  const StreamSmem sm = stream_smem(smem_raw, p.g.qkv, p.x_elems);
  if (!stream_init(sm, p.g.qkv)) {
    if (threadIdx.x == 0) flag_error(st, kErrPipelineTimeout);
    return;
  }
  if (threadIdx.x < 32) {  // producer: every weight stage of this CTA, in consumption order
    if (threadIdx.x == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (uint32_t l = 0; ok && l < p.n_layers; ++l) {
        ok = stream_produce(sm, p.g.qkv, p.maps + 4 * l, it) && stream_produce(sm, p.g.o, p.maps + 4 * l + 1, it) &&
             stream_produce(sm, p.g.gu, p.maps + 4 * l + 2, it) && stream_produce(sm, p.g.down, p.maps + 4 * l + 3, it);
      }
      if (ok) ok = stream_produce(sm, p.g.lm, p.maps + 4 * p.n_layers, it);
      if (!ok) flag_error(st, kErrPipelineTimeout);
    }
    return;
  }
  const uint32_t pos = st->position, n = pos + 1;
  const unsigned long long bar_base = st->bar_base;
  uint32_t tok = pos < st->prompt_len ? b.prompt[pos] : st->token;
  if (tok >= d.vocab) {
    if (blockIdx.x == 0 && ctid() == 0) flag_error(st, 1u);
    tok = 0;
  }
  const bf16 *x_embed = b.embed + static_cast<size_t>(tok) * d.H;
  if (blockIdx.x == 0)  // the residual stream starts as the embedding row
    for (uint32_t c = ctid(); c < d.H / 8; c += kConsumerThreads)
      reinterpret_cast<uint4 *>(b.x)[c] = reinterpret_cast<const uint4 *>(x_embed)[c];
  StepAttnShared<G> &as = *reinterpret_cast<StepAttnShared<G> *>(sm.xs);
  uint32_t ev = 0;
  auto stamp = [&]() {
    if (p.trace && ctid() == 0 && ev < p.trace_events) p.trace[static_cast<size_t>(blockIdx.x) * p.trace_events + ev] = global_ns();
    ++ev;
  };
  stamp();
  const uint32_t npc = pos_chunks_dev(d.max_seq), nch = (n + kPosChunk - 1) / kPosChunk;
  // Attention items: (kv head, run of cpi chunks), at most one item of a kv
  // head per CTA (ipk <= gridDim.x).
  const uint32_t cpi = (nch + gridDim.x - 1) / gridDim.x, ipk = (nch + cpi - 1) / cpi;
  const uint32_t attn_items = d.KVH_l * ipk;
  if (cpi > kMaxItemChunks || d.KVH_l > kMaxStepKvHeads) {  // the plan rules both out
    if (blockIdx.x == 0 && ctid() == 0) flag_error(st, kErrPipelineTimeout);
    return;
  }
  const bool tp = d.tp_size > 1;
  const unsigned long long x_base = st->x_base;
  uint32_t it = 0, nbar = 0, nx = 0;
  auto barrier = [&]() -> bool {
    ++nbar;
    return grid_barrier(p.bar, bar_base + static_cast<unsigned long long>(nbar) * gridDim.x, st, &bflag);
  };
  // epoch of the next cross-rank exchange (its words carry the low 32 bits)
  auto next_epoch = [&]() -> uint32_t { return static_cast<uint32_t>(x_base + (++nx)); };
  // Attention arrival counters only grow: every item of kv head h arrives
  // once per layer, so layer l of this step completes at base[h] + (l + 1) *
  // ipk. The bases are read before this CTA's first grid barrier; no CTA
  // arrives before passing it, so every CTA reads the same bases.
  __shared__ unsigned long long s_abase[kMaxStepKvHeads];
  if (ctid() < d.KVH_l) s_abase[ctid()] = *reinterpret_cast<volatile unsigned long long *>(p.acnt + ctid());
  consumer_sync();
  for (uint32_t l = 0; l < p.n_layers; ++l) {
    const LayerWeights w = p.layers[l];
    // trace events per layer: [staged, items, finished, barrier] x 6 phases
    // (tensor parallel: layers after the first were staged by the previous
    // layer's down-projection exchange)
    if (!tp || l == 0) stage_rms(l == 0 ? x_embed : b.x, w.in_norm, d.H, d.eps, sm.xs, sm.scratch);
    stamp();
    if (!qkv_items(d, b, sm, p.g.qkv, it)) { flag_error(st, kErrPipelineTimeout); return; }
    stamp();
    stamp();  // (no finishing phase: each attention item finishes its group's heads)
    if (!barrier()) return;
    stamp();
    stamp();
    {
      const unsigned long long full = static_cast<unsigned long long>(l + 1) * ipk;
      for (uint32_t item = blockIdx.x; item < attn_items; item += gridDim.x) {
        const uint32_t kvh = item / ipk, c0 = (item % ipk) * cpi, c1 = min(c0 + cpi, nch);
        if (!attn_item<G>(d, b, w, kvh, c0, c1, npc, n, as, [&]() {
              return grid_barrier(p.acnt + kvh, s_abase[kvh] + full, st, &bflag);
            }))
          return;
      }
    }
    stamp();
    stamp();
    stamp();  // (one attention phase: the trace keeps the stamps of two)
    stamp();
    stamp();
    stamp();
    if (!barrier()) return;
    stamp();
    stage_attn_parts(d, b, p.g.o, npc, n, sm.xs);
    stamp();
    if (tp) {
      const uint32_t ep = next_epoch();
      if (!rowpar_items_tp(d, b, sm, p.g.o, it, 0, ep)) { flag_error(st, kErrPipelineTimeout); return; }
      stamp();
      stamp();
      stamp();  // (no barrier: the staging below waits for the exchanged words themselves)
      if (!stage_residual_rms(d, b, 0, ep, b.x, b.x2, w.post_norm, sm.xs, sm.scratch, s_fail)) return;
    } else {
      if (!rowpar_items(d, b, sm, p.g.o, it)) { flag_error(st, kErrPipelineTimeout); return; }
      stamp();
      rowpar_finish(d, b, p.g.o, s_last);
      stamp();
      if (!barrier()) return;
      stamp();
      stage_rms(b.x, w.post_norm, d.H, d.eps, sm.xs, sm.scratch);
    }
    stamp();
    if (!gateup_items(d, b, sm, p.g.gu, it)) { flag_error(st, kErrPipelineTimeout); return; }
    stamp();
    stamp();
    if (!barrier()) return;
    stamp();
    stage_copy(b.h, d.I_l, sm.xs);
    stamp();
    if (tp) {
      const uint32_t ep = next_epoch();
      if (!rowpar_items_tp(d, b, sm, p.g.down, it, 1, ep)) { flag_error(st, kErrPipelineTimeout); return; }
      stamp();
      stamp();
      stamp();
      const bf16 *next_norm = l + 1 < p.n_layers ? p.layers[l + 1].in_norm : b.final_norm;
      if (!stage_residual_rms(d, b, 1, ep, b.x2, b.x, next_norm, sm.xs, sm.scratch, s_fail)) return;
    } else {
      if (!rowpar_items(d, b, sm, p.g.down, it)) { flag_error(st, kErrPipelineTimeout); return; }
      stamp();
      rowpar_finish(d, b, p.g.down, s_last);
      stamp();
      if (!barrier()) return;
      stamp();
    }
  }
  if (!tp) stage_rms(b.x, b.final_norm, d.H, d.eps, sm.xs, sm.scratch);
  stamp();
  // (tensor parallel: one more exchange, of the lm_head candidates)
  if (!lm_items_and_argmax(d, b, sm, p.g.lm, it, ls, pos, static_cast<uint64_t>(nbar) * gridDim.x,
                           tp ? x_base + nx + 1 : 0, tp ? nx + 1 : 0))
    flag_error(st, kErrPipelineTimeout);
  stamp();
}

template <int G>
cudaError_t launch_g(const StepPlan *plan, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kStreamThreads);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_step<G>, plan->p);
}

template <int G>
const void *step_kernel() {
  return reinterpret_cast<const void *>(k_step<G>);
}

}  // namespace

cudaError_t step_plan_create(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights *layers, uint32_t n_layers,
                             StepPlan **out) {
  *out = nullptr;
  auto plan = new StepPlan();
  StepParams &p = plan->p;
  p.d = d;
  p.b = b;
  p.n_layers = n_layers;
  const uint32_t K_o = d.QH_l * kHD;
  StepGeoms &g = p.g;
  g.qkv = make_geom(layers[0].wqkv, d.H, 0, (d.QH_l + 2 * d.KVH_l) * kHD, d.H / d.qkv_splits, d.qkv_splits);
  g.o = make_geom(layers[0].wo, K_o, 0, d.H, K_o / d.chunks_l, d.chunks_l);
  g.gu = make_geom(layers[0].wgu, d.H, 0, 2 * d.I_l, d.H, 1);
  g.down = make_geom(layers[0].wd, d.I_l, 0, d.H, d.I_l / d.chunks_l, d.chunks_l);
  g.lm = make_geom(b.lm_head, d.H, 0, d.V_l, d.H, 1);
  // One ring for every matrix: slot = the largest stage, as many slots (2-8)
  // as the per-CTA shared memory leaves after the activation/attention
  // region. The ring is how far the producer can run ahead while the
  // consumers are in attention or a barrier, so it gets all the room.
  uint32_t slot = 0;
  for (const StreamGeom *x : {&g.qkv, &g.o, &g.gu, &g.down, &g.lm}) slot = std::max(slot, stage_bytes(*x));
  plan->group = static_cast<int>(d.QH_l / d.KVH_l);
  size_t attn_bytes = 0;
  switch (plan->group) {
    case 1: attn_bytes = sizeof(StepAttnShared<1>); break;
    case 2: attn_bytes = sizeof(StepAttnShared<2>); break;
    case 4: attn_bytes = sizeof(StepAttnShared<4>); break;
    case 8: attn_bytes = sizeof(StepAttnShared<8>); break;
    default: delete plan; return cudaErrorInvalidValue;
  }
  const uint32_t stage_elems = std::max(std::max(d.H, K_o), d.I_l);
  p.x_elems = std::max<uint32_t>(stage_elems, static_cast<uint32_t>((attn_bytes + 1) / 2));

  int dev = 0, sms = 0, smem_optin = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) { delete plan; return e; }
  // Static shared memory of k_step (s_last, LmShared, flags) stays under 1 KB.
  const size_t budget = static_cast<size_t>(smem_optin) - 1024;
  uint32_t nslots = 8;
  while (nslots > 2) {
    g.qkv.slot = slot;
    g.qkv.stages = nslots;
    if (stream_smem_bytes(g.qkv, p.x_elems) <= budget) break;
    --nslots;
  }
  for (StreamGeom *x : {&g.qkv, &g.o, &g.gu, &g.down, &g.lm}) { x->slot = slot; x->stages = nslots; }
  plan->smem = stream_smem_bytes(g.qkv, p.x_elems);

  // Items a CTA owns in one phase must fit the deferred-arrival table; an
  // attention item holds at most kMaxItemChunks chunks of the context.
  plan->grid = static_cast<uint32_t>(sms);
  if (d.KVH_l > kMaxStepKvHeads || (pos_chunks(d.max_seq) + plan->grid - 1) / plan->grid > kMaxItemChunks) {
    delete plan;
    return cudaErrorInvalidConfiguration;
  }
  for (const StreamGeom *x : {&g.qkv, &g.o, &g.down})
    if ((x->items() + plan->grid - 1) / plan->grid > kMaxLocalItems) { delete plan; return cudaErrorInvalidConfiguration; }

  const void *kernel = nullptr;
  switch (plan->group) {
    case 1: kernel = step_kernel<1>(); break;
    case 2: kernel = step_kernel<2>(); break;
    case 4: kernel = step_kernel<4>(); break;
    default: kernel = step_kernel<8>(); break;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan->smem));
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kStreamThreads, plan->smem);
  if (e == cudaSuccess && per_sm < 1) e = cudaErrorCooperativeLaunchTooLarge;
  if (e != cudaSuccess) { delete plan; return e; }

  std::vector<CUtensorMap> maps(4 * n_layers + 1);
  for (uint32_t l = 0; l < n_layers && e == cudaSuccess; ++l) {
    e = make_tmap_2d_u16(&maps[4 * l], layers[l].wqkv, d.H, g.qkv.rows, d.H, g.qkv.box, kStageRows);
    if (e == cudaSuccess) e = make_tmap_2d_u16(&maps[4 * l + 1], layers[l].wo, K_o, d.H, K_o, g.o.box, kStageRows);
    if (e == cudaSuccess) e = make_tmap_2d_u16(&maps[4 * l + 2], layers[l].wgu, d.H, g.gu.rows, d.H, g.gu.box, kStageRows);
    if (e == cudaSuccess) e = make_tmap_2d_u16(&maps[4 * l + 3], layers[l].wd, d.I_l, d.H, d.I_l, g.down.box, kStageRows);
  }
  if (e == cudaSuccess) e = make_tmap_2d_u16(&maps[4 * n_layers], b.lm_head, d.H, d.V_l, d.H, g.lm.box, kStageRows);
  if (e == cudaSuccess) e = cudaMalloc(&plan->d_maps, maps.size() * sizeof(CUtensorMap));
  if (e == cudaSuccess) e = cudaMemcpy(plan->d_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&plan->d_layers, n_layers * sizeof(LayerWeights));
  if (e == cudaSuccess) e = cudaMemcpy(plan->d_layers, layers, n_layers * sizeof(LayerWeights), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && trace_enabled()) {
    p.trace_events = 1 + 24 * n_layers + 2;
    e = cudaMalloc(&p.trace, static_cast<size_t>(plan->grid) * p.trace_events * sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMemset(p.trace, 0, static_cast<size_t>(plan->grid) * p.trace_events * sizeof(uint64_t));
  }
  if (e == cudaSuccess) e = cudaMalloc(&plan->d_bar, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(plan->d_bar, 0, sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMalloc(&plan->d_acnt, d.KVH_l * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(plan->d_acnt, 0, d.KVH_l * sizeof(unsigned long long));
  if (e != cudaSuccess) { step_plan_destroy(plan); return e; }
  p.layers = plan->d_layers;
  p.maps = plan->d_maps;
  p.bar = plan->d_bar;
  p.acnt = plan->d_acnt;
  *out = plan;
  return cudaSuccess;
}

void step_plan_destroy(StepPlan *plan) {
  if (!plan) return;
  if (plan->p.trace) cudaFree(plan->p.trace);
  if (plan->d_maps) cudaFree(plan->d_maps);
  if (plan->d_layers) cudaFree(plan->d_layers);
  if (plan->d_bar) cudaFree(plan->d_bar);
  if (plan->d_acnt) cudaFree(plan->d_acnt);
  delete plan;
}

uint32_t step_grid(const StepPlan *plan) { return plan->grid; }

uint32_t step_trace(const StepPlan *plan, uint64_t *host, uint32_t capacity) {
  const uint32_t n = plan->p.trace ? plan->grid * plan->p.trace_events : 0;
  if (!n || !host) return n;
  cudaMemcpy(host, plan->p.trace, std::min(n, capacity) * sizeof(uint64_t), cudaMemcpyDeviceToHost);
  return n;
}

cudaError_t launch_step(const StepPlan *plan, cudaStream_t s) {
  switch (plan->group) {
    case 1: return launch_g<1>(plan, s);
    case 2: return launch_g<2>(plan, s);
    case 4: return launch_g<4>(plan, s);
    default: return launch_g<8>(plan, s);
  }
}

cudaError_t step_reset(const StepPlan *plan, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(plan->d_bar, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess) return e;
  return cudaMemsetAsync(&plan->p.b.state->bar_base, 0, sizeof(uint64_t), s);
}

}  // namespace xpu
