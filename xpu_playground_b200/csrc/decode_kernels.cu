// Multi-kernel Qwen3 decode step: one fused kernel per phase, captured into
// a CUDA graph with programmatic dependent launch between them (launch
// order and rounding points are described in decode.cuh). The math lives in
// decode_device.cuh, shared with the persistent path in decode_step.cu.
//
// Cross-CTA reductions (split-K partial sums, attention chunks, argmax) use
// the "last CTA finishes" pattern: each CTA publishes its partial results,
// fences, and bumps an arrival counter; the CTA that sees the final count
// reads every partial in a fixed order (so results never depend on arrival
// order), runs the epilogue and resets the counter for the next replay.
// Nothing in these kernels waits on another CTA.
#include "decode_device.cuh"
#include "xpu_internal.h"

namespace xpu {

namespace {

using namespace dec;

// Prologue of the streamed kernels: barriers, early launch of the next
// kernel, and the producer's whole life. Returns true in consumer threads.
__device__ __forceinline__ bool stream_begin(const StreamSmem &sm, const StreamGeom &g, const CUtensorMap *map,
                                             DecodeState *st) {
  if (!stream_init(sm, g)) {
    grid_dep_launch();
    grid_dep_wait();
    if (threadIdx.x == 0) flag_error(st, kErrPipelineTimeout);
    return false;
  }
  grid_dep_launch();
  if (threadIdx.x < 32) {
    uint32_t it = 0;
    if (threadIdx.x == 0 && !stream_produce(sm, g, map, it)) flag_error(st, kErrPipelineTimeout);
    return false;
  }
  grid_dep_wait();
  return true;
}

// ------------------------------------------------------------ embedding ----
__global__ void __launch_bounds__(256) k_embed(DecodeDims d, DecodeBuffers b) {
  grid_dep_launch();
  const DecodeState *st = b.state;
  const uint32_t pos = st->position;
  uint32_t tok = pos < st->prompt_len ? b.prompt[pos] : st->token;
  if (tok >= d.vocab) {  // a NaN step's sentinel or a bad id: read row 0, flag the state
    if (blockIdx.x == 0 && threadIdx.x == 0) b.state->error |= 1u;
    tok = 0;
  }
  const uint32_t c = blockIdx.x * 256 + threadIdx.x;
  if (c < d.H / 8)
    reinterpret_cast<uint4 *>(b.x)[c] =
        reinterpret_cast<const uint4 *>(b.embed)[static_cast<size_t>(tok) * (d.H / 8) + c];
}

__global__ void __launch_bounds__(kStreamThreads)
k_qkv(DecodeDims d, DecodeBuffers b, LayerWeights w, StreamGeom g, const __grid_constant__ CUtensorMap map) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint8_t s_last[kMaxLocalItems];
  const StreamSmem sm = stream_smem(smem_raw, g, d.H);
  if (!stream_begin(sm, g, &map, b.state)) return;
  const uint32_t pos = b.state->position;
  stage_rms(b.x, w.in_norm, d.H, d.eps, sm.xs, sm.scratch);
  uint32_t it = 0;
  if (!qkv_items(d, b, sm, g, it)) { flag_error(b.state, kErrPipelineTimeout); return; }
  qkv_finish(d, b, w, g, pos, s_last);
}

template <int G>
__global__ void __launch_bounds__(kStreamThreads) k_scores(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  __shared__ AttnShared<G> as;
  grid_dep_launch();
  grid_dep_wait();
  if (threadIdx.x < 32) return;
  const uint32_t n = b.state->position + 1;
  if (blockIdx.y * kPosChunk >= n) return;
  scores_item<G>(d, b, w, blockIdx.x, blockIdx.y, gridDim.y, n, as);
}

template <int G>
__global__ void __launch_bounds__(kStreamThreads) k_pv(DecodeDims d, DecodeBuffers b, LayerWeights w) {
  __shared__ AttnShared<G> as;
  grid_dep_launch();
  grid_dep_wait();
  if (threadIdx.x < 32) return;
  const uint32_t n = b.state->position + 1;
  if (blockIdx.y * kPosChunk >= n) return;
  pv_item<G>(d, b, w, blockIdx.x, blockIdx.y, gridDim.y, n, as);
}

__global__ void __launch_bounds__(kStreamThreads)
k_rowpar(DecodeDims d, DecodeBuffers b, StreamGeom g, const bf16 *xin, const __grid_constant__ CUtensorMap map) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ uint8_t s_last[kMaxLocalItems];
  const uint32_t K_l = g.kt * g.kparts;
  const StreamSmem sm = stream_smem(smem_raw, g, K_l);
  if (!stream_begin(sm, g, &map, b.state)) return;
  stage_copy(xin, K_l, sm.xs);
  uint32_t it = 0;
  if (!rowpar_items(d, b, sm, g, it)) { flag_error(b.state, kErrPipelineTimeout); return; }
  rowpar_finish(d, b, g, s_last);
}

__global__ void __launch_bounds__(kStreamThreads)
k_gateup(DecodeDims d, DecodeBuffers b, LayerWeights w, StreamGeom g, const __grid_constant__ CUtensorMap map) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const StreamSmem sm = stream_smem(smem_raw, g, d.H);
  if (!stream_begin(sm, g, &map, b.state)) return;
  stage_rms(b.x, w.post_norm, d.H, d.eps, sm.xs, sm.scratch);
  uint32_t it = 0;
  if (!gateup_items(d, b, sm, g, it)) flag_error(b.state, kErrPipelineTimeout);
}

__global__ void __launch_bounds__(kStreamThreads) k_lmhead(DecodeDims d, DecodeBuffers b, StreamGeom g,
                                                           const __grid_constant__ CUtensorMap map) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ LmShared ls;
  const StreamSmem sm = stream_smem(smem_raw, g, d.H);
  if (!stream_begin(sm, g, &map, b.state)) return;
  const uint32_t pos = b.state->position;
  stage_rms(b.x, b.final_norm, d.H, d.eps, sm.xs, sm.scratch);
  uint32_t it = 0;
  if (!lm_items_and_argmax(d, b, sm, g, it, ls, pos, 0)) flag_error(b.state, kErrPipelineTimeout);
}

}  // namespace

uint32_t pos_chunks(uint32_t max_seq) { return (max_seq + kPosChunk - 1) / kPosChunk; }

static uint32_t sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || count <= 0)
      count = 148;
  }
  return static_cast<uint32_t>(count);
}

// One streaming CTA per SM (a 128 KB ring of 32-row stages each).
static uint32_t stream_grid(const StreamGeom &g) {
  const uint32_t cap = sm_count(), items = g.items();
  return items < cap ? items : cap;
}

static StreamGeom lm_geom(const DecodeDims &d, const bf16 *lm_head) {
  return make_geom(lm_head, d.H, 0, d.V_l, d.H, 1);
}

uint32_t lmhead_ctas(const DecodeDims &d) { return stream_grid(lm_geom(d, nullptr)); }

// Tensor map over the whole weight matrix of a geometry: `cols` columns.
static cudaError_t geom_tmap(CUtensorMap *map, const StreamGeom &g, uint64_t cols) {
  return make_tmap_2d_u16(map, g.W, cols, g.rows, g.pitch, g.box, kStageRows);
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
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

static bool items_fit(const StreamGeom &g) {
  return (g.items() + stream_grid(g) - 1) / stream_grid(g) <= kMaxLocalItems;
}

cudaError_t launch_embed(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s) {
  const uint32_t grid = (d.H / 8 + 255) / 256;
  k_embed<<<grid, 256, 0, s>>>(d, b);
  return cudaGetLastError();
}

cudaError_t launch_qkv(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, cudaStream_t s) {
  const uint32_t rows = (d.QH_l + 2 * d.KVH_l) * kHD;
  const StreamGeom g = make_geom(w.wqkv, d.H, 0, rows, d.H / d.qkv_splits, d.qkv_splits);
  CUtensorMap map;
  cudaError_t e = geom_tmap(&map, g, d.H);
  if (e != cudaSuccess) return e;
  if (!items_fit(g)) return cudaErrorInvalidConfiguration;
  return launch_pdl(k_qkv, dim3(stream_grid(g)), dim3(kStreamThreads), stream_smem_bytes(g, d.H), s, d, b, w, g, map);
}

cudaError_t launch_attention(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, cudaStream_t s) {
  const dim3 grid(d.KVH_l, pos_chunks(d.max_seq)), block(kStreamThreads);
  cudaError_t e;
  switch (d.QH_l / d.KVH_l) {
    case 1: e = launch_pdl(k_scores<1>, grid, block, 0, s, d, b, w); return e ? e : launch_pdl(k_pv<1>, grid, block, 0, s, d, b, w);
    case 2: e = launch_pdl(k_scores<2>, grid, block, 0, s, d, b, w); return e ? e : launch_pdl(k_pv<2>, grid, block, 0, s, d, b, w);
    case 4: e = launch_pdl(k_scores<4>, grid, block, 0, s, d, b, w); return e ? e : launch_pdl(k_pv<4>, grid, block, 0, s, d, b, w);
    case 8: e = launch_pdl(k_scores<8>, grid, block, 0, s, d, b, w); return e ? e : launch_pdl(k_pv<8>, grid, block, 0, s, d, b, w);
    default: return cudaErrorInvalidValue;
  }
}

static cudaError_t launch_rowpar(const DecodeDims &d, const DecodeBuffers &b, const bf16 *W, uint32_t K_l,
                                 const bf16 *xin, cudaStream_t s) {
  const StreamGeom g = make_geom(W, K_l, 0, d.H, K_l / d.chunks_l, d.chunks_l);
  CUtensorMap map;
  cudaError_t e = geom_tmap(&map, g, K_l);
  if (e != cudaSuccess) return e;
  if (!items_fit(g)) return cudaErrorInvalidConfiguration;
  return launch_pdl(k_rowpar, dim3(stream_grid(g)), dim3(kStreamThreads), stream_smem_bytes(g, K_l), s, d, b, g, xin,
                    map);
}

cudaError_t launch_oproj(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, cudaStream_t s) {
  return launch_rowpar(d, b, w.wo, d.QH_l * kHD, b.attn, s);
}

cudaError_t launch_down(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, cudaStream_t s) {
  return launch_rowpar(d, b, w.wd, d.I_l, b.h, s);
}

cudaError_t launch_gateup(const DecodeDims &d, const DecodeBuffers &b, const LayerWeights &w, cudaStream_t s) {
  const StreamGeom g = make_geom(w.wgu, d.H, 0, 2 * d.I_l, d.H, 1);
  CUtensorMap map;
  cudaError_t e = geom_tmap(&map, g, d.H);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_gateup, dim3(stream_grid(g)), dim3(kStreamThreads), stream_smem_bytes(g, d.H), s, d, b, w, g,
                    map);
}

cudaError_t launch_lmhead(const DecodeDims &d, const DecodeBuffers &b, cudaStream_t s) {
  const StreamGeom g = lm_geom(d, b.lm_head);
  CUtensorMap map;
  cudaError_t e = geom_tmap(&map, g, d.H);
  if (e != cudaSuccess) return e;
  return launch_pdl(k_lmhead, dim3(stream_grid(g)), dim3(kStreamThreads), stream_smem_bytes(g, d.H), s, d, b, g, map);
}

}  // namespace xpu
