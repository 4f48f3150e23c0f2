// Qwen3 decode engine: weights, KV cache and the per-token CUDA graph.
//
// Replaces the reference's Engine (qwen3/main.cpp:118-329) and the Level Zero
// runtime it drives (qwen3/level_zero_runtime.cpp): instead of 508 launches
// each followed by a host synchronisation, one decode step is a captured
// CUDA graph of 2 + 6 * layers fused kernels (decode.cuh) that reads its
// input token and position from device memory, so prompt processing and
// greedy generation run back to back on the GPU without host round trips.
//
// Tensor parallelism (tp_size > 1) shards q/k/v and gate/up by rows (heads,
// intermediate units), o_proj/down by columns in canonical chunks, and the
// lm_head by vocabulary rows. Ranks are separate processes, one per GPU:
// each exports its exchange region as a CUDA IPC handle, the caller
// all-gathers the handles over its host process group and hands them to
// tp_connect, which maps the peers' regions (NVLink peer access). The
// persistent step kernel then exchanges partials through them.
//
// Batched decode (single GPU): an engine created with a batch capacity B
// holds B sequences' KV caches and steps up to B of them at once through a
// second CUDA graph (batch.cuh) over the same weights.
#include <algorithm>
#include <cmath>
#include <stdexcept>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "batch.cuh"
#include "decode.cuh"
#include "xpu_internal.h"

namespace xpu {

cudaError_t fill_normal_window(uint16_t *dst, uint64_t dst_ld, uint32_t row_step, uint64_t nrows,
                               uint64_t ncols, uint64_t src_cols, uint64_t r0, uint64_t c0,
                               uint64_t seed, uint64_t tag, float stddev, cudaStream_t s);
cudaError_t fill_value16(uint16_t *dst, uint64_t n, uint16_t bits, cudaStream_t s);

namespace {

struct CudaError : std::runtime_error {
  cudaError_t code;
  CudaError(cudaError_t c, const std::string &what)
      : std::runtime_error(what + ": " + cudaGetErrorName(c) + " (" + cudaGetErrorString(c) + ")"), code(c) {}
};

#define CK(expr)                                               \
  do {                                                         \
    cudaError_t e_ = (expr);                                   \
    if (e_ != cudaSuccess) throw CudaError(e_, #expr);         \
  } while (0)

struct InvalidArg : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// A bounded device-side wait gave up (DecodeState::error bit 4).
struct DeviceTimeout : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void check_state_error(uint32_t error) {
  if (error & 4u) throw DeviceTimeout("a decode kernel's bounded wait timed out (device error word " + std::to_string(error) + ")");
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

uint16_t host_bf16(float v) {  // RNE, finite inputs only (constants)
  uint32_t bits;
  std::memcpy(&bits, &v, 4);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<uint16_t>(bits >> 16);
}

// Where (part of) one checkpoint tensor lives on this rank: rows
// [r0, r0 + nr) and columns [c0, c0 + nc) of the global [rows x cols] tensor
// go to dst, row i of the window at dst + i * pitch elements.
struct Placement {
  uint16_t *dst;
  uint64_t pitch;
  uint64_t r0, nr, c0, nc, cols;
};

}  // namespace

class Qwen3Engine {
 public:
  Qwen3Engine(const xpu_qwen3_shape &shape, uint32_t max_seq, int device, uint32_t tp_rank,
              uint32_t tp_size, uint32_t max_batch = 1)
      : shape_(shape), max_seq_(max_seq), device_(device), rank_(tp_rank), tp_(tp_size), batch_cap_(max_batch) {
    validate();
    CK(cudaSetDevice(device_));
    CK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    plan();
    allocate();
    upload_rope();
  }

  ~Qwen3Engine() {
    cudaSetDevice(device_);
    if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
    if (batch_exec_) cudaGraphExecDestroy(batch_exec_);
    for (auto &kv : prefill_exec_) cudaGraphExecDestroy(kv.second);
    if (host_prefill_) cudaFreeHost(host_prefill_);
    if (plan_) step_plan_destroy(plan_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (void *p : peer_regions_) cudaIpcCloseMemHandle(p);
    for (void *p : allocations_) cudaFree(p);
    if (host_state_) cudaFreeHost(host_state_);
    if (host_seq_) cudaFreeHost(host_seq_);
    if (stream_) cudaStreamDestroy(stream_);
  }

  Qwen3Engine(const Qwen3Engine &) = delete;
  Qwen3Engine &operator=(const Qwen3Engine &) = delete;

  // ---------------------------------------------------------- weights ----
  std::vector<std::string> tensor_names() const {
    std::vector<std::string> names{"model.embed_tokens.weight", "model.norm.weight"};
    if (!shape_.tie_word_embeddings) names.push_back("lm_head.weight");
    static const char *suffix[] = {
        "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
        "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
        "self_attn.q_norm.weight", "self_attn.k_norm.weight", "mlp.gate_proj.weight",
        "mlp.up_proj.weight", "mlp.down_proj.weight"};
    for (uint32_t l = 0; l < shape_.num_hidden_layers; ++l)
      for (const char *s : suffix) names.push_back("model.layers." + std::to_string(l) + "." + s);
    return names;
  }

  // Global shape of a checkpoint tensor (rows, cols); vectors are 1 x n.
  void global_shape(const std::string &name, uint64_t &rows, uint64_t &cols) const {
    const uint64_t H = shape_.hidden_size, I = shape_.intermediate_size, V = shape_.vocab_size;
    const uint64_t Q = shape_.num_attention_heads * 128ull, KV = shape_.num_key_value_heads * 128ull;
    rows = 1;
    if (name == "model.embed_tokens.weight" || name == "lm_head.weight") { rows = V; cols = H; return; }
    if (name == "model.norm.weight") { cols = H; return; }
    const std::string suf = layer_suffix(name);
    if (suf == "input_layernorm.weight" || suf == "post_attention_layernorm.weight") { cols = H; return; }
    if (suf == "self_attn.q_norm.weight" || suf == "self_attn.k_norm.weight") { cols = 128; return; }
    if (suf == "self_attn.q_proj.weight") { rows = Q; cols = H; return; }
    if (suf == "self_attn.k_proj.weight" || suf == "self_attn.v_proj.weight") { rows = KV; cols = H; return; }
    if (suf == "self_attn.o_proj.weight") { rows = H; cols = Q; return; }
    if (suf == "mlp.gate_proj.weight" || suf == "mlp.up_proj.weight") { rows = I; cols = H; return; }
    if (suf == "mlp.down_proj.weight") { rows = H; cols = I; return; }
    throw InvalidArg("unknown Qwen3 tensor name: " + name);
  }

  std::vector<Placement> placements(const std::string &name) const {
    uint64_t rows, cols;
    global_shape(name, rows, cols);
    const uint64_t H = d_.H;
    if (name == "model.embed_tokens.weight") return {{embed_, H, 0, rows, 0, cols, cols}};
    if (name == "lm_head.weight") return {{lm_head_, H, d_.v_offset, d_.V_l, 0, cols, cols}};
    if (name == "model.norm.weight") return {{final_norm_, cols, 0, 1, 0, cols, cols}};
    const uint32_t l = layer_index(name);
    const Layer &L = layers_[l];
    const std::string suf = layer_suffix(name);
    const uint64_t qr = d_.QH_l * 128ull, kvr = d_.KVH_l * 128ull;
    if (suf == "input_layernorm.weight") return {{L.in_norm, cols, 0, 1, 0, cols, cols}};
    if (suf == "post_attention_layernorm.weight") return {{L.post_norm, cols, 0, 1, 0, cols, cols}};
    if (suf == "self_attn.q_norm.weight") return {{L.q_norm, cols, 0, 1, 0, cols, cols}};
    if (suf == "self_attn.k_norm.weight") return {{L.k_norm, cols, 0, 1, 0, cols, cols}};
    if (suf == "self_attn.q_proj.weight") return {{L.wqkv, H, rank_ * qr, qr, 0, H, H}};
    if (suf == "self_attn.k_proj.weight") return {{L.wqkv + qr * H, H, rank_ * kvr, kvr, 0, H, H}};
    if (suf == "self_attn.v_proj.weight") return {{L.wqkv + (qr + kvr) * H, H, rank_ * kvr, kvr, 0, H, H}};
    if (suf == "self_attn.o_proj.weight") return {{L.wo, qr, 0, H, rank_ * qr, qr, cols}};
    if (suf == "mlp.gate_proj.weight") return {{L.wgu, 2 * H, rank_ * d_.I_l, d_.I_l, 0, H, H}};
    if (suf == "mlp.up_proj.weight") return {{L.wgu + H, 2 * H, rank_ * d_.I_l, d_.I_l, 0, H, H}};
    if (suf == "mlp.down_proj.weight") return {{L.wd, d_.I_l, 0, H, rank_ * (uint64_t)d_.I_l, d_.I_l, cols}};
    throw InvalidArg("unknown Qwen3 tensor name: " + name);
  }

  uint32_t tensor_tag(const std::string &name) const {
    if (name == "model.embed_tokens.weight") return 0;
    if (name == "model.norm.weight") return 1;
    if (name == "lm_head.weight") return 2;
    static const char *suffix[] = {
        "input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
        "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
        "self_attn.q_norm.weight", "self_attn.k_norm.weight", "mlp.gate_proj.weight",
        "mlp.up_proj.weight", "mlp.down_proj.weight"};
    const std::string suf = layer_suffix(name);
    for (uint32_t j = 0; j < 11; ++j)
      if (suf == suffix[j]) return 3 + 11 * layer_index(name) + j;
    throw InvalidArg("unknown Qwen3 tensor name: " + name);
  }

  // Seeded synthetic checkpoint: norms 1, everything else N(0, stddev).
  void init_synthetic(uint64_t seed, float stddev) {
    CK(cudaSetDevice(device_));
    for (const std::string &name : tensor_names()) {
      const bool norm = name.size() >= 11 && name.compare(name.size() - 11, 11, "norm.weight") == 0;
      for (const Placement &p : placements(name)) {
        if (norm) {
          CK(fill_value16(p.dst, p.nc, host_bf16(1.0f), stream_));
        } else {
          CK(fill_normal_window(p.dst, p.pitch, 1, p.nr, p.nc, p.cols, p.r0, p.c0, seed,
                                tensor_tag(name), stddev, stream_));
        }
      }
    }
    CK(cudaStreamSynchronize(stream_));
    loaded_ = true;
  }

  // Copy (this rank's part of) a full tensor from host memory.
  void set_tensor(const std::string &name, const uint16_t *host, uint64_t elements) {
    CK(cudaSetDevice(device_));
    uint64_t rows, cols;
    global_shape(name, rows, cols);
    if (elements != rows * cols)
      throw InvalidArg("tensor " + name + " has " + std::to_string(rows * cols) + " elements, got " +
                       std::to_string(elements));
    for (const Placement &p : placements(name))
      CK(cudaMemcpy2DAsync(p.dst, p.pitch * 2, host + p.r0 * p.cols + p.c0, p.cols * 2, p.nc * 2, p.nr,
                           cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
    ++tensors_set_;
    if (tensors_set_ >= tensor_names().size()) loaded_ = true;
  }

  void mark_loaded() { loaded_ = true; }

  // Streams this rank's part of every tensor of a safetensors checkpoint
  // directory (validated against the engine's shape) to the GPU: file reads
  // into two pinned 64 MiB staging buffers alternate with their host->device
  // copies, so reading and copying overlap.
  void load_checkpoint(const std::string &dir) {
    xpu_qwen3_shape cfg{};
    read_qwen3_config(dir, &cfg, nullptr);
    auto same = [&](const char *what, double a, double b) {
      if (a != b)
        throw InvalidArg(std::string("checkpoint config does not match the engine: ") + what + " is " +
                         std::to_string(a) + ", engine has " + std::to_string(b));
    };
    same("hidden_size", cfg.hidden_size, shape_.hidden_size);
    same("intermediate_size", cfg.intermediate_size, shape_.intermediate_size);
    same("num_hidden_layers", cfg.num_hidden_layers, shape_.num_hidden_layers);
    same("num_attention_heads", cfg.num_attention_heads, shape_.num_attention_heads);
    same("num_key_value_heads", cfg.num_key_value_heads, shape_.num_key_value_heads);
    same("vocab_size", cfg.vocab_size, shape_.vocab_size);
    same("tie_word_embeddings", cfg.tie_word_embeddings, shape_.tie_word_embeddings);
    same("rms_norm_eps", cfg.rms_norm_eps, shape_.rms_norm_eps);
    same("rope_theta", cfg.rope_theta, shape_.rope_theta);
    std::vector<CkptTensor> tensors;
    try {
      tensors = index_qwen3_checkpoint(dir, shape_);
    } catch (const std::runtime_error &e) {
      throw InvalidArg(e.what());
    }
    CK(cudaSetDevice(device_));
    constexpr uint64_t kStaging = 64ull << 20;
    struct Staging {
      uint8_t *buf = nullptr;
      cudaEvent_t done = nullptr;
    } st[2];
    auto release = [&] {
      for (Staging &x : st) {
        if (x.done) cudaEventSynchronize(x.done), cudaEventDestroy(x.done);
        if (x.buf) cudaFreeHost(x.buf);
      }
    };
    try {
      for (Staging &x : st) {
        CK(cudaMallocHost(&x.buf, kStaging));
        CK(cudaEventCreateWithFlags(&x.done, cudaEventDisableTiming));
        CK(cudaEventRecord(x.done, stream_));
      }
      int k = 0;
      for (const CkptTensor &t : tensors) {
        FileReader file(t.path);
        for (const Placement &p : placements(t.name)) {
          const uint64_t row_bytes = p.cols * 2;
          const bool whole_rows = p.c0 == 0 && p.nc == p.cols && p.pitch == p.cols;
          const uint64_t rows_per = std::max<uint64_t>(1, kStaging / row_bytes);
          if (row_bytes > kStaging) throw InvalidArg("tensor row larger than the staging buffer: " + t.name);
          for (uint64_t r = 0; r < p.nr; r += rows_per) {
            const uint64_t rows = std::min(rows_per, p.nr - r);
            Staging &x = st[k];
            k ^= 1;
            CK(cudaEventSynchronize(x.done));  // the buffer's previous copy has finished
            file.read(x.buf, rows * row_bytes, t.offset + (p.r0 + r) * row_bytes);
            if (whole_rows)
              CK(cudaMemcpyAsync(p.dst + r * p.cols, x.buf, rows * row_bytes, cudaMemcpyHostToDevice, stream_));
            else
              CK(cudaMemcpy2DAsync(p.dst + r * p.pitch, p.pitch * 2, x.buf + p.c0 * 2, row_bytes, p.nc * 2, rows,
                                   cudaMemcpyHostToDevice, stream_));
            CK(cudaEventRecord(x.done, stream_));
          }
        }
      }
      CK(cudaStreamSynchronize(stream_));
    } catch (...) {
      release();
      throw;
    }
    release();
    loaded_ = true;
  }

  // 0 = persistent single kernel per step (default), 1 = CUDA graph of
  // per-phase kernels. Both compute identical bits.
  void set_mode(int mode) {
    if (mode != 0 && mode != 1) throw InvalidArg("decode mode must be 0 (persistent) or 1 (graph)");
    if (mode == 1 && tp_ > 1) throw InvalidArg("tensor-parallel decode runs in persistent mode (0) only");
    mode_ = mode;
  }

  // ------------------------------------------------- tensor parallel ----
  // CUDA IPC handle of this rank's exchange region.
  void tp_handle(void *out) const {
    if (tp_ == 1) throw InvalidArg("tp_handle: engine is not tensor parallel (tp_size 1)");
    cudaIpcMemHandle_t h;
    CK(cudaSetDevice(device_));
    CK(cudaIpcGetMemHandle(&h, xregion_));
    static_assert(sizeof(h) == XPU_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(out, &h, sizeof(h));
  }

  // Maps every peer's exchange region (handles[q] from rank q; this rank's
  // own entry is not used) and links all regions into the decode buffers.
  void tp_connect(const uint8_t *handles, uint32_t count) {
    if (tp_ == 1) throw InvalidArg("tp_connect: engine is not tensor parallel (tp_size 1)");
    if (count != tp_) throw InvalidArg("tp_connect: expected " + std::to_string(tp_) + " handles, got " + std::to_string(count));
    if (connected_) throw InvalidArg("tp_connect: already connected");
    CK(cudaSetDevice(device_));
    TpLinks links{};
    const uint32_t H = d_.H;
    region_base_.assign(tp_, nullptr);
    for (uint32_t q = 0; q < tp_; ++q) {
      uint8_t *base = xregion_;
      if (q != rank_) {
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + static_cast<size_t>(q) * XPU_TP_HANDLE_BYTES, sizeof(h));
        void *ptr = nullptr;
        CK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        peer_regions_.push_back(ptr);
        base = static_cast<uint8_t *>(ptr);
      }
      region_base_[q] = base;
      links.part[q] = reinterpret_cast<unsigned long long *>(base);
      links.lm[q] = reinterpret_cast<LmSlot *>(base + tp_region_lm_offset(H));
    }
    b_.tp = links;
    connected_ = true;
    if (plan_) {  // parameters hold the decode buffers: rebuild on next use
      step_plan_destroy(plan_);
      plan_ = nullptr;
    }
  }
  int mode() const { return mode_; }

  // ------------------------------------------------------------ decode ----
  // One step: input token at position (qwen3/main.cpp:159-226 Engine::decode).
  uint32_t decode(uint32_t token, uint32_t position) {
    if (position >= max_seq_) throw InvalidArg("position " + std::to_string(position) + " >= maximum sequence " + std::to_string(max_seq_));
    if (token >= shape_.vocab_size) throw InvalidArg("token id outside the vocabulary");
    ensure_graph();
    host_state_->token = token;
    host_state_->position = position;
    host_state_->prompt_len = 0;
    host_state_->error = 0;
    host_state_->steps = 0;
    write_state();
    launch_one(stream_);
    CK(cudaMemcpyAsync(host_state_, state_, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    after_step_check();
    return host_state_->next;
  }

  // Device-resident prompt + greedy generation: prompt[0..n) fed token by
  // token, then n_new greedy tokens; one host synchronisation at the end.
  // Returns the number of generated tokens written to out (stops after EOS
  // when stop_at_eos and the token is 151645 or 151643, main.cpp:345-352).
  uint32_t generate(const uint32_t *prompt, uint32_t n, uint32_t n_new, uint32_t *out, bool stop_at_eos) {
    if (n == 0) throw InvalidArg("at least one prompt token is required");
    if (static_cast<uint64_t>(n) + n_new > max_seq_) throw InvalidArg("prompt plus generation exceeds the maximum sequence");
    for (uint32_t i = 0; i < n; ++i)
      if (prompt[i] >= shape_.vocab_size) throw InvalidArg("prompt token id outside the vocabulary");
    ensure_graph();
    CK(cudaMemcpyAsync(prompt_, prompt, n * sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    *host_state_ = DecodeState{};
    host_state_->prompt_len = n;
    write_state();
    const uint32_t steps = n_new ? n + n_new - 1 : n;
    for (uint32_t i = 0; i < steps; ++i) launch_one(stream_);
    std::vector<uint32_t> log(n + n_new);
    CK(cudaMemcpyAsync(log.data(), log_, (n + n_new) * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(host_state_, state_, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    after_step_check();
    uint32_t count = 0;
    for (uint32_t i = 0; i < n_new; ++i) {
      const uint32_t t = log[n - 1 + i];
      out[count++] = t;
      if (t == 0xffffffffu) break;
      if (stop_at_eos && (t == 151645u || t == 151643u)) break;
    }
    return count;
  }

  // Set the device state without running (for device-resident loops).
  void set_state(uint32_t token, uint32_t position, uint32_t prompt_len) {
    *host_state_ = DecodeState{};
    host_state_->token = token;
    host_state_->position = position;
    host_state_->prompt_len = prompt_len;
    write_state();
    CK(cudaStreamSynchronize(stream_));
  }

  DecodeState get_state() {
    CK(cudaMemcpyAsync(host_state_, state_, sizeof(DecodeState), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    return *host_state_;
  }

  // Enqueue n device-resident steps on `stream` (or the engine's own).
  void enqueue_steps(uint32_t n, cudaStream_t stream) {
    ensure_graph();
    cudaStream_t s = stream ? stream : stream_;
    for (uint32_t i = 0; i < n; ++i) launch_one(s);
  }

  // Greedy tokens of positions [first, first + count) from the step log.
  void token_log(uint32_t first, uint32_t count, uint32_t *host) {
    if (static_cast<uint64_t>(first) + count > max_seq_) throw InvalidArg("token log range exceeds the maximum sequence");
    CK(cudaMemcpyAsync(host, log_ + first, count * sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }

  void logits(uint16_t *host, uint32_t count) {
    if (count > d_.V_l) throw InvalidArg("logit count exceeds this rank's vocabulary rows");
    CK(cudaMemcpyAsync(host, logits_, count * 2ull, cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }

  void sync() { CK(cudaStreamSynchronize(stream_)); }

  uint32_t trace(uint64_t *host, uint32_t capacity) {
    CK(cudaStreamSynchronize(stream_));
    return plan_ ? step_trace(plan_, host, capacity) : 0;
  }

  const DecodeDims &dims() const { return d_; }
  cudaStream_t stream() const { return stream_; }
  uint32_t kernels_per_step() const { return mode_ == 0 ? 1 : 2 + 6 * shape_.num_hidden_layers; }
  uint64_t weight_bytes() const { return weights_bytes_; }
  uint64_t bytes_per_token(uint32_t context) const {
    // weights streamed per step (embedding: one row) + K and V read for
    // `context` positions + the new K/V row written
    const uint64_t H = d_.H;
    uint64_t w = weights_bytes_ - embed_bytes_ + H * 2;
    if (shape_.tie_word_embeddings) w += static_cast<uint64_t>(d_.V_l) * H * 2;
    const uint64_t kv = 2ull * shape_.num_hidden_layers * d_.KVH_l * 128 * 2;
    return w + kv * context;
  }

  // ------------------------------------------------------ batched decode ----
  uint32_t batch_capacity() const { return batch_cap_; }

  // One step of sequences 0..n-1: tokens[s] at positions[s] (each sequence
  // reads and writes its own KV cache); next[s] = its greedy token.
  void batch_decode(uint32_t n, const uint32_t *tokens, const uint32_t *positions, uint32_t *next) {
    check_batch(n);
    for (uint32_t s = 0; s < n; ++s) {
      if (positions[s] >= max_seq_)
        throw InvalidArg("position " + std::to_string(positions[s]) + " >= maximum sequence " + std::to_string(max_seq_));
      if (tokens[s] >= shape_.vocab_size) throw InvalidArg("token id outside the vocabulary");
    }
    ensure_batch(n);
    for (uint32_t s = 0; s < n; ++s) host_seq_[s] = SeqState{tokens[s], positions[s], 0, 0};
    write_batch_state(n);
    CK(cudaGraphLaunch(batch_exec_, stream_));
    read_batch_state(n);
    after_batch_check();
    for (uint32_t s = 0; s < n; ++s) next[s] = host_seq_[s].next;
  }

  // Device-resident prompts + greedy generation for n sequences: prompt s
  // is lens[s] tokens (prompts holds them back to back); every step advances
  // every sequence one position, for max(lens) + n_new - 1 steps, with one
  // host synchronisation at the end. out[s * n_new + i] = generated token i
  // of sequence s; counts[s] as generate() (stops after EOS when asked).
  void batch_generate(uint32_t n, const uint32_t *prompts, const uint32_t *lens, uint32_t n_new, uint32_t *out,
                      uint32_t *counts, bool stop_at_eos) {
    check_batch(n);
    uint32_t steps = 0;
    uint64_t total = 0;
    for (uint32_t s = 0; s < n; ++s) {
      if (lens[s] == 0) throw InvalidArg("at least one prompt token is required per sequence");
      if (static_cast<uint64_t>(lens[s]) + n_new > max_seq_)
        throw InvalidArg("prompt plus generation exceeds the maximum sequence");
      for (uint32_t i = 0; i < lens[s]; ++i)
        if (prompts[total + i] >= shape_.vocab_size) throw InvalidArg("prompt token id outside the vocabulary");
      total += lens[s];
      steps = std::max(steps, n_new ? lens[s] + n_new - 1 : lens[s]);
    }
    ensure_batch(n);
    uint64_t off = 0;
    for (uint32_t s = 0; s < n; ++s) {
      CK(cudaMemcpyAsync(bprompt_ + static_cast<uint64_t>(s) * max_seq_, prompts + off, lens[s] * 4ull,
                         cudaMemcpyHostToDevice, stream_));
      off += lens[s];
      host_seq_[s] = SeqState{0, 0, lens[s], 0};
    }
    write_batch_state(n);
    for (uint32_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(batch_exec_, stream_));
    std::vector<uint32_t> log(static_cast<size_t>(n) * max_seq_);
    for (uint32_t s = 0; s < n; ++s)
      CK(cudaMemcpyAsync(log.data() + static_cast<size_t>(s) * max_seq_, blog_ + static_cast<size_t>(s) * max_seq_,
                         (lens[s] + n_new) * 4ull, cudaMemcpyDeviceToHost, stream_));
    read_batch_state(n);
    after_batch_check();
    for (uint32_t s = 0; s < n; ++s) {
      uint32_t count = 0;
      for (uint32_t i = 0; i < n_new; ++i) {
        const uint32_t t = log[static_cast<size_t>(s) * max_seq_ + lens[s] - 1 + i];
        out[static_cast<size_t>(s) * n_new + count++] = t;
        if (t == 0xffffffffu) break;
        if (stop_at_eos && (t == 151645u || t == 151643u)) break;
      }
      counts[s] = count;
    }
  }

  // Chunked prefill of the batch-1 sequence: prompt[0..n) goes through the
  // batched step 16 positions at a time (each position one "sequence" of a
  // batch sharing the batch-1 KV cache, so the projections are tcgen05
  // GEMMs over 16 tokens instead of 16 GEMV passes). The batch-1 state is
  // then set to continue at position n with the greedy token after the
  // prompt, which is returned (qwen3/main.cpp:343-344 feeds the prompt
  // token by token instead). Single GPU only.
  uint32_t prefill(const uint32_t *prompt, uint32_t n) {
    if (tp_ > 1) throw InvalidArg("chunked prefill runs on one GPU (tp_size 1)");
    if (n == 0) throw InvalidArg("at least one prompt token is required");
    if (n > max_seq_) throw InvalidArg("prompt exceeds the maximum sequence");
    for (uint32_t i = 0; i < n; ++i)
      if (prompt[i] >= shape_.vocab_size) throw InvalidArg("prompt token id outside the vocabulary");
    if (!loaded_) throw InvalidArg("no weights: call init_synthetic, load a checkpoint or set every tensor");
    if (!bb_.x) allocate_batch();
    CK(cudaSetDevice(device_));
    const uint32_t chunks = (n + kMaxBatch - 1) / kMaxBatch;
    if (prefill_cap_ < chunks) {
      if (host_prefill_) CK(cudaFreeHost(host_prefill_));
      host_prefill_ = nullptr;
      CK(cudaMallocHost(&host_prefill_, static_cast<size_t>(chunks) * kMaxBatch * sizeof(SeqState)));
      prefill_cap_ = chunks;
    }
    CK(cudaStreamSynchronize(stream_));  // the staging area may still feed an earlier call
    *host_berr_ = 0;
    CK(cudaMemcpyAsync(bb_.error, host_berr_, sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    uint32_t last = 0;
    for (uint32_t k = 0; k < chunks; ++k) {
      const uint32_t c = std::min<uint32_t>(kMaxBatch, n - k * kMaxBatch);
      SeqState *st = host_prefill_ + static_cast<size_t>(k) * kMaxBatch;
      for (uint32_t s = 0; s < c; ++s) st[s] = SeqState{prompt[k * kMaxBatch + s], k * kMaxBatch + s, 0, 0};
      CK(cudaMemcpyAsync(bb_.seq, st, c * sizeof(SeqState), cudaMemcpyHostToDevice, stream_));
      CK(cudaGraphLaunch(prefill_graph(c), stream_));
      last = c - 1;
    }
    SeqState tail{};
    CK(cudaMemcpyAsync(&tail, bb_.seq + last, sizeof(SeqState), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(host_berr_, bb_.error, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
    after_batch_check();
    if (*host_berr_ & 1u) throw InvalidArg("prefill met a NaN/Inf logit or an invalid token");
    *host_state_ = DecodeState{};
    host_state_->token = tail.next;
    host_state_->next = tail.next;
    host_state_->position = n;
    write_state();
    CK(cudaMemcpyAsync(log_ + (n - 1), &tail.next, sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
    CK(cudaStreamSynchronize(stream_));
    return tail.next;
  }

  // Dense prefill (compute-bound): the prompt's positions go through each
  // layer together, in segments of up to kPrefillSegment positions, the
  // projections as tcgen05 GEMMs against the stored weights (prefill.cu);
  // then the lm_head GEMV and greedy pick of the last position. o_proj and
  // down are the canonical K chunks summed in a fixed tree (decode.cuh), so
  // every tensor-parallel size computes the same bits: under tensor
  // parallelism each rank sums its own chunks, the owner of each row sums the
  // ranks' subtrees over NVLink, and the normalised rows are copied to the
  // other ranks before the next GEMM. Leaves the engine at position n with
  // the greedy token after the prompt, which is returned, and the last
  // position's logits (this rank's vocabulary shard) in logits().
  static constexpr uint32_t kPrefillSegment = 2048;
  uint32_t prefill_cap() const { return std::min(max_seq_, kPrefillSegment); }

  uint32_t dense_prefill(const uint32_t *prompt, uint32_t n) {
    if (n == 0) throw InvalidArg("at least one prompt token is required");
    if (n > max_seq_) throw InvalidArg("prompt exceeds the maximum sequence");
    for (uint32_t i = 0; i < n; ++i)
      if (prompt[i] >= shape_.vocab_size) throw InvalidArg("prompt token id outside the vocabulary");
    if (!loaded_) throw InvalidArg("no weights: call init_synthetic, load a checkpoint or set every tensor");
    if (broken_)
      throw InvalidArg("a tensor-parallel exchange timed out earlier: destroy and recreate the engines on every rank");
    if (tp_ > 1 && !connected_) throw InvalidArg("tensor-parallel engine not connected: call xpu_qwen3_tp_connect");
    CK(cudaSetDevice(device_));
    const uint32_t H = d_.H, I = d_.I_l, QH = d_.QH_l, KVH = d_.KVH_l, R = (QH + 2 * KVH) * kHD;
    const uint32_t cap = prefill_cap(), chunks_l = d_.chunks_l;
    const uint64_t plane = static_cast<uint64_t>(cap) * H;
    if (!pf_x_) {
      pf_x_ = dev_alloc<uint16_t>(plane);
      pf_big_ = dev_alloc<uint16_t>(static_cast<uint64_t>(cap) * std::max(R, 2 * I));
      pf_h_ = dev_alloc<uint16_t>(static_cast<uint64_t>(cap) * I);
      pf_q_ = dev_alloc<uint16_t>(static_cast<uint64_t>(cap) * QH * kHD);
      pf_att_ = dev_alloc<uint16_t>(static_cast<uint64_t>(cap) * QH * kHD);
      // canonical-chunk partials (at tp 8 each rank holds one chunk, which
      // the GEMM writes straight into the exchange region)
      if (tp_ == 1 || chunks_l > 1) pf_chunks_ = dev_alloc<float>(chunks_l * plane);
      pf_xn_ = tp_ == 1 ? dev_alloc<uint16_t>(plane)
                        : reinterpret_cast<uint16_t *>(xregion_ + pf_xn_offset(H, cap));
      pf_tok_ = dev_alloc<uint32_t>(cap + 1);
      pf_err_ = dev_alloc<uint32_t>(1);
      CK(cudaMemset(pf_err_, 0, sizeof(uint32_t)));
    }
    const float eps = d_.eps;
    cudaStream_t s = stream_;
    for (uint32_t p0 = 0; p0 < n; p0 += cap) {
      const uint32_t M = std::min(cap, n - p0);
      const uint32_t rows_per = (M + tp_ - 1) / tp_;
      const uint32_t row0 = std::min(M, rank_ * rows_per), rows = std::min(M, row0 + rows_per) - row0;
      // Row-parallel projection `which` (0 o_proj, 1 down) of A [M][K_l]
      // against W [H][K_l], then x += its sum over all chunks and xn =
      // RMSNorm(x) with `norm`, for every row on every rank.
      auto rowpar = [&](uint32_t which, const uint16_t *A, const uint16_t *W, uint32_t K_l, const uint16_t *norm) {
        const uint32_t Kc = K_l / chunks_l;
        PfTree tree{};
        PfWait wait{};
        if (tp_ == 1) {
          CK(gemm_chunks_launch(A, W, pf_chunks_, M, H, Kc, chunks_l, s));
          tree.n = chunks_l;
          for (uint32_t c = 0; c < chunks_l; ++c) tree.in[c] = pf_chunks_ + c * static_cast<uint64_t>(M) * H;
          CK(prefill_reduce_rms(tree, wait, pf_x_, norm, pf_xn_, 0, M, H, eps, s));
          return;
        }
        const unsigned long long epoch = ++pf_epoch_;
        float *mine = pf_part(rank_, which);
        if (chunks_l == 1) {
          CK(gemm_chunks_launch(A, W, mine, M, H, Kc, 1, s));
        } else {
          CK(gemm_chunks_launch(A, W, pf_chunks_, M, H, Kc, chunks_l, s));
          PfTree own{};
          own.n = chunks_l;
          for (uint32_t c = 0; c < chunks_l; ++c) own.in[c] = pf_chunks_ + c * static_cast<uint64_t>(M) * H;
          CK(prefill_presum(own, mine, static_cast<uint64_t>(M) * H, s));
        }
        CK(prefill_signal(pf_flag(rank_, which), epoch, s));
        tree.n = tp_;
        wait.count = tp_;
        wait.epoch = epoch;
        wait.err = pf_err_;
        for (uint32_t q = 0; q < tp_; ++q) {
          tree.in[q] = pf_part(q, which);
          wait.flag[q] = pf_flag(q, which);
        }
        CK(prefill_reduce_rms(tree, wait, pf_x_, norm, pf_xn_, row0, rows, H, eps, s));
        CK(prefill_signal(pf_flag(rank_, 2 + which), epoch, s));
        PfGather g{};
        for (uint32_t q = 0; q < tp_; ++q) {
          g.src[q] = reinterpret_cast<const uint16_t *>(region_base_[q] + pf_xn_offset(H, cap));
          g.flag[q] = pf_flag(q, 2 + which);
        }
        g.epoch = epoch;
        g.tp = tp_;
        g.rank = rank_;
        g.rows_per = rows_per;
        g.err = pf_err_;
        CK(prefill_gather(g, pf_xn_, M, H, s));
      };
      if (tp_ > 1 && p0 > 0) {
        // every rank has copied the previous segment's last rows from this
        // one before this rank overwrites its xn
        PfWait w{};
        w.count = tp_;
        w.epoch = pf_epoch_;
        w.err = pf_err_;
        for (uint32_t q = 0; q < tp_; ++q) w.flag[q] = pf_flag(q, 4);
        CK(prefill_wait(w, s));
      }
      CK(cudaMemcpyAsync(pf_tok_, prompt + p0, M * sizeof(uint32_t), cudaMemcpyHostToDevice, s));
      CK(prefill_embed(embed_, pf_tok_, pf_x_, M, H, s));
      CK(prefill_rms(pf_x_, layers_[0].in_norm, pf_xn_, M, H, eps, s));
      for (size_t l = 0; l < layers_.size(); ++l) {
        const Layer &L = layers_[l];
        CK(gemm_launch_ex(false, true, pf_xn_, L.wqkv, pf_big_, M, R, H, s));
        CK(prefill_heads(pf_big_, L.q_norm, L.k_norm, cos_, sin_, pf_q_, L.kcache, L.vcache, p0, M, QH, KVH, eps, s));
        CK(prefill_attention(pf_q_, L.kcache, L.vcache, pf_att_, p0, M, QH, KVH, s));
        rowpar(0, pf_att_, L.wo, QH * kHD, L.post_norm);
        CK(gemm_launch_ex(false, true, pf_xn_, L.wgu, pf_big_, M, 2 * I, H, s));
        CK(prefill_swiglu(pf_big_, pf_h_, M, I, s));
        rowpar(1, pf_h_, L.wd, I, l + 1 < layers_.size() ? layers_[l + 1].in_norm : final_norm_);
      }
      if (tp_ > 1 && p0 + M < n) CK(prefill_signal(pf_flag(rank_, 4), pf_epoch_, s));
      if (p0 + M == n) {
        const uint16_t *last = pf_xn_ + static_cast<uint64_t>(M - 1) * H;
        CK(gemv_launch(reinterpret_cast<const __nv_bfloat16 *>(lm_head_), reinterpret_cast<const __nv_bfloat16 *>(last),
                       reinterpret_cast<__nv_bfloat16 *>(logits_), d_.V_l, H, s));
        PfPick pick{};
        pick.tp = tp_;
        pick.rank = rank_;
        pick.v_offset = d_.v_offset;
        pick.err = pf_err_;
        if (tp_ > 1) {
          pick.epoch = ++pf_epoch_;
          for (uint32_t q = 0; q < tp_; ++q)
            pick.slots[q] = reinterpret_cast<LmSlot *>(region_base_[q] + pf_region_offset(H) + kPfLmOffset);
        }
        CK(prefill_pick(logits_, d_.V_l, pick, pf_tok_ + cap, s));
      }
    }
    uint32_t next = 0, err = 0;
    CK(cudaMemcpyAsync(&next, pf_tok_ + cap, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(&err, pf_err_, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (take_device_error()) throw DeviceTimeout("a prefill GEMM pipeline timed out");
    if (err) {
      broken_ = true;  // the ranks' exchange epochs may now disagree
      throw DeviceTimeout("a tensor-parallel prefill exchange timed out: destroy and recreate the engines on every rank");
    }
    if (next == 0xffffffffu) throw InvalidArg("prefill met a NaN/Inf logit");
    *host_state_ = DecodeState{};
    host_state_->token = next;
    host_state_->next = next;
    host_state_->position = n;
    write_state();
    CK(cudaMemcpyAsync(log_ + (n - 1), &next, sizeof(uint32_t), cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
    return next;
  }

  // Set sequences 0..n-1 (token, position) without running; enqueue_steps
  // then advances them device-resident.
  void batch_set_state(uint32_t n, const uint32_t *tokens, const uint32_t *positions) {
    check_batch(n);
    for (uint32_t s = 0; s < n; ++s)
      if (positions[s] >= max_seq_ || tokens[s] >= shape_.vocab_size) throw InvalidArg("token or position out of range");
    ensure_batch(n);
    for (uint32_t s = 0; s < n; ++s) host_seq_[s] = SeqState{tokens[s], positions[s], 0, 0};
    write_batch_state(n);
    CK(cudaStreamSynchronize(stream_));
  }

  // Sequences 0..n-1 of the current batch: last greedy token and next position.
  uint32_t batch_get_state(uint32_t n, uint32_t *tokens, uint32_t *positions) {
    if (!batch_exec_ || n > batch_n_) throw InvalidArg("no batch of that size is set up");
    read_batch_state(n);
    for (uint32_t s = 0; s < n; ++s) {
      if (tokens) tokens[s] = host_seq_[s].next;
      if (positions) positions[s] = host_seq_[s].position;
    }
    return *host_berr_;
  }

  void batch_enqueue_steps(uint32_t steps, cudaStream_t stream) {
    if (!batch_exec_) throw InvalidArg("no batch set up: call batch_set_state, batch_decode or batch_generate first");
    cudaStream_t s = stream ? stream : stream_;
    for (uint32_t i = 0; i < steps; ++i) CK(cudaGraphLaunch(batch_exec_, s));
  }

  // Per-kernel timeline of the batched steps since the last call
  // (XPU_BATCH_TRACE=1): [slot][8] globaltimer ns, see BatchBuffers::trace;
  // returns the number of values written (0 when tracing is off). Resets it.
  uint32_t batch_trace(uint64_t *host, uint32_t capacity) {
    if (!btrace_) return 0;
    const uint32_t total = kBatchTraceSlots * kBatchTraceValues;
    const uint32_t n = std::min<uint32_t>(capacity, total);
    CK(cudaStreamSynchronize(stream_));
    if (host && n) CK(cudaMemcpy(host, btrace_, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    std::vector<unsigned long long> init(total, 0);
    for (uint32_t i = 0; i < kBatchTraceSlots; ++i) init[kBatchTraceValues * i] = init[kBatchTraceValues * i + 3] = ~0ull;
    CK(cudaMemcpy(btrace_, init.data(), init.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice));
    return host ? n : 0;
  }

  void batch_logits(uint32_t seq, uint16_t *host, uint32_t count) {
    if (seq >= kMaxBatch) throw InvalidArg("sequence index outside the batch (16 rows)");
    if (!bb_.logits) throw InvalidArg("no batched step has run");
    if (count > bd_.vocab) throw InvalidArg("logit count exceeds the vocabulary rows of this rank");
    CK(cudaMemcpyAsync(host, bb_.logits + static_cast<size_t>(seq) * bd_.vocab, count * 2ull,
                       cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }

  // embed + norm, 5 per layer (qkv, attention, o_proj, gate/up, down), lm_head,
  // argmax; tensor parallel: + 1 exchange per row-parallel GEMM and the epoch
  // update
  uint32_t batch_kernels_per_step() const {
    return tp_ > 1 ? 7 * shape_.num_hidden_layers + 4 : 5 * shape_.num_hidden_layers + 3;
  }

  // Bytes one batched step of n sequences must move: the weights once, plus
  // every sequence's K and V over `context` positions.
  uint64_t batch_bytes_per_step(uint32_t n, uint32_t context) const {
    const uint64_t kv = 2ull * shape_.num_hidden_layers * d_.KVH_l * 128 * 2;
    return bytes_per_token(0) + static_cast<uint64_t>(n) * kv * context;
  }

 private:
  void check_batch(uint32_t n) const {
    if (broken_)
      throw InvalidArg("a tensor-parallel exchange timed out earlier: destroy and recreate the engines on every rank");
    if (tp_ > 1 && !connected_) throw InvalidArg("tensor-parallel engine not connected: call xpu_qwen3_tp_connect");
    if (n < 1 || n > batch_cap_)
      throw InvalidArg("batch of " + std::to_string(n) + " sequences outside [1, " + std::to_string(batch_cap_) +
                       "] (the engine's batch capacity)");
  }

  void write_batch_state(uint32_t n) {
    *host_berr_ = 0;
    CK(cudaMemcpyAsync(bb_.seq, host_seq_, n * sizeof(SeqState), cudaMemcpyHostToDevice, stream_));
    CK(cudaMemcpyAsync(bb_.error, host_berr_, sizeof(uint32_t), cudaMemcpyHostToDevice, stream_));
  }

  void read_batch_state(uint32_t n) {
    CK(cudaMemcpyAsync(host_seq_, bb_.seq, n * sizeof(SeqState), cudaMemcpyDeviceToHost, stream_));
    CK(cudaMemcpyAsync(host_berr_, bb_.error, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream_));
    CK(cudaStreamSynchronize(stream_));
  }

  // A timed-out wait leaves arrival counters mid-count: clear them (and the
  // error word) before reporting, so the next call starts clean.
  void after_batch_check() {
    const uint32_t err = *host_berr_;
    if ((err & 4u) && tp_ > 1) broken_ = true;  // the ranks' exchange epochs may now disagree
    if (err & 4u) {
      CK(cudaMemsetAsync(bb_.cnt_tile, 0, batch_max_tiles(bd_) * sizeof(unsigned), stream_));
      CK(cudaMemsetAsync(bb_.cnt_attn, 0, kMaxBatch * bd_.KVH * sizeof(unsigned), stream_));
      CK(cudaMemsetAsync(bb_.error, 0, sizeof(uint32_t), stream_));
      CK(cudaStreamSynchronize(stream_));
      check_state_error(err);
    }
  }

  template <typename T>
  T *dev_zeros(uint64_t count) {
    T *p = dev_alloc<T>(count);
    CK(cudaMemset(p, 0, std::max<uint64_t>(count * sizeof(T), 16)));
    return p;
  }

  void allocate_batch() {
    CK(cudaSetDevice(device_));
    const auto &s = shape_;
    bd_ = BatchDims{};
    bd_.H = s.hidden_size;
    bd_.I = d_.I_l;  // this rank's share (everything on one GPU)
    bd_.QH = d_.QH_l;
    bd_.KVH = d_.KVH_l;
    bd_.vocab = d_.V_l;
    bd_.tp = tp_;
    bd_.rank = rank_;
    bd_.v_offset = d_.v_offset;
    bd_.tokens = s.vocab_size;
    bd_.layers = s.num_hidden_layers;
    bd_.max_seq = max_seq_;
    bd_.nchunks = pos_chunks(max_seq_);
    bd_.batch = 1;
    bd_.eps = s.rms_norm_eps;
    bd_.seq_rows = max_seq_;
    const uint64_t B = kMaxBatch, H = bd_.H, Q = bd_.QH * 128ull;
    BatchBuffers b{};
    b.x = dev_zeros<bf16>(B * H);
    b.xn = dev_zeros<bf16>(B * H);
    b.qkv = dev_zeros<bf16>(B * (Q + 2ull * bd_.KVH * 128));
    b.q = dev_zeros<bf16>(B * Q);
    b.attn = dev_zeros<bf16>(B * Q);
    b.h = dev_zeros<bf16>(B * bd_.I);
    b.logits = dev_zeros<uint16_t>(B * bd_.vocab);
    b.scores = dev_zeros<float>(B * bd_.QH * max_seq_);
    b.stats = dev_zeros<float>(B * bd_.QH * bd_.nchunks * 2);
    b.attn_part = dev_zeros<float>(B * Q * bd_.nchunks);
    b.gemm_part = dev_zeros<float>(static_cast<uint64_t>(batch_gemm_grid()) * 2 * B * 128);
    b.ssq = dev_zeros<float>((H / 128) * B);
    b.cnt_tile = dev_zeros<unsigned>(batch_max_tiles(bd_));
    b.cnt_attn = dev_zeros<unsigned>(B * bd_.KVH);
    b.cand = dev_zeros<ArgBest>(B * batch_lm_tiles(bd_.vocab));
    b.cand_bad = dev_zeros<uint32_t>(B * batch_lm_tiles(bd_.vocab));
    b.seq = dev_zeros<SeqState>(B);
    b.error = dev_zeros<uint32_t>(1);
    bprompt_ = dev_zeros<uint32_t>(B * max_seq_);
    blog_ = dev_zeros<uint32_t>(B * max_seq_);
    b.prompt = bprompt_;
    b.log = blog_;
    b.cos_t = reinterpret_cast<const bf16 *>(cos_);
    b.sin_t = reinterpret_cast<const bf16 *>(sin_);
    b.embed = reinterpret_cast<const bf16 *>(embed_);
    b.final_norm = reinterpret_cast<const bf16 *>(final_norm_);
    b.lm_head = reinterpret_cast<const bf16 *>(lm_head_);
    b.kv_seq_stride = static_cast<uint64_t>(max_seq_) * bd_.KVH * 128;
    if (tp_ > 1) {
      const size_t off = batch_region_offset(static_cast<uint32_t>(H), prefill_cap());
      for (uint32_t q = 0; q < tp_; ++q) {
        uint8_t *base = region_base_[q] + off;
        b.xflag[q] = reinterpret_cast<unsigned long long *>(base);
        b.xlm[q] = reinterpret_cast<LmSlot *>(base + kBatchLmOffset);
        b.xpart[q] = reinterpret_cast<float *>(base + kBatchPartOffset);
      }
      b.xepoch = dev_zeros<unsigned long long>(1);
      b.xdone = dev_zeros<unsigned>(1);
    }
    const char *trace_env = std::getenv("XPU_BATCH_TRACE");
    if (trace_env && trace_env[0] == '1') {
      b.trace = dev_alloc<unsigned long long>(kBatchTraceSlots * kBatchTraceValues);
      btrace_ = b.trace;
    }
    bb_ = b;
    CK(cudaMallocHost(&host_seq_, kMaxBatch * sizeof(SeqState) + 16));
    host_berr_ = reinterpret_cast<uint32_t *>(host_seq_ + kMaxBatch);
  }

  // The prefill graph for chunks of c positions (built once per c).
  cudaGraphExec_t prefill_graph(uint32_t c) {
    auto it = prefill_exec_.find(c);
    if (it != prefill_exec_.end()) return it->second;
    BatchDims d = bd_;
    d.batch = c;
    d.seq_rows = 0;
    BatchBuffers b = bb_;
    b.kv_seq_stride = 0;
    std::vector<LayerWeights> lw(shape_.num_hidden_layers);
    for (uint32_t l = 0; l < shape_.num_hidden_layers; ++l) lw[l] = layer_weights(l);
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    const cudaError_t rec = record_batch_step(d, b, lw.data(), shape_.num_hidden_layers, stream_, true);
    const cudaError_t end = cudaStreamEndCapture(stream_, &graph);
    if (rec != cudaSuccess || end != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      CK(rec != cudaSuccess ? rec : end);
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(e);
    prefill_exec_[c] = exec;
    return exec;
  }

  // Builds (once per batch size) the batched step graph for n sequences.
  void ensure_batch(uint32_t n) {
    if (!loaded_) throw InvalidArg("no weights: call init_synthetic, load a checkpoint or set every tensor");
    if (!bb_.x) allocate_batch();
    if (batch_exec_ && batch_n_ == n) return;
    CK(cudaSetDevice(device_));
    CK(cudaStreamSynchronize(stream_));
    if (batch_exec_) {
      CK(cudaGraphExecDestroy(batch_exec_));
      batch_exec_ = nullptr;
    }
    bd_.batch = n;
    std::vector<LayerWeights> lw(shape_.num_hidden_layers);
    for (uint32_t l = 0; l < shape_.num_hidden_layers; ++l) lw[l] = layer_weights(l);
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    const cudaError_t rec = record_batch_step(bd_, bb_, lw.data(), shape_.num_hidden_layers, stream_);
    const cudaError_t end = cudaStreamEndCapture(stream_, &graph);
    if (rec != cudaSuccess || end != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      CK(rec != cudaSuccess ? rec : end);
    }
    const cudaError_t e = cudaGraphInstantiate(&batch_exec_, graph, 0);
    cudaGraphDestroy(graph);
    CK(e);
    batch_n_ = n;
  }

  struct Layer {
    uint16_t *in_norm, *post_norm, *q_norm, *k_norm, *wqkv, *wo, *wgu, *wd, *kcache, *vcache;
  };

  static std::string layer_suffix(const std::string &name) {
    const std::string prefix = "model.layers.";
    if (name.compare(0, prefix.size(), prefix) != 0) return "";
    const size_t dot = name.find('.', prefix.size());
    return dot == std::string::npos ? "" : name.substr(dot + 1);
  }

  uint32_t layer_index(const std::string &name) const {
    const std::string prefix = "model.layers.";
    if (name.compare(0, prefix.size(), prefix) != 0) throw InvalidArg("unknown Qwen3 tensor name: " + name);
    const size_t dot = name.find('.', prefix.size());
    const std::string digits = name.substr(prefix.size(), dot - prefix.size());
    if (digits.empty() || digits.find_first_not_of("0123456789") != std::string::npos)
      throw InvalidArg("bad layer index in " + name);
    const unsigned long l = std::stoul(digits);
    if (l >= shape_.num_hidden_layers) throw InvalidArg("layer index out of range in " + name);
    return static_cast<uint32_t>(l);
  }

  void validate() const {
    const auto &s = shape_;
    auto req = [](bool ok, const char *what) {
      if (!ok) throw InvalidArg(std::string("unsupported Qwen3 shape: ") + what);
    };
    req(s.hidden_size > 0 && s.hidden_size % 128 == 0, "hidden_size must be a positive multiple of 128");
    req(s.num_key_value_heads > 0 && s.num_attention_heads % s.num_key_value_heads == 0,
        "num_attention_heads must be a multiple of num_key_value_heads");
    const uint32_t g = s.num_attention_heads / s.num_key_value_heads;
    req(g == 1 || g == 2 || g == 4 || g == 8, "query heads per key/value head must be 1, 2, 4 or 8");
    req(s.intermediate_size > 0 && s.intermediate_size % 64 == 0, "intermediate_size must be a multiple of 64");
    req(s.num_hidden_layers > 0 && s.vocab_size > 0, "layers and vocabulary must be positive");
    req(max_seq_ > 0 && max_seq_ <= 40960, "maximum sequence must be in [1, 40960]");
    req(tp_ == 1 || tp_ == 2 || tp_ == 4 || tp_ == 8, "tensor-parallel size must be 1, 2, 4 or 8");
    req(rank_ < tp_, "tensor-parallel rank out of range");
    req(s.num_key_value_heads % tp_ == 0 && s.num_attention_heads % tp_ == 0,
        "heads must divide evenly across tensor-parallel ranks");
    req(s.intermediate_size % (64 * tp_) == 0, "intermediate_size / tp must be a multiple of 64");
    req(s.vocab_size % tp_ == 0 && (s.vocab_size / tp_) % 2 == 0, "vocabulary must split evenly");
    req(batch_cap_ >= 1 && batch_cap_ <= kMaxBatch, "batch capacity must be in [1, 16]");
  }

  void plan() {
    const auto &s = shape_;
    d_ = DecodeDims{};
    d_.H = s.hidden_size;
    d_.I_l = s.intermediate_size / tp_;
    d_.QH_l = s.num_attention_heads / tp_;
    d_.KVH_l = s.num_key_value_heads / tp_;
    d_.vocab = s.vocab_size;
    d_.V_l = s.vocab_size / tp_;
    d_.v_offset = rank_ * d_.V_l;
    d_.max_seq = max_seq_;
    d_.qkv_splits = d_.H >= 2048 ? d_.H / 1024 : 1;
    d_.chunks_l = kCanonChunks / tp_;
    d_.chunk0 = rank_ * d_.chunks_l;
    d_.tp_size = tp_;
    d_.tp_rank = rank_;
    d_.eps = s.rms_norm_eps;
  }

  template <typename T>
  T *dev_alloc(uint64_t count) {
    void *p = nullptr;
    const cudaError_t e = cudaMalloc(&p, std::max<uint64_t>(count * sizeof(T), 16));
    if (e != cudaSuccess) throw CudaError(e, "cudaMalloc of " + std::to_string(count * sizeof(T)) + " bytes");
    allocations_.push_back(p);
    return static_cast<T *>(p);
  }

  void allocate() {
    const auto &s = shape_;
    const uint64_t H = d_.H, L = s.num_hidden_layers;
    const uint64_t qr = d_.QH_l * 128ull, kvr = d_.KVH_l * 128ull;
    // One weight arena, every tensor 4 KiB aligned (qwen3/model.cpp:481-491).
    struct Item { uint16_t **slot; uint64_t elems; };
    std::vector<Item> items;
    layers_.assign(L, Layer{});
    items.push_back({&embed_, static_cast<uint64_t>(s.vocab_size) * H});
    items.push_back({&final_norm_, H});
    if (!s.tie_word_embeddings) items.push_back({&lm_head_, static_cast<uint64_t>(d_.V_l) * H});
    for (uint64_t l = 0; l < L; ++l) {
      Layer &Y = layers_[l];
      items.push_back({&Y.in_norm, H});
      items.push_back({&Y.post_norm, H});
      items.push_back({&Y.q_norm, 128});
      items.push_back({&Y.k_norm, 128});
      items.push_back({&Y.wqkv, (qr + 2 * kvr) * H});
      items.push_back({&Y.wo, H * qr});
      items.push_back({&Y.wgu, 2ull * d_.I_l * H});
      items.push_back({&Y.wd, H * d_.I_l});
    }
    uint64_t offset = 0;
    std::vector<uint64_t> offsets;
    for (const Item &it : items) {
      offset = align_up(offset, 4096);
      offsets.push_back(offset);
      offset += it.elems * 2;
    }
    weights_bytes_ = offset;
    embed_bytes_ = static_cast<uint64_t>(s.vocab_size) * H * 2;
    uint8_t *arena = dev_alloc<uint8_t>(offset);
    for (size_t i = 0; i < items.size(); ++i) *items[i].slot = reinterpret_cast<uint16_t *>(arena + offsets[i]);
    if (s.tie_word_embeddings) lm_head_ = embed_ + static_cast<uint64_t>(d_.v_offset) * H;

    // [batch capacity][max_seq][kv heads][128] per layer; sequence 0 is the
    // batch-1 path's cache.
    const uint64_t cache_layer = static_cast<uint64_t>(batch_cap_) * max_seq_ * kvr;
    uint16_t *kc = dev_alloc<uint16_t>(cache_layer * L), *vc = dev_alloc<uint16_t>(cache_layer * L);
    CK(cudaMemset(kc, 0, cache_layer * L * 2));
    CK(cudaMemset(vc, 0, cache_layer * L * 2));
    for (uint64_t l = 0; l < L; ++l) {
      layers_[l].kcache = kc + l * cache_layer;
      layers_[l].vcache = vc + l * cache_layer;
    }
    cos_ = dev_alloc<uint16_t>(static_cast<uint64_t>(max_seq_) * 128);
    sin_ = dev_alloc<uint16_t>(static_cast<uint64_t>(max_seq_) * 128);

    const uint32_t npc = pos_chunks(max_seq_);
    const uint64_t rows_qkv = qr + 2 * kvr;
    b_ = DecodeBuffers{};
    b_.x = dev_alloc<bf16>(H);
    b_.x2 = dev_alloc<bf16>(H);
    if (tp_ > 1) {
      // decode exchange, the dense prefill exchange of one segment, the
      // batched step's exchange (every engine accepts batch 1)
      const size_t bytes = batch_region_end(static_cast<uint32_t>(H), prefill_cap());
      xregion_ = dev_alloc<uint8_t>(bytes);
      CK(cudaMemset(xregion_, 0, bytes));
    }
    b_.q = dev_alloc<bf16>(qr);
    b_.attn = dev_alloc<bf16>(qr);
    b_.h = dev_alloc<bf16>(d_.I_l);
    b_.part_qkv = dev_alloc<float>(d_.qkv_splits * rows_qkv);
    b_.part = dev_alloc<float>(kCanonChunks * H);
    b_.scores = dev_alloc<float>(static_cast<uint64_t>(d_.QH_l) * max_seq_);
    b_.stats = dev_alloc<float>(static_cast<uint64_t>(d_.QH_l) * npc * 2);
    b_.attn_part = dev_alloc<float>(static_cast<uint64_t>(d_.QH_l) * npc * 128);
    // lm_head candidates: one per CTA of either decode path (the persistent
    // step runs one CTA per SM, the graph path up to lmhead_ctas).
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_));
    const uint32_t lm_ctas = std::max<uint32_t>(lmhead_ctas(d_), static_cast<uint32_t>(sms));
    b_.lm_best = dev_alloc<ArgBest>(lm_ctas);
    b_.lm_bad = dev_alloc<uint32_t>(lm_ctas);
    logits_ = dev_alloc<uint16_t>(d_.V_l);
    b_.logits = logits_;
    const uint64_t heads_qkv = d_.QH_l + 2ull * d_.KVH_l;
    n_counters_ = heads_qkv + d_.KVH_l + H / kTileRows + 1;
    counters_ = dev_alloc<unsigned>(n_counters_);
    CK(cudaMemset(counters_, 0, n_counters_ * sizeof(unsigned)));
    b_.cnt_qkv = counters_;
    b_.cnt_attn = counters_ + heads_qkv;
    b_.cnt_tile = b_.cnt_attn + d_.KVH_l;
    b_.cnt_lm = b_.cnt_tile + H / kTileRows;
    state_ = dev_alloc<DecodeState>(1);
    CK(cudaMemset(state_, 0, sizeof(DecodeState)));
    b_.state = state_;
    prompt_ = dev_alloc<uint32_t>(max_seq_);
    log_ = dev_alloc<uint32_t>(max_seq_);
    b_.prompt = prompt_;
    b_.log = log_;
    b_.cos_t = reinterpret_cast<const bf16 *>(cos_);
    b_.sin_t = reinterpret_cast<const bf16 *>(sin_);
    b_.embed = reinterpret_cast<const bf16 *>(embed_);
    b_.final_norm = reinterpret_cast<const bf16 *>(final_norm_);
    b_.lm_head = reinterpret_cast<const bf16 *>(lm_head_);
    CK(cudaMallocHost(&host_state_, sizeof(DecodeState)));
  }

  // RoPE tables as transformers builds them (FP32 inv_freq = 1/theta^(2i/128),
  // FP32 angle, FP32 cos/sin, bf16), frequency d % 64 for dimension d.
  void upload_rope() {
    std::vector<uint16_t> c(static_cast<size_t>(max_seq_) * 128), s(c.size());
    float inv[64];
    const float theta = static_cast<float>(shape_.rope_theta);
    for (int i = 0; i < 64; ++i) inv[i] = 1.0f / std::pow(theta, static_cast<float>(2 * i) / 128.0f);
    for (uint32_t p = 0; p < max_seq_; ++p)
      for (uint32_t dd = 0; dd < 128; ++dd) {
        const float angle = static_cast<float>(p) * inv[dd % 64];
        c[static_cast<size_t>(p) * 128 + dd] = host_bf16(std::cos(angle));
        s[static_cast<size_t>(p) * 128 + dd] = host_bf16(std::sin(angle));
      }
    CK(cudaMemcpy(cos_, c.data(), c.size() * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(sin_, s.data(), s.size() * 2, cudaMemcpyHostToDevice));
  }

  LayerWeights layer_weights(uint32_t l) const {
    const Layer &Y = layers_[l];
    auto c = [](const uint16_t *p) { return reinterpret_cast<const bf16 *>(p); };
    return LayerWeights{c(Y.in_norm), c(Y.post_norm), c(Y.q_norm), c(Y.k_norm), c(Y.wqkv), c(Y.wo),
                        c(Y.wgu), c(Y.wd), reinterpret_cast<bf16 *>(Y.kcache),
                        reinterpret_cast<bf16 *>(Y.vcache)};
  }

  void record_step(cudaStream_t s) {
    CK(launch_embed(d_, b_, s));
    for (uint32_t l = 0; l < shape_.num_hidden_layers; ++l) {
      const LayerWeights w = layer_weights(l);
      CK(launch_qkv(d_, b_, w, s));
      CK(launch_attention(d_, b_, w, s));
      CK(launch_oproj(d_, b_, w, s));
      CK(launch_gateup(d_, b_, w, s));
      CK(launch_down(d_, b_, w, s));
    }
    CK(launch_lmhead(d_, b_, s));
  }

  // Host -> device copy of the step inputs (every field before bar_base,
  // which only the device advances).
  void write_state() {
    CK(cudaMemcpyAsync(state_, host_state_, offsetof(DecodeState, bar_base), cudaMemcpyHostToDevice, stream_));
  }

  // A timed-out step leaves the grid barrier mid-count: re-arm it and clear
  // the sticky bit before reporting, so the next call starts clean.
  void after_step_check() {
    const uint32_t err = host_state_->error;
    if ((err & 4u) && tp_ > 1) {
      // The ranks' exchange epochs may now disagree: the engines cannot resume.
      broken_ = true;
      check_state_error(err);
    }
    if (err & 4u) {
      // Re-arm the grid barrier and every arrival counter (a step that gave
      // up can leave any of them mid-count).
      if (plan_) CK(step_reset(plan_, stream_));
      CK(cudaMemsetAsync(counters_, 0, n_counters_ * sizeof(unsigned), stream_));
      host_state_->error = 0;
      write_state();
      CK(cudaStreamSynchronize(stream_));
      check_state_error(err);
    }
  }

  void launch_one(cudaStream_t s) {
    if (mode_ == 0) CK(launch_step(plan_, s));
    else CK(cudaGraphLaunch(graph_exec_, s));
  }

  void ensure_graph() {
    if (!loaded_) throw InvalidArg("no weights: call init_synthetic, load a checkpoint or set every tensor");
    if (broken_)
      throw InvalidArg("a tensor-parallel exchange timed out earlier: destroy and recreate the engines on every rank");
    if (tp_ > 1 && !connected_) throw InvalidArg("tensor-parallel engine not connected: call xpu_qwen3_tp_connect");
    if (tp_ > 1 && mode_ != 0) throw InvalidArg("tensor-parallel decode runs in persistent mode (0) only");
    if (mode_ == 0) {
      if (!plan_) {
        CK(cudaSetDevice(device_));
        std::vector<LayerWeights> lw(shape_.num_hidden_layers);
        for (uint32_t l = 0; l < shape_.num_hidden_layers; ++l) lw[l] = layer_weights(l);
        CK(step_plan_create(d_, b_, lw.data(), shape_.num_hidden_layers, &plan_));
      }
      return;
    }
    if (graph_exec_) return;
    CK(cudaSetDevice(device_));
    cudaGraph_t graph = nullptr;
    CK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
      record_step(stream_);
    } catch (...) {
      cudaStreamEndCapture(stream_, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    CK(cudaStreamEndCapture(stream_, &graph));
    const cudaError_t e = cudaGraphInstantiate(&graph_exec_, graph, 0);
    cudaGraphDestroy(graph);
    CK(e);
  }

  xpu_qwen3_shape shape_;
  uint32_t max_seq_;
  int device_;
  uint32_t rank_, tp_;
  DecodeDims d_{};
  DecodeBuffers b_{};
  cudaStream_t stream_ = nullptr;
  cudaGraphExec_t graph_exec_ = nullptr;
  StepPlan *plan_ = nullptr;
  int mode_ = 0;
  std::vector<void *> allocations_;
  std::vector<Layer> layers_;
  uint16_t *embed_ = nullptr, *final_norm_ = nullptr, *lm_head_ = nullptr;
  uint16_t *cos_ = nullptr, *sin_ = nullptr, *logits_ = nullptr;
  uint32_t *prompt_ = nullptr, *log_ = nullptr;
  DecodeState *state_ = nullptr, *host_state_ = nullptr;
  uint64_t weights_bytes_ = 0, embed_bytes_ = 0;
  size_t tensors_set_ = 0;
  bool loaded_ = false;
  unsigned *counters_ = nullptr;          // every arrival counter of the decode step
  uint64_t n_counters_ = 0;
  uint8_t *xregion_ = nullptr;            // this rank's exchange region (tp_size > 1)
  std::vector<void *> peer_regions_;      // peers' regions mapped through CUDA IPC
  bool connected_ = false, broken_ = false;
  // batched decode
  uint32_t batch_cap_ = 1;
  BatchDims bd_{};
  BatchBuffers bb_{};
  cudaGraphExec_t batch_exec_ = nullptr;
  uint32_t batch_n_ = 0;
  uint32_t *bprompt_ = nullptr, *blog_ = nullptr;
  SeqState *host_seq_ = nullptr;
  uint32_t *host_berr_ = nullptr;
  unsigned long long *btrace_ = nullptr;  // batched step trace (XPU_BATCH_TRACE=1)
  // dense prefill buffers (one segment of up to kPrefillSegment positions);
  // under tensor parallelism xn, the subtree sums and the flags live in the
  // exchange regions (decode.cuh)
  uint16_t *pf_x_ = nullptr, *pf_xn_ = nullptr, *pf_big_ = nullptr, *pf_h_ = nullptr, *pf_q_ = nullptr,
           *pf_att_ = nullptr;
  float *pf_chunks_ = nullptr;            // [chunks_l][M][H] canonical-chunk partials
  uint32_t *pf_tok_ = nullptr, *pf_err_ = nullptr;
  unsigned long long pf_epoch_ = 0;       // prefill exchanges so far (the same on every rank)
  std::vector<uint8_t *> region_base_;    // exchange region of rank q (own or IPC-mapped)
  float *pf_part(uint32_t q, uint32_t which) const {
    return reinterpret_cast<float *>(region_base_[q] + pf_part_offset(d_.H)) +
           static_cast<uint64_t>(which) * prefill_cap() * d_.H;
  }
  unsigned long long *pf_flag(uint32_t q, uint32_t which) const {
    return reinterpret_cast<unsigned long long *>(region_base_[q] + pf_region_offset(d_.H)) + which;
  }
  std::map<uint32_t, cudaGraphExec_t> prefill_exec_;  // chunked-prefill graphs by chunk size
  SeqState *host_prefill_ = nullptr;                 // pinned per-chunk step states
  uint32_t prefill_cap_ = 0;
};

}  // namespace xpu

// ------------------------------------------------------------- C ABI ----
using xpu::Qwen3Engine;

struct xpu_qwen3_engine {
  std::unique_ptr<Qwen3Engine> impl;
};

namespace {

template <typename F>
int guarded(F &&f) {
  try {
    f();
    return XPU_OK;
  } catch (const xpu::CudaError &e) {
    return xpu::fail(e.code == cudaErrorMemoryAllocation ? XPU_ERR_NO_MEMORY : XPU_ERR_CUDA, e.what());
  } catch (const xpu::InvalidArg &e) {
    return xpu::fail(XPU_ERR_INVALID, e.what());
  } catch (const xpu::DeviceTimeout &e) {
    return xpu::fail(XPU_ERR_TIMEOUT, e.what());
  } catch (const std::exception &e) {
    return xpu::fail(XPU_ERR_INVALID, e.what());
  } catch (...) {
    return xpu::fail(XPU_ERR_INVALID, "unknown exception");
  }
}

Qwen3Engine &eng(xpu_qwen3_engine *e) {
  if (!e || !e->impl) throw xpu::InvalidArg("null engine");
  return *e->impl;
}

}  // namespace

extern "C" {

int xpu_qwen3_create(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                     uint32_t tp_rank, uint32_t tp_size, xpu_qwen3_engine **out) {
  return guarded([&] {
    if (!shape || !out) throw xpu::InvalidArg("xpu_qwen3_create: null pointer");
    *out = nullptr;
    auto holder = std::make_unique<xpu_qwen3_engine>();
    holder->impl = std::make_unique<Qwen3Engine>(*shape, maximum_sequence, device, tp_rank, tp_size);
    *out = holder.release();
  });
}

int xpu_qwen3_create_batched(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                             uint32_t max_batch, xpu_qwen3_engine **out) {
  return guarded([&] {
    if (!shape || !out) throw xpu::InvalidArg("xpu_qwen3_create_batched: null pointer");
    *out = nullptr;
    auto holder = std::make_unique<xpu_qwen3_engine>();
    holder->impl = std::make_unique<Qwen3Engine>(*shape, maximum_sequence, device, 0, 1, max_batch);
    *out = holder.release();
  });
}

int xpu_qwen3_create_batched_tp(const xpu_qwen3_shape *shape, uint32_t maximum_sequence, int device,
                                uint32_t tp_rank, uint32_t tp_size, uint32_t max_batch, xpu_qwen3_engine **out) {
  return guarded([&] {
    if (!shape || !out) throw xpu::InvalidArg("xpu_qwen3_create_batched_tp: null pointer");
    *out = nullptr;
    auto holder = std::make_unique<xpu_qwen3_engine>();
    holder->impl = std::make_unique<Qwen3Engine>(*shape, maximum_sequence, device, tp_rank, tp_size, max_batch);
    *out = holder.release();
  });
}

int xpu_qwen3_destroy(xpu_qwen3_engine *engine) {
  return guarded([&] { delete engine; });
}

int xpu_qwen3_tp_handle(xpu_qwen3_engine *engine, void *handle) {
  return guarded([&] {
    if (!handle) throw xpu::InvalidArg("xpu_qwen3_tp_handle: null pointer");
    eng(engine).tp_handle(handle);
  });
}

int xpu_qwen3_tp_connect(xpu_qwen3_engine *engine, const void *handles, uint32_t count) {
  return guarded([&] {
    if (!handles) throw xpu::InvalidArg("xpu_qwen3_tp_connect: null pointer");
    eng(engine).tp_connect(static_cast<const uint8_t *>(handles), count);
  });
}

int xpu_qwen3_load_checkpoint(xpu_qwen3_engine *engine, const char *model_dir) {
  return guarded([&] {
    if (!model_dir) throw xpu::InvalidArg("xpu_qwen3_load_checkpoint: null pointer");
    eng(engine).load_checkpoint(model_dir);
  });
}

int xpu_qwen3_init_synthetic(xpu_qwen3_engine *engine, uint64_t seed, float stddev) {
  return guarded([&] { eng(engine).init_synthetic(seed, stddev); });
}

int xpu_qwen3_set_tensor(xpu_qwen3_engine *engine, const char *name, const uint16_t *host_bf16,
                         uint64_t elements) {
  return guarded([&] {
    if (!name || !host_bf16) throw xpu::InvalidArg("xpu_qwen3_set_tensor: null pointer");
    eng(engine).set_tensor(name, host_bf16, elements);
  });
}

int xpu_qwen3_decode(xpu_qwen3_engine *engine, uint32_t token, uint32_t position, uint32_t *next_token) {
  int status = guarded([&] {
    if (!next_token) throw xpu::InvalidArg("xpu_qwen3_decode: null pointer");
    *next_token = eng(engine).decode(token, position);
  });
  if (status == XPU_OK && *next_token == 0xffffffffu)
    return xpu::fail(XPU_ERR_NONFINITE, "model produced a NaN or infinity in vocabulary logits");
  return status;
}

int xpu_qwen3_generate(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len,
                       uint32_t max_new_tokens, int stop_at_eos, uint32_t *out_tokens,
                       uint32_t *out_count) {
  int status = guarded([&] {
    if (!prompt || !out_count || (max_new_tokens && !out_tokens))
      throw xpu::InvalidArg("xpu_qwen3_generate: null pointer");
    *out_count = eng(engine).generate(prompt, prompt_len, max_new_tokens, out_tokens, stop_at_eos != 0);
  });
  if (status == XPU_OK && *out_count && out_tokens[*out_count - 1] == 0xffffffffu)
    return xpu::fail(XPU_ERR_NONFINITE, "model produced a NaN or infinity in vocabulary logits");
  return status;
}

int xpu_qwen3_set_state(xpu_qwen3_engine *engine, uint32_t token, uint32_t position, uint32_t prompt_len) {
  return guarded([&] { eng(engine).set_state(token, position, prompt_len); });
}

int xpu_qwen3_get_state(xpu_qwen3_engine *engine, uint32_t *token, uint32_t *position, uint32_t *error) {
  return guarded([&] {
    const xpu::DecodeState s = eng(engine).get_state();
    if (token) *token = s.next;
    if (position) *position = s.position;
    if (error) *error = s.error;
  });
}

int xpu_qwen3_enqueue_steps(xpu_qwen3_engine *engine, uint32_t steps, void *stream) {
  return guarded([&] { eng(engine).enqueue_steps(steps, static_cast<cudaStream_t>(stream)); });
}

int xpu_qwen3_prefill_dense(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len,
                            uint32_t *next_token) {
  return guarded([&] {
    if (!prompt || !next_token) throw xpu::InvalidArg("xpu_qwen3_prefill_dense: null pointer");
    *next_token = eng(engine).dense_prefill(prompt, prompt_len);
  });
}

int xpu_qwen3_token_log(xpu_qwen3_engine *engine, uint32_t first_position, uint32_t count, uint32_t *host_out) {
  return guarded([&] {
    if (count && !host_out) throw xpu::InvalidArg("xpu_qwen3_token_log: null pointer");
    if (count) eng(engine).token_log(first_position, count, host_out);
  });
}

int xpu_qwen3_logits(xpu_qwen3_engine *engine, uint16_t *host_out, uint32_t count) {
  return guarded([&] {
    if (!host_out) throw xpu::InvalidArg("xpu_qwen3_logits: null pointer");
    eng(engine).logits(host_out, count);
  });
}

int xpu_qwen3_info(xpu_qwen3_engine *engine, xpu_qwen3_info_t *info) {
  return guarded([&] {
    if (!info) throw xpu::InvalidArg("xpu_qwen3_info: null pointer");
    Qwen3Engine &e = eng(engine);
    info->weight_bytes = e.weight_bytes();
    info->kernels_per_step = e.kernels_per_step();
    info->vocab_rows = e.dims().V_l;
    info->vocab_offset = e.dims().v_offset;
    info->stream = e.stream();
  });
}

uint64_t xpu_qwen3_bytes_per_token(xpu_qwen3_engine *engine, uint32_t context) {
  if (!engine || !engine->impl) return 0;
  return engine->impl->bytes_per_token(context);
}

int xpu_qwen3_trace(xpu_qwen3_engine *engine, uint64_t *host_ns, uint32_t capacity, uint32_t *count) {
  return guarded([&] {
    if (!count) throw xpu::InvalidArg("xpu_qwen3_trace: null pointer");
    *count = eng(engine).trace(host_ns, capacity);
  });
}

int xpu_qwen3_set_mode(xpu_qwen3_engine *engine, int mode) {
  return guarded([&] { eng(engine).set_mode(mode); });
}

int xpu_qwen3_synchronize(xpu_qwen3_engine *engine) {
  return guarded([&] { eng(engine).sync(); });
}

int xpu_qwen3_prefill(xpu_qwen3_engine *engine, const uint32_t *prompt, uint32_t prompt_len, uint32_t *next_token) {
  int status = guarded([&] {
    if (!prompt || !next_token) throw xpu::InvalidArg("xpu_qwen3_prefill: null pointer");
    *next_token = eng(engine).prefill(prompt, prompt_len);
  });
  if (status == XPU_OK && *next_token == 0xffffffffu)
    return xpu::fail(XPU_ERR_NONFINITE, "model produced a NaN or infinity in vocabulary logits");
  return status;
}

int xpu_qwen3_batch_decode(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *tokens,
                           const uint32_t *positions, uint32_t *next_tokens) {
  int status = guarded([&] {
    if (!tokens || !positions || !next_tokens) throw xpu::InvalidArg("xpu_qwen3_batch_decode: null pointer");
    eng(engine).batch_decode(batch, tokens, positions, next_tokens);
  });
  if (status == XPU_OK)
    for (uint32_t s = 0; s < batch; ++s)
      if (next_tokens[s] == 0xffffffffu)
        return xpu::fail(XPU_ERR_NONFINITE, "model produced a NaN or infinity in vocabulary logits");
  return status;
}

int xpu_qwen3_batch_generate(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *prompts,
                             const uint32_t *prompt_lens, uint32_t max_new_tokens, int stop_at_eos,
                             uint32_t *out_tokens, uint32_t *out_counts) {
  int status = guarded([&] {
    if (!prompts || !prompt_lens || !out_counts || (max_new_tokens && !out_tokens))
      throw xpu::InvalidArg("xpu_qwen3_batch_generate: null pointer");
    eng(engine).batch_generate(batch, prompts, prompt_lens, max_new_tokens, out_tokens, out_counts,
                               stop_at_eos != 0);
  });
  if (status == XPU_OK)
    for (uint32_t s = 0; s < batch; ++s)
      if (out_counts[s] && out_tokens[static_cast<size_t>(s) * max_new_tokens + out_counts[s] - 1] == 0xffffffffu)
        return xpu::fail(XPU_ERR_NONFINITE, "model produced a NaN or infinity in vocabulary logits");
  return status;
}

int xpu_qwen3_batch_set_state(xpu_qwen3_engine *engine, uint32_t batch, const uint32_t *tokens,
                              const uint32_t *positions) {
  return guarded([&] {
    if (!tokens || !positions) throw xpu::InvalidArg("xpu_qwen3_batch_set_state: null pointer");
    eng(engine).batch_set_state(batch, tokens, positions);
  });
}

int xpu_qwen3_batch_get_state(xpu_qwen3_engine *engine, uint32_t batch, uint32_t *tokens, uint32_t *positions,
                              uint32_t *error) {
  return guarded([&] {
    const uint32_t e = eng(engine).batch_get_state(batch, tokens, positions);
    if (error) *error = e;
  });
}

int xpu_qwen3_batch_enqueue_steps(xpu_qwen3_engine *engine, uint32_t steps, void *stream) {
  return guarded([&] { eng(engine).batch_enqueue_steps(steps, static_cast<cudaStream_t>(stream)); });
}

int xpu_qwen3_batch_logits(xpu_qwen3_engine *engine, uint32_t sequence, uint16_t *host_out, uint32_t count) {
  return guarded([&] {
    if (!host_out) throw xpu::InvalidArg("xpu_qwen3_batch_logits: null pointer");
    eng(engine).batch_logits(sequence, host_out, count);
  });
}

uint64_t xpu_qwen3_batch_bytes_per_step(xpu_qwen3_engine *engine, uint32_t batch, uint32_t context) {
  if (!engine || !engine->impl) return 0;
  return engine->impl->batch_bytes_per_step(batch, context);
}

int xpu_qwen3_batch_trace(xpu_qwen3_engine *engine, uint64_t *host_ns, uint32_t capacity, uint32_t *count) {
  return guarded([&] {
    if (!count) throw xpu::InvalidArg("xpu_qwen3_batch_trace: null pointer");
    *count = eng(engine).batch_trace(host_ns, capacity);
  });
}

uint32_t xpu_qwen3_batch_kernels_per_step(xpu_qwen3_engine *engine) {
  if (!engine || !engine->impl) return 0;
  return engine->impl->batch_kernels_per_step();
}

}  // extern "C"
