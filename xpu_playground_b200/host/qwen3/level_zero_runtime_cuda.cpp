// CUDA implementation of the reference's Qwen3 kernel runtime API
// (qwen3/level_zero_runtime.hpp:13-52, qwen3/level_zero_runtime.cpp): the
// eight Qwen kernel entries of qwen3/kernels_entry.cpp:8-72 run as
// libxpu_cuda's xpu_qwen_* entry points on one CUDA stream.
//
// This file compiles against either declaration of the class: the
// reference's own header (with host/ze_shim on the include path for its
// handle types) or host/qwen3_api/level_zero_runtime.hpp. It therefore keeps
// all of its state in a side table keyed by the runtime object and touches
// only the two members both declarations have (device_name_,
// device_memory_).
//
// Behaviour follows the reference: the runtime owns its allocations and
// frees them in the destructor; copies and launches are synchronous; a
// fragment that matches no kernel or several throws; arguments are checked
// by count and size against the kernel's parameter list; CUDA failures throw
// std::runtime_error with the call, file and line. Attention launches are
// serialised per device across runtime objects (they share the library's
// attention scratch); every other launch runs concurrently as before.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "level_zero_runtime.hpp"
#include "xpu_cuda.h"

namespace qwen3 {
namespace {

// Reference kernel constants the launch widths refer to (qwen3/kernels.hpp:20-22).
constexpr std::uint32_t kKvHeadsRef = 8;

[[noreturn]] void throw_cuda(cudaError_t e, const char *expression, const char *file, int line) {
  std::ostringstream out;
  out << expression << " failed at " << file << ':' << line << " (CUDA error " << static_cast<int>(e) << ' '
      << cudaGetErrorName(e) << ": " << cudaGetErrorString(e) << ')';
  throw std::runtime_error(out.str());
}

#define CUDA_CHECK(expression)                                              \
  do {                                                                      \
    const cudaError_t check_result_ = (expression);                         \
    if (check_result_ != cudaSuccess) throw_cuda(check_result_, #expression, __FILE__, __LINE__); \
  } while (false)

void xpu_check(int status, const std::string &entry) {
  if (status != XPU_OK) throw std::runtime_error(entry + " failed: " + xpu_last_error());
}

// Typed view of a checked argument list.
struct Args {
  const std::vector<KernelArgument> &a;
  template <typename T>
  T get(std::size_t i) const {
    T v;
    std::memcpy(&v, a[i].value, sizeof(T));
    return v;
  }
};

using Launcher = int (*)(const Args &, std::uint32_t work_items, cudaStream_t);

struct Entry {
  const char *name;                  // the reference module's kernel names contain these
  std::vector<std::size_t> sizes;    // parameter sizes, in order
  Launcher launch;
  bool shared_scratch = false;       // runs on the library's per-device scratch array
};

constexpr std::size_t P = sizeof(void *), U = sizeof(std::uint32_t), F = sizeof(float);

const std::vector<Entry> &entries() {
  static const std::vector<Entry> table = {
      {"QwenEmbeddingLevelZeroEntry", {P, P, U},
       [](const Args &a, std::uint32_t work_items, cudaStream_t s) {
         // work_items = row width (main.cpp:162: kHiddenSize)
         return xpu_qwen_embedding(a.get<const uint16_t *>(0), a.get<uint16_t *>(1), a.get<uint32_t>(2),
                                   work_items, s);
       }},
      {"QwenRmsNormLevelZeroEntry", {P, P, P, U, F},
       [](const Args &a, std::uint32_t, cudaStream_t s) {
         return xpu_qwen_rms_norm(a.get<const uint16_t *>(0), a.get<const uint16_t *>(1), a.get<uint16_t *>(2),
                                  a.get<uint32_t>(3), a.get<float>(4), s);
       }},
      {"QwenGemvLevelZeroEntry", {P, P, P, U, U},
       [](const Args &a, std::uint32_t, cudaStream_t s) {
         return xpu_qwen_gemv(a.get<const uint16_t *>(0), a.get<const uint16_t *>(1), a.get<uint16_t *>(2),
                              a.get<uint32_t>(3), a.get<uint32_t>(4), s);
       }},
      {"QwenQkvRopeCacheLevelZeroEntry", {P, P, P, P, P, P, P, P, P, U, U},
       [](const Args &a, std::uint32_t work_items, cudaStream_t s) {
         // work_items = query heads (main.cpp:183); 8 key/value heads.
         return xpu_qwen_qkv_rope_cache(a.get<uint16_t *>(0), a.get<uint16_t *>(1), a.get<const uint16_t *>(2),
                                        a.get<const uint16_t *>(3), a.get<const uint16_t *>(4),
                                        a.get<const uint16_t *>(5), a.get<const uint16_t *>(6),
                                        a.get<uint16_t *>(7), a.get<uint16_t *>(8), a.get<uint32_t>(9),
                                        a.get<uint32_t>(10), work_items, kKvHeadsRef, s);
       }},
      {"QwenAttentionLevelZeroEntry", {P, P, P, P, U},
       [](const Args &a, std::uint32_t work_items, cudaStream_t s) {
         // work_items = query heads (main.cpp:191); the split-softmax scratch
         // is the library's fixed array, as the reference passes none.
         return xpu_qwen_attention_noalloc(a.get<const uint16_t *>(0), a.get<const uint16_t *>(1),
                                           a.get<const uint16_t *>(2), a.get<uint16_t *>(3), a.get<uint32_t>(4),
                                           work_items, kKvHeadsRef, s);
       },
       true},
      {"QwenAddLevelZeroEntry", {P, P, U},
       [](const Args &a, std::uint32_t, cudaStream_t s) {
         return xpu_qwen_add(a.get<uint16_t *>(0), a.get<const uint16_t *>(1), a.get<uint32_t>(2), s);
       }},
      {"QwenSiluMultiplyLevelZeroEntry", {P, P, U},
       [](const Args &a, std::uint32_t, cudaStream_t s) {
         return xpu_qwen_silu_multiply(a.get<uint16_t *>(0), a.get<const uint16_t *>(1), a.get<uint32_t>(2), s);
       }},
      {"QwenArgmaxLevelZeroEntry", {P, P, U},
       [](const Args &a, std::uint32_t, cudaStream_t s) {
         return xpu_qwen_argmax(a.get<const uint16_t *>(0), a.get<uint32_t *>(1), a.get<uint32_t>(2), s);
       }},
  };
  return table;
}

struct State {
  int device = 0;
  cudaStream_t stream = nullptr;
  int cc_major = 0, cc_minor = 0;
  std::vector<void *> allocations;  // cudaMalloc bases, freed by the destructor
};

std::mutex g_mutex;
std::map<const LevelZeroRuntime *, std::unique_ptr<State>> g_states;

// Attention runs on one scratch array per device shared by every caller of
// xpu_qwen_attention_noalloc, so two runtimes on one device (each on its own
// stream, possibly driven from two threads) must not have attention in
// flight at the same time: a launch of such an entry holds its device's
// lock until its stream has drained.
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_locks[kMaxScratchDevices];

State &state_of(const LevelZeroRuntime *rt) {
  std::lock_guard<std::mutex> lock(g_mutex);
  auto it = g_states.find(rt);
  if (it == g_states.end()) throw std::runtime_error("LevelZeroRuntime used after destruction");
  return *it->second;
}

}  // namespace

LevelZeroRuntime::LevelZeroRuntime(const std::string &module_path) {
  (void)module_path;
  auto st = std::make_unique<State>();
  CUDA_CHECK(cudaGetDevice(&st->device));
  cudaDeviceProp prop{};
  CUDA_CHECK(cudaGetDeviceProperties(&prop, st->device));
  st->cc_major = prop.major;
  st->cc_minor = prop.minor;
  CUDA_CHECK(cudaStreamCreateWithFlags(&st->stream, cudaStreamNonBlocking));
  device_name_ = prop.name;
  device_memory_ = prop.totalGlobalMem;
  std::lock_guard<std::mutex> lock(g_mutex);
  g_states[this] = std::move(st);
}

LevelZeroRuntime::~LevelZeroRuntime() {
  std::unique_ptr<State> st;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_states.find(this);
    if (it == g_states.end()) return;
    st = std::move(it->second);
    g_states.erase(it);
  }
  cudaSetDevice(st->device);
  if (st->stream) cudaStreamSynchronize(st->stream);
  for (void *p : st->allocations) cudaFree(p);
  if (st->stream) cudaStreamDestroy(st->stream);
}

void LevelZeroRuntime::require_bmg_and_memory(std::uint64_t required_bytes) const {
  const State &st = state_of(this);
  if (st.cc_major != 10)
    throw std::runtime_error("unsupported GPU '" + device_name_ +
                             "': the Qwen3 kernels are built for sm_100a (B200)");
  constexpr std::uint64_t reserve = 512ULL << 20;
  if (device_memory_ < required_bytes || device_memory_ - required_bytes < reserve)
    throw std::runtime_error("insufficient GPU memory: need " +
                             std::to_string((required_bytes + (1ULL << 20) - 1) >> 20) +
                             " MiB plus a 512 MiB reserve, device reports " + std::to_string(device_memory_ >> 20) +
                             " MiB");
}

void *LevelZeroRuntime::allocate_device(std::uint64_t bytes, std::uint64_t alignment) {
  State &st = state_of(this);
  if (alignment == 0 || (alignment & (alignment - 1)))
    throw std::runtime_error("allocate_device: alignment must be a power of two");
  CUDA_CHECK(cudaSetDevice(st.device));
  // cudaMalloc returns 256-byte aligned memory; larger alignments over-allocate.
  const std::uint64_t extra = alignment > 256 ? alignment : 0;
  void *base = nullptr;
  CUDA_CHECK(cudaMalloc(&base, std::max<std::uint64_t>(bytes + extra, 1)));
  st.allocations.push_back(base);
  const auto addr = reinterpret_cast<std::uintptr_t>(base);
  return reinterpret_cast<void *>((addr + alignment - 1) & ~static_cast<std::uintptr_t>(alignment - 1));
}

void LevelZeroRuntime::copy_to_device(void *destination, const void *source, std::size_t bytes) {
  State &st = state_of(this);
  CUDA_CHECK(cudaMemcpyAsync(destination, source, bytes, cudaMemcpyHostToDevice, st.stream));
  CUDA_CHECK(cudaStreamSynchronize(st.stream));
}

void LevelZeroRuntime::copy_from_device(void *destination, const void *source, std::size_t bytes) {
  State &st = state_of(this);
  CUDA_CHECK(cudaMemcpyAsync(destination, source, bytes, cudaMemcpyDeviceToHost, st.stream));
  CUDA_CHECK(cudaStreamSynchronize(st.stream));
}

void LevelZeroRuntime::launch(const std::string &entry_fragment, std::uint32_t work_items,
                              const std::vector<KernelArgument> &arguments) {
  State &st = state_of(this);
  const Entry *selected = nullptr;
  for (const Entry &e : entries())
    if (std::string(e.name).find(entry_fragment) != std::string::npos) {
      if (selected) throw std::runtime_error("ambiguous Qwen3 kernel entry: " + entry_fragment);
      selected = &e;
    }
  if (!selected) throw std::runtime_error("Qwen3 kernel is absent from module: " + entry_fragment);
  if (arguments.size() != selected->sizes.size())
    throw std::runtime_error(entry_fragment + " takes " + std::to_string(selected->sizes.size()) +
                             " arguments, got " + std::to_string(arguments.size()));
  for (std::size_t i = 0; i != arguments.size(); ++i)
    if (arguments[i].size != selected->sizes[i] || !arguments[i].value)
      throw std::runtime_error("rejected argument " + std::to_string(i) + " (" + std::to_string(arguments[i].size) +
                               " bytes) for " + entry_fragment + ": expected " +
                               std::to_string(selected->sizes[i]) + " bytes");
  CUDA_CHECK(cudaSetDevice(st.device));
  std::unique_lock<std::mutex> scratch_lock;
  if (selected->shared_scratch) {
    if (st.device < 0 || st.device >= kMaxScratchDevices)
      throw std::runtime_error("device ordinal beyond the scratch lock table: " + std::to_string(st.device));
    scratch_lock = std::unique_lock<std::mutex>(g_scratch_locks[st.device]);
  }
  xpu_check(selected->launch(Args{arguments}, work_items, st.stream), entry_fragment);
  const cudaError_t e = cudaStreamSynchronize(st.stream);
  if (e != cudaSuccess) throw_cuda(e, entry_fragment.c_str(), __FILE__, __LINE__);
}

}  // namespace qwen3
