// The Qwen3 kernel runtime API of the reference (qwen3/level_zero_runtime.hpp:
// KernelArgument, LevelZeroRuntime, kernel_argument), declared for the CUDA
// implementation in host/qwen3/level_zero_runtime_cuda.cpp so that callers
// written for the reference (its Engine in qwen3/main.cpp, its
// tests/test_gpu_dispatch.cpp) keep their source. The class keeps its name so
// that those callers need no edit; it runs the eight kernel entries of
// libxpu_cuda on a B200.
//
// Semantics as in the reference: the runtime owns every device allocation
// and frees them when destroyed; it is not copyable; every call is
// synchronous (one CUDA stream, waited for after each copy and launch);
// failures throw std::runtime_error naming the CUDA error and the call;
// launch() picks the one kernel whose name contains the fragment (none or
// several: throws) and checks the argument count and sizes against the
// kernel's parameter list (mismatch: throws).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace qwen3 {

struct KernelArgument {
  std::size_t size;
  const void *value;
};

class LevelZeroRuntime {
 public:
  // module_path names the reference's AOT kernel module; here the kernels are
  // linked in (libxpu_cuda), so the path is accepted and not read.
  explicit LevelZeroRuntime(const std::string &module_path);
  ~LevelZeroRuntime();
  LevelZeroRuntime(const LevelZeroRuntime &) = delete;
  LevelZeroRuntime &operator=(const LevelZeroRuntime &) = delete;

  // Requires an sm_100 (B200-class) GPU with required_bytes + 512 MiB of
  // memory (the reference requires an Intel BMG GPU; the name is kept).
  void require_bmg_and_memory(std::uint64_t required_bytes) const;
  void *allocate_device(std::uint64_t bytes, std::uint64_t alignment = 4096);
  void copy_to_device(void *destination, const void *source, std::size_t bytes);
  void copy_from_device(void *destination, const void *source, std::size_t bytes);
  void launch(const std::string &entry_fragment, std::uint32_t work_items,
              const std::vector<KernelArgument> &arguments);

  const std::string &device_name() const { return device_name_; }
  std::uint64_t device_memory() const { return device_memory_; }

 private:
  std::string device_name_;
  std::uint64_t device_memory_ = 0;
};

template <typename T>
KernelArgument kernel_argument(const T &value) {
  return KernelArgument{sizeof(T), &value};
}

}  // namespace qwen3
