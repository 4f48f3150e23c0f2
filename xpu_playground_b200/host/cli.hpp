// Shared pieces of the benchmark programs (gemv, gemm, peak_mem_2d,
// peak_compute_dpas): the reference's option rules, CUDA error checks, device
// buffers, per-launch event timing and 16-bit conversions.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <charconv>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "xpu_cuda.h"

namespace xpu_cli {

// A positive integer option value (gemv.cpp:34-43): the whole text must
// parse and the value must be non-zero.
template <typename T>
T positive(std::string_view text, std::string_view option) {
  T value{};
  const auto parsed = std::from_chars(text.data(), text.data() + text.size(), value);
  if (parsed.ec != std::errc{} || parsed.ptr != text.data() + text.size() || !value)
    throw std::invalid_argument(std::string(option) + " requires a positive integer");
  return value;
}

inline void cuda_check(cudaError_t error, const char *what) {
  if (error != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(error));
}

inline void xpu_check(int status, const char *what) {
  if (status != XPU_OK) throw std::runtime_error(std::string(what) + ": " + xpu_last_error());
}

// Owning device allocation (freed on every exit path).
template <typename T>
class DeviceArray {
 public:
  explicit DeviceArray(size_t count) : count_(count) {
    void *p = nullptr;
    if (cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) throw std::bad_alloc();
    ptr_ = static_cast<T *>(p);
  }
  ~DeviceArray() { cudaFree(ptr_); }
  DeviceArray(const DeviceArray &) = delete;
  DeviceArray &operator=(const DeviceArray &) = delete;
  T *get() const { return ptr_; }
  size_t size() const { return count_; }

 private:
  T *ptr_ = nullptr;
  size_t count_ = 0;
};

// Device time of one launch: events on both sides on the legacy stream,
// waited for before returning (the reference waits on each launch's event).
class LaunchTimer {
 public:
  LaunchTimer() {
    cuda_check(cudaEventCreate(&start_), "cudaEventCreate");
    cuda_check(cudaEventCreate(&stop_), "cudaEventCreate");
  }
  ~LaunchTimer() {
    cudaEventDestroy(start_);
    cudaEventDestroy(stop_);
  }
  LaunchTimer(const LaunchTimer &) = delete;
  LaunchTimer &operator=(const LaunchTimer &) = delete;
  template <typename Launch>
  double seconds(Launch &&launch) {
    cuda_check(cudaEventRecord(start_, nullptr), "cudaEventRecord");
    launch();
    cuda_check(cudaEventRecord(stop_, nullptr), "cudaEventRecord");
    cuda_check(cudaEventSynchronize(stop_), "kernel");
    float ms = 0.0f;
    cuda_check(cudaEventElapsedTime(&ms, start_, stop_), "cudaEventElapsedTime");
    return static_cast<double>(ms) * 1e-3;
  }

 private:
  cudaEvent_t start_ = nullptr, stop_ = nullptr;
};

// Median of a sorted, non-empty vector (gemv.cpp:134-137).
inline double median_sorted(const std::vector<double> &v) {
  const size_t mid = v.size() / 2;
  return v.size() & 1 ? v[mid] : (v[mid - 1] + v[mid]) * 0.5;
}

inline std::string device_name() {
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  cudaDeviceProp prop{};
  cuda_check(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties");
  return prop.name;
}

inline int device_attribute(cudaDeviceAttr attr) {
  int dev = 0, value = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  cuda_check(cudaDeviceGetAttribute(&value, attr, dev), "cudaDeviceGetAttribute");
  return value;
}

inline std::string driver_version() {
  int v = 0;
  cuda_check(cudaDriverGetVersion(&v), "cudaDriverGetVersion");
  return std::to_string(v / 1000) + "." + std::to_string((v % 1000) / 10);
}

// Round-to-nearest-even float -> bf16 bits; NaN stays NaN (model.cpp:497-502).
inline uint16_t float_to_bf16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((bits >> 16) | 0x40u);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<uint16_t>(bits >> 16);
}

inline float bf16_to_float(uint16_t v) {
  const uint32_t bits = static_cast<uint32_t>(v) << 16;
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// IEEE binary16 through the compiler's _Float16 (round to nearest even).
inline uint16_t float_to_fp16(float value) {
  const _Float16 h = static_cast<_Float16>(value);
  uint16_t bits;
  std::memcpy(&bits, &h, 2);
  return bits;
}

inline float fp16_to_float(uint16_t v) {
  _Float16 h;
  std::memcpy(&h, &v, 2);
  return static_cast<float>(h);
}

inline uint16_t to16(float value, bool fp16) { return fp16 ? float_to_fp16(value) : float_to_bf16(value); }
inline float from16(uint16_t v, bool fp16) { return fp16 ? fp16_to_float(v) : bf16_to_float(v); }

}  // namespace xpu_cli
