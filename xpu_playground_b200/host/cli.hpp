// Shared pieces of the host programs (gemv, gemm, peak_mem_2d,
// peak_compute_dpas, peak_sycl, qwen3): a declarative command-line table,
// CUDA error checks, device buffers, per-launch event timing and 16-bit
// conversions.
//
// Command lines. A program lists its flags once in a FlagTable (name, value
// kind, destination) and calls parse(); the table walks argv, and every
// problem it meets is thrown as a FlagError naming what went wrong (no
// value, not a count, not one of the choices, unknown flag). The wording of
// the message belongs to the program: benchmark_message() gives the
// benchmark programs' texts ("--m requires a positive integer", ...), and
// the qwen3 program formats its own. "-h"/"--help" anywhere a flag may
// stand makes parse() return false after the program's usage text went to
// stdout, so library entries can return 0 instead of ending the process.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <functional>
#include <iostream>
#include <limits>
#include <stdexcept>
#include <string>
#include <string_view>
#include <vector>

#include "xpu_cuda.h"

namespace xpu_cli {

// ------------------------------------------------------------ command line --

enum class FlagProblem { kNoValue, kNotCount, kNotChoice, kUnknown };

struct FlagError : std::runtime_error {
  FlagError(FlagProblem p, std::string f, std::string v, std::string allowed)
      : std::runtime_error(f), problem(p), flag(std::move(f)), value(std::move(v)), choices(std::move(allowed)) {}
  FlagProblem problem;
  std::string flag, value;
  std::string choices;  // kNotChoice: the accepted values joined with " or "
};

// Decimal unsigned count. Strict form: digits only. Lenient form (what
// std::stoull accepts, for the qwen3 program): leading white space and one
// sign, where "-" wraps like stoull does; returns false when the text is
// not entirely a number or overflows 64 bits.
inline bool read_count(std::string_view text, bool lenient, uint64_t &out) {
  size_t i = 0;
  bool negative = false;
  if (lenient) {
    while (i < text.size() && (text[i] == ' ' || (text[i] >= '\t' && text[i] <= '\r'))) ++i;
    if (i < text.size() && (text[i] == '+' || text[i] == '-')) negative = text[i++] == '-';
  }
  if (i == text.size()) return false;
  uint64_t v = 0;
  for (; i < text.size(); ++i) {
    const unsigned digit = static_cast<unsigned char>(text[i]) - '0';
    if (digit > 9) return false;
    if (v > (std::numeric_limits<uint64_t>::max() - digit) / 10) return false;
    v = v * 10 + digit;
  }
  out = negative ? 0 - v : v;
  return true;
}

class FlagTable {
 public:
  using Usage = std::function<void(std::ostream &)>;

  explicit FlagTable(Usage usage) : usage_(std::move(usage)) {}

  // A count stored into every destination (one flag may set several, like
  // --size for m, n and k). Zero is refused unless allow_zero; values above
  // the narrowest destination's range are refused.
  template <typename... T>
  FlagTable &count(std::string_view name, bool allow_zero, T *...dst) {
    const uint64_t limit = std::min({static_cast<uint64_t>(std::numeric_limits<T>::max())...});
    entries_.push_back({std::string(name), [=](std::string_view v) {
                          uint64_t x = 0;
                          if (!read_count(v, lenient_, x) || x > limit || (!allow_zero && x == 0))
                            throw FlagError(FlagProblem::kNotCount, std::string(name), std::string(v), "");
                          ((*dst = static_cast<T>(x)), ...);
                        }});
    return *this;
  }

  // One of a fixed set of words; each word runs its action.
  FlagTable &choice(std::string_view name, std::vector<std::pair<std::string, std::function<void()>>> words) {
    std::string allowed;
    for (const auto &w : words) allowed += (allowed.empty() ? "" : " or ") + w.first;
    entries_.push_back({std::string(name), [=](std::string_view v) {
                          for (const auto &w : words)
                            if (v == w.first) return w.second();
                          throw FlagError(FlagProblem::kNotChoice, std::string(name), std::string(v), allowed);
                        }});
    return *this;
  }

  // Free text (a path, "-").
  FlagTable &text(std::string_view name, std::string *dst) {
    entries_.push_back({std::string(name), [dst](std::string_view v) { *dst = std::string(v); }});
    return *this;
  }

  // Counts are read the way std::stoull reads them (see read_count).
  FlagTable &lenient_counts() {
    lenient_ = true;
    return *this;
  }

  // Walks argv[1..argc): every flag takes the next word as its value.
  // Returns false after printing the usage for -h/--help.
  bool parse(int argc, char **argv) {
    for (int i = 1; i < argc; i += 2) {
      const std::string_view flag(argv[i]);
      if (flag == "-h" || flag == "--help") {
        usage_(std::cout);
        return false;
      }
      if (i + 1 >= argc) throw FlagError(FlagProblem::kNoValue, std::string(flag), "", "");
      const auto hit = std::find_if(entries_.begin(), entries_.end(), [&](const Entry &e) { return e.name == flag; });
      if (hit == entries_.end()) throw FlagError(FlagProblem::kUnknown, std::string(flag), argv[i + 1], "");
      hit->apply(argv[i + 1]);
      hit->given = true;
    }
    return true;
  }

  // Whether the last parse() met the flag.
  bool given(std::string_view name) const {
    return std::any_of(entries_.begin(), entries_.end(), [&](const Entry &e) { return e.name == name && e.given; });
  }

 private:
  struct Entry {
    std::string name;
    std::function<void(std::string_view)> apply;
    bool given = false;
  };
  Usage usage_;
  std::vector<Entry> entries_;
  bool lenient_ = false;
};

// The benchmark programs' wording of a command-line problem
// (gemv.cpp:34-64, peak_mem_2d.cpp:69-99 in the reference).
inline std::string benchmark_message(const FlagError &e) {
  switch (e.problem) {
    case FlagProblem::kNoValue: return e.flag + " requires a value";
    case FlagProblem::kNotCount: return e.flag + " requires a positive integer";
    case FlagProblem::kNotChoice: return e.flag + " must be " + e.choices;
    case FlagProblem::kUnknown: break;
  }
  return "unknown option: " + e.flag;
}

// Runs a benchmark program body behind the C ABI: its problems print
// "Error: <what>" on stderr and give 1; no exception leaves.
template <typename Body>
int guarded_main(Body &&body) {
  try {
    return body();
  } catch (const FlagError &e) {
    std::cerr << "Error: " << benchmark_message(e) << '\n';
  } catch (const std::exception &e) {
    std::cerr << "Error: " << e.what() << '\n';
  }
  return 1;
}

// ------------------------------------------------------------------ device --

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
// waited for before returning.
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

// Median and best of per-launch rates (the programs report both).
struct RateSummary {
  double median = 0.0, best = 0.0;
};

inline RateSummary summarize(std::vector<double> rates) {
  RateSummary s;
  if (rates.empty()) return s;
  std::sort(rates.begin(), rates.end());
  const size_t n = rates.size();
  s.median = (n % 2) ? rates[n / 2] : 0.5 * (rates[n / 2 - 1] + rates[n / 2]);
  s.best = rates.back();
  return s;
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

// ---------------------------------------------------------- 16-bit codecs --

// Round-to-nearest-even float -> bf16 bits, NaN kept quiet: the bit rule of
// the reference's host converter (model.cpp:497-502).
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
