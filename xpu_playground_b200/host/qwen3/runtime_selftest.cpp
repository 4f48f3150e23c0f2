// Self-test of the CUDA implementation of the reference's Qwen3 kernel
// runtime API: the error behaviour the reference defines
// (qwen3/level_zero_runtime.cpp:230-247: absent and ambiguous fragments,
// rejected arguments), allocation alignment, the memory requirement, and two
// launches through the fragment table checked on the host. Prints
// "runtime selftest: PASS on <device>" and exits 0, or names the failure and
// exits 1.
#include <cstdint>
#include <cstring>
#include <functional>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

#include "level_zero_runtime.hpp"

namespace {

void expect_throw(const std::function<void()> &f, const std::string &needle) {
  try {
    f();
  } catch (const std::runtime_error &e) {
    if (std::string(e.what()).find(needle) == std::string::npos)
      throw std::runtime_error("wrong error: '" + std::string(e.what()) + "', expected '" + needle + "'");
    return;
  }
  throw std::runtime_error("no error raised, expected '" + needle + "'");
}

std::uint16_t bf16(float v) {
  std::uint32_t bits;
  std::memcpy(&bits, &v, 4);
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return static_cast<std::uint16_t>(bits >> 16);
}

float f32(std::uint16_t b) {
  const std::uint32_t bits = static_cast<std::uint32_t>(b) << 16;
  float v;
  std::memcpy(&v, &bits, 4);
  return v;
}

}  // namespace

int main() {
  try {
    qwen3::LevelZeroRuntime rt("qwen3_kernels.bin");
    if (rt.device_name().empty() || rt.device_memory() == 0) throw std::runtime_error("no device properties");
    rt.require_bmg_and_memory(256ULL << 20);
    expect_throw([&] { rt.require_bmg_and_memory(1ULL << 50); }, "insufficient GPU memory");

    for (std::uint64_t align : {64ULL, 256ULL, 4096ULL, 65536ULL}) {
      void *p = rt.allocate_device(100, align);
      if (reinterpret_cast<std::uintptr_t>(p) % align) throw std::runtime_error("allocation not aligned");
    }

    const std::uint32_t width = 96;
    std::vector<std::uint16_t> left(width), right(width), out(width);
    for (std::uint32_t i = 0; i < width; ++i) {
      left[i] = bf16(static_cast<float>(i % 7) * 0.25f);
      right[i] = bf16(static_cast<float>(i % 5) * 0.5f);
    }
    auto *d_left = static_cast<std::uint16_t *>(rt.allocate_device(width * 2, 64));
    auto *d_right = static_cast<std::uint16_t *>(rt.allocate_device(width * 2, 64));
    rt.copy_to_device(d_left, left.data(), width * 2);
    rt.copy_to_device(d_right, right.data(), width * 2);

    using qwen3::kernel_argument;
    expect_throw([&] { rt.launch("QwenMissing", 1, {}); }, "absent from module: QwenMissing");
    expect_throw([&] { rt.launch("Qwen", 1, {}); }, "ambiguous Qwen3 kernel entry: Qwen");
    expect_throw([&] { rt.launch("QwenAdd", width / 32, {kernel_argument(d_left), kernel_argument(d_right)}); },
                 "takes 3 arguments, got 2");
    const std::uint64_t wide = width;
    expect_throw([&] {
      rt.launch("QwenAdd", width / 32, {kernel_argument(d_left), kernel_argument(d_right), kernel_argument(wide)});
    }, "rejected argument 2 (8 bytes)");

    rt.launch("QwenAdd", width / 32, {kernel_argument(d_left), kernel_argument(d_right), kernel_argument(width)});
    rt.copy_from_device(out.data(), d_left, width * 2);
    for (std::uint32_t i = 0; i < width; ++i)  // kernels.hpp:194-207: bf16(l + r), exact for these values
      if (out[i] != bf16(f32(left[i]) + f32(right[i]))) throw std::runtime_error("QwenAdd result");

    const std::uint32_t token = 2;
    auto *d_out = static_cast<std::uint16_t *>(rt.allocate_device(width * 2, 64));
    rt.launch("QwenEmbedding", 32, {kernel_argument(static_cast<const std::uint16_t *>(d_right)),
                                    kernel_argument(d_out), kernel_argument(token)});
    std::vector<std::uint16_t> row(32);
    rt.copy_from_device(row.data(), d_out, 64);
    for (std::uint32_t i = 0; i < 32; ++i)
      if (row[i] != right[token * 32 + i]) throw std::runtime_error("QwenEmbedding result");

    std::cout << "runtime selftest: PASS on " << rt.device_name() << '\n';
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "runtime selftest: " << e.what() << '\n';
    return 1;
  }
}
