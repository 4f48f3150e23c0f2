// `gemm` benchmark program: C = A.B on the tensor cores through xpu_gemm.
// Flags, defaults, the constant inputs with their closed-form check and the
// output lines are the reference program's interface (gemm.cpp:17-155);
// shapes are used as given (the kernel predicates edge tiles, nothing is
// padded).
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

struct GemmRun {
  uint32_t m = 4096, n = 4096, k = 4096;
  unsigned iterations = 20, warmups = 5;
  bool fp16 = false;
};

FlagTable gemm_flags(GemmRun &r, const char *program) {
  FlagTable t([program](std::ostream &out) {
    out << "Usage: " << program << " [--size N | --m M --n N --k K] [--type bf16|fp16]\n"
        << "       [--iterations N] [--warmups N]\n";
  });
  t.count("--size", false, &r.m, &r.n, &r.k)
      .count("--m", false, &r.m)
      .count("--n", false, &r.n)
      .count("--k", false, &r.k)
      .count("--iterations", false, &r.iterations)
      .count("--warmups", false, &r.warmups)
      .choice("--type", {{"bf16", [&r] { r.fp16 = false; }}, {"fp16", [&r] { r.fp16 = true; }}});
  return t;
}

// Device buffer of `count` copies of one 16-bit value.
void fill_constant(uint16_t *dst, size_t count, uint16_t bits) {
  const std::vector<uint16_t> host(count, bits);
  cuda_check(cudaMemcpy(dst, host.data(), count * 2, cudaMemcpyHostToDevice), "copy operand");
}

int bench(const GemmRun &r) {
  const size_t na = size_t{r.m} * r.k, nb = size_t{r.k} * r.n, nc = size_t{r.m} * r.n;
  DeviceArray<uint16_t> A(na), B(nb), C(nc);
  // A = 0.5 and B = 0.25 everywhere, so every element of C is k / 8
  // (the reference's check, gemm.cpp:81-85 and 109-117).
  fill_constant(A.get(), na, to16(0.5f, r.fp16));
  fill_constant(B.get(), nb, to16(0.25f, r.fp16));
  cuda_check(cudaMemset(C.get(), 0, nc * 2), "clear C");

  const int dtype = r.fp16 ? XPU_FP16 : XPU_BF16;
  LaunchTimer timer;
  const auto once = [&] {
    return timer.seconds(
        [&] { xpu_check(xpu_gemm(dtype, A.get(), B.get(), C.get(), r.m, r.n, r.k, nullptr), "xpu_gemm"); });
  };
  for (unsigned w = 0; w < r.warmups; ++w) once();
  const double flop = 2.0 * r.m * static_cast<double>(r.n) * r.k;
  std::vector<double> tflops;
  tflops.reserve(r.iterations);
  for (unsigned it = 0; it < r.iterations; ++it) tflops.push_back(flop / once() / 1e12);
  uint32_t device_flags = 0;
  xpu_check(xpu_device_status(&device_flags), "xpu_device_status");
  if (device_flags) throw std::runtime_error("GEMM pipeline timed out on the device");

  // the first (up to) 64 elements of row 0
  std::vector<uint16_t> row(std::min<uint32_t>(r.n, 64));
  cuda_check(cudaMemcpy(row.data(), C.get(), row.size() * 2, cudaMemcpyDeviceToHost), "copy C");
  const float want = 0.125f * static_cast<float>(r.k), slack = std::max(0.5f, 0.01f * want);
  const auto off = std::find_if(row.begin(), row.end(),
                                [&](uint16_t v) { return std::abs(from16(v, r.fp16) - want) > slack; });
  if (off != row.end())
    throw std::runtime_error("GEMM verification failed: expected " + std::to_string(want) + ", got " +
                             std::to_string(from16(*off, r.fp16)));

  const RateSummary s = summarize(std::move(tflops));
  std::cout << "Type: " << (r.fp16 ? "FP16" : "BF16") << ", shape: " << r.m << 'x' << r.n << 'x' << r.k << '\n'
            << std::fixed << std::setprecision(2) << "Median: " << s.median << " TFLOP/s\n"
            << "Best:   " << s.best << " TFLOP/s\n"
            << "Verification: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_gemm(int argc, char **argv) {
  return guarded_main([&] {
    GemmRun r;
    if (!gemm_flags(r, argv[0]).parse(argc, argv)) return 0;
    std::cout << "Device: " << device_name() << '\n';
    return bench(r);
  });
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_gemm(argc, argv); }
#endif
