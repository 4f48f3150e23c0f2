// `gemv` benchmark program: y = A.x through xpu_gemv. Flags, defaults,
// input hashes, the spot check of the first 64 rows and the output lines
// are the reference program's interface (gemv.cpp:20-170); shapes are used
// as given (the kernel predicates its edges, nothing is padded).
#include <iomanip>
#include <iostream>
#include <numeric>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

struct GemvRun {
  uint32_t m = 16384, k = 16384;
  unsigned iterations = 50, warmups = 5;
  bool fp16 = false;
};

FlagTable gemv_flags(GemvRun &r, const char *program) {
  FlagTable t([program](std::ostream &out) {
    out << "Usage: " << program << " [--size N | --m M --k K] [--type bf16|fp16]\n"
        << "       [--iterations N] [--warmups N]\n";
  });
  t.count("--size", false, &r.m, &r.k)
      .count("--m", false, &r.m)
      .count("--k", false, &r.k)
      .count("--iterations", false, &r.iterations)
      .count("--warmups", false, &r.warmups)
      .choice("--type", {{"bf16", [&r] { r.fp16 = false; }}, {"fp16", [&r] { r.fp16 = true; }}});
  return t;
}

// The reference's deterministic inputs (gemv.cpp:91-104), by flat index:
// matrix 0.25 + (mix(i) & 255) / 1024 with an integer avalanche mix, vector
// 0.5 + ((i * 747796405) >> 16 & 127) / 512.
uint32_t avalanche(uint32_t h) {
  h = (h ^ (h >> 16)) * 0x7feb352du;
  h = (h ^ (h >> 15)) * 0x846ca68bu;
  return h ^ (h >> 16);
}
float matrix_value(size_t i) { return 0.25f + static_cast<float>(avalanche(static_cast<uint32_t>(i)) & 0xffu) / 1024.0f; }
float vector_value(uint32_t i) { return 0.5f + static_cast<float>(((i * 747796405u) >> 16) & 0x7fu) / 512.0f; }

// Rows [0, rows) of y against an FP32 left-to-right dot product of the
// decoded inputs; a row fails when it is off by more than max(1, 1% of the
// expected value). Returns the first failing row, or -1.
long first_bad_row(const std::vector<uint16_t> &A, const std::vector<uint16_t> &x, const std::vector<uint16_t> &y,
                   uint32_t k, bool fp16) {
  std::vector<float> xf(k);
  std::transform(x.begin(), x.end(), xf.begin(), [fp16](uint16_t v) { return from16(v, fp16); });
  for (size_t row = 0; row < y.size(); ++row) {
    const uint16_t *a = A.data() + row * k;
    const float want = std::inner_product(xf.begin(), xf.end(), a, 0.0f, std::plus<float>(),
                                          [fp16](float xv, uint16_t av) { return from16(av, fp16) * xv; });
    if (std::abs(from16(y[row], fp16) - want) > std::max(1.0f, 0.01f * std::abs(want))) return static_cast<long>(row);
  }
  return -1;
}

int bench(const GemvRun &r) {
  const size_t n = static_cast<size_t>(r.m) * r.k;
  std::vector<uint16_t> hA(n), hx(r.k);
  for (size_t i = 0; i < n; ++i) hA[i] = to16(matrix_value(i), r.fp16);
  for (uint32_t i = 0; i < r.k; ++i) hx[i] = to16(vector_value(i), r.fp16);
  DeviceArray<uint16_t> A(n), x(r.k), y(r.m);
  cuda_check(cudaMemcpy(A.get(), hA.data(), n * 2, cudaMemcpyHostToDevice), "copy matrix");
  cuda_check(cudaMemcpy(x.get(), hx.data(), size_t{r.k} * 2, cudaMemcpyHostToDevice), "copy vector");

  const int dtype = r.fp16 ? XPU_FP16 : XPU_BF16;
  LaunchTimer timer;
  const auto once = [&] {
    return timer.seconds([&] { xpu_check(xpu_gemv(dtype, A.get(), x.get(), y.get(), r.m, r.k, nullptr), "xpu_gemv"); });
  };
  for (unsigned w = 0; w < r.warmups; ++w) once();
  const double work = 2.0 * static_cast<double>(n);  // FLOP per launch, and matrix bytes per launch
  std::vector<double> gflops;
  gflops.reserve(r.iterations);
  for (unsigned it = 0; it < r.iterations; ++it) gflops.push_back(work / once() / 1e9);

  std::vector<uint16_t> head(std::min<uint32_t>(r.m, 64));
  cuda_check(cudaMemcpy(head.data(), y.get(), head.size() * 2, cudaMemcpyDeviceToHost), "copy output");
  if (first_bad_row(hA, hx, head, r.k, r.fp16) >= 0) throw std::runtime_error("GEMV verification failed");

  // bytes moved per launch equal the FLOP count (2 bytes per element, 2 FLOP per element)
  const RateSummary s = summarize(std::move(gflops));
  std::cout << "Type: " << (r.fp16 ? "FP16" : "BF16") << ", shape: " << r.m << 'x' << r.k << '\n'
            << std::fixed << std::setprecision(2) << "Median: " << s.median << " GFLOP/s, " << s.median << " GB/s\n"
            << "Best:   " << s.best << " GFLOP/s, " << s.best << " GB/s\n"
            << "Verification: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_gemv(int argc, char **argv) {
  return guarded_main([&] {
    GemvRun r;
    if (!gemv_flags(r, argv[0]).parse(argc, argv)) return 0;
    std::cout << "Device: " << device_name() << '\n';
    return bench(r);
  });
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_gemv(argc, argv); }
#endif
