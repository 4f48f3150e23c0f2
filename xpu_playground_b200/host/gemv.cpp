// `gemv` benchmark: y = A.x through xpu_gemv, with the reference program's
// flags, defaults, hash-generated inputs, timing loop, 64-row check and
// output lines (gemv.cpp:20-170). Shapes are used as given (no padding).
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

struct Options {
  uint32_t m = 16384, k = 16384;
  unsigned iterations = 50, warmups = 5;
  bool fp16 = false;
};

[[noreturn]] void usage(const char *program, int status) {
  std::ostream &out = status ? std::cerr : std::cout;
  out << "Usage: " << program << " [--size N | --m M --k K] [--type bf16|fp16]\n"
      << "       [--iterations N] [--warmups N]\n";
  std::exit(status);
}

Options parse(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string_view arg(argv[i]);
    if (arg == "-h" || arg == "--help") usage(argv[0], 0);
    if (++i == argc) throw std::invalid_argument(std::string(arg) + " requires a value");
    const std::string_view value(argv[i]);
    if (arg == "--size") o.m = o.k = positive<uint32_t>(value, arg);
    else if (arg == "--m") o.m = positive<uint32_t>(value, arg);
    else if (arg == "--k") o.k = positive<uint32_t>(value, arg);
    else if (arg == "--iterations") o.iterations = positive<unsigned>(value, arg);
    else if (arg == "--warmups") o.warmups = positive<unsigned>(value, arg);
    else if (arg == "--type" && value == "fp16") o.fp16 = true;
    else if (arg == "--type" && value == "bf16") o.fp16 = false;
    else if (arg == "--type") throw std::invalid_argument("--type must be bf16 or fp16");
    else throw std::invalid_argument("unknown option: " + std::string(arg));
  }
  return o;
}

uint32_t hash_u32(uint32_t bits) {
  bits ^= bits >> 16;
  bits *= 0x7feb352du;
  bits ^= bits >> 15;
  bits *= 0x846ca68bu;
  bits ^= bits >> 16;
  return bits;
}

int run(const Options &o) {
  const size_t elements = static_cast<size_t>(o.m) * o.k;
  DeviceArray<uint16_t> matrix(elements), vector(o.k), output(o.m);
  // gemv.cpp:91-104: matrix 0.25 + (hash(i) & 255) / 1024, vector
  // 0.5 + ((i * 747796405 >> 16) & 127) / 512, i the flat element index.
  std::vector<uint16_t> hm(elements), hv(o.k);
  for (size_t i = 0; i < elements; ++i)
    hm[i] = to16(0.25f + static_cast<float>(hash_u32(static_cast<uint32_t>(i)) & 255u) / 1024.0f, o.fp16);
  for (uint32_t i = 0; i < o.k; ++i) {
    const uint32_t bits = i * 747796405u;
    hv[i] = to16(0.5f + static_cast<float>((bits >> 16) & 127u) / 512.0f, o.fp16);
  }
  cuda_check(cudaMemcpy(matrix.get(), hm.data(), elements * 2, cudaMemcpyHostToDevice), "copy matrix");
  cuda_check(cudaMemcpy(vector.get(), hv.data(), o.k * 2, cudaMemcpyHostToDevice), "copy vector");

  const int dtype = o.fp16 ? XPU_FP16 : XPU_BF16;
  auto launch = [&] {
    xpu_check(xpu_gemv(dtype, matrix.get(), vector.get(), output.get(), o.m, o.k, nullptr), "xpu_gemv");
  };
  LaunchTimer timer;
  for (unsigned i = 0; i < o.warmups; ++i) timer.seconds(launch);
  const long double operations = 2.0L * o.m * o.k, matrix_bytes = 2.0L * o.m * o.k;
  std::vector<double> rates, bandwidths;
  for (unsigned i = 0; i < o.iterations; ++i) {
    const double elapsed = timer.seconds(launch);
    rates.push_back(static_cast<double>(operations) / elapsed / 1e9);
    bandwidths.push_back(static_cast<double>(matrix_bytes) / elapsed / 1e9);
  }
  // gemv.cpp:118-131: FP32 serial sums of the first 64 rows, max(1, 1%).
  std::vector<uint16_t> check(std::min<uint32_t>(o.m, 64));
  cuda_check(cudaMemcpy(check.data(), output.get(), check.size() * 2, cudaMemcpyDeviceToHost), "copy output");
  for (size_t row = 0; row < check.size(); ++row) {
    float expected = 0.0f;
    for (uint32_t col = 0; col < o.k; ++col)
      expected += from16(hm[row * o.k + col], o.fp16) * from16(hv[col], o.fp16);
    const float tolerance = std::max(1.0f, std::abs(expected) * 0.01f);
    if (std::abs(from16(check[row], o.fp16) - expected) > tolerance)
      throw std::runtime_error("GEMV verification failed");
  }
  std::sort(rates.begin(), rates.end());
  std::sort(bandwidths.begin(), bandwidths.end());
  std::cout << "Type: " << (o.fp16 ? "FP16" : "BF16") << ", shape: " << o.m << 'x' << o.k << '\n'
            << std::fixed << std::setprecision(2) << "Median: " << median_sorted(rates) << " GFLOP/s, "
            << median_sorted(bandwidths) << " GB/s\n"
            << "Best:   " << rates.back() << " GFLOP/s, " << bandwidths.back() << " GB/s\n"
            << "Verification: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_gemv(int argc, char **argv) {
  try {
    const Options options = parse(argc, argv);
    const std::string device = device_name();
    std::cout << "Device: " << device << '\n';
    return run(options);
  } catch (const std::exception &e) {
    std::cerr << "Error: " << e.what() << '\n';
    return 1;
  }
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_gemv(argc, argv); }
#endif
