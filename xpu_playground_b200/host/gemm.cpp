// `gemm` benchmark: C = A.B on the tensor cores through xpu_gemm, with the
// reference program's flags, defaults, timing loop, closed-form check and
// output lines (gemm.cpp:17-155). Shapes are used as given: the kernel
// predicates edge tiles, so nothing is padded.
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

struct Options {
  uint32_t m = 4096, n = 4096, k = 4096;
  unsigned iterations = 20, warmups = 5;
  bool fp16 = false;
};

[[noreturn]] void usage(const char *program, int status) {
  std::ostream &out = status ? std::cerr : std::cout;
  out << "Usage: " << program << " [--size N | --m M --n N --k K] [--type bf16|fp16]\n"
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
    if (arg == "--size") o.m = o.n = o.k = positive<uint32_t>(value, arg);
    else if (arg == "--m") o.m = positive<uint32_t>(value, arg);
    else if (arg == "--n") o.n = positive<uint32_t>(value, arg);
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

int run(const Options &o) {
  const size_t as = static_cast<size_t>(o.m) * o.k, bs = static_cast<size_t>(o.k) * o.n,
               cs = static_cast<size_t>(o.m) * o.n;
  DeviceArray<uint16_t> a(as), b(bs), c(cs);
  {
    // gemm.cpp:81-85: A = 0.5, B = 0.25 everywhere.
    std::vector<uint16_t> ha(as, to16(0.5f, o.fp16));
    cuda_check(cudaMemcpy(a.get(), ha.data(), as * 2, cudaMemcpyHostToDevice), "copy A");
    std::vector<uint16_t> hb(bs, to16(0.25f, o.fp16));
    cuda_check(cudaMemcpy(b.get(), hb.data(), bs * 2, cudaMemcpyHostToDevice), "copy B");
    cuda_check(cudaMemset(c.get(), 0, cs * 2), "clear C");
  }
  const int dtype = o.fp16 ? XPU_FP16 : XPU_BF16;
  auto launch = [&] { xpu_check(xpu_gemm(dtype, a.get(), b.get(), c.get(), o.m, o.n, o.k, nullptr), "xpu_gemm"); };
  LaunchTimer timer;
  for (unsigned i = 0; i < o.warmups; ++i) timer.seconds(launch);
  const long double flops = 2.0L * o.m * o.n * o.k;
  std::vector<double> rates;
  for (unsigned i = 0; i < o.iterations; ++i) rates.push_back(static_cast<double>(flops) / timer.seconds(launch) / 1e12);
  uint32_t flags = 0;
  xpu_check(xpu_device_status(&flags), "xpu_device_status");
  if (flags) throw std::runtime_error("GEMM pipeline timed out on the device");

  std::vector<uint16_t> check(std::min<uint32_t>(o.n, 64));
  cuda_check(cudaMemcpy(check.data(), c.get(), check.size() * 2, cudaMemcpyDeviceToHost), "copy C");
  const float expected = o.k * 0.125f;
  const float tolerance = std::max(0.5f, expected * 0.01f);
  for (uint16_t v : check)
    if (std::abs(from16(v, o.fp16) - expected) > tolerance)
      throw std::runtime_error("GEMM verification failed: expected " + std::to_string(expected) + ", got " +
                               std::to_string(from16(v, o.fp16)));
  std::sort(rates.begin(), rates.end());
  std::cout << "Type: " << (o.fp16 ? "FP16" : "BF16") << ", shape: " << o.m << 'x' << o.n << 'x' << o.k << '\n'
            << std::fixed << std::setprecision(2) << "Median: " << median_sorted(rates) << " TFLOP/s\nBest:   "
            << rates.back() << " TFLOP/s\nVerification: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_gemm(int argc, char **argv) {
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
int main(int argc, char **argv) { return run_gemm(argc, argv); }
#endif
