// `peak_compute_dpas` (dense BF16 tensor-core calibrator) through
// xpu_peak_compute, with the reference program's flags, timing loop,
// closed-form checksum and output lines (peak_compute_dpas.cpp:24-222).
// --work-items is the number of CTAs (default: one per SM); each issues
// rounds x 8 tcgen05 MMAs of 128x256x16. The percentage is of the B200's
// nominal dense BF16 peak (the reference prints its B70's).
#include <cmath>
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

constexpr double kPeakTFlops = 2250.0;  // B200 dense BF16, nominal
constexpr uint64_t kFlopsPerMma = 2ull * 128 * 256 * 16;
constexpr uint64_t kMmasPerRound = 8;

struct Options {
  size_t work_items = 0;  // 0: one CTA per SM
  unsigned rounds = 8192;
  unsigned iterations = 1000;
};

[[noreturn]] void usage(const char *program, int status) {
  std::ostream &out = status == 0 ? std::cout : std::cerr;
  out << "Usage: " << program << " [--work-items N] [--rounds N] [--iterations N]\n"
      << "  --work-items N  CTAs, one tensor-core issuer each (default: one per SM)\n"
      << "  --rounds N      eight-MMA batches per CTA (default: 8192)\n"
      << "  --iterations N  timed kernel launches (default: 1000)\n";
  std::exit(status);
}

Options parse(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string_view arg(argv[i]);
    if (arg == "--help" || arg == "-h") usage(argv[0], 0);
    if (i + 1 == argc) throw std::invalid_argument(std::string(arg) + " requires a value");
    if (arg == "--work-items") o.work_items = positive<size_t>(argv[++i], "--work-items");
    else if (arg == "--rounds") o.rounds = positive<unsigned>(argv[++i], "--rounds");
    else if (arg == "--iterations") o.iterations = positive<unsigned>(argv[++i], "--iterations");
    else throw std::invalid_argument("unknown option: " + std::string(arg));
  }
  return o;
}

}  // namespace

extern "C" int run_peak_compute_dpas(int argc, char **argv) {
  try {
    Options o = parse(argc, argv);
    const int sms = device_attribute(cudaDevAttrMultiProcessorCount);
    if (o.work_items == 0) o.work_items = static_cast<size_t>(sms);
    if (o.work_items > 0x7fffffffu) throw std::invalid_argument("--work-items is too large");
    const std::string device = device_name(), driver = driver_version();
    std::cout << "Device: " << device << '\n'
              << "Driver: " << driver << '\n'
              << "Compute units: " << sms << '\n';
    DeviceArray<float> sink(o.work_items);
    cuda_check(cudaMemset(sink.get(), 0, o.work_items * sizeof(float)), "clear sink");
    const long double total_flops = static_cast<long double>(o.work_items) * o.rounds * kMmasPerRound * kFlopsPerMma;
    std::cout << "MMA shape: 128x256x16 BF16, " << kFlopsPerMma << " FLOP/instruction\n"
              << "Launch: " << o.work_items << " CTAs x " << o.rounds << " rounds x " << kMmasPerRound
              << " MMA = " << std::fixed << std::setprecision(3) << static_cast<double>(total_flops / 1.0e12L)
              << " TFLOP/launch\n";
    auto launch = [&] {
      xpu_check(xpu_peak_compute(sink.get(), static_cast<uint32_t>(o.work_items), o.rounds, nullptr),
                "xpu_peak_compute");
    };
    LaunchTimer timer;
    for (unsigned i = 0; i < 3; ++i) timer.seconds(launch);
    std::vector<double> tflops;
    for (unsigned i = 0; i < o.iterations; ++i)
      tflops.push_back(static_cast<double>(total_flops) / timer.seconds(launch) / 1e12);
    uint32_t flags = 0;
    xpu_check(xpu_device_status(&flags), "xpu_device_status");
    if (flags) throw std::runtime_error("tensor-core wait timed out on the device");
    float first = 0.0f, last = 0.0f;
    cuda_check(cudaMemcpy(&first, sink.get(), sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
    cuda_check(cudaMemcpy(&last, sink.get() + o.work_items - 1, sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
    // Accumulator initial offsets 0 + 1, plus 4 per MMA in each element.
    const float expected = 1.0f + static_cast<float>(kMmasPerRound) * o.rounds * 4.0f;
    const float tolerance = std::max(1.0f, expected * 1.0e-5f);
    if (std::abs(first - expected) > tolerance || std::abs(last - expected) > tolerance)
      throw std::runtime_error("MMA checksum verification failed");
    std::sort(tflops.begin(), tflops.end());
    const double median = median_sorted(tflops), best = tflops.back();
    std::cout << std::fixed << std::setprecision(2) << "Median BF16 compute: " << median << " TFLOP/s ("
              << (100.0 * median / kPeakTFlops) << "% of " << std::setprecision(1) << kPeakTFlops << " TFLOP/s)\n"
              << std::setprecision(2) << "Best BF16 compute:   " << best << " TFLOP/s (" << (100.0 * best / kPeakTFlops)
              << "% of " << std::setprecision(1) << kPeakTFlops << " TFLOP/s)\n"
              << "Checksum: PASS\n";
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "Error: " << e.what() << '\n';
  }
  return 1;
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_peak_compute_dpas(argc, argv); }
#endif
