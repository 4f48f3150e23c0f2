// `peak_compute_dpas` program: the dense BF16 tensor-core calibrator on
// xpu_peak_compute. Flags, the timing loop's shape, the closed-form
// checksum and the output lines are the reference program's interface
// (peak_compute_dpas.cpp:24-222). --work-items counts CTAs (default: one
// per SM), each issuing rounds x 8 tcgen05 MMAs of 128x256x16; the
// percentage is of the B200's nominal dense BF16 peak.
#include <cmath>
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

constexpr double kNominalTFlops = 2250.0;  // B200 dense BF16
constexpr uint64_t kMmaFlop = 2ull * 128 * 256 * 16;
constexpr uint64_t kMmasPerRound = 8;

struct ComputeRun {
  size_t work_items = 0;  // 0: one CTA per SM
  unsigned rounds = 8192;
  unsigned iterations = 1000;
};

FlagTable compute_flags(ComputeRun &r, const char *program) {
  FlagTable t([program](std::ostream &out) {
    out << "Usage: " << program << " [--work-items N] [--rounds N] [--iterations N]\n"
        << "  --work-items N  CTAs, one tensor-core issuer each (default: one per SM)\n"
        << "  --rounds N      eight-MMA batches per CTA (default: 8192)\n"
        << "  --iterations N  timed kernel launches (default: 1000)\n";
  });
  t.count("--work-items", false, &r.work_items).count("--rounds", false, &r.rounds).count("--iterations", false, &r.iterations);
  return t;
}

int calibrate(ComputeRun r) {
  const int sms = device_attribute(cudaDevAttrMultiProcessorCount);
  if (!r.work_items) r.work_items = static_cast<size_t>(sms);
  if (r.work_items > 0x7fffffffu) throw std::invalid_argument("--work-items is too large");
  std::cout << "Device: " << device_name() << '\n'
            << "Driver: " << driver_version() << '\n'
            << "Compute units: " << sms << '\n';
  const double flop = static_cast<double>(r.work_items) * r.rounds * kMmasPerRound * kMmaFlop;
  std::cout << "MMA shape: 128x256x16 BF16, " << kMmaFlop << " FLOP/instruction\n"
            << "Launch: " << r.work_items << " CTAs x " << r.rounds << " rounds x " << kMmasPerRound
            << " MMA = " << std::fixed << std::setprecision(3) << flop / 1.0e12 << " TFLOP/launch\n";

  DeviceArray<float> sums(r.work_items);
  cuda_check(cudaMemset(sums.get(), 0, r.work_items * sizeof(float)), "clear sink");
  LaunchTimer timer;
  const auto once = [&] {
    return timer.seconds([&] {
      xpu_check(xpu_peak_compute(sums.get(), static_cast<uint32_t>(r.work_items), r.rounds, nullptr), "xpu_peak_compute");
    });
  };
  for (int w = 0; w < 3; ++w) once();
  std::vector<double> tflops;
  for (unsigned it = 0; it < r.iterations; ++it) tflops.push_back(flop / once() / 1e12);
  uint32_t device_flags = 0;
  xpu_check(xpu_device_status(&device_flags), "xpu_device_status");
  if (device_flags) throw std::runtime_error("tensor-core wait timed out on the device");

  // Each element of the two accumulators starts at 0 and 1 and gains 4 per
  // MMA (ones . quarter-ones over K = 16); the CTA checksum adds one element
  // of each: 1 + 8 x 4 x rounds.
  const float want = 1.0f + 4.0f * static_cast<float>(kMmasPerRound) * static_cast<float>(r.rounds);
  const float slack = std::max(1.0f, 1.0e-5f * want);
  float ends[2] = {0.0f, 0.0f};
  cuda_check(cudaMemcpy(&ends[0], sums.get(), sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
  cuda_check(cudaMemcpy(&ends[1], sums.get() + r.work_items - 1, sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
  for (float got : ends)
    if (std::abs(got - want) > slack) throw std::runtime_error("MMA checksum verification failed");

  const RateSummary s = summarize(std::move(tflops));
  const auto line = [](const char *label, double v) {
    std::cout << std::fixed << std::setprecision(2) << label << v << " TFLOP/s (" << 100.0 * v / kNominalTFlops
              << "% of " << std::setprecision(1) << kNominalTFlops << " TFLOP/s)\n";
  };
  line("Median BF16 compute: ", s.median);
  line("Best BF16 compute:   ", s.best);
  std::cout << "Checksum: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_peak_compute_dpas(int argc, char **argv) {
  return guarded_main([&] {
    ComputeRun r;
    if (!compute_flags(r, argv[0]).parse(argc, argv)) return 0;
    return calibrate(r);
  });
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_peak_compute_dpas(argc, argv); }
#endif
