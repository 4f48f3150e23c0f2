// `peak_mem_2d` (DRAM read-bandwidth calibrator) through xpu_peak_mem_read,
// with the reference program's flags, defaults, surface geometry, checksum
// verification and output lines (peak_mem_2d.cpp:29-244). The percentage is
// of the B200's nominal HBM3e bandwidth (the reference prints its B70's).
#include <cmath>
#include <iomanip>
#include <iostream>
#include <limits>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

constexpr size_t kMiB = 1024 * 1024;
constexpr double kPeakGBs = 7700.0;  // B200 HBM3e, nominal
constexpr size_t kSurfaceWidth = 1024, kUnitWidth = 16, kUnitRows = 32, kBlockRows = 8;
constexpr size_t kBytesPerUnit = kUnitWidth * kUnitRows * sizeof(float);  // 2 KiB

struct Options {
  size_t size_mib = 1024;
  unsigned iterations = 100;
};

[[noreturn]] void usage(const char *program, int status) {
  std::ostream &out = status == 0 ? std::cout : std::cerr;
  out << "Usage: " << program << " [--size-mib N] [--iterations N]\n"
      << "  --size-mib N    DRAM read surface size (default: 1024)\n"
      << "  --iterations N  Timed kernel launches (default: 100)\n";
  std::exit(status);
}

Options parse(int argc, char **argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string_view arg(argv[i]);
    if (arg == "--help" || arg == "-h") usage(argv[0], 0);
    if (i + 1 == argc) throw std::invalid_argument(std::string(arg) + " requires a value");
    if (arg == "--size-mib") o.size_mib = positive<size_t>(argv[++i], "--size-mib");
    else if (arg == "--iterations") o.iterations = positive<unsigned>(argv[++i], "--iterations");
    else throw std::invalid_argument("unknown option: " + std::string(arg));
  }
  return o;
}

// peak_mem_2d.cpp:36-47.
float input_value(size_t index) {
  uint32_t bits = static_cast<uint32_t>(index);
  bits ^= bits >> 16;
  bits *= 0x7feb352du;
  bits ^= bits >> 15;
  bits *= 0x846ca68bu;
  bits ^= bits >> 16;
  return 1.0f + static_cast<float>(bits & 0xffffu) * (1.0f / 65536.0f);
}

// peak_mem_2d.cpp:49-59.
float expected_checksum(size_t unit, size_t surface_height) {
  const size_t x = (unit % (kSurfaceWidth / kUnitWidth)) * kUnitWidth;
  const size_t y = (unit / (kSurfaceWidth / kUnitWidth)) * kUnitRows;
  if (y + 3 * kBlockRows >= surface_height) throw std::logic_error("checksum coordinate is outside the surface");
  float result = 0.0f;
  for (size_t load = 0; load < 4; ++load) result += input_value(x + (y + load * kBlockRows) * kSurfaceWidth);
  return result;
}

}  // namespace

extern "C" int run_peak_mem_2d(int argc, char **argv) {
  try {
    const Options o = parse(argc, argv);
    if (o.size_mib > std::numeric_limits<size_t>::max() / kMiB) throw std::invalid_argument("--size-mib is too large");
    const std::string device = device_name(), driver = driver_version();
    std::cout << "Device: " << device << '\n' << "Driver: " << driver << '\n';
    const size_t bytes = o.size_mib * kMiB;
    constexpr size_t row_bytes = kSurfaceWidth * sizeof(float);
    if (bytes % (row_bytes * kUnitRows) != 0) throw std::invalid_argument("surface size must be a multiple of 128 KiB");
    size_t free_bytes = 0, total_bytes = 0;
    cuda_check(cudaMemGetInfo(&free_bytes, &total_bytes), "cudaMemGetInfo");
    if (bytes > free_bytes) throw std::runtime_error("requested surface exceeds the device's free memory");
    const size_t elements = bytes / sizeof(float);
    const size_t surface_height = bytes / row_bytes;
    if (surface_height > std::numeric_limits<uint32_t>::max()) throw std::invalid_argument("--size-mib is too large");
    const size_t units = bytes / kBytesPerUnit;
    DeviceArray<float> input(elements), sink(units);
    xpu_check(xpu_peak_mem_fill(input.get(), elements, nullptr), "xpu_peak_mem_fill");
    cuda_check(cudaMemset(sink.get(), 0, units * sizeof(float)), "clear sink");
    cuda_check(cudaDeviceSynchronize(), "fill");
    std::cout << "Surface: " << o.size_mib << " MiB, " << kSurfaceWidth << " x " << surface_height << " floats\n"
              << "Traffic: " << (kBytesPerUnit / 1024) << " KiB/read unit, " << units << " units\n";
    auto launch = [&] {
      xpu_check(xpu_peak_mem_read(input.get(), sink.get(), static_cast<uint32_t>(surface_height), nullptr),
                "xpu_peak_mem_read");
    };
    LaunchTimer timer;
    for (unsigned i = 0; i < 3; ++i) timer.seconds(launch);
    std::vector<double> bandwidths;
    for (unsigned i = 0; i < o.iterations; ++i) bandwidths.push_back(static_cast<double>(bytes) / timer.seconds(launch) / 1e9);
    uint32_t flags = 0;
    xpu_check(xpu_device_status(&flags), "xpu_device_status");
    if (flags) throw std::runtime_error("read pipeline timed out on the device");
    float first = 0.0f, last = 0.0f;
    cuda_check(cudaMemcpy(&first, sink.get(), sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
    cuda_check(cudaMemcpy(&last, sink.get() + units - 1, sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
    if (std::abs(first - expected_checksum(0, surface_height)) > 1.0e-5f ||
        std::abs(last - expected_checksum(units - 1, surface_height)) > 1.0e-5f)
      throw std::runtime_error("checksum verification failed");
    std::sort(bandwidths.begin(), bandwidths.end());
    const double median = median_sorted(bandwidths), best = bandwidths.back();
    std::cout << std::fixed << std::setprecision(2) << "Median read bandwidth: " << median << " GB/s ("
              << (100.0 * median / kPeakGBs) << "% of " << std::setprecision(1) << kPeakGBs << " GB/s)\n"
              << std::setprecision(2) << "Best read bandwidth:   " << best << " GB/s (" << (100.0 * best / kPeakGBs)
              << "% of " << std::setprecision(1) << kPeakGBs << " GB/s)\n"
              << "Checksum: PASS\n";
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "Error: " << e.what() << '\n';
  }
  return 1;
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_peak_mem_2d(argc, argv); }
#endif
