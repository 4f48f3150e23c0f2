// `peak_mem_2d` program: the DRAM read-bandwidth calibrator on
// xpu_peak_mem_read. Flags, defaults, the surface geometry, the checksum
// rule for the first and last read unit and the output lines are the
// reference program's interface (peak_mem_2d.cpp:29-244); the percentage is
// of the B200's nominal HBM3e bandwidth.
#include <cmath>
#include <iomanip>
#include <iostream>

#include "cli.hpp"
#include "xpu_bench.h"

namespace {

using namespace xpu_cli;

constexpr double kNominalGBs = 7700.0;  // B200 HBM3e
// Surface: rows of 1024 floats; a read unit is a 16-float x 32-row block
// (2 KiB) whose checksum adds the unit's first column at rows 0, 8, 16, 24.
constexpr size_t kRowFloats = 1024, kUnitCols = 16, kUnitRows = 32, kProbeStride = 8, kProbes = 4;
constexpr size_t kUnitBytes = kUnitCols * kUnitRows * sizeof(float);
constexpr size_t kUnitsPerBand = kRowFloats / kUnitCols;

struct ReadRun {
  size_t size_mib = 1024;
  unsigned iterations = 100;
};

FlagTable read_flags(ReadRun &r, const char *program) {
  FlagTable t([program](std::ostream &out) {
    out << "Usage: " << program << " [--size-mib N] [--iterations N]\n"
        << "  --size-mib N    DRAM read surface size (default: 1024)\n"
        << "  --iterations N  Timed kernel launches (default: 100)\n";
  });
  t.count("--size-mib", false, &r.size_mib).count("--iterations", false, &r.iterations);
  return t;
}

// Surface element i: 1 + (16 low bits of an avalanche mix of i) / 65536, an
// irregular finite fill (peak_mem_2d.cpp:36-47 gives the mix).
float surface_value(size_t i) {
  uint32_t h = static_cast<uint32_t>(i);
  h = (h ^ (h >> 16)) * 0x7feb352du;
  h = (h ^ (h >> 15)) * 0x846ca68bu;
  h ^= h >> 16;
  return 1.0f + static_cast<float>(h & 0xffffu) / 65536.0f;
}

float unit_checksum(size_t unit, size_t rows) {
  const size_t col = (unit % kUnitsPerBand) * kUnitCols, row0 = (unit / kUnitsPerBand) * kUnitRows;
  if (row0 + (kProbes - 1) * kProbeStride >= rows) throw std::logic_error("checksum coordinate is outside the surface");
  float sum = 0.0f;
  for (size_t p = 0; p < kProbes; ++p) sum += surface_value((row0 + p * kProbeStride) * kRowFloats + col);
  return sum;
}

int calibrate(const ReadRun &r) {
  constexpr size_t kMiB = size_t{1} << 20;
  if (r.size_mib > std::numeric_limits<size_t>::max() / kMiB) throw std::invalid_argument("--size-mib is too large");
  std::cout << "Device: " << device_name() << '\n' << "Driver: " << driver_version() << '\n';
  const size_t bytes = r.size_mib * kMiB, band_bytes = kRowFloats * sizeof(float) * kUnitRows;
  if (bytes % band_bytes) throw std::invalid_argument("surface size must be a multiple of 128 KiB");
  size_t free_bytes = 0, total_bytes = 0;
  cuda_check(cudaMemGetInfo(&free_bytes, &total_bytes), "cudaMemGetInfo");
  if (bytes > free_bytes) throw std::runtime_error("requested surface exceeds the device's free memory");
  const size_t rows = bytes / (kRowFloats * sizeof(float)), units = bytes / kUnitBytes;
  if (rows > std::numeric_limits<uint32_t>::max()) throw std::invalid_argument("--size-mib is too large");

  DeviceArray<float> surface(bytes / sizeof(float)), sums(units);
  xpu_check(xpu_peak_mem_fill(surface.get(), surface.size(), nullptr), "xpu_peak_mem_fill");
  cuda_check(cudaMemset(sums.get(), 0, units * sizeof(float)), "clear sink");
  cuda_check(cudaDeviceSynchronize(), "fill");
  std::cout << "Surface: " << r.size_mib << " MiB, " << kRowFloats << " x " << rows << " floats\n"
            << "Traffic: " << kUnitBytes / 1024 << " KiB/read unit, " << units << " units\n";

  LaunchTimer timer;
  const auto once = [&] {
    return timer.seconds([&] {
      xpu_check(xpu_peak_mem_read(surface.get(), sums.get(), static_cast<uint32_t>(rows), nullptr), "xpu_peak_mem_read");
    });
  };
  for (int w = 0; w < 3; ++w) once();
  std::vector<double> gbs;
  for (unsigned it = 0; it < r.iterations; ++it) gbs.push_back(static_cast<double>(bytes) / once() / 1e9);
  uint32_t device_flags = 0;
  xpu_check(xpu_device_status(&device_flags), "xpu_device_status");
  if (device_flags) throw std::runtime_error("read pipeline timed out on the device");

  float ends[2] = {0.0f, 0.0f};
  cuda_check(cudaMemcpy(&ends[0], sums.get(), sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
  cuda_check(cudaMemcpy(&ends[1], sums.get() + units - 1, sizeof(float), cudaMemcpyDeviceToHost), "copy sink");
  const size_t probe_units[2] = {0, units - 1};
  for (int e = 0; e < 2; ++e)
    if (std::abs(ends[e] - unit_checksum(probe_units[e], rows)) > 1.0e-5f)
      throw std::runtime_error("checksum verification failed");

  const RateSummary s = summarize(std::move(gbs));
  const auto line = [](const char *label, double v) {
    std::cout << std::fixed << std::setprecision(2) << label << v << " GB/s (" << 100.0 * v / kNominalGBs << "% of "
              << std::setprecision(1) << kNominalGBs << " GB/s)\n";
  };
  line("Median read bandwidth: ", s.median);
  line("Best read bandwidth:   ", s.best);
  std::cout << "Checksum: PASS\n";
  return 0;
}

}  // namespace

extern "C" int run_peak_mem_2d(int argc, char **argv) {
  return guarded_main([&] {
    ReadRun r;
    if (!read_flags(r, argv[0]).parse(argc, argv)) return 0;
    return calibrate(r);
  });
}

#ifdef XPU_STANDALONE_HOST
int main(int argc, char **argv) { return run_peak_mem_2d(argc, argv); }
#endif
