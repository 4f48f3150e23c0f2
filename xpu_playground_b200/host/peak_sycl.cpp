// `peak_sycl` program: one front end for the four benchmarks. `peak_sycl
// MODE ARGS...` runs MODE's benchmark entry of libxpu_bench.so in this
// process with ARGS, so every mode keeps its own options, messages and
// defaults. The program name, the modes, the usage text and the error
// lines are the reference dispatcher's interface (peak_sycl.cpp:10-56).
// The benchmark sees the path of its stand-alone program (beside this one)
// as argv[0], which is what its usage line prints.
#include <unistd.h>

#include <array>
#include <iostream>
#include <string>
#include <vector>

#include "xpu_bench.h"

namespace {

struct Mode {
  const char *word;     // first argument of peak_sycl
  const char *program;  // stand-alone program of the same benchmark
  int (*entry)(int, char **);
};

constexpr std::array<Mode, 4> kModes{{{"mem", "peak_mem_2d", run_peak_mem_2d},
                                       {"compute", "peak_compute_dpas", run_peak_compute_dpas},
                                       {"gemv", "gemv", run_gemv},
                                       {"gemm", "gemm", run_gemm}}};

void print_usage(const std::string &self) {
  std::cout << "Usage:\n"
            << "  " << self << " mem [--size-mib N] [--iterations N]\n"
            << "  " << self << " compute [--work-items N] [--rounds N] [--iterations N]\n"
            << "  " << self << " gemv [--size N | --m M --k K] [--type bf16|fp16]\n"
            << "  " << self << " gemm [--size N | --m M --n N --k K] [--type bf16|fp16]\n";
}

// Directory of this executable ("." when it cannot be resolved).
std::string own_directory() {
  std::vector<char> buf(4096);
  const ssize_t n = readlink("/proc/self/exe", buf.data(), buf.size() - 1);
  if (n <= 0) return ".";
  const std::string path(buf.data(), static_cast<size_t>(n));
  const size_t slash = path.rfind('/');
  return slash == std::string::npos ? "." : path.substr(0, slash);
}

int fail(const std::string &what) {
  std::cerr << "Error: " << what << '\n';
  return 1;
}

}  // namespace

int main(int argc, char **argv) {
  const std::string self = argv[0];
  if (argc < 2) {
    print_usage(self);
    return fail("missing benchmark mode");
  }
  const std::string word = argv[1];
  if (word == "-h" || word == "--help") {
    print_usage(self);
    return 0;
  }
  for (const Mode &m : kModes) {
    if (word != m.word) continue;
    std::string program = own_directory() + "/" + m.program;
    std::vector<char *> args(argv + 1, argv + argc);
    args[0] = program.data();
    args.push_back(nullptr);
    return m.entry(argc - 1, args.data());
  }
  return fail("unknown benchmark mode: " + word);
}
