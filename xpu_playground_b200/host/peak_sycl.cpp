// `peak_sycl` mode dispatcher (peak_sycl.cpp:8-56): `peak_sycl MODE ARGS...`
// runs the sibling benchmark program for MODE with the remaining arguments,
// so each keeps its own options, diagnostics and defaults. The name is kept
// so that scripts written for the reference run unchanged.
#include <unistd.h>

#include <exception>
#include <filesystem>
#include <iostream>
#include <stdexcept>
#include <string>

namespace {

void usage(const char *program) {
  std::cout << "Usage:\n"
            << "  " << program << " mem [--size-mib N] [--iterations N]\n"
            << "  " << program << " compute [--work-items N] [--rounds N] [--iterations N]\n"
            << "  " << program << " gemv [--size N | --m M --k K] [--type bf16|fp16]\n"
            << "  " << program << " gemm [--size N | --m M --n N --k K] [--type bf16|fp16]\n";
}

[[noreturn]] void run_sibling(const char *program, char **argv) {
  const auto self = std::filesystem::canonical("/proc/self/exe");
  const auto target = self.parent_path() / program;
  argv[0] = const_cast<char *>(target.c_str());
  execv(target.c_str(), argv);
  throw std::runtime_error("cannot execute " + target.string());
}

}  // namespace

int main(int argc, char **argv) {
  try {
    if (argc < 2) {
      usage(argv[0]);
      throw std::invalid_argument("missing benchmark mode");
    }
    const std::string mode = argv[1];
    if (mode == "-h" || mode == "--help") {
      usage(argv[0]);
      return 0;
    }
    if (mode == "mem") run_sibling("peak_mem_2d", argv + 1);
    if (mode == "compute") run_sibling("peak_compute_dpas", argv + 1);
    if (mode == "gemv") run_sibling("gemv", argv + 1);
    if (mode == "gemm") run_sibling("gemm", argv + 1);
    throw std::invalid_argument("unknown benchmark mode: " + mode);
  } catch (const std::exception &error) {
    std::cerr << "Error: " << error.what() << '\n';
    return 1;
  }
}
