/* Benchmark entry points of libxpu_bench.so (and the programs of the same
 * names). Each takes the program's command line (argv[0] = program name),
 * prints the reference program's output lines, returns 0 on success and 1
 * after printing "Error: <what>" on stderr. No C++ exception crosses the
 * boundary.
 */
#ifndef XPU_BENCH_H
#define XPU_BENCH_H

#ifdef __cplusplus
extern "C" {
#endif

/* gemv [--size N | --m M --k K] [--type bf16|fp16] [--iterations N] [--warmups N]
 * Replaces run_gemv (gemv.cpp:157-170). */
int run_gemv(int argc, char **argv);

/* gemm [--size N | --m M --n N --k K] [--type bf16|fp16] [--iterations N] [--warmups N]
 * Replaces run_gemm (gemm.cpp:135-155). */
int run_gemm(int argc, char **argv);

/* peak_mem_2d [--size-mib N] [--iterations N]
 * Replaces run_peak_mem_2d (peak_mem_2d.cpp:124-244). */
int run_peak_mem_2d(int argc, char **argv);

/* peak_compute_dpas [--work-items N] [--rounds N] [--iterations N]
 * Replaces run_peak_compute_dpas (peak_compute_dpas.cpp:102-222);
 * --work-items counts CTAs. */
int run_peak_compute_dpas(int argc, char **argv);

#ifdef __cplusplus
}
#endif

#endif /* XPU_BENCH_H */
