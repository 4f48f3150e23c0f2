// GQA decode attention for callers that cannot allocate device memory.
//
// xpu_qwen_attention needs a caller-provided FP32 workspace for its split over
// 128-position chunks. Some callers cannot provide one: a host whose caching
// allocator owns the whole device, a serving loop that must never call
// cudaMalloc/cudaFree after start-up (both can synchronise the device and
// stall every stream), or a plugin host that hands a kernel only its input and
// output buffers. This entry point runs the same kernels with the workspace in
// a fixed array in this library's device memory instead.
//
// The array, g_noalloc_attention_scratch, is a file-scope __device__ variable
// of kNoAllocScratchBytes (6 MiB: enough for 32 query heads at 40,960
// positions). It occupies that much memory on every device where this code
// is loaded, until the process exits. In host code the variable's name is
// only a host-side stand-in, so its device address is looked up with
// cudaGetSymbolAddress (with that device current) on the first call for a
// device and cached; the first call on a device therefore does this set-up
// and should come before any stream capture. The cache is keyed by the
// device's current context as well, so a cudaDeviceReset (which gives the
// device a new context, with the array at a possibly different address)
// makes the next call look the address up again.
#include <cuda.h>

#include <mutex>
#include <string>

#include "xpu_internal.h"

namespace xpu {

constexpr size_t kNoAllocScratchBytes = size_t(6) << 20;

static __device__ __align__(256) float g_noalloc_attention_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchAddress {
  unsigned long long context = 0;  // driver id of the context the address belongs to
  float *ptr = nullptr;
};
ScratchAddress g_scratch[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long *);

// Driver id of the context current on this thread; 0 when there is none or
// the driver does not report it (then the address is looked up every call).
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of the scratch array on the current device: looked up on
// the first call for that device (and again after its context changed).
cudaError_t noalloc_scratch(float **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchAddress &slot = g_scratch[dev];
  const unsigned long long context = current_context_id();
  if (!slot.ptr || context == 0 || context != slot.context) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_attention_scratch);
    if (e != cudaSuccess) return e;
    slot.ptr = static_cast<float *>(p);
    slot.context = current_context_id();  // the lookup made the context current if it was not
  }
  *out = slot.ptr;
  return cudaSuccess;
}

}  // namespace
}  // namespace xpu

extern "C" int xpu_qwen_attention_noalloc(const uint16_t *query, const uint16_t *key_cache,
                                          const uint16_t *value_cache, uint16_t *output, uint32_t position,
                                          uint32_t query_heads, uint32_t key_value_heads, void *stream) {
  using namespace xpu;
  try {
    if (!query || !key_cache || !value_cache || !output)
      return fail(XPU_ERR_INVALID, "xpu_qwen_attention_noalloc: null pointer");
    if (key_value_heads == 0 || query_heads % key_value_heads != 0)
      return fail(XPU_ERR_INVALID, "xpu_qwen_attention_noalloc: query_heads must be a multiple of key_value_heads");
    const uint32_t group = query_heads / key_value_heads;
    if (group != 1 && group != 2 && group != 4 && group != 8)
      return fail(XPU_ERR_UNSUPPORTED,
                  "xpu_qwen_attention_noalloc: query_heads / key_value_heads must be 1, 2, 4 or 8");
    if (position == UINT32_MAX) return fail(XPU_ERR_INVALID, "xpu_qwen_attention_noalloc: position out of range");
    const size_t need = qwen_attention_workspace(query_heads, position + 1);
    if (need > kNoAllocScratchBytes)
      return fail(XPU_ERR_INVALID, "xpu_qwen_attention_noalloc: " + std::to_string(query_heads) +
                                       " query heads at position " + std::to_string(position) + " need " +
                                       std::to_string(need) + " bytes of scratch, more than the fixed " +
                                       std::to_string(kNoAllocScratchBytes) +
                                       "; use xpu_qwen_attention with a caller-owned workspace");
    float *scratch = nullptr;
    cudaError_t e = noalloc_scratch(&scratch);
    if (e != cudaSuccess) return cuda_status(e, "xpu_qwen_attention_noalloc: scratch address");
    // No slot needs clearing: the merge reads only the (max, sum, acc) slots
    // that this call's chunk kernel writes first.
    return cuda_status(qwen_attention_launch(query, key_cache, value_cache, output, position, query_heads,
                                             key_value_heads, scratch, static_cast<cudaStream_t>(stream)),
                       "xpu_qwen_attention_noalloc");
  } catch (const std::exception &ex) {
    return fail(XPU_ERR_INVALID, std::string("exception: ") + ex.what());
  }
}
