// ops_status.cu -- the device status word of the operator entry points, and
// qwen_ops_status.
//
// Operator entry points enqueue kernels and return before they run, so a
// failure that only the device sees (a bounded wait that gave up, a length
// out of range) cannot be their return value.  Those kernels record it in a
// per-device status word instead -- a file-scope __device__ array, so
// recording needs no allocation -- and qwen_ops_status() synchronises a stream
// and reports (then clears) what was recorded.  The first error wins until
// it is read.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "../../include/qwen_b200.h"
#include "qwen_common.cuh"
#include "qwen_internal.h"
#include "status.h"

namespace qwen {

// [0] first error code (DeviceError), [1..3] detail of the kernel that set it.
static __device__ __align__(16) int g_ops_status[4];

// cuCtxGetCurrent through the runtime's driver entry point table (the library
// does not link libcuda directly, so it loads on machines without a driver).
static CUresult current_context(CUcontext* ctx) {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(f);
  });
  *ctx = nullptr;
  return fn ? fn(ctx) : CUDA_ERROR_NOT_INITIALIZED;
}

// Device address of a __device__ symbol, looked up once per device and
// context: a new primary context (after cudaDeviceReset, or a context the host
// application created) gets its own lookup.
int symbol_address_cached(DeviceSymbolCache& cache, int (*lookup)(void**), void** out) {
  int dev = 0;
  if (int rc = cuda_status(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= DeviceSymbolCache::kMaxDevices)
    return set_error(QWEN_ERR_INVALID_ARGUMENT, "device %d beyond %d", dev,
                     DeviceSymbolCache::kMaxDevices);
  CUcontext ctx = nullptr;
  current_context(&ctx);  // null until the runtime has made a context current here
  std::lock_guard<std::mutex> lk(cache.mu);
  if (!ctx || cache.ctx[dev] != (void*)ctx || !cache.addr[dev]) {
    void* p = nullptr;
    // (cudaGetSymbolAddress also initialises the device's primary context when needed)
    if (int rc = lookup(&p)) return rc;
    if (current_context(&ctx) != CUDA_SUCCESS || !ctx)
      return set_error(QWEN_ERR_CUDA, "no current CUDA context on device %d", dev);
    cache.addr[dev] = p;
    cache.ctx[dev] = (void*)ctx;
  }
  *out = cache.addr[dev];
  return QWEN_OK;
}

static DeviceSymbolCache g_status_cache;

static int lookup_status(void** p) {
  return cuda_status(cudaGetSymbolAddress(p, g_ops_status), "cudaGetSymbolAddress(status word)");
}

int ops_status_word(int** out) {
  void* p = nullptr;
  QWEN_TRY(symbol_address_cached(g_status_cache, lookup_status, &p));
  *out = reinterpret_cast<int*>(p);
  return QWEN_OK;
}

}  // namespace qwen

using namespace qwen;

extern "C" int qwen_ops_status(void* stream) {
  int* word = nullptr;
  QWEN_TRY(ops_status_word(&word));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int h[4] = {0, 0, 0, 0};
  QWEN_CUDA(cudaMemcpyAsync(h, word, sizeof(h), cudaMemcpyDeviceToHost, st), "cudaMemcpyAsync(status)");
  QWEN_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  if (h[0] == kDevOk) return QWEN_OK;
  QWEN_CUDA(cudaMemsetAsync(word, 0, sizeof(h), st), "cudaMemsetAsync(status)");
  QWEN_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  if (h[0] == kDevWaitTimeout)
    return set_error(QWEN_ERR_DEVICE_TIMEOUT, "an operator kernel's bounded device wait gave up");
  return set_error(QWEN_ERR_INVALID_ARGUMENT,
                   "an operator kernel saw an out-of-range length or index on the device");
}
