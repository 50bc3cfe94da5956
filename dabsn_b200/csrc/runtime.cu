// Host runtime shared by the C-ABI entry points: error reporting and per-device
// kernel attribute caching.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <map>
#include <utility>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
std::mutex g_prep_mu;
// (kernel, device) -> largest dynamic shared-memory limit set so far.  The
// limit only ever grows, so a launch that needs less never lowers it under
// another configuration that needs more.
std::map<std::pair<const void*, int>, int> g_prepared;
}  // namespace

namespace dabsn {

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

// Identity of the current CUDA context (the driver's cuCtxGetCurrent, reached
// through the runtime's entry-point query so the library needs no -lcuda).
// Cached device addresses are keyed on it: after cudaDeviceReset the primary
// context, and with it every module's device symbols, is created anew.
const void* current_context() {
  using GetCtx = int (*)(void**);
  static GetCtx fn = []() -> GetCtx {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<GetCtx>(p);
    return nullptr;
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Raise the dynamic shared-memory limit of `kernel` on the current device the
// first time it is launched there with at least `smem_bytes`.
bool kernel_prepared(const void* kernel, int smem_bytes) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_prep_mu);
  auto key = std::make_pair(kernel, dev);
  auto it = g_prepared.find(key);
  if (it != g_prepared.end() && it->second >= smem_bytes) return true;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_bytes);
  if (err != cudaSuccess) {
    set_error("cudaFuncSetAttribute(smem=%d): %s", smem_bytes, cudaGetErrorString(err));
    return false;
  }
  g_prepared[key] = smem_bytes;
  return true;
}

int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(err));
    return DABSN_ERR_LAUNCH;
  }
  return DABSN_OK;
}

}  // namespace dabsn

__device__ int g_dabsn_status[1];

namespace dabsn {
// Device address of the status word on the current device (looked up once per
// device, context and host thread).
int* device_status() {
  static thread_local int dev_cached = -1;
  static thread_local const void* ctx_cached = nullptr;
  static thread_local int* ptr = nullptr;
  const int dev = current_device();
  const void* ctx = current_context();
  if (dev != dev_cached || ctx != ctx_cached || ptr == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dabsn_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    ptr = static_cast<int*>(p);
    dev_cached = dev;
    ctx_cached = ctx;
  }
  return ptr;
}
}  // namespace dabsn

// Status word of the bounded device waits on the current device (0 = none
// timed out).  Reading it synchronises the device; diagnostics and tests.
extern "C" int dabsn_device_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_dabsn_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(g_dabsn_status, &z, sizeof(int));
  }
  return v;
}

extern "C" const char* dabsn_version(void) { return "dabsn_b200 0.1.0 (sm_100a)"; }
extern "C" const char* dabsn_last_error(void) { return g_last_error; }
