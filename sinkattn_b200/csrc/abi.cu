// abi.cu — host-side plumbing of the C ABI: thread-local error messages,
// the driver's cuTensorMapEncodeTiled resolved through the runtime (so the
// library needs no -lcuda), and cached per-device SM counts.

#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <set>
#include <tuple>

#include "sa_common.cuh"

namespace sa {

namespace {
thread_local char g_err[512] = "";
std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;
int g_sm_count[64] = {};
// (device, kernel, attribute, value) already applied by func_attr_once
std::set<std::tuple<int, const void*, int, int>> g_attrs;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t e, const char* what) {
  set_error("%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  return SA_ECUDA;
}

EncodeTiledFn encode_tiled_fn() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode != nullptr) return g_encode;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
    set_error("cannot resolve cuTensorMapEncodeTiled (%s)",
              e != cudaSuccess ? cudaGetErrorString(e) : "symbol not found");
    return nullptr;
  }
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return g_encode;
}

int sm_count_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_sm_count[dev] > 0) return g_sm_count[dev];
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_sm_count[dev] = n;
  }
  return n;
}

int func_attr_once(const void* func, cudaFuncAttribute attr, int value) {
  int dev = 0;
  SA_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_mu);
  const auto key = std::make_tuple(dev, func, (int)attr, value);
  if (g_attrs.count(key) != 0) return SA_OK;
  SA_CUDA_TRY(cudaFuncSetAttribute(func, attr, value));
  g_attrs.insert(key);
  return SA_OK;
}

}  // namespace sa

extern "C" const char* sa_last_error(void) { return sa::g_err; }

extern "C" int sa_version(void) { return 1; }

extern "C" int sa_device_sm_count(void) { return sa::sm_count_current_device(); }
