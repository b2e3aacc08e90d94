// Error state, driver entry point and device error flag for the C ABI.
#include <cstring>
#include <mutex>

#include "host_common.h"

namespace tmb {

__device__ int g_device_error = 0;

namespace {
thread_local char t_msg[512] = {0};
}

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
  va_end(ap);
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TM_OK;
  return set_error(TM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// The flag's device address, looked up once per device (with that device
// current) and cached: the first launch on a device does the lookup, so that
// first launch must come before any stream capture on that device.
int* device_error_flag() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

}  // namespace tmb

extern "C" {

int tm_abi_version(void) { return 1; }

const char* tm_last_error(void) { return tmb::t_msg; }

int tm_device_error(int* code_out) {
  if (!code_out) return tmb::set_error(TM_ERR_INVALID_ARGUMENT, "tm_device_error: null output");
  int v = 0;
  int st = tmb::check_cuda(cudaDeviceSynchronize(), "tm_device_error: synchronize");
  if (st) return st;
  st = tmb::check_cuda(cudaMemcpyFromSymbol(&v, tmb::g_device_error, sizeof(int)),
                      "tm_device_error: read flag");
  if (st) return st;
  const int zero = 0;
  st = tmb::check_cuda(cudaMemcpyToSymbol(tmb::g_device_error, &zero, sizeof(int)),
                      "tm_device_error: clear flag");
  if (st) return st;
  *code_out = v;
  return TM_OK;
}

}  // extern "C"
