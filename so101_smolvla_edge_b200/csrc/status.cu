// The device status word kernels record bounded-wait timeouts into, and the library version.
#include <mutex>

#include "common.cuh"

namespace so101 {

__device__ int g_device_status = 0;

int* status_ptr() {
  // one address per device, looked up on first use (cudaGetSymbolAddress needs the device current)
  static int* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

bool g_pdl = false;
bool pdl_enabled() { return g_pdl; }

thread_local cudaError_t g_last_error = cudaSuccess;

int launch_error(cudaError_t e) {
  g_last_error = e;
  cudaGetLastError();  // a failed launch leaves no sticky error; clear the non-sticky one
  return SO101_ERR_LAUNCH;
}

}  // namespace so101

extern "C" int so101_set_pdl(int enable) {
  so101::g_pdl = enable != 0;
  return SO101_OK;
}

extern "C" int so101_device_status(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, so101::g_device_status, sizeof(int)) != cudaSuccess) return SO101_ERR_LAUNCH;
  return v;
}

extern "C" int so101_clear_device_status(void) {
  const int zero = 0;
  return cudaMemcpyToSymbol(so101::g_device_status, &zero, sizeof(int)) == cudaSuccess ? SO101_OK
                                                                                       : SO101_ERR_LAUNCH;
}

extern "C" const char* so101_last_error(void) {
  return so101::g_last_error == cudaSuccess ? "" : cudaGetErrorString(so101::g_last_error);
}

extern "C" const char* so101_version(void) { return "so101_b200 0.1.0 sm_100a"; }
