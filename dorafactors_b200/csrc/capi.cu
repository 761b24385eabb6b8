// Library-wide C ABI entry points: version, status text, CUDA error text and
// the device error word.
#include <atomic>
#include <cstdio>
#include <cstring>

#include "dora_common.cuh"

namespace dora {

__device__ int g_device_error = 0;

static thread_local char g_last_cuda_error[256] = "";
static std::atomic<unsigned long long> g_launches{0};

void count_launches(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }

int set_cuda_error(cudaError_t e) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return DORA_ERR_CUDA;
}

}  // namespace dora

using namespace dora;

extern "C" int dora_version(void) { return 100; }  // 0.1.0

extern "C" const char* dora_status_string(int status) {
  switch (status) {
    case DORA_OK: return "ok";
    case DORA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DORA_ERR_UNSUPPORTED: return "unsupported";
    case DORA_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case DORA_ERR_CUDA: return "CUDA error";
    case DORA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* dora_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" unsigned long long dora_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int dora_device_error(int reset, int* out) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_cuda_error(e);
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (e != cudaSuccess) return set_cuda_error(e);
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return set_cuda_error(e);
  }
  if (out) *out = v;
  return DORA_OK;
}
