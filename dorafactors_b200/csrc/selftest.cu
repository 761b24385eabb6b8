// Self-test of the bounded-wait path every tcgen05 kernel relies on: one thread
// waits, with the kernels' own mbarrier wait loop but a short cycle limit, on a
// barrier phase that nothing completes.  The wait must give up, record
// DORA_ERR_DEVICE_TIMEOUT in the device error word and return, leaving the
// context usable.  No trap, no fault, no unbounded spin.
#include "tc_common.cuh"

namespace dora {
namespace tc {

__global__ void bounded_wait_selftest_kernel(long long limit_cycles, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival that never comes
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    bool done = mbar_try_wait(&bar, 0);
    while (!done && clock64() - t0 <= limit_cycles) done = mbar_try_wait(&bar, 0);
    if (!done) record_device_error(DORA_ERR_DEVICE_TIMEOUT);
    *gave_up = done ? 0 : 1;
  }
}

}  // namespace tc
}  // namespace dora

using namespace dora;

extern "C" int dora_selftest_bounded_wait(long long limit_cycles, int* gave_up_host, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > tc::kWaitCycles || !gave_up_host) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* d = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d), sizeof(int), st);
  if (e != cudaSuccess) return set_cuda_error(e);
  tc::bounded_wait_selftest_kernel<<<1, 32, 0, st>>>(limit_cycles, d);
  int rc = check_launch();
  if (rc == DORA_OK) {
    e = cudaMemcpyAsync(gave_up_host, d, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = set_cuda_error(e);
  }
  cudaFreeAsync(d, st);
  return rc;
}
