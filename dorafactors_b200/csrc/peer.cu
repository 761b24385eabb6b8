// Peer-writable device buffers for the row-sharded layer's fused all-gather.
//
// dora_linear_output_fwd_allgather stores into every rank's output buffer
// through pointers valid in the storing process.  These functions make such
// buffers with plain CUDA IPC: each rank allocates its buffer with cudaMalloc
// (IPC needs the base of an allocation, which a caching allocator's tensors
// need not be), exports a 64-byte handle, the ranks exchange handles through
// their process group, and each opens the others' handles (peer access
// enabled lazily).  The mapping is an ordinary NVLink peer mapping: no
// multicast object is created, so a rank that exits cannot leave memory bound
// to one.
//
// Teardown order is the caller's: every importer closes its mappings of a
// buffer before the exporter frees it.
#include <string.h>

#include "dora_common.cuh"

using namespace dora;

static_assert(sizeof(cudaIpcMemHandle_t) == DORA_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int dora_peer_buffer_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes == 0) return DORA_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return set_cuda_error(e);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_cuda_error(e);
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return DORA_OK;
}

extern "C" int dora_peer_buffer_open(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) return DORA_ERR_INVALID_ARGUMENT;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_cuda_error(e);
  *ptr = p;
  return DORA_OK;
}

extern "C" int dora_peer_buffer_close(void* ptr) {
  if (!ptr) return DORA_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? DORA_OK : set_cuda_error(e);
}

extern "C" int dora_peer_buffer_free(void* ptr) {
  if (!ptr) return DORA_ERR_INVALID_ARGUMENT;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? DORA_OK : set_cuda_error(e);
}
