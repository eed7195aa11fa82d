// Set-up of the sequence-shard exchange buffers: one device buffer per rank,
// shared with the other ranks' processes through CUDA IPC handles (plain peer
// mappings over NVLink; no multicast object is created).  These calls
// allocate and map memory; they run once per decoder, never inside a step.
#include "tq_common.cuh"

#include <string.h>

using namespace tq;

static_assert(sizeof(cudaIpcMemHandle_t) == TQ_IPC_HANDLE_BYTES, "IPC handle size");

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return TQ_OK;
  cudaGetLastError();
  set_last_cuda_error(e);
  return TQ_E_CUDA;
}

extern "C" {

int tq_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return TQ_E_ARG;
  void* p = nullptr;
  int s = cuda_status(cudaMalloc(&p, bytes));
  if (s != TQ_OK) return s;
  s = cuda_status(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  if (s == TQ_OK) s = cuda_status(cudaIpcGetMemHandle(&h, p));
  if (s == TQ_OK) s = cuda_status(cudaDeviceSynchronize());
  if (s != TQ_OK) {
    cudaFree(p);
    return s;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return TQ_OK;
}

int tq_exchange_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return TQ_E_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  int s = cuda_status(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  if (s != TQ_OK) return s;
  *ptr = p;
  return TQ_OK;
}

int tq_exchange_close(void* ptr) {
  if (!ptr) return TQ_E_ARG;
  return cuda_status(cudaIpcCloseMemHandle(ptr));
}

int tq_exchange_free(void* ptr) {
  if (!ptr) return TQ_E_ARG;
  return cuda_status(cudaFree(ptr));
}

}  // extern "C"
