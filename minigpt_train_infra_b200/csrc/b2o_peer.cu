// Peer memory for the fused ZeRO-1 collectives: device buffers other processes of the node map
// into their own address space, with legacy CUDA IPC (cudaMalloc + cudaIpcGetMemHandle /
// cudaIpcOpenMemHandle).  Accesses through these mappings are plain loads and stores over
// NVLink; no multicast object is created.
#include <cuda_runtime.h>

#include <cstring>

#include "b200_optim.h"

static_assert(sizeof(cudaIpcMemHandle_t) == B2O_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int b2o_peer_alloc(size_t bytes, void** ptr_out) {
  if (!ptr_out || bytes == 0) return B2O_ERR_ARG;
  *ptr_out = nullptr;
  return cudaMalloc(ptr_out, bytes) == cudaSuccess ? B2O_OK : B2O_ERR_CUDA;
}

extern "C" int b2o_peer_free(void* ptr) {
  if (!ptr) return B2O_ERR_ARG;
  return cudaFree(ptr) == cudaSuccess ? B2O_OK : B2O_ERR_CUDA;
}

extern "C" int b2o_peer_export(void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return B2O_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return B2O_ERR_CUDA;
  std::memcpy(handle_out, &h, sizeof(h));
  return B2O_OK;
}

extern "C" int b2o_peer_import(const void* handle, void** ptr_out) {
  if (!handle || !ptr_out) return B2O_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr_out = nullptr;
  return cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? B2O_OK
             : B2O_ERR_CUDA;
}

extern "C" int b2o_peer_close(void* ptr) {
  if (!ptr) return B2O_ERR_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? B2O_OK : B2O_ERR_CUDA;
}
