// Exchange buffers of the vocabulary-parallel top-1 merge: allocation, IPC
// handles and peer mappings (host side; the device side is gsp_peer.cuh).
#include <cuda_runtime.h>

#include <cstring>

#include "../../include/gsp_b200.h"
#include "gsp_internal.h"

using namespace gsp;

static_assert(sizeof(cudaIpcMemHandle_t) == GSP_IPC_HANDLE_BYTES, "IPC handle size");
static_assert(kMaxPeers == GSP_MAX_PEERS, "peer count");

extern "C" {

size_t gsp_peer_exchange_bytes(int32_t world_size, int32_t max_batch) {
  if (world_size < 1 || world_size > kMaxPeers || max_batch < 1) return 0;
  return peer_exchange_bytes_for((size_t)world_size, (size_t)max_batch);
}

int32_t gsp_peer_exchange_alloc(size_t bytes, void** buffer, void* ipc_handle) {
  const char* fn = "gsp_peer_exchange_alloc";
  if (!buffer || !ipc_handle || bytes < kPeerKeysOffset)
    return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: need buffer, ipc_handle and at least %zu bytes", fn,
                        (size_t)kPeerKeysOffset);
  *buffer = nullptr;
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, bytes);
  if (err == cudaSuccess) err = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
  if (err != cudaSuccess) {
    if (p) cudaFree(p);
    return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return GSP_OK;
}

int32_t gsp_peer_exchange_open(const void* ipc_handle, void** peer_buffer) {
  const char* fn = "gsp_peer_exchange_open";
  if (!ipc_handle || !peer_buffer) return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: null argument", fn);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
  *peer_buffer = p;
  return GSP_OK;
}

int32_t gsp_peer_exchange_close(void* peer_buffer) {
  if (!peer_buffer) return GSP_OK;
  const cudaError_t err = cudaIpcCloseMemHandle(peer_buffer);
  if (err != cudaSuccess)
    return record_error(GSP_ERR_CUDA, "gsp_peer_exchange_close: %s", cudaGetErrorString(err));
  return GSP_OK;
}

int32_t gsp_peer_exchange_reset(void* buffer, int32_t world_size, int32_t max_batch) {
  const char* fn = "gsp_peer_exchange_reset";
  if (!buffer || world_size < 1 || world_size > kMaxPeers || max_batch < 1)
    return record_error(GSP_ERR_INVALID_ARGUMENT, "%s: bad buffer, world size or max_batch", fn);
  const cudaError_t err = cudaMemset(buffer, 0, peer_exchange_bytes_for((size_t)world_size, (size_t)max_batch));
  if (err != cudaSuccess) return record_error(GSP_ERR_CUDA, "%s: %s", fn, cudaGetErrorString(err));
  return GSP_OK;
}

int32_t gsp_peer_exchange_free(void* buffer) {
  if (!buffer) return GSP_OK;
  const cudaError_t err = cudaFree(buffer);
  if (err != cudaSuccess) return record_error(GSP_ERR_CUDA, "gsp_peer_exchange_free: %s", cudaGetErrorString(err));
  return GSP_OK;
}

}  // extern "C"
