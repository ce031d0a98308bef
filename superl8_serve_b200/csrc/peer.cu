// Set-up-time peer plumbing for stage-to-stage stores over NVLink: peer access between GPUs
// of one process, and CUDA IPC for one-process-per-GPU pipelines (a receive buffer is
// allocated by its owner, exported as a 64-byte handle and mapped by the producer rank).
// None of these run on the decode hot path.
#include <cstring>

#include "common.cuh"

using namespace s8b;

extern "C" int s8b_enable_peer_access(int dev, int peer) {
  if (dev == peer) return S8B_OK;
  int can = 0;
  if (cudaDeviceCanAccessPeer(&can, dev, peer) != cudaSuccess || !can) {
    cudaGetLastError();
    return S8B_ERR_PEER;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(dev);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  cudaSetDevice(prev);
  if (e == cudaErrorPeerAccessAlreadyEnabled || e == cudaSuccess) {
    cudaGetLastError();
    return S8B_OK;
  }
  record_cuda_error(e);
  return S8B_ERR_PEER;
}

extern "C" int s8b_ipc_alloc(size_t bytes, void **ptr, void *handle_out) {
  if (!ptr || !handle_out || bytes == 0) return S8B_ERR_ARG;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  cudaMemset(*ptr, 0, bytes);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  return S8B_OK;
}

extern "C" int s8b_ipc_free(void *ptr) {
  if (!ptr) return S8B_OK;
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return S8B_OK;
}

extern "C" int s8b_ipc_open(const void *handle, void **ptr) {
  if (!handle || !ptr) return S8B_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_PEER;
  }
  return S8B_OK;
}

extern "C" int s8b_ipc_close(void *ptr) {
  if (!ptr) return S8B_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return S8B_OK;
}

extern "C" int s8b_ipc_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

// One stream-ordered copy between any two addresses the device can reach (device, peer, IPC
// mapped or pinned host), for set-up and host I/O around the decode step.
extern "C" int s8b_memcpy_async(void *dst, const void *src, size_t bytes, void *stream) {
  if (!dst || !src) return S8B_ERR_ARG;
  if (bytes == 0) return S8B_OK;
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, (cudaStream_t)stream);
  if (e != cudaSuccess) {
    record_cuda_error(e);
    return S8B_ERR_CUDA;
  }
  return S8B_OK;
}
