// Host-side symmetric-memory helpers: device buffers allocated outside any caching allocator (so an IPC handle
// names exactly one buffer), CUDA IPC export/import, and peer access between devices of one process.
//
// A handle is opened on the importing process's current device with lazy peer access, so the returned pointer
// is valid for kernels running on that device and reaches the exporting GPU's memory over NVLink. (Opening it in
// the exporting device's context instead yields a pointer that kernels on the importing device cannot use.)
#include <cuda_runtime.h>
#include <cstring>

extern "C" {

int sdc_symm_alloc(unsigned long long bytes, void** ptr) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  *ptr = p;
  return 0;
}

int sdc_symm_free(void* ptr) { return static_cast<int>(cudaFree(ptr)); }

int sdc_ipc_handle(void* ptr, void* out) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return static_cast<int>(e);
  std::memcpy(out, &h, sizeof(h));
  return 0;
}

int sdc_ipc_handle_bytes() { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int sdc_ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int sdc_ipc_close(void* ptr) { return static_cast<int>(cudaIpcCloseMemHandle(ptr)); }

// Lets kernels on the current device read and write `peer`'s memory directly (one process, several GPUs).
int sdc_enable_peer_access(int peer) {
  int can = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceCanAccessPeer(&can, dev, peer);
  if (!can) return -1;
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return 0;
  }
  return static_cast<int>(e);
}

}  // extern "C"
