// Host runtime helpers exported with a C ABI: raw device allocations for
// receive rings (so their CUDA IPC handles cover exactly the ring), IPC
// export/import, peer access, device error-word reads, and events.
//
// Rings are allocated with cudaMalloc instead of the PyTorch caching
// allocator because a CUDA IPC handle names a whole allocation: with the
// caching allocator the importer would also need the offset inside a
// larger segment.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

namespace {
// Switches the calling thread to `device` and back to the device that was
// current before, so a helper never leaves another device's context current
// for the caller's next launch.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
}  // namespace

extern "C" {

int kvs_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

int kvs_malloc(int device, uint64_t bytes, void** out) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return -2;
  *out = p;
  return 0;
}

int kvs_free(int device, void* p) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  return cudaFree(p) == cudaSuccess ? 0 : -2;
}

int kvs_memset(void* p, int value, uint64_t bytes, void* stream) {
  return cudaMemsetAsync(p, value, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess ? 0
                                                                                          : -1;
}

// 64-byte opaque handle.
int kvs_ipc_get_handle(int device, void* ptr, uint8_t* handle_out) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) return -2;
  std::memcpy(handle_out, &h, sizeof(h));
  return static_cast<int>(sizeof(h));
}

int kvs_ipc_open_handle(int device, const uint8_t* handle, void** out) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return -2;
  *out = p;
  return 0;
}

int kvs_ipc_close_handle(int device, void* p) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  return cudaIpcCloseMemHandle(p) == cudaSuccess ? 0 : -2;
}

// 1 if `device` can address `peer` directly, 0 if not, negative on error.
int kvs_can_access_peer(int device, int peer) {
  int ok = 0;
  if (cudaDeviceCanAccessPeer(&ok, device, peer) != cudaSuccess) return -1;
  return ok;
}

int kvs_enable_peer_access(int device, int peer) {
  DeviceGuard guard(device);
  if (!guard.ok) return -1;
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return 0;
  }
  return e == cudaSuccess ? 0 : -2;
}

const char* kvs_last_error_string(void) { return cudaGetErrorString(cudaGetLastError()); }

int kvs_stream_sync(void* stream) {
  return cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) == cudaSuccess ? 0 : -1;
}

int kvs_library_version(void) { return 1; }

}  // extern "C"
