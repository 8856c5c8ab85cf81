// Library-level plumbing: error reporting, device error word, peer access / IPC helpers.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

__device__ int g_hx_device_error = 0;

namespace hx {
static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HX_OK;
  set_error("%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
  return HX_ERR_CUDA;
}
}  // namespace hx

extern "C" {

int hx_abi_version(void) { return 1; }

const char* hx_last_error(void) { return hx::g_last_error; }

int hx_device_error(int clear) {
  int err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return -hx::cuda_status((cudaError_t)err, "cudaDeviceSynchronize");
  int value = 0;
  if (cudaMemcpyFromSymbol(&value, g_hx_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear) {
    int zero = 0;
    cudaMemcpyToSymbol(g_hx_device_error, &zero, sizeof(int));
  }
  return value;
}

int hx_sm_count(void) {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return n;
}

int hx_enable_peer_access(int peer_device) {
  int dev = 0;
  int s = hx::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (s) return s;
  if (peer_device == dev) return HX_OK;
  int can = 0;
  s = hx::cuda_status(cudaDeviceCanAccessPeer(&can, dev, peer_device), "cudaDeviceCanAccessPeer");
  if (s) return s;
  if (!can) {
    hx::set_error("device %d cannot access peer %d", dev, peer_device);
    return HX_ERR_UNSUPPORTED;
  }
  cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return HX_OK;
  }
  return hx::cuda_status(e, "cudaDeviceEnablePeerAccess");
}

int hx_ipc_get_handle(const void* device_ptr, void* handle_out_64_bytes) {
  HX_REQUIRE(device_ptr && handle_out_64_bytes, "hx_ipc_get_handle: null pointer");
  cudaIpcMemHandle_t h;
  int s = hx::cuda_status(cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr)),
                          "cudaIpcGetMemHandle");
  if (s) return s;
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  memcpy(handle_out_64_bytes, &h, sizeof(h));
  return HX_OK;
}

int hx_ipc_open_handle(const void* handle_64_bytes, void** device_ptr_out) {
  HX_REQUIRE(handle_64_bytes && device_ptr_out, "hx_ipc_open_handle: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle_64_bytes, sizeof(h));
  return hx::cuda_status(cudaIpcOpenMemHandle(device_ptr_out, h, cudaIpcMemLazyEnablePeerAccess),
                         "cudaIpcOpenMemHandle");
}

int hx_ipc_close_handle(void* device_ptr) {
  return hx::cuda_status(cudaIpcCloseMemHandle(device_ptr), "cudaIpcCloseMemHandle");
}

int hx_peer_copy(void* dst, int dst_device, const void* src, int src_device, size_t bytes,
                 void* stream) {
  if (bytes == 0) return HX_OK;
  HX_REQUIRE(dst && src, "hx_peer_copy: null pointer");
  return hx::cuda_status(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, bytes,
                                             (cudaStream_t)stream),
                         "cudaMemcpyPeerAsync");
}

}  // extern "C"
