// Library-level plumbing: error reporting, device error word, peer access / IPC helpers.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

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

namespace {
struct MapKey {
  uintptr_t ptr;
  int rank, dtype, dev;
  uint64_t dims[5], strides[5];
  uint32_t box[5];
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
    size_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return h;
  }
};
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}
}  // namespace

int make_tensor_map(CUtensorMap* out, const void* ptr, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int dtype) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  if (rank < 1 || rank > 5) {
    hx::set_error("make_tensor_map: rank %d", rank);
    return HX_ERR_INVALID;
  }
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.ptr = (uintptr_t)ptr;
  key.rank = rank;
  key.dtype = dtype;
  cudaGetDevice(&key.dev);
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i > 0) key.strides[i] = strides_bytes[i - 1];
  }
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return HX_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) {
    hx::set_error("cuTensorMapEncodeTiled unavailable");
    return HX_ERR_CUDA;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  CUtensorMapDataType dt = dtype == HX_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, dt, rank, const_cast<void*>(ptr), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    hx::set_error("cuTensorMapEncodeTiled failed (%d), rank %d, dims[0]=%llu", (int)r, rank,
                  (unsigned long long)dims[0]);
    return HX_ERR_CUDA;
  }
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 65536) cache.clear();
  cache.emplace(key, *out);
  return HX_OK;
}

int device_sm_count() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int n = 148;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = n;
  }
  return sms[dev];
}

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

int hx_mem_range(const void* device_ptr, void** base_out, size_t* size_out) {
  HX_REQUIRE(device_ptr && base_out && size_out, "hx_mem_range: null pointer");
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  if (!fn) {
    hx::set_error("cuMemGetAddressRange unavailable");
    return HX_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = fn(&base, &size, (CUdeviceptr)device_ptr);
  if (r != CUDA_SUCCESS) {
    hx::set_error("cuMemGetAddressRange failed (%d)", (int)r);
    return HX_ERR_CUDA;
  }
  *base_out = (void*)base;
  *size_out = size;
  return HX_OK;
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
