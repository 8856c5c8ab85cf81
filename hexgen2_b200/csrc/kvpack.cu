// K9: live-position gather-pack of KV caches into one contiguous buffer (and the inverse).
//
// The reference sends the live slice of every layer's cache, t[:, :L].contiguous()
// (hexgen2/model.py:81), as one NCCL message per layer (hexgen2/transport.py:54-59), and the
// decode side copies it back into a capacity-sized cache (hexgen2/model.py:103-109). Here one
// launch moves the live rows of every request and every layer: the source of request r is
// viewed as [n_outer][cap_rows][row_bytes] and its first live_rows[r] rows of every outer
// slice land densely at dst + dst_offsets[r]. When dst is a peer GPU's buffer (peer access or
// an IPC mapping), the stores cross NVLink directly, so pack and transfer are one pass.
// Pure byte movement: 16-byte vector loads/stores, 4 vectors in flight per thread.
#include "common.cuh"

namespace {

constexpr int kPackThreads = 256;
constexpr int kUnroll = 4;

struct PackGeom {
  int64_t n_outer, outer_stride, row_stride, row_vecs;
};

// Maps flat vector index v of request r to (outer, row, chunk) and returns the byte offset
// inside the capacity-sized cache. Idx is 32-bit when every request's vector count fits (the
// usual case: 80 layers x 4096 rows x 256 vectors < 2^32), which keeps the two divisions
// per vector cheap.
template <typename Idx>
HX_DEVICE int64_t cache_offset(Idx v, Idx live, const PackGeom& g) {
  const Idx row_vecs = (Idx)g.row_vecs;
  const Idx per_outer = live * row_vecs;
  const Idx outer = v / per_outer;
  const Idx rem = v - outer * per_outer;
  const Idx row = rem / row_vecs;
  const Idx c = rem - row * row_vecs;
  return (int64_t)outer * g.outer_stride + (int64_t)row * g.row_stride + (int64_t)c * 16;
}

template <bool kPack, typename Idx>
__global__ void __launch_bounds__(kPackThreads) kv_pack_kernel(
    const uint64_t* __restrict__ cache_ptrs, const int64_t* __restrict__ live_rows,
    const int64_t* __restrict__ packed_offsets, uint8_t* packed, PackGeom g) {
  const int r = blockIdx.y;
  const uint64_t live = (uint64_t)live_rows[r];
  const uint64_t total = (uint64_t)g.n_outer * live * (uint64_t)g.row_vecs;
  uint8_t* cache = reinterpret_cast<uint8_t*>(cache_ptrs[r]);
  uint8_t* pk = packed + packed_offsets[r];
  const uint64_t stride = (uint64_t)gridDim.x * kPackThreads * kUnroll;
  for (uint64_t base = ((uint64_t)blockIdx.x * kPackThreads * kUnroll) + threadIdx.x; base < total;
       base += stride) {
    uint4 buf[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint64_t v = base + (uint64_t)u * kPackThreads;
      if (v < total) {
        if (kPack)
          buf[u] = __ldg(reinterpret_cast<const uint4*>(cache + cache_offset<Idx>((Idx)v, (Idx)live, g)));
        else
          buf[u] = __ldg(reinterpret_cast<const uint4*>(pk + v * 16));
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const uint64_t v = base + (uint64_t)u * kPackThreads;
      if (v < total) {
        if (kPack)
          *reinterpret_cast<uint4*>(pk + v * 16) = buf[u];
        else
          *reinterpret_cast<uint4*>(cache + cache_offset<Idx>((Idx)v, (Idx)live, g)) = buf[u];
      }
    }
  }
}

int launch(bool pack, const uint64_t* cache_ptrs, const int64_t* live_rows,
           const int64_t* packed_offsets, void* packed, int64_t n_req, int64_t n_outer,
           int64_t outer_stride_bytes, int64_t row_stride_bytes, int64_t row_bytes,
           int64_t max_live_rows, cudaStream_t stream) {
  HX_REQUIRE(cache_ptrs && live_rows && packed_offsets && packed, "hx_kv_pack: null pointer");
  HX_REQUIRE(row_bytes > 0 && row_bytes % 16 == 0 && outer_stride_bytes % 16 == 0 &&
                 row_stride_bytes % 16 == 0 && (uintptr_t)packed % 16 == 0,
             "hx_kv_pack: rows, strides and buffers must be 16-byte multiples");
  HX_REQUIRE(n_outer >= 0 && max_live_rows >= 0 && n_req >= 0 && n_req < 65536,
             "hx_kv_pack: bad sizes");
  if (n_req == 0 || n_outer == 0 || max_live_rows == 0) return HX_OK;
  PackGeom g{n_outer, outer_stride_bytes, row_stride_bytes, row_bytes / 16};
  const int64_t max_vecs = n_outer * max_live_rows * (row_bytes / 16);
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Enough CTAs to keep ~8 resident per SM across all requests.
  int64_t want = ceil_div(max_vecs, (int64_t)kPackThreads * kUnroll);
  int64_t cap = std::max<int64_t>(1, (int64_t)sms * 8 / n_req);
  int gx = (int)std::min<int64_t>(std::max<int64_t>(want, 1), std::max<int64_t>(cap, 1));
  dim3 grid(gx, (unsigned)n_req);
  // 32-bit index math when no request can hold 2^32 vectors (plus the grid stride's headroom).
  const bool small = max_vecs + (int64_t)gx * kPackThreads * kUnroll < (int64_t(1) << 32);
  if (pack && small)
    kv_pack_kernel<true, uint32_t><<<grid, kPackThreads, 0, stream>>>(
        cache_ptrs, live_rows, packed_offsets, (uint8_t*)packed, g);
  else if (pack)
    kv_pack_kernel<true, uint64_t><<<grid, kPackThreads, 0, stream>>>(
        cache_ptrs, live_rows, packed_offsets, (uint8_t*)packed, g);
  else if (small)
    kv_pack_kernel<false, uint32_t><<<grid, kPackThreads, 0, stream>>>(
        cache_ptrs, live_rows, packed_offsets, (uint8_t*)packed, g);
  else
    kv_pack_kernel<false, uint64_t><<<grid, kPackThreads, 0, stream>>>(
        cache_ptrs, live_rows, packed_offsets, (uint8_t*)packed, g);
  HX_LAUNCH_CHECK("kv_pack_kernel");
  return HX_OK;
}

}  // namespace

extern "C" {

int hx_kv_pack(const uint64_t* src_ptrs, const int64_t* live_rows, const int64_t* dst_offsets,
               int64_t n_req, int64_t n_outer, int64_t outer_stride_bytes,
               int64_t row_stride_bytes, int64_t row_bytes, int64_t max_live_rows, void* dst,
               void* stream) {
  return launch(true, src_ptrs, live_rows, dst_offsets, dst, n_req, n_outer, outer_stride_bytes,
                row_stride_bytes, row_bytes, max_live_rows, (cudaStream_t)stream);
}

int hx_kv_unpack(const void* src, const int64_t* src_offsets, const int64_t* live_rows,
                 const uint64_t* dst_ptrs, int64_t n_req, int64_t n_outer,
                 int64_t outer_stride_bytes, int64_t row_stride_bytes, int64_t row_bytes,
                 int64_t max_live_rows, void* stream) {
  return launch(false, dst_ptrs, live_rows, src_offsets, const_cast<void*>(src), n_req, n_outer,
                outer_stride_bytes, row_stride_bytes, row_bytes, max_live_rows,
                (cudaStream_t)stream);
}

}  // extern "C"
