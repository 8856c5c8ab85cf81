// Greedy sampling: row-wise argmax with torch.argmax tie-breaking (first maximal index).
// Replaces logits.argmax(-1) at hexgen2/model.py:82 and :117. One CTA per row.
#include "common.cuh"

namespace {

HX_DEVICE void better(float& bv, int64_t& bi, float v, int64_t i) {
  // NaN propagates as the maximum, like torch.argmax.
  if (v > bv || (v == bv && i < bi) || (isnan(v) && !isnan(bv)) ||
      (isnan(v) && isnan(bv) && i < bi)) {
    bv = v;
    bi = i;
  }
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ logits, int64_t cols, int64_t ld,
                              int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const T* row = logits + (int64_t)blockIdx.x * ld;
  float bv = -INFINITY;
  int64_t bi = cols;  // sentinel larger than any index
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte load
  if (sizeof(T) < 4 && ((uintptr_t)row % 16) == 0) {
    // 16-byte loads, four in flight per thread before any compare; the order of the compares
    // does not matter (better() prefers the larger value, then the smaller index).
    const int64_t nvec = cols / V;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    for (int64_t base = threadIdx.x; base < nvec; base += 4 * (int64_t)blockDim.x) {
      uint4 raw[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t vi = base + (int64_t)u * blockDim.x;
        raw[u] = vi < nvec ? rv[vi] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t vi = base + (int64_t)u * blockDim.x;
        if (vi >= nvec) break;
        const T* e = reinterpret_cast<const T*>(&raw[u]);
#pragma unroll
        for (int j = 0; j < V; ++j) better(bv, bi, DT<T>::to_f(e[j]), vi * V + j);
      }
    }
    for (int64_t i = nvec * V + threadIdx.x; i < cols; i += blockDim.x)
      better(bv, bi, DT<T>::to_f(row[i]), i);
  } else {
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) better(bv, bi, DT<T>::to_f(row[i]), i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, ov, oi);
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(bv, bi, sv[w], si[w]);
    out[blockIdx.x] = bi < cols ? bi : 0;
  }
}

}  // namespace

extern "C" int hx_argmax(const void* logits, int64_t rows, int64_t cols, int64_t ld,
                         int64_t* out_idx, int dtype, void* stream) {
  HX_REQUIRE(logits && out_idx && cols > 0 && ld >= cols, "hx_argmax: bad arguments");
  if (rows == 0) return HX_OK;
  HX_DISPATCH_DTYPE(dtype, T, {
    const int s = hx::cuda_status(
        launch_ex(argmax_kernel<T>, dim3((unsigned)rows), dim3(1024), 0, (cudaStream_t)stream, 1,
                  (const T*)logits, cols, ld, out_idx),
        "argmax_kernel launch");
    if (s) return s;
    HX_LAUNCH_CHECK("argmax_kernel");
  });
  return HX_OK;
}
