// K6: token embedding, fused residual-add + RMSNorm (and embedding + first-layer RMSNorm).
//
// Numerics follow hexgen/hexgen_core/modules/rms_norm.py:13-15 and block.py:126-129:
//   residual = round(h + residual)                         (activation dtype)
//   n        = round(float(residual) * rsqrt(mean(float(residual)^2) + eps))
//   out      = round(float(n) * float(weight))
// One CTA normalises one row; loads/stores are 16-byte vectors when the row allows it
// (16-bit rows up to 8192 wide: one vector per thread, one block barrier).
// HBM-bound: per row the kernel reads x (+add) and writes residual_out + out once.
#include "common.cuh"

namespace {

constexpr int kNormThreads = 256;

template <typename T>
struct Vec {
  static constexpr int N = 16 / sizeof(T);
  T v[N];
};

template <typename T>
HX_DEVICE float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float total = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) total += red[i];
  return total;
}

// x/add/residual_out/out rows are addressed via the row strides. `table_ids` switches the
// input to an embedding lookup (x = table, row index from ids).
template <typename T, bool kVec>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(
    const T* __restrict__ x, const T* __restrict__ add, T* __restrict__ residual_out,
    T* __restrict__ out, const T* __restrict__ weight, const int64_t* __restrict__ ids,
    int64_t hidden, int64_t in_stride, int64_t out_stride, float eps) {
  extern __shared__ float smem_row[];  // hidden floats: the residual row in f32
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const T* xr = ids ? x + ids[row] * hidden : x + row * in_stride;
  const T* ar = add ? add + row * in_stride : nullptr;
  float ss = 0.f;
  if (kVec) {
    constexpr int N = Vec<T>::N;
    const int64_t nv = hidden / N;
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
      Vec<T> a = *reinterpret_cast<const Vec<T>*>(xr + i * N);
      Vec<T> b;
      if (ar) b = *reinterpret_cast<const Vec<T>*>(ar + i * N);
      Vec<T> r;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float f = DT<T>::to_f(a.v[j]);
        if (ar) f = round_to<T>(f + DT<T>::to_f(b.v[j]));
        r.v[j] = DT<T>::from_f(f);
        smem_row[i * N + j] = f;
        ss += f * f;
      }
      if (residual_out) *reinterpret_cast<Vec<T>*>(residual_out + row * out_stride + i * N) = r;
    }
  } else {
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
      float f = DT<T>::to_f(xr[i]);
      if (ar) f = round_to<T>(f + DT<T>::to_f(ar[i]));
      smem_row[i] = f;
      if (residual_out) residual_out[row * out_stride + i] = DT<T>::from_f(f);
      ss += f * f;
    }
  }
  const float total = block_sum<T>(ss, red);
  const float rstd = rsqrtf(total / (float)hidden + eps);
  if (kVec) {
    constexpr int N = Vec<T>::N;
    const int64_t nv = hidden / N;
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
      Vec<T> w = *reinterpret_cast<const Vec<T>*>(weight + i * N);
      Vec<T> o;
#pragma unroll
      for (int j = 0; j < N; ++j) {
        float n = round_to<T>(smem_row[i * N + j] * rstd);
        o.v[j] = DT<T>::from_f(n * DT<T>::to_f(w.v[j]));
      }
      *reinterpret_cast<Vec<T>*>(out + row * out_stride + i * N) = o;
    }
  } else {
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
      float n = round_to<T>(smem_row[i] * rstd);
      out[row * out_stride + i] = DT<T>::from_f(n * DT<T>::to_f(weight[i]));
    }
  }
}

// One CTA per row, one 16-byte vector per thread (16-bit types, hidden a multiple of 8 up to
// 8192): every load of the row is issued at once and there is a single block barrier, which
// keeps latency low for the few rows of a decode step and is fully parallel for prefill rows.
// The residual is rounded to T before it is stored, so keeping it packed in T is exact.
template <typename T>
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(
    const T* __restrict__ x, const T* __restrict__ add, T* __restrict__ residual_out,
    T* __restrict__ out, const T* __restrict__ weight, const int64_t* __restrict__ ids,
    int64_t hidden, int64_t in_stride, int64_t out_stride, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const int64_t off = (int64_t)t * 8;
  const T* xr = ids ? x + ids[row] * hidden : x + row * in_stride;
  uint4 v = *reinterpret_cast<const uint4*>(xr + off);
  const uint4 wv = *reinterpret_cast<const uint4*>(weight + off);
  T* e = reinterpret_cast<T*>(&v);
  if (add) {
    const uint4 av = *reinterpret_cast<const uint4*>(add + row * in_stride + off);
    const T* ae = reinterpret_cast<const T*>(&av);
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = DT<T>::from_f(DT<T>::to_f(e[j]) + DT<T>::to_f(ae[j]));
  }
  if (residual_out) *reinterpret_cast<uint4*>(residual_out + row * out_stride + off) = v;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float f = DT<T>::to_f(e[j]);
    ss += f * f;
  }
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float total = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) total += red[i];
  const float rstd = rsqrtf(total / (float)hidden + eps);
  const T* we = reinterpret_cast<const T*>(&wv);
  T o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
    o[j] = DT<T>::from_f(round_to<T>(DT<T>::to_f(e[j]) * rstd) * DT<T>::to_f(we[j]));
  *reinterpret_cast<uint4*>(out + row * out_stride + off) = *reinterpret_cast<const uint4*>(o);
}

template <typename T>
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const T* __restrict__ table,
                                 int64_t vocab_start, int64_t vocab_rows, int64_t hidden,
                                 T* __restrict__ out) {
  const int64_t row = blockIdx.x;
  const int64_t id = ids[row] - vocab_start;
  const bool valid = id >= 0 && id < vocab_rows;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x)
    out[row * hidden + i] = valid ? table[id * hidden + i] : DT<T>::from_f(0.f);
}

template <typename T>
int launch_rmsnorm(const void* x, const void* add, void* residual_out, void* out,
                   const void* weight, const int64_t* ids, int64_t rows, int64_t hidden,
                   int64_t in_stride, int64_t out_stride, float eps, cudaStream_t stream) {
  if (rows == 0) return HX_OK;
  constexpr int N = 16 / sizeof(T);
  const bool vec = (hidden % N == 0) && (in_stride % N == 0) && (out_stride % N == 0) &&
                   ((uintptr_t)x % 16 == 0) && ((uintptr_t)out % 16 == 0) &&
                   ((uintptr_t)weight % 16 == 0) && (!add || (uintptr_t)add % 16 == 0) &&
                   (!residual_out || (uintptr_t)residual_out % 16 == 0);
  if constexpr (sizeof(T) == 2) {
    if (vec && hidden % 256 == 0 && hidden <= 8192) {
      const int s = hx::cuda_status(
          launch_ex(rmsnorm_vec_kernel<T>, dim3((unsigned)rows), dim3((unsigned)(hidden / 8)), 0,
                    stream, 1, (const T*)x, (const T*)add, (T*)residual_out, (T*)out,
                    (const T*)weight, ids, hidden, in_stride, out_stride, eps),
          "rmsnorm_vec_kernel launch");
      if (s) return s;
      HX_LAUNCH_CHECK("rmsnorm_vec_kernel");
      return HX_OK;
    }
  }
  const size_t smem = (size_t)hidden * sizeof(float);
  HX_REQUIRE(smem <= 200 * 1024, "hx_rmsnorm: hidden %lld too large", (long long)hidden);
  auto kern = vec ? rmsnorm_kernel<T, true> : rmsnorm_kernel<T, false>;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int s = hx::cuda_status(
      launch_ex(kern, dim3((unsigned)rows), dim3(kNormThreads), smem, stream, 1, (const T*)x,
                (const T*)add, (T*)residual_out, (T*)out, (const T*)weight, ids, hidden,
                in_stride, out_stride, eps),
      "rmsnorm_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("rmsnorm_kernel");
  return HX_OK;
}

}  // namespace

extern "C" {

int hx_rmsnorm(const void* x, const void* add, void* residual_out, void* out,
               const void* weight, int64_t rows, int64_t hidden, int64_t in_stride,
               int64_t out_stride, float eps, int dtype, void* stream) {
  HX_REQUIRE(x && out && weight && hidden > 0 && rows >= 0, "hx_rmsnorm: bad arguments");
  HX_REQUIRE(in_stride >= hidden && out_stride >= hidden, "hx_rmsnorm: bad strides");
  HX_DISPATCH_DTYPE(dtype, T,
                    return launch_rmsnorm<T>(x, add, residual_out, out, weight, nullptr, rows,
                                             hidden, in_stride, out_stride, eps,
                                             (cudaStream_t)stream));
  return HX_OK;
}

int hx_embed_rmsnorm(const int64_t* ids, int64_t rows, const void* table, int64_t hidden,
                     const void* weight, float eps, void* residual_out, void* normed_out,
                     int dtype, void* stream) {
  HX_REQUIRE(ids && table && weight && normed_out && residual_out && hidden > 0,
             "hx_embed_rmsnorm: bad arguments");
  HX_DISPATCH_DTYPE(dtype, T,
                    return launch_rmsnorm<T>(table, nullptr, residual_out, normed_out, weight,
                                             ids, rows, hidden, hidden, hidden, eps,
                                             (cudaStream_t)stream));
  return HX_OK;
}

int hx_embedding(const int64_t* ids, int64_t rows, const void* table, int64_t vocab_start,
                 int64_t vocab_rows, int64_t hidden, void* out, int dtype, void* stream) {
  HX_REQUIRE(ids && table && out && hidden > 0, "hx_embedding: bad arguments");
  if (rows == 0) return HX_OK;
  HX_DISPATCH_DTYPE(dtype, T, {
    embedding_kernel<T><<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(
        ids, (const T*)table, vocab_start, vocab_rows, hidden, (T*)out);
    HX_LAUNCH_CHECK("embedding_kernel");
  });
  return HX_OK;
}

}  // extern "C"
