// K3: rotary embedding on q/k fused with the KV-cache write.
//
// Follows the flash_attn RotaryEmbedding used by the native model (hexgen/hexgen_core/
// modules/mha.py:382-384, :557; flash-attn 2.7.4.post1 layers/rotary.py): cos/sin tables are
// computed in f32 and cached in the activation dtype, the rotation is evaluated in f32
//   o0 = x0 * cos - x1 * sin,  o1 = x0 * sin + x1 * cos
// and stored in the activation dtype. Pairs are (x[2i], x[2i+1]) when interleaved (the
// native Llama layout after remap_state_dict.py:88-103) or (x[i], x[i+d/2]) otherwise.
// The cache write reproduces _update_kv_cache (mha.py:255-288):
//   cache[b0 + b, pos, 0] = rope(k);  cache[b0 + b, pos, 1] = v.
// One thread handles one rotation pair (or two v elements); HBM-bound.
#include "common.cuh"

namespace {

template <typename T, bool kInterleaved>
__global__ void rotary_cache_kernel(const T* __restrict__ qkv, int64_t seqlen, int n_heads,
                                    int n_heads_kv, int head_dim, const int32_t* __restrict__ pos_start,
                                    const T* __restrict__ cos_t, const T* __restrict__ sin_t,
                                    int64_t table_rows, T* __restrict__ q_out, T* __restrict__ cache,
                                    int64_t cache_batch_stride, int64_t cache_seq_stride,
                                    int64_t cache_batch_offset, int64_t cache_max_seq) {
  const int64_t token = blockIdx.x;  // b * seqlen + s
  const int64_t b = token / seqlen, s = token % seqlen;
  const int64_t pos = (int64_t)pos_start[b] + s;
  if (pos < 0 || pos >= cache_max_seq || pos >= table_rows) {
    if (threadIdx.x == 0) record_device_error(HX_DEVERR_BAD_ARGUMENT);
    return;
  }
  const int half = head_dim / 2;
  const int n_qk = n_heads + n_heads_kv;         // heads that get rotated
  const int total_pairs = n_qk * half;            // rotation pairs for this token
  const int v_pairs = n_heads_kv * half;          // v elements copied two at a time
  const T* src = qkv + token * (int64_t)(n_heads + 2 * n_heads_kv) * head_dim;
  T* kv_dst = cache + (cache_batch_offset + b) * cache_batch_stride + pos * cache_seq_stride;
  const T* cs = cos_t + pos * half;
  const T* sn = sin_t + pos * half;
  for (int p = threadIdx.x; p < total_pairs + v_pairs; p += blockDim.x) {
    if (p < total_pairs) {
      const int h = p / half, i = p % half;
      const int i0 = kInterleaved ? 2 * i : i;
      const int i1 = kInterleaved ? 2 * i + 1 : i + half;
      const T* xh = src + (int64_t)h * head_dim;
      const float x0 = DT<T>::to_f(xh[i0]), x1 = DT<T>::to_f(xh[i1]);
      const float c = DT<T>::to_f(cs[i]), sv = DT<T>::to_f(sn[i]);
      const float o0 = x0 * c - x1 * sv;
      const float o1 = x0 * sv + x1 * c;
      T* dst;
      if (h < n_heads) {
        dst = q_out + (token * n_heads + h) * (int64_t)head_dim;
      } else {
        dst = kv_dst + (int64_t)(h - n_heads) * head_dim;  // k slot: [0, hk, :]
      }
      dst[i0] = DT<T>::from_f(o0);
      dst[i1] = DT<T>::from_f(o1);
    } else {
      const int e = (p - total_pairs) * 2;  // element index inside [n_heads_kv * head_dim]
      const T* vsrc = src + (int64_t)n_qk * head_dim;
      T* vdst = kv_dst + (int64_t)n_heads_kv * head_dim;  // v slot: [1, :, :]
      vdst[e] = vsrc[e];
      vdst[e + 1] = vsrc[e + 1];
    }
  }
}

// Interleaved layout, vectorised: one thread per 16-byte chunk of the packed qkv row. A chunk
// of q or k holds whole (x[2i], x[2i+1]) pairs, so the rotation needs only the matching
// cos/sin entries of the same position; v chunks are copied. Grid = tokens x chunks.
template <typename T>
__global__ void __launch_bounds__(256) rotary_vec_kernel(
    const T* __restrict__ qkv, int64_t n_tokens, int64_t seqlen, int n_heads, int n_heads_kv,
    int head_dim, const int32_t* __restrict__ pos_start, const T* __restrict__ cos_t,
    const T* __restrict__ sin_t, int64_t table_rows, T* __restrict__ q_out, T* __restrict__ cache,
    int64_t cache_batch_stride, int64_t cache_seq_stride, int64_t cache_batch_offset,
    int64_t cache_max_seq) {
  constexpr int N = 16 / sizeof(T);
  const int chunks = (n_heads + 2 * n_heads_kv) * head_dim / N;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_tokens * chunks) return;
  const int64_t token = i / chunks;
  const int c = (int)(i - token * chunks);
  const int64_t b = token / seqlen, s = token - b * seqlen;
  const int64_t pos = (int64_t)pos_start[b] + s;
  if (pos < 0 || pos >= cache_max_seq || pos >= table_rows) {
    record_device_error(HX_DEVERR_BAD_ARGUMENT);
    return;
  }
  const int elem = c * N;
  const int head = elem / head_dim, within = elem - head * head_dim;
  const uint4 raw = *reinterpret_cast<const uint4*>(qkv + token * (int64_t)chunks * N + elem);
  T* kv_dst = cache + (cache_batch_offset + b) * cache_batch_stride + pos * cache_seq_stride;
  if (head >= n_heads + n_heads_kv) {  // v: plain copy into the cache's v slot
    *reinterpret_cast<uint4*>(kv_dst + (int64_t)n_heads_kv * head_dim +
                              (int64_t)(head - n_heads - n_heads_kv) * head_dim + within) = raw;
    return;
  }
  const T* x = reinterpret_cast<const T*>(&raw);
  const int half = head_dim / 2;
  const T* cs = cos_t + pos * half + within / 2;
  const T* sn = sin_t + pos * half + within / 2;
  T o[N];
#pragma unroll
  for (int p = 0; p < N / 2; ++p) {
    const float x0 = DT<T>::to_f(x[2 * p]), x1 = DT<T>::to_f(x[2 * p + 1]);
    const float cv = DT<T>::to_f(cs[p]), sv = DT<T>::to_f(sn[p]);
    o[2 * p] = DT<T>::from_f(x0 * cv - x1 * sv);
    o[2 * p + 1] = DT<T>::from_f(x0 * sv + x1 * cv);
  }
  T* dst = head < n_heads ? q_out + token * (int64_t)n_heads * head_dim + elem
                          : kv_dst + (int64_t)(head - n_heads) * head_dim + within;
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
}

}  // namespace

extern "C" int hx_rotary_cache_write(const void* qkv, int64_t batch, int64_t seqlen,
                                     int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                                     const int32_t* pos_start, const void* cos_table,
                                     const void* sin_table, int64_t table_rows, int interleaved,
                                     void* q_out, void* cache, int64_t cache_batch_stride,
                                     int64_t cache_seq_stride, int64_t cache_batch_offset,
                                     int64_t cache_max_seq, int dtype, void* stream) {
  HX_REQUIRE(qkv && pos_start && cos_table && sin_table && q_out && cache,
             "hx_rotary_cache_write: null pointer");
  HX_REQUIRE(head_dim > 0 && head_dim % 2 == 0 && n_heads > 0 && n_heads_kv > 0 &&
                 n_heads % n_heads_kv == 0,
             "hx_rotary_cache_write: bad head configuration");
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim, "hx_rotary_cache_write: bad stride");
  if (batch == 0 || seqlen == 0) return HX_OK;
  const int threads = 128;
  const int esz = dtype == HX_F32 ? 4 : 2;
  const bool vec = interleaved && (head_dim * esz) % 16 == 0 && (uintptr_t)qkv % 16 == 0 &&
                   (uintptr_t)q_out % 16 == 0 && (uintptr_t)cache % 16 == 0 &&
                   (cache_seq_stride * esz) % 16 == 0 && (cache_batch_stride * esz) % 16 == 0;
  if (vec) {
    HX_DISPATCH_DTYPE(dtype, T, {
      const int64_t n_tokens = batch * seqlen;
      const int64_t total = n_tokens * (n_heads + 2 * n_heads_kv) * head_dim / (16 / sizeof(T));
      rotary_vec_kernel<T><<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
          (const T*)qkv, n_tokens, seqlen, (int)n_heads, (int)n_heads_kv, (int)head_dim,
          pos_start, (const T*)cos_table, (const T*)sin_table, table_rows, (T*)q_out, (T*)cache,
          cache_batch_stride, cache_seq_stride, cache_batch_offset, cache_max_seq);
      HX_LAUNCH_CHECK("rotary_vec_kernel");
    });
    return HX_OK;
  }
  HX_DISPATCH_DTYPE(dtype, T, {
    auto kern = interleaved ? rotary_cache_kernel<T, true> : rotary_cache_kernel<T, false>;
    kern<<<(unsigned)(batch * seqlen), threads, 0, (cudaStream_t)stream>>>(
        (const T*)qkv, seqlen, (int)n_heads, (int)n_heads_kv, (int)head_dim, pos_start,
        (const T*)cos_table, (const T*)sin_table, table_rows, (T*)q_out, (T*)cache,
        cache_batch_stride, cache_seq_stride, cache_batch_offset, cache_max_seq);
    HX_LAUNCH_CHECK("rotary_cache_kernel");
  });
  return HX_OK;
}
