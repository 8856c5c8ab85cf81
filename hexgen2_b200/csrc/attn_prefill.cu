// K4: causal prefill attention over the KV cache (CUDA-core kernel: f32 and head_dim 32;
// f16/bf16 with head_dim 64/128 run on the tcgen05 kernel in attn_prefill_tc.cu).
//
// Semantics: flash_attn_kvpacked_func(q, kv, causal=True) as called by the native model
// during prefill (hexgen/hexgen_core/modules/mha.py:566-569), with FlashAttention-2's
// bottom-right causal alignment: query s of sequence b sits at absolute position
// p = pos_start[b] + s and attends to cache keys 0..p. Numerics follow FlashAttention-2: f32
// scores and online softmax (base 2), probabilities rounded to the activation dtype before the
// P.V product, f32 accumulation, output O / l rounded to the activation dtype.
//
// One CTA = 64 queries of one head; K/V tiles of 64 keys are staged through shared memory as
// f32 and both products are register-blocked (4 x 8 scores, 4 x D/8 outputs per thread).
#include "common.cuh"

namespace {

constexpr int kQ = 64, kK = 64, kThreads = 128;

template <int D>
struct PSmem {
  float qt[D][kQ];          // Q^T, pre-scaled by softmax_scale * log2(e)
  float kt[D][kK + 4];      // K^T
  float v[kK][D + 4];       // V
  float p[kQ][kK + 4];      // probabilities (rounded to T)
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) prefill_attn_kernel(
    const T* __restrict__ q, const T* __restrict__ cache, int64_t cbs, int64_t css,
    int64_t cache_batch_offset, const int32_t* __restrict__ pos_start, int seqlen_q,
    int n_heads, int n_heads_kv, int causal, float scale_log2, T* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PSmem<D>& sm = *reinterpret_cast<PSmem<D>*>(smem_raw);
  const int qblk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (n_heads / n_heads_kv);
  const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;  // 16 x 8 thread grid
  const int q0 = qblk * kQ;
  const int p0 = pos_start[b];
  const int nq = min(kQ, seqlen_q - q0);
  // Load Q^T (scaled).
  for (int i = tid; i < kQ * D; i += kThreads) {
    const int r = i / D, d = i % D;
    float x = 0.f;
    if (r < nq) x = DT<T>::to_f(q[(((int64_t)b * seqlen_q + q0 + r) * n_heads + h) * D + d]);
    sm.qt[d][r] = x * scale_log2;
  }
  float o[4][D / 8];
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) o[i][j] = 0.f;
  }
  // Exclusive key bound: with causal masking the last query of the block sees keys
  // <= p0 + q0 + nq - 1; without it every query sees all p0 + seqlen_q keys.
  const int key_end = causal ? p0 + q0 + nq : p0 + seqlen_q;
  const T* kb = cache + (cache_batch_offset + b) * cbs + (int64_t)hk * D;
  const T* vb = kb + (int64_t)n_heads_kv * D;
  for (int k0 = 0; k0 < key_end; k0 += kK) {
    const int nk = min(kK, key_end - k0);
    __syncthreads();
    for (int i = tid; i < kK * D; i += kThreads) {
      const int r = i / D, d = i % D;
      float kx = 0.f, vx = 0.f;
      if (r < nk) {
        const int64_t off = (int64_t)(k0 + r) * css + d;
        kx = DT<T>::to_f(kb[off]);
        vx = DT<T>::to_f(vb[off]);
      }
      sm.kt[d][r] = kx;
      sm.v[r][d] = vx;
    }
    __syncthreads();
    float s[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) s[i][j] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
      const float4 qa = *reinterpret_cast<const float4*>(&sm.qt[d][ty * 4]);
      const float4 ka = *reinterpret_cast<const float4*>(&sm.kt[d][tx * 8]);
      const float4 kc = *reinterpret_cast<const float4*>(&sm.kt[d][tx * 8 + 4]);
      const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
      const float kv[8] = {ka.x, ka.y, ka.z, ka.w, kc.x, kc.y, kc.z, kc.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
    // Causal mask + online softmax; the 8 threads of a row group are consecutive lanes.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      const int qpos = p0 + q0 + r;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int key = k0 + tx * 8 + j;
        if (tx * 8 + j >= nk || (causal && key > qpos) || r >= nq) s[i][j] = -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      const float m_new = fmaxf(m_run[i], mx);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = exp2f(m_run[i] - m_use);
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float pv = exp2f(s[i][j] - m_use);
        psum += pv;
        sm.p[r][tx * 8 + j] = round_to<T>(pv);
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 1);
      psum += __shfl_xor_sync(0xffffffffu, psum, 2);
      psum += __shfl_xor_sync(0xffffffffu, psum, 4);
      l_run[i] = l_run[i] * alpha + psum;
      m_run[i] = m_new;
#pragma unroll
      for (int j = 0; j < D / 8; ++j) o[i][j] *= alpha;
    }
    __syncwarp();
    __syncthreads();
    for (int key = 0; key < nk; ++key) {
      float vv[D / 8];
#pragma unroll
      for (int j = 0; j < D / 8; ++j) vv[j] = sm.v[key][tx + 8 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float pv = sm.p[ty * 4 + i][key];
#pragma unroll
        for (int j = 0; j < D / 8; ++j) o[i][j] = fmaf(pv, vv[j], o[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty * 4 + i;
    if (r >= nq) continue;
    T* orow = out + (((int64_t)b * seqlen_q + q0 + r) * n_heads + h) * D;
    const float inv = l_run[i] > 0.f ? 1.f / l_run[i] : 0.f;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) orow[tx + 8 * j] = DT<T>::from_f(o[i][j] * inv);
  }
}

template <typename T, int D>
int launch_prefill(const void* q, const void* cache, int64_t cbs, int64_t css, int64_t cbo,
                   const int32_t* pos_start, int64_t batch, int64_t seqlen_q, int64_t n_heads,
                   int64_t n_heads_kv, int causal, float scale, void* out, cudaStream_t stream) {
  const size_t smem = sizeof(PSmem<D>);
  auto kern = prefill_attn_kernel<T, D>;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(ceil_div(seqlen_q, kQ), (unsigned)n_heads, (unsigned)batch);
  kern<<<grid, kThreads, smem, stream>>>((const T*)q, (const T*)cache, cbs, css, cbo, pos_start,
                                         (int)seqlen_q, (int)n_heads, (int)n_heads_kv, causal,
                                         scale * 1.4426950408889634f, (T*)out);
  HX_LAUNCH_CHECK("prefill_attn_kernel");
  return HX_OK;
}

}  // namespace

int prefill_attention_tc(const void* q, const void* cache, int64_t cbs, int64_t css, int64_t cbo,
                         const int32_t* pos_start, int64_t B, int64_t S, int64_t hq, int64_t hk,
                         int64_t d, int causal, float scale, void* out, int dtype,
                         cudaStream_t stream);

int prefill_attention_tc_varlen(const void* q, const void* cache, int64_t cbs, int64_t css,
                                int64_t cache_rows, const int32_t* seq_off, const int32_t* slots,
                                const int32_t* pos_start, const int32_t* items,
                                int64_t n_prompts, int64_t n_items, int64_t total_rows,
                                int64_t hq, int64_t hk, int64_t d, int causal, float scale,
                                void* out, int dtype, cudaStream_t stream);

extern "C" int hx_prefill_attention_varlen(
    const void* q, const void* cache, int64_t cache_batch_stride, int64_t cache_seq_stride,
    int64_t cache_rows, const int32_t* seq_offsets, const int32_t* slots,
    const int32_t* pos_start, const int32_t* items, int64_t n_prompts, int64_t n_items,
    int64_t total_rows, int64_t n_heads, int64_t n_heads_kv, int64_t head_dim, int causal,
    float softmax_scale, void* out, int dtype, void* stream) {
  HX_REQUIRE(q && cache && seq_offsets && slots && pos_start && items && out,
             "hx_prefill_attention_varlen: null pointer");
  HX_REQUIRE(n_heads_kv > 0 && n_heads % n_heads_kv == 0, "hx_prefill_attention_varlen: bad heads");
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim && cache_rows > 0 && n_prompts >= 0 &&
                 n_items >= 0 && total_rows >= 0,
             "hx_prefill_attention_varlen: bad sizes");
  if (n_prompts == 0 || n_items == 0 || total_rows == 0) return HX_OK;
  return prefill_attention_tc_varlen(q, cache, cache_batch_stride, cache_seq_stride, cache_rows,
                                     seq_offsets, slots, pos_start, items, n_prompts, n_items,
                                     total_rows, n_heads, n_heads_kv, head_dim, causal,
                                     softmax_scale, out, dtype, (cudaStream_t)stream);
}

extern "C" int hx_prefill_attention(const void* q, const void* cache, int64_t cache_batch_stride,
                                    int64_t cache_seq_stride, int64_t cache_batch_offset,
                                    const int32_t* pos_start, int64_t batch, int64_t seqlen_q,
                                    int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                                    int causal, float softmax_scale, void* out, int dtype,
                                    void* stream) {
  HX_REQUIRE(q && cache && pos_start && out, "hx_prefill_attention: null pointer");
  HX_REQUIRE(n_heads_kv > 0 && n_heads % n_heads_kv == 0, "hx_prefill_attention: bad heads");
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim, "hx_prefill_attention: bad stride");
  if (batch == 0 || seqlen_q == 0) return HX_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // f16/bf16 with head_dim 64/128: tcgen05 kernel; everything else: the CUDA-core kernel.
  const int tc = prefill_attention_tc(q, cache, cache_batch_stride, cache_seq_stride,
                                      cache_batch_offset, pos_start, batch, seqlen_q, n_heads,
                                      n_heads_kv, head_dim, causal, softmax_scale, out, dtype, s);
  if (tc != HX_ERR_UNSUPPORTED) return tc;
#define HX_PREFILL_CASE(DIM)                                                                  \
  case DIM:                                                                                   \
    HX_DISPATCH_DTYPE(dtype, T,                                                               \
                      return launch_prefill<T, DIM>(q, cache, cache_batch_stride,             \
                                                    cache_seq_stride, cache_batch_offset,     \
                                                    pos_start, batch, seqlen_q, n_heads,      \
                                                    n_heads_kv, causal, softmax_scale, out, s)); \
    break;
  switch (head_dim) {
    HX_PREFILL_CASE(32)
    HX_PREFILL_CASE(64)
    HX_PREFILL_CASE(128)
    default:
      hx::set_error("hx_prefill_attention: head_dim %lld unsupported", (long long)head_dim);
      return HX_ERR_UNSUPPORTED;
  }
#undef HX_PREFILL_CASE
  return HX_OK;
}
