// K5: single-query decode attention over the KV cache, split along the key axis.
//
// Semantics: flash_attn_kvpacked_func(q, kv, causal=False) with q_len = 1 as called by the
// native model during decode (hexgen/hexgen_core/modules/mha.py:565-569): for each query head h
// (KV head h / G, G = n_heads / n_heads_kv) out = softmax(q.K^T * scale) V over the live keys.
// Numerics follow FlashAttention-2: f32 scores, f32 online softmax in base 2, probabilities
// rounded to the activation dtype before the P.V product, f32 accumulation, l from the f32
// probabilities, final O / l rounded to the activation dtype.
//
// Layout: cache [B_cap, max_seq, 2, n_heads_kv, D] (the reference's per-layer cache layout),
// rows of one key position are contiguous. One CTA = (split, kv head, sequence); it streams its
// key range through shared memory in 64-key tiles with 16-byte cp.async loads (double
// buffered), serves all G query heads of the KV head from one copy of K/V, and writes an
// unnormalised partial (o, m, l) per query head. A second kernel merges the splits.
// HBM-bound: algorithmic bytes = 2 * n_heads_kv * D * L * sizeof(T) per sequence.
#include <mutex>

#include "common.cuh"

namespace {

constexpr int kThreads = 128;
constexpr int kTile = 64;      // keys per shared-memory tile
constexpr int kMaxGroup = 16;  // max query heads per KV head handled by one CTA

HX_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
HX_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
HX_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Key splits (whole 128-key tiles); shared by the launcher and the workspace query. Splits of
// at most 512 keys keep work items short and balanced across ragged lengths; small batches
// split further (down to single tiles) so that ~4 items per SM exist.
struct SplitPlan {
  int splits, chunk;
};
SplitPlan decode_splits(int64_t batch, int64_t n_heads, int64_t max_len) {
  const int64_t tiles = std::max<int64_t>(1, (max_len + 127) / 128);
  const int64_t units = std::max<int64_t>(1, batch * n_heads);
  int64_t splits = std::max<int64_t>((max_len + 511) / 512, (148 * 4 + units - 1) / units);
  splits = std::min<int64_t>(std::max<int64_t>(splits, 1), tiles);
  const int64_t chunk_tiles = (tiles + splits - 1) / splits;
  splits = (tiles + chunk_tiles - 1) / chunk_tiles;
  return {(int)std::min<int64_t>(splits, 4096), (int)(chunk_tiles * 128)};
}

template <typename T, int D>
struct Smem {
  static constexpr int kPitch = D + 8;  // +16 bytes per row: conflict-free 16B row reads
  T k[2][kTile][kPitch];
  T v[2][kTile][kPitch];
  float q[kMaxGroup][D];
  float s[kMaxGroup][kTile];
  float alpha[kMaxGroup];
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads) decode_split_kernel(
    const T* __restrict__ q, const T* __restrict__ cache, int64_t cbs, int64_t css,
    const int32_t* __restrict__ seqlens, int n_heads, int n_heads_kv, int chunk,
    float scale_log2, T* __restrict__ out, float* __restrict__ ws_o, float* __restrict__ ws_ml,
    int n_splits) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem<T, D>& sm = *reinterpret_cast<Smem<T, D>*>(smem_raw);
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = n_heads / n_heads_kv;
  const int tid = threadIdx.x;
  const int len = seqlens[b];
  const int start = split * chunk;
  const int end = min(start + chunk, len);

  // Per-thread owned outputs: idx = tid + j * kThreads over G * D.
  constexpr int kMaxOwned = kMaxGroup * D / kThreads;
  const int owned = (G * D + kThreads - 1) / kThreads;
  float acc[kMaxOwned];
#pragma unroll
  for (int j = 0; j < kMaxOwned; ++j) acc[j] = 0.f;

  const int64_t row_base = (int64_t)b * n_heads * D;  // q/out row of head 0
  if (start >= end) {
    // Empty split: partials that the merge ignores.
    if (n_splits > 1) {
      for (int i = tid; i < G; i += kThreads) {
        const int64_t slot = ((int64_t)b * n_heads + hk * G + i) * n_splits + split;
        ws_ml[slot * 2] = -INFINITY;
        ws_ml[slot * 2 + 1] = 0.f;
      }
      for (int idx = tid; idx < G * D; idx += kThreads) {
        const int g = idx / D, e = idx % D;
        const int64_t slot = ((int64_t)b * n_heads + hk * G + g) * n_splits + split;
        ws_o[slot * D + e] = 0.f;
      }
    }
    return;
  }

  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D, e = idx % D;
    sm.q[g][e] = DT<T>::to_f(q[row_base + (int64_t)(hk * G + g) * D + e]);
  }
  // Running max (base-2, scaled) and sum per query head: kept by warp (g % 4) lane 0, in smem.
  __shared__ float m_run[kMaxGroup], l_run[kMaxGroup];
  if (tid < kMaxGroup) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
  }

  const T* kbase = cache + (int64_t)b * cbs + (int64_t)hk * D;
  const T* vbase = kbase + (int64_t)n_heads_kv * D;
  constexpr int kVecPerRow = D * sizeof(T) / 16;
  auto load_tile = [&](int buf, int t0) {
    const int n = min(kTile, end - t0);
    for (int i = tid; i < n * kVecPerRow; i += kThreads) {
      const int r = i / kVecPerRow, c = i % kVecPerRow;
      const int64_t goff = (int64_t)(t0 + r) * css + c * (16 / sizeof(T));
      cp_async16(&sm.k[buf][r][c * (16 / sizeof(T))], kbase + goff);
      cp_async16(&sm.v[buf][r][c * (16 / sizeof(T))], vbase + goff);
    }
    cp_async_commit();
  };

  const int n_tiles = (end - start + kTile - 1) / kTile;
  load_tile(0, start);
  for (int t = 0; t < n_tiles; ++t) {
    const int buf = t & 1;
    const int t0 = start + t * kTile;
    const int n = min(kTile, end - t0);
    if (t + 1 < n_tiles) {
      load_tile(buf ^ 1, t0 + kTile);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // Scores: pair p -> (key = p % kTile, g = p / kTile).
    for (int p = tid; p < G * kTile; p += kThreads) {
      const int key = p % kTile, g = p / kTile;
      float sc = -INFINITY;
      if (key < n) {
        float dot = 0.f;
        const T* kr = sm.k[buf][key];
#pragma unroll
        for (int c = 0; c < D; c += 16 / sizeof(T)) {
          uint4 raw = *reinterpret_cast<const uint4*>(kr + c);
          const T* kv = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int j = 0; j < (int)(16 / sizeof(T)); ++j) dot += sm.q[g][c + j] * DT<T>::to_f(kv[j]);
        }
        sc = dot * scale_log2;
      }
      sm.s[g][key] = sc;
    }
    __syncthreads();
    // Online softmax, one warp per query head (warps loop over heads).
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += kThreads / 32) {
      const float s0 = sm.s[g][lane], s1 = sm.s[g][lane + 32];
      const float tmax = warp_max(fmaxf(s0, s1));
      const float m_old = m_run[g];
      const float m_new = fmaxf(m_old, tmax);
      const float p0 = exp2f(s0 - m_new), p1 = exp2f(s1 - m_new);
      const float psum = warp_sum(p0 + p1);
      const float alpha = exp2f(m_old - m_new);
      sm.s[g][lane] = round_to<T>(p0);
      sm.s[g][lane + 32] = round_to<T>(p1);
      __syncwarp();
      if (lane == 0) {
        m_run[g] = m_new;
        l_run[g] = l_run[g] * alpha + psum;
        sm.alpha[g] = alpha;
      }
    }
    __syncthreads();
    // P.V accumulation.
#pragma unroll
    for (int j = 0; j < kMaxOwned; ++j) {
      if (j < owned) {
        const int idx = tid + j * kThreads;
        if (idx < G * D) {
          const int g = idx / D, e = idx % D;
          float a = acc[j] * sm.alpha[g];
          for (int key = 0; key < n; ++key) a += sm.s[g][key] * DT<T>::to_f(sm.v[buf][key][e]);
          acc[j] = a;
        }
      }
    }
    __syncthreads();
  }

  if (n_splits == 1) {
#pragma unroll
    for (int j = 0; j < kMaxOwned; ++j) {
      const int idx = tid + j * kThreads;
      if (j < owned && idx < G * D) {
        const int g = idx / D, e = idx % D;
        const float l = l_run[g];
        out[row_base + (int64_t)(hk * G + g) * D + e] = DT<T>::from_f(l > 0.f ? acc[j] / l : 0.f);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < kMaxOwned; ++j) {
      const int idx = tid + j * kThreads;
      if (j < owned && idx < G * D) {
        const int g = idx / D, e = idx % D;
        const int64_t slot = ((int64_t)b * n_heads + hk * G + g) * n_splits + split;
        ws_o[slot * D + e] = acc[j];
      }
    }
    for (int g = tid; g < G; g += kThreads) {
      const int64_t slot = ((int64_t)b * n_heads + hk * G + g) * n_splits + split;
      ws_ml[slot * 2] = m_run[g];
      ws_ml[slot * 2 + 1] = l_run[g];
    }
  }
}

// ------------------------------------------------------------------------------------------
// Register-resident kernel for G = n_heads / n_heads_kv <= 2 (MHA, light GQA), 16-bit dtypes.
// Four lanes share one key row (lane s of the group reads 16-byte chunks s, s+4, ... so each
// load instruction covers whole sectors), eight key groups per warp, two keys per group in
// flight; every warp keeps its own online-softmax state for its keys (no __syncthreads in the
// key loop) and the 32 partial states of a CTA are merged at the end.
// ------------------------------------------------------------------------------------------
constexpr int kLPK = 4;                      // lanes per key row
constexpr int kGroups = 32 / kLPK;           // key groups per warp

// kUnroll keys per key group are in flight per iteration (2 for MHA, 1 when G = 2 keeps the
// second query's state in registers).
template <typename T, int D, int G, int kUnroll = (G == 1 ? 2 : 1)>
__global__ void __launch_bounds__(kThreads) decode_warp_kernel(
    const T* __restrict__ q, const T* __restrict__ cache, int64_t cbs, int64_t css,
    const int32_t* __restrict__ seqlens, int n_heads, int n_heads_kv, int chunk,
    float scale_log2, T* __restrict__ out, float* __restrict__ ws_o, float* __restrict__ ws_ml,
    int n_splits) {
  constexpr int VPL = D / (8 * kLPK);  // 16-byte vectors per lane per row
  constexpr int EPL = VPL * 8;          // elements per lane
  constexpr int kWarpKeys = kGroups * kUnroll;  // keys per warp per iteration
  __shared__ float sm_m[kThreads / 32][G], sm_l[kThreads / 32][G];
  __shared__ float sm_acc[kThreads / 32][G][D];
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kg = lane >> 2, sl = lane & 3;
  const int len = seqlens[b];
  const int start = split * chunk;
  const int end = min(start + chunk, len);
  if (start >= end) {
    if (n_splits > 1) {
      for (int idx = tid; idx < G * D; idx += kThreads) {
        const int g = idx / D, e = idx % D;
        const int64_t slot = ((int64_t)b * n_heads + hk * G + g) * n_splits + split;
        ws_o[slot * D + e] = 0.f;
        if (e == 0) {
          ws_ml[slot * 2] = -INFINITY;
          ws_ml[slot * 2 + 1] = 0.f;
        }
      }
    }
    return;
  }
  // Query slice of this lane (pre-scaled into the base-2 softmax domain).
  float qv[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const T* qr = q + ((int64_t)b * n_heads + hk * G + g) * D;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qr + (j * kLPK + sl) * 8);
      const T* qe = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int t = 0; t < 8; ++t) qv[g][j * 8 + t] = DT<T>::to_f(qe[t]) * scale_log2;
    }
  }
  float m[G], l[G], acc[G][EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) acc[g][i] = 0.f;
  }
  const T* kbase = cache + (int64_t)b * cbs + (int64_t)hk * D;
  const T* vbase = kbase + (int64_t)n_heads_kv * D;
  for (int base = start + warp * kWarpKeys; base < end; base += (kThreads / 32) * kWarpKeys) {
    uint4 kr[kUnroll][VPL], vr[kUnroll][VPL];
    bool valid[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int key = base + u * kGroups + kg;
      valid[u] = key < end;
      const int64_t off = (int64_t)key * css;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        if (valid[u]) {
          kr[u][j] = __ldg(reinterpret_cast<const uint4*>(kbase + off + (j * kLPK + sl) * 8));
          vr[u][j] = __ldg(reinterpret_cast<const uint4*>(vbase + off + (j * kLPK + sl) * 8));
        } else {
          kr[u][j] = make_uint4(0, 0, 0, 0);
          vr[u][j] = make_uint4(0, 0, 0, 0);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float s[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
          const T* ke = reinterpret_cast<const T*>(&kr[u][j]);
#pragma unroll
          for (int t = 0; t < 8; ++t) dot = fmaf(qv[g][j * 8 + t], DT<T>::to_f(ke[t]), dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        s[u] = valid[u] ? dot : -INFINITY;
      }
      float mb = m[g];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) mb = fmaxf(mb, s[u]);
      const float m_use = mb == -INFINITY ? 0.f : mb;
      const float alpha = exp2f(m[g] - m_use);
      float p[kUnroll], psum = 0.f;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        p[u] = exp2f(s[u] - m_use);
        psum += p[u];
        p[u] = round_to<T>(p[u]);
      }
      l[g] = l[g] * alpha + psum;
      m[g] = mb;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          float a = acc[g][j * 8 + t] * alpha;
#pragma unroll
          for (int u = 0; u < kUnroll; ++u)
            a = fmaf(p[u], DT<T>::to_f(reinterpret_cast<const T*>(&vr[u][j])[t]), a);
          acc[g][j * 8 + t] = a;
        }
      }
    }
  }
  // Merge the 8 key groups of the warp (lanes with equal slice index).
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float M = m[g];
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 4));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 8));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 16));
    const float sc = (m[g] == -INFINITY) ? 0.f : exp2f(m[g] - M);
    float L = l[g] * sc;
    L += __shfl_xor_sync(0xffffffffu, L, 4);
    L += __shfl_xor_sync(0xffffffffu, L, 8);
    L += __shfl_xor_sync(0xffffffffu, L, 16);
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      float a = acc[g][i] * sc;
      a += __shfl_xor_sync(0xffffffffu, a, 4);
      a += __shfl_xor_sync(0xffffffffu, a, 8);
      a += __shfl_xor_sync(0xffffffffu, a, 16);
      acc[g][i] = a;
    }
    if (kg == 0) {
#pragma unroll
      for (int j = 0; j < VPL; ++j)
#pragma unroll
        for (int t = 0; t < 8; ++t) sm_acc[warp][g][(j * kLPK + sl) * 8 + t] = acc[g][j * 8 + t];
      if (sl == 0) {
        sm_m[warp][g] = M;
        sm_l[warp][g] = L;
      }
    }
  }
  __syncthreads();
  // Merge the 4 warps and write the output (one split) or the split partial.
  for (int idx = tid; idx < G * D; idx += kThreads) {
    const int g = idx / D, e = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) M = fmaxf(M, sm_m[w][g]);
    float L = 0.f, A = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      const float mw = sm_m[w][g];
      if (mw == -INFINITY) continue;
      const float sc = exp2f(mw - M);
      L += sm_l[w][g] * sc;
      A += sm_acc[w][g][e] * sc;
    }
    if (n_splits == 1) {
      out[((int64_t)b * n_heads + hk * G + g) * D + e] = DT<T>::from_f(L > 0.f ? A / L : 0.f);
    } else {
      const int64_t slot = ((int64_t)b * n_heads + hk * G + g) * n_splits + split;
      ws_o[slot * D + e] = A;
      if (e == 0) {
        ws_ml[slot * 2] = M;
        ws_ml[slot * 2 + 1] = L;
      }
    }
  }
}

// Merge split partials: one CTA per (sequence, query head), one thread per output element.
template <typename T, int D>
__global__ void decode_merge_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_ml,
                                    int n_splits, T* __restrict__ out) {
  const int64_t bh = blockIdx.x;
  const float* ml = ws_ml + bh * n_splits * 2;
  float m = -INFINITY;
  for (int s = 0; s < n_splits; ++s) m = fmaxf(m, ml[2 * s]);
  float l = 0.f, o = 0.f;
  for (int e = threadIdx.x; e < D; e += blockDim.x) {
    l = 0.f;
    o = 0.f;
    for (int s = 0; s < n_splits; ++s) {
      const float ms = ml[2 * s];
      if (ms == -INFINITY) continue;
      const float w = exp2f(ms - m);
      l += ml[2 * s + 1] * w;
      o += ws_o[(bh * n_splits + s) * D + e] * w;
    }
    out[bh * D + e] = DT<T>::from_f(l > 0.f ? o / l : 0.f);
  }
}

}  // namespace

int decode_attention_tma(const void* q, const void* cache, int64_t cbs, int64_t css,
                         const int32_t* seqlens, int64_t batch, int64_t n_heads,
                         int64_t n_heads_kv, int64_t head_dim, float scale, void* out, void* ws,
                         size_t ws_bytes, int dtype, cudaStream_t stream);
size_t decode_tma_workspace(int64_t batch, int64_t n_heads, int64_t head_dim);

namespace {

template <typename T, int D>
int launch_decode(const void* q, const void* cache, int64_t cbs, int64_t css,
                  const int32_t* seqlens, int64_t batch, int64_t n_heads, int64_t n_heads_kv,
                  int64_t max_len, float scale, void* out, void* ws, size_t ws_bytes,
                  cudaStream_t stream) {
  {
    // Main path (f16/bf16, head_dim 64/128, <= 2 query heads per KV head): balanced TMA kernel.
    const int dt = sizeof(T) == 4 ? HX_F32 : (std::is_same<T, __half>::value ? HX_F16 : HX_BF16);
    const int s = decode_attention_tma(q, cache, cbs, css, seqlens, batch, n_heads, n_heads_kv, D,
                                       scale, out, ws, ws_bytes, dt, stream);
    if (s != HX_ERR_UNSUPPORTED) return s;
  }
  const SplitPlan sp = decode_splits(batch, n_heads, max_len);
  const int splits = sp.splits, chunk = sp.chunk;
  float* ws_o = nullptr;
  float* ws_ml = nullptr;
  if (splits > 1) {
    const size_t need = (size_t)batch * n_heads * splits * (D + 2) * sizeof(float);
    HX_REQUIRE(ws && ws_bytes >= need, "hx_decode_attention: workspace too small (%zu < %zu)",
               ws_bytes, need);
    ws_o = (float*)ws;
    ws_ml = ws_o + (size_t)batch * n_heads * splits * D;
  }
  dim3 grid(splits, (unsigned)n_heads_kv, (unsigned)batch);
  const float scale_log2 = scale * 1.4426950408889634f;
  const int64_t group = n_heads / n_heads_kv;
  bool done = false;
  if constexpr (sizeof(T) == 2 && D >= 64) {
    if (group <= 2) {
      auto wk = group == 1 ? decode_warp_kernel<T, D, 1> : decode_warp_kernel<T, D, 2>;
      wk<<<grid, kThreads, 0, stream>>>((const T*)q, (const T*)cache, cbs, css, seqlens,
                                        (int)n_heads, (int)n_heads_kv, chunk, scale_log2,
                                        (T*)out, ws_o, ws_ml, splits);
      HX_LAUNCH_CHECK("decode_warp_kernel");
      done = true;
    }
  }
  if (!done) {
  const size_t smem = sizeof(Smem<T, D>);
  auto kern = decode_split_kernel<T, D>;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, kThreads, smem, stream>>>((const T*)q, (const T*)cache, cbs, css, seqlens,
                                         (int)n_heads, (int)n_heads_kv, chunk, scale_log2,
                                         (T*)out, ws_o, ws_ml, splits);
  HX_LAUNCH_CHECK("decode_split_kernel");
  }
  if (splits > 1) {
    decode_merge_kernel<T, D><<<(unsigned)(batch * n_heads), D, 0, stream>>>(ws_o, ws_ml, splits,
                                                                            (T*)out);
    HX_LAUNCH_CHECK("decode_merge_kernel");
  }
  return HX_OK;
}

}  // namespace

extern "C" {

size_t hx_decode_attention_workspace(int64_t batch, int64_t n_heads, int64_t head_dim,
                                     int64_t max_seqlen_k) {
  // The larger of the two paths' needs: the balanced TMA kernel (f16/bf16, head_dim 64/128) and
  // the fixed-split kernels (other shapes and dtypes).
  if (batch <= 0 || n_heads <= 0 || head_dim <= 0 || max_seqlen_k <= 0) return 0;
  const int splits = decode_splits(batch, n_heads, max_seqlen_k).splits;
  const size_t split_need =
      splits <= 1 ? 0 : (size_t)batch * n_heads * splits * (head_dim + 2) * sizeof(float);
  const size_t tma_need =
      (head_dim == 64 || head_dim == 128) ? decode_tma_workspace(batch, n_heads, head_dim) : 0;
  return std::max(split_need, tma_need);
}

int hx_decode_attention(const void* q, const void* cache, int64_t cache_batch_stride,
                        int64_t cache_seq_stride, const int32_t* seqlens_k, int64_t batch,
                        int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                        int64_t max_seqlen_k, float softmax_scale, void* out, void* workspace,
                        size_t workspace_bytes, int dtype, void* stream) {
  HX_REQUIRE(q && cache && seqlens_k && out, "hx_decode_attention: null pointer");
  HX_REQUIRE(n_heads_kv > 0 && n_heads % n_heads_kv == 0 && n_heads / n_heads_kv <= kMaxGroup,
             "hx_decode_attention: unsupported head grouping %lld/%lld", (long long)n_heads,
             (long long)n_heads_kv);
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim, "hx_decode_attention: bad stride");
  if (batch == 0 || max_seqlen_k == 0) return HX_OK;
  const int esz = dtype == HX_F32 ? 4 : 2;
  HX_REQUIRE(((uintptr_t)cache % 16 == 0) && (cache_seq_stride * esz) % 16 == 0 &&
                 (cache_batch_stride * esz) % 16 == 0,
             "hx_decode_attention: cache must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
#define HX_DECODE_CASE(DIM)                                                                   \
  case DIM:                                                                                   \
    HX_DISPATCH_DTYPE(dtype, T,                                                               \
                      return launch_decode<T, DIM>(q, cache, cache_batch_stride,              \
                                                   cache_seq_stride, seqlens_k, batch,        \
                                                   n_heads, n_heads_kv, max_seqlen_k,         \
                                                   softmax_scale, out, workspace,             \
                                                   workspace_bytes, s));                      \
    break;
  switch (head_dim) {
    HX_DECODE_CASE(32)
    HX_DECODE_CASE(64)
    HX_DECODE_CASE(128)
    default:
      hx::set_error("hx_decode_attention: head_dim %lld unsupported", (long long)head_dim);
      return HX_ERR_UNSUPPORTED;
  }
#undef HX_DECODE_CASE
  return HX_OK;
}

// ------------------------------------------------------------------------------------------
// No-allocation variant: the split partials live in a file-scope device array.
// ------------------------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_decode_noalloc_scratch[HX_DECODE_NOALLOC_SCRATCH_BYTES];

int hx_decode_attention_noalloc(const void* q, const void* cache, int64_t cache_batch_stride,
                                int64_t cache_seq_stride, const int32_t* seqlens_k,
                                int64_t batch, int64_t n_heads, int64_t n_heads_kv,
                                int64_t head_dim, int64_t max_seqlen_k, float softmax_scale,
                                void* out, int dtype, void* stream) {
  // In host code g_decode_noalloc_scratch names a host-side stand-in, not device memory: the
  // device address is looked up once per device, with that device current.
  static std::mutex mu;
  static void* scratch_ptr[64] = {nullptr};
  int dev = 0;
  int s = hx::cuda_status(cudaGetDevice(&dev), "cudaGetDevice");
  if (s) return s;
  HX_REQUIRE(dev >= 0 && dev < 64, "hx_decode_attention_noalloc: device %d out of range", dev);
  const size_t need = hx_decode_attention_workspace(batch, n_heads, head_dim, max_seqlen_k);
  HX_REQUIRE(need <= HX_DECODE_NOALLOC_SCRATCH_BYTES,
             "hx_decode_attention_noalloc: this shape needs %zu bytes of split scratch, more than "
             "the %u-byte static array (batch %lld, heads %lld, head_dim %lld, max_seqlen_k %lld)",
             need, HX_DECODE_NOALLOC_SCRATCH_BYTES, (long long)batch, (long long)n_heads,
             (long long)head_dim, (long long)max_seqlen_k);
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> g(mu);
    if (!scratch_ptr[dev]) {
      s = hx::cuda_status(cudaGetSymbolAddress(&scratch_ptr[dev], g_decode_noalloc_scratch),
                          "cudaGetSymbolAddress(decode scratch)");
      if (s) {
        scratch_ptr[dev] = nullptr;
        return s;
      }
    }
    ptr = scratch_ptr[dev];
  }
  return hx_decode_attention(q, cache, cache_batch_stride, cache_seq_stride, seqlens_k, batch,
                             n_heads, n_heads_kv, head_dim, max_seqlen_k, softmax_scale, out, ptr,
                             HX_DECODE_NOALLOC_SCRATCH_BYTES, dtype, stream);
}

}  // extern "C"
