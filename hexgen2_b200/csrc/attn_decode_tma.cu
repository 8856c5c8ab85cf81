// K5 (main path): persistent TMA-fed decode attention for f16/bf16, head_dim 64/128, up to 2
// query heads per KV head (MHA and light GQA). Semantics and numerics are those of
// attn_decode.cu (flash_attn_kvpacked_func with q_len 1, FlashAttention-2 rounding points).
//
// Balanced partition. The live keys of every (sequence, kv head) pair form a run of 128-key
// tiles; the runs of all pairs, sequence-major, make one list of T tiles (T is computed on the
// device from seqlens, so ragged batches inside a CUDA graph need no host work). CTA c of G
// (one per SM) takes tiles [c*T/G, (c+1)*T/G): every CTA streams the same number of KV bytes
// whatever the length mix. A run that lies wholly inside one CTA's range is finished by that CTA
// (output written directly). A run cut by a range boundary leaves one partial (o, m, l) per
// contributing CTA: the CTA where the run ends in the middle of writes slot 2c + 1, the CTAs
// where it continues write slot 2c, and decode_tma_merge_kernel combines them in CTA order.
//   warp 0      TMA producer: K and V boxes [128 keys x 64 elements] (SWIZZLE_128B) straight
//               out of the cache ([B, max_seq, 2*hkv, d] as a 4D tensor map) into a ring of
//               64 KB (d=128) stages; ~192 KB stay in flight per SM, which is what keeps HBM busy.
//   warps 1-4   consumers: warp w owns keys [32w, 32w+32) of each tile, one key per lane.
//               QK: the lane reads its key's row (the swizzle makes 8 consecutive rows hit 8
//               different 16-byte slots, so no bank conflicts) against q held in shared memory;
//               online softmax across the warp with shuffles; PV: for each valid key, the warp
//               reads that V row (lane = 4 (or 2) output dims) and accumulates.
//               Each warp keeps its own (m, l, o); the four are merged at the run's end.
// Cache rows past a sequence's length are never used: their scores are masked and P.V stops
// at the last valid key, so stale cache bits cannot leak in.
#include "common.cuh"

namespace {

constexpr int kTileKeys = 128;
constexpr int kBoxBytes = kTileKeys * 128;  // [128 keys x 64 elements] swizzled box
constexpr int kConsumers = 4;
constexpr int kThreadsTma = 32 * (1 + kConsumers);
constexpr int kMaxSeqs = 2048;              // sequences per call (tile prefix kept in smem)

template <int D>
struct DLay {
  static constexpr int kChunks = D / 64;
  static constexpr int kStageBytes = 2 * kChunks * kBoxBytes;  // K + V
  static constexpr int kStages = D == 128 ? 3 : 6;
  static constexpr int kRing = kStages * kStageBytes;
};

struct DecArgs {
  const void* q;
  void* out;
  float* ws_o;   // [2 * grid][G][D] partial outputs
  float* ws_ml;  // [2 * grid][G][2] partial (m, l)
  int* ws_pre;   // [batch + 1] tile prefix (written by CTA 0 for the merge kernel)
  const int32_t* seqlens;
  int n_heads, n_heads_kv, batch, max_seq;
  float scale_log2;
};

HX_DEVICE void named_barrier_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumers) : "memory");
}

HX_DEVICE int live_len(const DecArgs& a, int b) {
  return min(max(a.seqlens[b], 0), a.max_seq);
}

// First CTA (of `grid`) whose tile range [c*T/grid, (c+1)*T/grid) contains tile u.
HX_DEVICE int cta_of(int64_t u, int64_t T, int grid) {
  return (int)(((u + 1) * grid - 1) / T);
}

// One run piece of this CTA's range: sequence b, kv head hk, tiles [t_lo, t_hi) of the run,
// run bounds [seg0, seg1) in the global tile list.
struct Piece {
  int b, hk, t_lo, t_hi;
  int64_t seg0, seg1;
};

// Walks the pieces of [u0, u1) in order; `pre` is the per-sequence prefix of tiles x hkv.
struct PieceWalker {
  const int* pre;
  int hkv, b;
  int64_t u, u1;
  HX_DEVICE PieceWalker(const int* pre_, int hkv_, int batch, int64_t u0, int64_t u1_)
      : pre(pre_), hkv(hkv_), b(0), u(u0), u1(u1_) {
    // Largest b with pre[b] <= u0 (binary search over the monotone prefix).
    int lo = 0, hi = batch;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pre[mid] <= u0) lo = mid; else hi = mid - 1;
    }
    b = lo;
  }
  HX_DEVICE bool next(Piece& p) {
    if (u >= u1) return false;
    while (pre[b + 1] <= u) ++b;
    const int tiles = (pre[b + 1] - pre[b]) / hkv;
    const int64_t rel = u - pre[b];
    const int hk = (int)(rel / tiles);
    p.b = b;
    p.hk = hk;
    p.seg0 = pre[b] + (int64_t)hk * tiles;
    p.seg1 = p.seg0 + tiles;
    const int64_t e = p.seg1 < u1 ? p.seg1 : u1;
    p.t_lo = (int)(u - p.seg0);
    p.t_hi = (int)(e - p.seg0);
    u = e;
    return true;
  }
};

template <typename T, int D, int G>
__global__ void __launch_bounds__(kThreadsTma, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tmKV, const DecArgs a) {
  using L = DLay<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* q_s = reinterpret_cast<float*>(ring + L::kRing);                 // [G][D]
  float* mo = q_s + G * D;                                               // [4][G][D]
  float* ml = mo + kConsumers * G * D;                                    // [4][G][2]
  uint64_t* full = reinterpret_cast<uint64_t*>(ml + kConsumers * G * 2 + 2);
  uint64_t* empty = full + L::kStages;
  int* pre = reinterpret_cast<int*>(empty + L::kStages);                  // [batch + 1]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hkv = a.n_heads_kv;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmKV);
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    fence_mbar_init();
  }
  pdl_wait();  // q, the cache rows and seqlens come from earlier kernels
  pdl_trigger();
  if (warp == 1) {
    // Tile prefix over sequences: pre[b] = hkv * sum_{b' < b} ceil(len_b' / 128).
    int carry = 0;
    if (lane == 0) pre[0] = 0;
    for (int base = 0; base < a.batch; base += 32) {
      const int b = base + lane;
      int v = b < a.batch ? hkv * ((live_len(a, b) + kTileKeys - 1) / kTileKeys) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      if (b < a.batch) pre[b + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const int64_t total = pre[a.batch];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= a.batch; i += blockDim.x) a.ws_pre[i] = pre[i];
  if (total == 0) return;
  const int64_t u0 = (int64_t)blockIdx.x * total / gridDim.x;
  const int64_t u1 = (int64_t)(blockIdx.x + 1) * total / gridDim.x;
  if (u0 >= u1) return;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      PieceWalker w(pre, hkv, a.batch, u0, u1);
      Piece p;
      while (w.next(p)) {
        for (int t = p.t_lo; t < p.t_hi; ++t) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) goto producer_done;
          ++issued;
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          uint8_t* kb = ring + stage * L::kStageBytes;
          uint8_t* vb = kb + L::kChunks * kBoxBytes;
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c) {
            tma_load_4d(kb + c * kBoxBytes, &tmKV, &full[stage], c * 64, p.hk, t * kTileKeys, p.b);
            tma_load_4d(vb + c * kBoxBytes, &tmKV, &full[stage], c * 64, hkv + p.hk, t * kTileKeys, p.b);
          }
          if (++stage == L::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      // Loads older than the last kStages were released by the consumers before their stage
      // was reused; let the newest ones land (bounded) before this warp leaves.
      for (uint32_t i = issued > (uint32_t)L::kStages ? issued - L::kStages : 0; i < issued; ++i)
        mbar_wait(&full[i % L::kStages], (i / L::kStages) & 1);
    }
    return;  // the producer warp takes no part in the consumer barriers below
  }

  // ------------------------------------------------------------------ consumers
  const int cw = warp - 1;                 // consumer warp 0..3
  const int ct = threadIdx.x - 32;         // consumer thread 0..127
  constexpr int kDims = D / 32;            // output dims per lane (4 or 2)
  const int e0 = lane * kDims;
  const int e_chunk = e0 / 64, e_unit = (e0 % 64) / 8, e_within = e0 % 8;
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  // Every consumer warp walks the same piece / tile / barrier sequence even after a failed
  // (timed-out) wait, only skipping the work, so no warp is left waiting at a named barrier.
  PieceWalker walker(pre, hkv, a.batch, u0, u1);
  Piece pc;
  while (walker.next(pc)) {
    const int b = pc.b, hk = pc.hk;
    const int len = live_len(a, b);
    const int start = pc.t_lo * kTileKeys;
    const int end = min(pc.t_hi * kTileKeys, len);
    for (int idx = ct; idx < G * D; idx += 32 * kConsumers) {
      const int g = idx / D, e = idx % D;
      q_s[g * D + e] = DT<T>::to_f(reinterpret_cast<const T*>(a.q)[((int64_t)b * a.n_heads + hk * G + g) * D + e]) * a.scale_log2;
    }
    named_barrier_consumers();
    float m[G], l[G], o[G][kDims];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m[g] = -INFINITY;
      l[g] = 0.f;
#pragma unroll
      for (int i = 0; i < kDims; ++i) o[g][i] = 0.f;
    }
    for (int key0 = start; key0 < end; key0 += kTileKeys) {
      if (ok && !mbar_wait_warp(&full[stage], phase)) ok = false;
      if (!ok) {
        if (++stage == L::kStages) {
          stage = 0;
          phase ^= 1;
        }
        continue;
      }
      const uint8_t* kb = ring + stage * L::kStageBytes;
      const uint8_t* vb = kb + L::kChunks * kBoxBytes;
      const int r = cw * 32 + lane;  // this lane's key row in the tile
      const int kw0 = key0 + cw * 32;
      const bool valid = kw0 + lane < end;
      const int n_valid = max(0, min(32, end - kw0));
      // QK with eight independent partial sums per head (one per element of a 16-byte chunk)
      // so the FMA latency chain is 16 deep instead of D deep.
      float part[G][8];
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < 8; ++j) part[g][j] = 0.f;
#pragma unroll
      for (int u = 0; u < D / 8; ++u) {
        const int c = u >> 3, uu = u & 7;
        const uint4 raw = *reinterpret_cast<const uint4*>(kb + c * kBoxBytes + r * 128 + ((uu ^ (r & 7)) << 4));
        const T* ke = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(q_s + g * D + u * 8);
          const float4 qb = *reinterpret_cast<const float4*>(q_s + g * D + u * 8 + 4);
          part[g][0] = fmaf(qa.x, DT<T>::to_f(ke[0]), part[g][0]);
          part[g][1] = fmaf(qa.y, DT<T>::to_f(ke[1]), part[g][1]);
          part[g][2] = fmaf(qa.z, DT<T>::to_f(ke[2]), part[g][2]);
          part[g][3] = fmaf(qa.w, DT<T>::to_f(ke[3]), part[g][3]);
          part[g][4] = fmaf(qb.x, DT<T>::to_f(ke[4]), part[g][4]);
          part[g][5] = fmaf(qb.y, DT<T>::to_f(ke[5]), part[g][5]);
          part[g][6] = fmaf(qb.z, DT<T>::to_f(ke[6]), part[g][6]);
          part[g][7] = fmaf(qb.w, DT<T>::to_f(ke[7]), part[g][7]);
        }
      }
      float dot[G];
#pragma unroll
      for (int g = 0; g < G; ++g)
        dot[g] = ((part[g][0] + part[g][1]) + (part[g][2] + part[g][3])) +
                 ((part[g][4] + part[g][5]) + (part[g][6] + part[g][7]));
      float pr[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float s = valid ? dot[g] : -INFINITY;
        const float m_new = fmaxf(m[g], warp_max(s));
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = exp2f(m[g] - m_use);
        const float p = valid ? exp2f(s - m_use) : 0.f;
        l[g] = l[g] * alpha + warp_sum(p);
        m[g] = m_new;
        pr[g] = round_to<T>(p);
#pragma unroll
        for (int i = 0; i < kDims; ++i) o[g][i] *= alpha;
      }
      auto load_v = [&](int k, float (&vf)[kDims]) {
        const int row = cw * 32 + k;
        const uint8_t* vrow = vb + e_chunk * kBoxBytes + row * 128 + ((e_unit ^ (row & 7)) << 4) + e_within * 2;
        if constexpr (kDims == 4) {
          const uint2 raw = *reinterpret_cast<const uint2*>(vrow);
          const T* ve = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) vf[i] = DT<T>::to_f(ve[i]);
        } else {
          const uint32_t raw = *reinterpret_cast<const uint32_t*>(vrow);
          const T* ve = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int i = 0; i < 2; ++i) vf[i] = DT<T>::to_f(ve[i]);
        }
      };
      if (n_valid == 32) {
        // Full 32-key slice: unrolled, two accumulator sets to halve the FMA chain.
        float o2[G][kDims];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < kDims; ++i) o2[g][i] = 0.f;
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float v0[kDims], v1[kDims];
          load_v(k, v0);
          load_v(k + 1, v1);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float p0 = __shfl_sync(0xffffffffu, pr[g], k);
            const float p1 = __shfl_sync(0xffffffffu, pr[g], k + 1);
#pragma unroll
            for (int i = 0; i < kDims; ++i) {
              o[g][i] = fmaf(p0, v0[i], o[g][i]);
              o2[g][i] = fmaf(p1, v1[i], o2[g][i]);
            }
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < kDims; ++i) o[g][i] += o2[g][i];
      } else {
        for (int k = 0; k < n_valid; ++k) {
          float vf[kDims];
          load_v(k, vf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pk = __shfl_sync(0xffffffffu, pr[g], k);
#pragma unroll
            for (int i = 0; i < kDims; ++i) o[g][i] = fmaf(pk, vf[i], o[g][i]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == L::kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    // Merge the four consumer warps' states.
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int i = 0; i < kDims; ++i) mo[(cw * G + g) * D + e0 + i] = o[g][i];
      if (lane == 0) {
        ml[(cw * G + g) * 2] = m[g];
        ml[(cw * G + g) * 2 + 1] = l[g];
      }
    }
    named_barrier_consumers();
    const bool whole = pc.seg0 >= u0 && pc.seg1 <= u1;
    const int64_t slot = 2 * (int64_t)blockIdx.x + (pc.seg0 < u0 ? 0 : 1);
    for (int idx = ct; ok && idx < G * D; idx += 32 * kConsumers) {
      const int g = idx / D, e = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, ml[(w * G + g) * 2]);
      float Ls = 0.f, A = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        const float mw = ml[(w * G + g) * 2];
        if (mw == -INFINITY) continue;
        const float sc = exp2f(mw - M);
        Ls += ml[(w * G + g) * 2 + 1] * sc;
        A += mo[(w * G + g) * D + e] * sc;
      }
      if (whole) {
        const int64_t h = (int64_t)b * a.n_heads + hk * G + g;
        reinterpret_cast<T*>(a.out)[h * D + e] = DT<T>::from_f(Ls > 0.f ? A / Ls : 0.f);
      } else {
        a.ws_o[(slot * G + g) * D + e] = A;
        if (e == 0) {
          a.ws_ml[(slot * G + g) * 2] = M;
          a.ws_ml[(slot * G + g) * 2 + 1] = Ls;
        }
      }
    }
    named_barrier_consumers();
  }
}

// Combines the partials of runs that were cut by a CTA range boundary; one CTA per
// (sequence, kv head), one thread per (query head of the group, output element). Runs of an
// empty sequence get a zero output; runs finished by one CTA are left as written.
template <typename T, int D, int G>
__global__ void decode_tma_merge_kernel(const DecArgs a, int grid) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x / a.n_heads_kv, hk = blockIdx.x % a.n_heads_kv;
  const int g = threadIdx.x / D, e = threadIdx.x % D;
  const int64_t total = a.ws_pre[a.batch];
  const int tiles = (a.ws_pre[b + 1] - a.ws_pre[b]) / a.n_heads_kv;
  const int64_t h = (int64_t)b * a.n_heads + hk * G + g;
  if (tiles == 0) {
    reinterpret_cast<T*>(a.out)[h * D + e] = DT<T>::from_f(0.f);
    return;
  }
  const int64_t seg0 = a.ws_pre[b] + (int64_t)hk * tiles, seg1 = seg0 + tiles;
  const int c0 = cta_of(seg0, total, grid), c1 = cta_of(seg1 - 1, total, grid);
  if (c0 == c1) return;
  float M = -INFINITY;
  for (int c = c0; c <= c1; ++c) {
    const int64_t slot = c == c0 ? 2 * (int64_t)c + 1 : 2 * (int64_t)c;
    M = fmaxf(M, a.ws_ml[(slot * G + g) * 2]);
  }
  float Ls = 0.f, A = 0.f;
  for (int c = c0; c <= c1; ++c) {
    const int64_t slot = c == c0 ? 2 * (int64_t)c + 1 : 2 * (int64_t)c;
    const float mc = a.ws_ml[(slot * G + g) * 2];
    if (mc == -INFINITY) continue;
    const float sc = exp2f(mc - M);
    Ls += a.ws_ml[(slot * G + g) * 2 + 1] * sc;
    A += a.ws_o[(slot * G + g) * D + e] * sc;
  }
  reinterpret_cast<T*>(a.out)[h * D + e] = DT<T>::from_f(Ls > 0.f ? A / Ls : 0.f);
}

template <typename T, int D, int G>
int launch(const CUtensorMap& map, const DecArgs& args, int grid, cudaStream_t stream) {
  using L = DLay<D>;
  const size_t smem = (size_t)L::kRing + 1024 +
                      sizeof(float) * (G * D + kConsumers * G * D + kConsumers * G * 2 + 2) +
                      2 * L::kStages * sizeof(uint64_t) + sizeof(int) * (kMaxSeqs + 1) + 64;
  auto kern = decode_tma_kernel<T, D, G>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem),
                            "cudaFuncSetAttribute(decode_tma)");
    if (s) return s;
    attr[dev & 63] = true;
  }
  int s = hx::cuda_status(launch_ex(kern, dim3(grid), dim3(kThreadsTma), smem, stream, 1, map, args),
                          "decode_tma_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("decode_tma_kernel");
  s = hx::cuda_status(launch_ex(decode_tma_merge_kernel<T, D, G>,
                                dim3((unsigned)(args.batch * args.n_heads_kv)), dim3(G * D), 0,
                                stream, 1, args, grid),
                      "decode_tma_merge_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("decode_tma_merge_kernel");
  return HX_OK;
}

}  // namespace

// Workspace of the balanced path: partials of 2 slots per CTA (each for a whole query-head
// group, bounded here by n_heads) plus the tile prefix.
size_t decode_tma_workspace(int64_t batch, int64_t n_heads, int64_t head_dim) {
  const int64_t slots = 2 * (int64_t)device_sm_count();
  return (size_t)slots * n_heads * (head_dim + 2) * sizeof(float) + (size_t)(batch + 1) * sizeof(int) + 256;
}

// Returns HX_ERR_UNSUPPORTED (without launching) for shapes this kernel does not cover.
int decode_attention_tma(const void* q, const void* cache, int64_t cbs, int64_t css,
                         const int32_t* seqlens, int64_t batch, int64_t n_heads,
                         int64_t n_heads_kv, int64_t head_dim, float scale, void* out, void* ws,
                         size_t ws_bytes, int dtype, cudaStream_t stream) {
  const int64_t group = n_heads / n_heads_kv;
  if ((dtype != HX_BF16 && dtype != HX_F16) || (head_dim != 64 && head_dim != 128) || group > 2 ||
      batch > kMaxSeqs || css % 8 || cbs % css || (uintptr_t)cache % 16)
    return HX_ERR_UNSUPPORTED;
  const int64_t max_seq = cbs / css;
  const int64_t max_tiles = (max_seq + kTileKeys - 1) / kTileKeys;
  if (batch * n_heads_kv * max_tiles > INT32_MAX / 2) return HX_ERR_UNSUPPORTED;
  const size_t need = decode_tma_workspace(batch, n_heads, head_dim);
  HX_REQUIRE(ws && ws_bytes >= need, "hx_decode_attention: workspace too small (%zu < %zu)",
             ws_bytes, need);
  HX_REQUIRE((uintptr_t)ws % 16 == 0, "hx_decode_attention: workspace must be 16-byte aligned");
  CUtensorMap map;
  const uint64_t dims[4] = {(uint64_t)head_dim, (uint64_t)(2 * n_heads_kv), (uint64_t)max_seq,
                            (uint64_t)batch};
  const uint64_t strides[3] = {(uint64_t)head_dim * 2, (uint64_t)css * 2, (uint64_t)cbs * 2};
  const uint32_t box[4] = {64, 1, (uint32_t)kTileKeys, 1};
  int s = make_tensor_map(&map, cache, 4, dims, strides, box, dtype);
  if (s) return s;
  const int grid = device_sm_count();
  const int64_t slots = 2 * (int64_t)grid;
  float* ws_o = (float*)ws;
  float* ws_ml = ws_o + slots * group * head_dim;
  int* ws_pre = (int*)(ws_ml + slots * group * 2);
  DecArgs args{q, out, ws_o, ws_ml, ws_pre, seqlens, (int)n_heads, (int)n_heads_kv, (int)batch,
               (int)max_seq, scale * 1.4426950408889634f};
#define HX_DEC_TMA(TT, DD, GG) return launch<TT, DD, GG>(map, args, grid, stream)
  if (dtype == HX_BF16) {
    if (head_dim == 128) { if (group == 1) HX_DEC_TMA(__nv_bfloat16, 128, 1); HX_DEC_TMA(__nv_bfloat16, 128, 2); }
    if (group == 1) HX_DEC_TMA(__nv_bfloat16, 64, 1);
    HX_DEC_TMA(__nv_bfloat16, 64, 2);
  }
  if (head_dim == 128) { if (group == 1) HX_DEC_TMA(__half, 128, 1); HX_DEC_TMA(__half, 128, 2); }
  if (group == 1) HX_DEC_TMA(__half, 64, 1);
  HX_DEC_TMA(__half, 64, 2);
#undef HX_DEC_TMA
}
