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
// where it continues write slot 2c, and decode_tma_merge_kernel combines them in CTA order
// (CTAs whose range is empty, which happens when there are fewer tiles than CTAs, are skipped).
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

// Whether CTA c of `grid` owns at least one tile (small batches leave some CTAs without work;
// their partial slots are never written and must not be merged).
HX_DEVICE bool cta_has_tiles(int c, int64_t T, int grid) {
  return (int64_t)c * T / grid < (int64_t)(c + 1) * T / grid;
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

// Issues the K and V loads of one 128-key tile into a ring stage and arms its barrier. A tile
// with fewer live keys (the last of a run) is fetched in 32-row boxes, only as many as hold
// live keys (SWIZZLE_128B is a function of the shared-memory address, so the partial boxes land
// exactly where the full box would have put those rows); rows past them keep stale bytes that
// the consumers never use.
template <int kChunks>
HX_DEVICE void load_kv_tile(uint8_t* kb, uint64_t* bar, const CUtensorMap* full_map,
                            const CUtensorMap* map32, int hk, int hkv, int key0, int b,
                            int live_rows) {
  uint8_t* vb = kb + kChunks * kBoxBytes;
  if (live_rows >= kTileKeys) {
    mbar_arrive_expect_tx(bar, 2 * kChunks * kBoxBytes);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      tma_load_4d(kb + c * kBoxBytes, full_map, bar, c * 64, hk, key0, b);
      tma_load_4d(vb + c * kBoxBytes, full_map, bar, c * 64, hkv + hk, key0, b);
    }
    return;
  }
  const int n32 = (live_rows + 31) / 32;
  mbar_arrive_expect_tx(bar, 2 * kChunks * n32 * 32 * 128);
  for (int i = 0; i < n32; ++i) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      tma_load_4d(kb + c * kBoxBytes + i * 32 * 128, map32, bar, c * 64, hk, key0 + i * 32, b);
      tma_load_4d(vb + c * kBoxBytes + i * 32 * 128, map32, bar, c * 64, hkv + hk, key0 + i * 32, b);
    }
  }
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kThreadsTma, 1)
    decode_tma_kernel(const __grid_constant__ CUtensorMap tmKV,
                      const __grid_constant__ CUtensorMap tmKV32, const DecArgs a) {
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
    prefetch_tensormap(&tmKV32);
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
          load_kv_tile<L::kChunks>(ring + stage * L::kStageBytes, &full[stage], &tmKV, &tmKV32,
                                   p.hk, hkv, t * kTileKeys, p.b,
                                   live_len(a, p.b) - t * kTileKeys);
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
        mbar_wait_drain(&full[i % L::kStages], (i / L::kStages) & 1);
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
  // The query and live length of the next piece are loaded while the current one runs, so a
  // piece boundary costs no global-memory round trip.
  constexpr int kQPer = (G * D + 32 * kConsumers - 1) / (32 * kConsumers);
  PieceWalker walker(pre, hkv, a.batch, u0, u1);
  Piece pc, pn;
  T qn[kQPer];
  int len_n = 0;
  auto prefetch = [&](const Piece& x) {
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
      const int idx = ct + i * 32 * kConsumers;
      if (idx < G * D)
        qn[i] = reinterpret_cast<const T*>(a.q)[((int64_t)x.b * a.n_heads + x.hk * G) * D + idx];
    }
    len_n = live_len(a, x.b);
  };
  bool have = walker.next(pc);
  if (have) prefetch(pc);
  while (have) {
    const int b = pc.b, hk = pc.hk;
    const int len = len_n;
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
      const int idx = ct + i * 32 * kConsumers;
      if (idx < G * D) q_s[idx] = DT<T>::to_f(qn[i]) * a.scale_log2;
    }
    const bool have_next = walker.next(pn);
    if (have_next) prefetch(pn);
    const int start = pc.t_lo * kTileKeys;
    const int end = min(pc.t_hi * kTileKeys, len);
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
      {
        // 32-key slice, unrolled, two accumulator sets to halve the FMA chain. Keys past the
        // live range (the last tile of a run) are skipped by predication: their V rows may hold
        // stale bytes, so they must not enter an FMA even with p = 0.
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
          const bool use0 = k < n_valid, use1 = k + 1 < n_valid;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float p0 = __shfl_sync(0xffffffffu, pr[g], k);
            const float p1 = __shfl_sync(0xffffffffu, pr[g], k + 1);
#pragma unroll
            for (int i = 0; i < kDims; ++i) {
              if (use0) o[g][i] = fmaf(p0, v0[i], o[g][i]);
              if (use1) o2[g][i] = fmaf(p1, v1[i], o2[g][i]);
            }
          }
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < kDims; ++i) o[g][i] += o2[g][i];
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
    // No barrier here: the next piece writes q_s (read only in the tile loops, which every
    // thread left before the barrier above) and then meets at its own start barrier before
    // anything rewrites mo / ml.
    pc = pn;
    have = have_next;
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
    if (!cta_has_tiles(c, total, grid)) continue;
    const int64_t slot = c == c0 ? 2 * (int64_t)c + 1 : 2 * (int64_t)c;
    M = fmaxf(M, a.ws_ml[(slot * G + g) * 2]);
  }
  float Ls = 0.f, A = 0.f;
  for (int c = c0; c <= c1; ++c) {
    if (!cta_has_tiles(c, total, grid)) continue;
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
int launch(const CUtensorMap& map, const CUtensorMap& map32, const DecArgs& args, int grid,
           cudaStream_t stream) {
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
  int s = hx::cuda_status(launch_ex(kern, dim3(grid), dim3(kThreadsTma), smem, stream, 1, map, map32, args),
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

// ------------------------------------------------------------------------------------------
// Tensor-core variant for grouped queries (2..16 query heads per KV head): the same balanced
// partition and TMA ring, with QK and PV on tcgen05.
//   S^T = K Q^T   M = 128 keys, N = 16 (the group's query heads, padded), K = head_dim
//   O^T = V^T P   M = head_dim (128; for head_dim 64 the upper 64 rows are unused), N = 16,
//                 K = 128 keys, V read MN-major straight from the TMA tile
//   warp 0      TMA: the group's q rows once per run (16-row box), K/V tiles into the ring.
//   warp 1      one thread issues the MMAs; S of tile j+1 is issued before P.V of tile j.
//   warps 2-5   thread r = key r of the tile: loads its 16 scores, per-head tile max by a
//               transpose-reduce over the warp (16 shuffles) and a double-buffered exchange
//               across the four warps, online softmax in base 2 (FlashAttention-2 rounding:
//               P rounded to the activation dtype, l from the f32 probabilities), writes P^T
//               into shared memory in the SW128 K-major layout; then as thread r = output
//               element r it adds the previous tile's P.V into registers with the rescale.
// ------------------------------------------------------------------------------------------
constexpr int kTcThreads = 192;
constexpr int kNq = 16;                      // MMA N: query heads per group, padded

template <int D>
struct TcLay {
  static constexpr int kChunks = D / 64;
  static constexpr int kStageBytes = 2 * kChunks * kBoxBytes;   // K + V
  static constexpr int kStages = D == 128 ? 3 : 5;
  static constexpr int kRing = kStages * kStageBytes;
  static constexpr int kPad = D == 64 ? kBoxBytes : 0;           // target of the unused A rows
  static constexpr int kQ = kRing + kPad;                        // 2 x [16 x D] q tiles
  static constexpr int kQBytes = kChunks * kNq * 128;
  static constexpr int kP = kQ + 2 * kQBytes;                    // 2 x [16 x 128 keys] P^T
  static constexpr int kPBytes = 2 * kNq * 128;
  static constexpr int kRed = kP + 2 * kPBytes;                  // floats [2][4][16] + [4][16]
  static constexpr int kBar = kRed + (2 * 4 * kNq + 4 * kNq) * 4;
  static constexpr int kPre = kBar + 32 * 8;
  static constexpr size_t kSmem = 1024 + (size_t)kPre + sizeof(int) * (kMaxSeqs + 1) + 64;
};

// Per-head reduction over the 32 lanes of a warp of 16 values per lane (max or sum): after it,
// lanes 2k and 2k+1 hold the result for head (lane >> 1) & 15 in v[0].
template <bool kMax>
HX_DEVICE float head_reduce(float (&v)[16], int lane) {
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int mask = 16 >> step;
    const int half = 8 >> step;
    const bool upper = lane & mask;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < half) {
        const float send = upper ? v[i] : v[i + half];
        const float recv = __shfl_xor_sync(0xffffffffu, send, mask);
        const float keep = upper ? v[i + half] : v[i];
        v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
      }
    }
  }
  const float o = __shfl_xor_sync(0xffffffffu, v[0], 1);
  return kMax ? fmaxf(v[0], o) : v[0] + o;
}

// Flat walk over the tiles of a CTA's range: piece index, tile, first / last of the piece.
struct TileWalker {
  PieceWalker w;
  Piece p;
  int t, piece;
  bool have;
  HX_DEVICE TileWalker(const int* pre, int hkv, int batch, int64_t u0, int64_t u1)
      : w(pre, hkv, batch, u0, u1), t(0), piece(-1), have(false) {}
  HX_DEVICE bool next() {
    if (have && t + 1 < p.t_hi) {
      ++t;
      return true;
    }
    if (!w.next(p)) return false;
    have = true;
    ++piece;
    t = p.t_lo;
    return true;
  }
  HX_DEVICE bool first() const { return t == p.t_lo; }
  HX_DEVICE bool last() const { return t == p.t_hi - 1; }
};

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmKV,
                     const __grid_constant__ CUtensorMap tmKV32,
                     const __grid_constant__ CUtensorMap tmQ, const DecArgs a) {
  using L = TcLay<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* wred = reinterpret_cast<float*>(sm + L::kRed);          // [2][4][16] tile maxima
  float* lred = wred + 2 * 4 * kNq;                               // [4][16] l sums
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint64_t* kv_full = bars;                    // [kStages]
  uint64_t* kv_empty = bars + L::kStages;      // [kStages]
  uint64_t* q_full = bars + 2 * L::kStages;    // [2]
  uint64_t* q_empty = q_full + 2;              // [2]
  uint64_t* s_full = q_empty + 2;              // [2]
  uint64_t* s_empty = s_full + 2;              // [2]
  uint64_t* p_full = s_empty + 2;              // [2]
  uint64_t* o_full = p_full + 2;               // [2]
  uint64_t* o_empty = o_full + 2;              // [2]
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* pre = reinterpret_cast<int*>(sm + L::kPre);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hkv = a.n_heads_kv;
  const int G = a.n_heads / hkv;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmKV);
    prefetch_tensormap(&tmKV32);
    prefetch_tensormap(&tmQ);
    for (int s = 0; s < L::kStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 64);  // S[2] at columns 0/16, O[2] at 32/48
    tmem_relinquish();
  }
  pdl_wait();  // q, the cache rows and seqlens come from earlier kernels
  pdl_trigger();
  if (warp == 2) {
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
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t total = pre[a.batch];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= a.batch; i += blockDim.x) a.ws_pre[i] = pre[i];
  const int64_t u0 = total ? (int64_t)blockIdx.x * total / gridDim.x : 0;
  const int64_t u1 = total ? (int64_t)(blockIdx.x + 1) * total / gridDim.x : 0;

  if (warp == 0) {
    if (lane == 0 && u0 < u1) {
      TileWalker tw(pre, hkv, a.batch, u0, u1);
      int j = 0, nq = 0;  // K/V tiles and query rows issued
      bool aborted = false;
      while (tw.next()) {
        if (tw.first()) {
          const int qb = tw.piece & 1;
          if (!mbar_wait(&q_empty[qb], ((tw.piece >> 1) & 1) ^ 1)) { aborted = true; break; }
          mbar_arrive_expect_tx(&q_full[qb], L::kQBytes);
          const int row = tw.p.b * a.n_heads + tw.p.hk * G;
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c)
            tma_load_2d(sm + L::kQ + qb * L::kQBytes + c * kNq * 128, &tmQ, &q_full[qb], c * 64, row);
          ++nq;
        }
        const int st = j % L::kStages;
        if (!mbar_wait(&kv_empty[st], ((j / L::kStages) & 1) ^ 1)) { aborted = true; break; }
        load_kv_tile<L::kChunks>(sm + st * L::kStageBytes, &kv_full[st], &tmKV, &tmKV32, tw.p.hk,
                                 hkv, tw.t * kTileKeys, tw.p.b,
                                 live_len(a, tw.p.b) - tw.t * kTileKeys);
        ++j;
      }
      if (aborted) {
        // The consumers may have given up as well: let the newest loads (each the latest use of
        // its buffer) land before the CTA's shared memory is released.
        for (int i = j > L::kStages ? j - L::kStages : 0; i < j; ++i)
          mbar_wait_drain(&kv_full[i % L::kStages], (i / L::kStages) & 1);
        for (int i = nq > 2 ? nq - 2 : 0; i < nq; ++i) mbar_wait_drain(&q_full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && u0 < u1) {
      constexpr uint32_t idesc_s = make_idesc_f16<T>(128, kNq);
      constexpr uint32_t idesc_o = make_idesc_f16<T>(128, kNq, 1, 0);
      TileWalker ws(pre, hkv, a.batch, u0, u1);
      int ns = 0;  // S tiles issued
      bool ok = true;
      auto issue_s = [&]() -> bool {
        const int j = ns;
        const int st = j % L::kStages;
        const int qb = ws.piece & 1;
        if (ws.first() && !mbar_wait(&q_full[qb], (ws.piece >> 1) & 1)) return false;
        if (!mbar_wait(&kv_full[st], (j / L::kStages) & 1)) return false;
        if (!mbar_wait(&s_empty[j & 1], ((j >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sm + st * L::kStageBytes);
        const uint32_t qa = smem_u32(sm + L::kQ + qb * L::kQBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int c = kk >> 2, o = (kk & 3) * 32;
          tc_mma_f16(tmem + (j & 1) * kNq, sw128_kmajor_desc(ka + c * kBoxBytes + o),
                     sw128_kmajor_desc(qa + c * kNq * 128 + o), idesc_s, kk ? 1u : 0u);
        }
        tc_commit(&s_full[j & 1]);
        if (ws.last()) tc_commit(&q_empty[qb]);  // q buffer free once these MMAs complete
        ++ns;
        return true;
      };
      if (ws.next()) ok = issue_s();
      for (int j = 0; ok && j < ns; ++j) {
        if (ws.next() && !issue_s()) ok = false;
        const int st = j % L::kStages;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1)) break;
        if (!mbar_wait(&o_empty[j & 1], ((j >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t va = smem_u32(sm + st * L::kStageBytes + L::kChunks * kBoxBytes);
        const uint32_t pa = smem_u32(sm + L::kP + (j & 1) * L::kPBytes);
#pragma unroll
        for (int kk = 0; kk < kTileKeys / 16; ++kk) {
          const int c = kk >> 2, o = (kk & 3) * 32;
          tc_mma_f16(tmem + 32 + (j & 1) * kNq,
                     sw128_mnmajor_desc(va + kk * 16 * 128, kBoxBytes, 1024),
                     sw128_kmajor_desc(pa + c * kNq * 128 + o), idesc_o, kk ? 1u : 0u);
        }
        tc_commit(&o_full[j & 1]);
        tc_commit(&kv_empty[st]);
      }
      tc_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (u0 < u1) {
    // Softmax / output warps. Thread r: key r of a tile (scores), element r of the output.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    TileWalker tw(pre, hkv, a.batch, u0, u1);
    int j = 0;
    bool ok = true;
    float m_run[kNq], l_part[kNq], o[kNq], alpha_prev[kNq];
    int b = 0, hk = 0, end = 0;
    int64_t seg0 = 0, seg1 = 0;
    auto correct = [&](int jj, const float (&al)[kNq]) {
      const bool got = mbar_wait_warp(&o_full[jj & 1], (jj >> 1) & 1);
      tc_fence_after();
      if (got) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(lane_addr + 32 + (jj & 1) * kNq, v);
        tc_wait_ld();
#pragma unroll
        for (int h = 0; h < kNq; ++h) o[h] = o[h] * al[h] + __uint_as_float(v[h]);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[jj & 1]);
      return got;
    };
    auto finish = [&]() {
      // l = sum over the 128 key-threads of their partial sums.
      float t[kNq];
#pragma unroll
      for (int h = 0; h < kNq; ++h) t[h] = l_part[h];
      const float part = head_reduce<false>(t, lane);
      if ((lane & 1) == 0) lred[quarter * kNq + ((lane >> 1) & 15)] = part;
      ok = named_bar_and(1, 128, ok);
      float l_fin[kNq];
#pragma unroll
      for (int h = 0; h < kNq; ++h)
        l_fin[h] = (lred[h] + lred[kNq + h]) + (lred[2 * kNq + h] + lred[3 * kNq + h]);
      const bool whole = seg0 >= u0 && seg1 <= u1;
      const int64_t slot = 2 * (int64_t)blockIdx.x + (seg0 < u0 ? 0 : 1);
      if (ok && r < D) {
#pragma unroll
        for (int g = 0; g < kNq; ++g) {
          if (g >= G) break;
          const int64_t hrow = (int64_t)b * a.n_heads + hk * G + g;
          if (whole) {
            reinterpret_cast<T*>(a.out)[hrow * D + r] = DT<T>::from_f(l_fin[g] > 0.f ? o[g] / l_fin[g] : 0.f);
          } else {
            a.ws_o[(slot * G + g) * D + r] = o[g];
            if (r == 0) {
              a.ws_ml[(slot * G + g) * 2] = m_run[g];
              a.ws_ml[(slot * G + g) * 2 + 1] = l_fin[g];
            }
          }
        }
      }
      ok = named_bar_and(1, 128, ok);  // lred is reused by the next run
    };
    while (ok && tw.next()) {
      if (tw.first()) {
        b = tw.p.b;
        hk = tw.p.hk;
        seg0 = tw.p.seg0;
        seg1 = tw.p.seg1;
        end = min(tw.p.t_hi * kTileKeys, live_len(a, b));
#pragma unroll
        for (int h = 0; h < kNq; ++h) {
          m_run[h] = -INFINITY;
          l_part[h] = 0.f;
          o[h] = 0.f;
        }
      }
      const bool got = mbar_wait_warp(&s_full[j & 1], (j >> 1) & 1);
      tc_fence_after();
      float sc[kNq];
      const bool valid = tw.t * kTileKeys + r < end;
      if (got) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(lane_addr + (j & 1) * kNq, v);
        tc_wait_ld();
#pragma unroll
        for (int h = 0; h < kNq; ++h) sc[h] = valid ? __uint_as_float(v[h]) * a.scale_log2 : -INFINITY;
      } else {
#pragma unroll
        for (int h = 0; h < kNq; ++h) sc[h] = -INFINITY;
      }
      float t[kNq];
#pragma unroll
      for (int h = 0; h < kNq; ++h) t[h] = sc[h];
      const float wm = head_reduce<true>(t, lane);
      float* wr = wred + (j & 1) * 4 * kNq;
      if ((lane & 1) == 0) wr[quarter * kNq + ((lane >> 1) & 15)] = wm;
      ok = named_bar_and(1, 128, ok && got);
      if (!ok) break;
      float alpha[kNq];
#pragma unroll
      for (int h = 0; h < kNq; ++h) {
        const float tmax = fmaxf(fmaxf(wr[h], wr[kNq + h]), fmaxf(wr[2 * kNq + h], wr[3 * kNq + h]));
        const float m_new = fmaxf(m_run[h], tmax);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        alpha[h] = exp2f(m_run[h] - m_use);
        const float pv = valid ? exp2f(sc[h] - m_use) : 0.f;
        l_part[h] = l_part[h] * alpha[h] + pv;
        m_run[h] = m_new;
        sc[h] = pv;
      }
      // Cache rows past the live keys may hold any bits (NaN included): zero their V rows so
      // 0 * stale never reaches the P.V product.
      if (!valid) {
        uint8_t* vrow = sm + (j % L::kStages) * L::kStageBytes + L::kChunks * kBoxBytes + r * 128;
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(vrow + c * kBoxBytes + u * 16) = make_uint4(0, 0, 0, 0);
      }
      // P^T row h (query head), column r (key) in the SW128 K-major layout of the MMA's B.
      uint8_t* pb = sm + L::kP + (j & 1) * L::kPBytes + (r >> 6) * (kNq * 128);
      const int unit = (r & 63) >> 3;
#pragma unroll
      for (int h = 0; h < kNq; ++h) {
        if (h >= G) break;
        const int rr = h & 7;
        *reinterpret_cast<T*>(pb + (h >> 3) * 1024 + rr * 128 + ((unit ^ rr) << 4) + (r & 7) * 2) =
            DT<T>::from_f(sc[h]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&s_empty[j & 1]);
      mbar_arrive(&p_full[j & 1]);
      if (!tw.first()) ok = correct(j - 1, alpha_prev) && ok;
#pragma unroll
      for (int h = 0; h < kNq; ++h) alpha_prev[h] = alpha[h];
      if (tw.last()) {
        ok = correct(j, alpha_prev) && ok;
        finish();
      }
      ++j;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 64);
}

// Combines the partials of cut runs for a runtime group size: one CTA per (sequence, kv head),
// one thread per (query head of the group, output element). One pass over the contributing
// CTAs with an online rescale; the loads of different contributors do not depend on each
// other, so they overlap.
template <typename T, int D>
__global__ void decode_tc_merge_kernel(const DecArgs a, int grid) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x / a.n_heads_kv, hk = blockIdx.x % a.n_heads_kv;
  const int G = a.n_heads / a.n_heads_kv;
  const int64_t total = a.ws_pre[a.batch];
  const int tiles = (a.ws_pre[b + 1] - a.ws_pre[b]) / a.n_heads_kv;
  int c0 = 0, c1 = -1;
  if (tiles > 0) {
    const int64_t seg0 = a.ws_pre[b] + (int64_t)hk * tiles, seg1 = seg0 + tiles;
    c0 = cta_of(seg0, total, grid);
    c1 = cta_of(seg1 - 1, total, grid);
    if (c0 == c1) return;  // finished by one CTA, output already written
  }
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, e = idx % D;
    const int64_t h = (int64_t)b * a.n_heads + hk * G + g;
    float M = -INFINITY, Ls = 0.f, A = 0.f;
#pragma unroll 4
    for (int c = c0; c <= c1; ++c) {
      if (!cta_has_tiles(c, total, grid)) continue;
      const int64_t slot = c == c0 ? 2 * (int64_t)c + 1 : 2 * (int64_t)c;
      const float mc = a.ws_ml[(slot * G + g) * 2];
      const float lc = a.ws_ml[(slot * G + g) * 2 + 1];
      const float oc = a.ws_o[(slot * G + g) * D + e];
      if (mc == -INFINITY) continue;
      const float mn = fmaxf(M, mc);
      const float sa = exp2f(M - mn), sb = exp2f(mc - mn);
      Ls = Ls * sa + lc * sb;
      A = A * sa + oc * sb;
      M = mn;
    }
    reinterpret_cast<T*>(a.out)[h * D + e] = DT<T>::from_f(Ls > 0.f ? A / Ls : 0.f);
  }
}

template <typename T, int D>
int launch_tc(const CUtensorMap& map, const CUtensorMap& map32, const CUtensorMap& qmap,
              const DecArgs& args, int grid, cudaStream_t stream) {
  using L = TcLay<D>;
  auto kern = decode_tc_kernel<T, D>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::kSmem),
                            "cudaFuncSetAttribute(decode_tc)");
    if (s) return s;
    attr[dev & 63] = true;
  }
  int s = hx::cuda_status(launch_ex(kern, dim3(grid), dim3(kTcThreads), L::kSmem, stream, 1, map, map32, qmap, args),
                          "decode_tc_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("decode_tc_kernel");
  const int G = args.n_heads / args.n_heads_kv;
  s = hx::cuda_status(launch_ex(decode_tc_merge_kernel<T, D>,
                                dim3((unsigned)(args.batch * args.n_heads_kv)),
                                dim3((unsigned)std::min(G * D, 1024)), 0, stream, 1, args, grid),
                      "decode_tc_merge_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("decode_tc_merge_kernel");
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
  if ((dtype != HX_BF16 && dtype != HX_F16) || (head_dim != 64 && head_dim != 128) || group > 16 ||
      batch > kMaxSeqs || css % 8 || cbs % css || (uintptr_t)cache % 16 || (uintptr_t)q % 16)
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
  CUtensorMap map32;  // 32-row boxes for the partial last tile of a run
  const uint32_t box32[4] = {64, 1, 32, 1};
  s = make_tensor_map(&map32, cache, 4, dims, strides, box32, dtype);
  if (s) return s;
  const int grid = device_sm_count();
  const int64_t slots = 2 * (int64_t)grid;
  float* ws_o = (float*)ws;
  float* ws_ml = ws_o + slots * group * head_dim;
  int* ws_pre = (int*)(ws_ml + slots * group * 2);
  DecArgs args{q, out, ws_o, ws_ml, ws_pre, seqlens, (int)n_heads, (int)n_heads_kv, (int)batch,
               (int)max_seq, scale * 1.4426950408889634f};
  if (group > 2) {
    // Grouped queries: QK and PV on tcgen05 (q rows of a group = one 16-row TMA box).
    CUtensorMap qmap;
    const uint64_t qdims[2] = {(uint64_t)head_dim, (uint64_t)(batch * n_heads)};
    const uint64_t qstrides[1] = {(uint64_t)head_dim * 2};
    const uint32_t qbox[2] = {64, (uint32_t)kNq};
    s = make_tensor_map(&qmap, q, 2, qdims, qstrides, qbox, dtype);
    if (s) return s;
    if (dtype == HX_BF16)
      return head_dim == 128 ? launch_tc<__nv_bfloat16, 128>(map, map32, qmap, args, grid, stream)
                             : launch_tc<__nv_bfloat16, 64>(map, map32, qmap, args, grid, stream);
    return head_dim == 128 ? launch_tc<__half, 128>(map, map32, qmap, args, grid, stream)
                           : launch_tc<__half, 64>(map, map32, qmap, args, grid, stream);
  }
#define HX_DEC_TMA(TT, DD, GG) return launch<TT, DD, GG>(map, map32, args, grid, stream)
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
