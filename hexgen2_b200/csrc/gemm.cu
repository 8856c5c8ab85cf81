// K1/K2/K7/K8: projection GEMMs C = A * B^T (nn.Linear) with fused epilogues.
//
// f16/bf16: a persistent, warp-specialised tcgen05 kernel.
//   warp 0      TMA producer: A [BM x 64] and B [BN x 64] K-major tiles, SWIZZLE_128B, into a
//               kStages-deep shared-memory ring (full/empty mbarriers).
//   warp 1      MMA issuer: one thread issues tcgen05.mma kind::f16 (M=128, N=BN, K=16) into a
//               double-buffered f32 accumulator in tensor memory; tcgen05.commit frees each
//               smem stage and publishes each finished accumulator.
//   warps 2-5   epilogue: tcgen05.ld 32 columns at a time (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), applies the epilogue, stores to global memory.
//   The accumulator of tile i+1 is computed while tile i is being stored.
// Decode-shaped problems (few tiles) split K across CTAs; partial sums go to a caller-provided
// f32 workspace and a small kernel reduces them in split order and applies the epilogue.
// f32: a CUDA-core tiled kernel with exact f32 products (the reference's f32 path).
//
// Epilogues reproduce the reference's rounding points:
//   NONE      c = round(acc)
//   RESIDUAL  c = round(round(acc) + r)                  (block.py:155-158 residual add)
//   SWIGLU    u = round(acc_up), g = round(acc_gate), c = round(u * round(silu(g)))
//             (mlp.py:79-87; fc1 rows must be interleaved in blocks of 16: [up16|gate16]...)
#include "common.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 x 2 bytes = one 128-byte swizzle row
constexpr int kGemmThreads = 192;

// kSwap: decode-shaped problems (M = batch <= 64) run with the operands swapped: the MMA's
// 128-row side walks the weight rows (output features) and its N side is the batch, so no
// tensor-core work or shared-memory bandwidth is spent on padding rows. Those configurations
// use small rings (<= ~110 KB) so two CTAs fit on an SM.
template <int BN, bool kSwap = false>
struct Cfg {
  static constexpr int kStages = kSwap ? (BN <= 16 ? 6 : (BN <= 32 ? 5 : 4))
                                       : (BN == 256 ? 4 : (BN == 128 ? 6 : 8));
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two accumulators
  static constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 1024 /*align*/ + 512;
};

// Destination of the fused Wqkv epilogue (HX_EPI_QKV_ROTARY).
struct QkvArgs {
  void* q_out;
  void* cache;
  int64_t cbs, css, cbo, max_seq, table_rows;
  const int32_t* pos_start;
  const void* cos;
  const void* sin;
  int n_heads, n_heads_kv, head_dim, seqlen;
};

// Workspace layout (f16/bf16): [0, 64 KiB) per-tile arrival counters of the stream-K fixup
// (zero between calls), then the f32 partial sums.
constexpr size_t kFlagBytes = 64 * 1024;

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, k_splits, kb_per_split, k_blocks;
  void* C;
  int64_t ldc;
  const void* R;
  int64_t ldr;
  float* ws;        // split-K partials [k_splits][M][N]; stream-K partials [ctas][segs][M][128]
  uint32_t* flags;  // stream-K per-tile arrival counters
  int ctas, segs;   // stream-K: CTAs sharing the units, max tile segments per CTA
  QkvArgs qkv;
};

HX_DEVICE float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Fused Wqkv epilogue for the feature pair (n, n+1), n even, of row m = b * seqlen + s: the
// values are rounded like the reference's Linear output; q and k pairs are rotated (f32 math
// on the dtype-cached cos/sin, as flash_attn's rotary) and q goes to q_out, k and v to the cache
// row of position pos_start[b] + s (the packed [k; v] part of a row is exactly the cache's
// [2, hkv, d] row layout).
template <typename T>
HX_DEVICE void qkv_store_pair(const GemmArgs& a, int m, int n, float v0, float v1) {
  if (m >= a.M || n >= a.N) return;
  const QkvArgs& q = a.qkv;
  const int b = m / q.seqlen, s = m - b * q.seqlen;
  const int64_t pos = (int64_t)q.pos_start[b] + s;
  if (pos < 0 || pos >= q.max_seq || pos >= q.table_rows) {
    record_device_error(HX_DEVERR_BAD_ARGUMENT);
    return;
  }
  float x0 = round_to<T>(v0), x1 = round_to<T>(v1);
  const int hqd = q.n_heads * q.head_dim;
  if (n < hqd + q.n_heads_kv * q.head_dim) {
    const int64_t i = pos * (q.head_dim / 2) + ((n % q.head_dim) >> 1);
    const float c = DT<T>::to_f(reinterpret_cast<const T*>(q.cos)[i]);
    const float sn = DT<T>::to_f(reinterpret_cast<const T*>(q.sin)[i]);
    const float o0 = x0 * c - x1 * sn;
    const float o1 = x0 * sn + x1 * c;
    x0 = o0;
    x1 = o1;
  }
  T* dst = n < hqd ? reinterpret_cast<T*>(q.q_out) + (int64_t)m * hqd + n
                   : reinterpret_cast<T*>(q.cache) + (q.cbo + b) * q.cbs + pos * q.css + (n - hqd);
  T pair[2] = {DT<T>::from_f(x0), DT<T>::from_f(x1)};
  *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(pair);
}

// Applies the epilogue to 32 accumulator columns [n0, n0+32) of row m and stores them.
template <typename T, int EPI>
HX_DEVICE void epilogue_store(const GemmArgs& a, int m, int n0, const float* v) {
  if (m >= a.M) return;
  if (EPI == HX_EPI_QKV_ROTARY) {
    const QkvArgs& q = a.qkv;
    if (q.head_dim % 32 != 0 || n0 + 32 > a.N) {
#pragma unroll
      for (int j = 0; j < 16; ++j) qkv_store_pair<T>(a, m, n0 + 2 * j, v[2 * j], v[2 * j + 1]);
      return;
    }
    // The 32 columns lie in one head: one destination row, 16 consecutive cos/sin entries.
    const int b = m / q.seqlen, s = m - b * q.seqlen;
    const int64_t pos = (int64_t)q.pos_start[b] + s;
    if (pos < 0 || pos >= q.max_seq || pos >= q.table_rows) {
      record_device_error(HX_DEVERR_BAD_ARGUMENT);
      return;
    }
    const int hqd = q.n_heads * q.head_dim;
    const int within = n0 % q.head_dim;
    T out[32];
    if (n0 < hqd + q.n_heads_kv * q.head_dim) {
      const T* cs = reinterpret_cast<const T*>(q.cos) + pos * (q.head_dim / 2) + within / 2;
      const T* sn = reinterpret_cast<const T*>(q.sin) + pos * (q.head_dim / 2) + within / 2;
      T cv[16], sv[16];
      *reinterpret_cast<uint4*>(cv) = *reinterpret_cast<const uint4*>(cs);
      *reinterpret_cast<uint4*>(cv + 8) = *reinterpret_cast<const uint4*>(cs + 8);
      *reinterpret_cast<uint4*>(sv) = *reinterpret_cast<const uint4*>(sn);
      *reinterpret_cast<uint4*>(sv + 8) = *reinterpret_cast<const uint4*>(sn + 8);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float x0 = round_to<T>(v[2 * j]), x1 = round_to<T>(v[2 * j + 1]);
        const float c = DT<T>::to_f(cv[j]), sn2 = DT<T>::to_f(sv[j]);
        out[2 * j] = DT<T>::from_f(x0 * c - x1 * sn2);
        out[2 * j + 1] = DT<T>::from_f(x0 * sn2 + x1 * c);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) out[j] = DT<T>::from_f(v[j]);
    }
    T* dst = n0 < hqd ? reinterpret_cast<T*>(q.q_out) + (int64_t)m * hqd + n0
                      : reinterpret_cast<T*>(q.cache) + (q.cbo + b) * q.cbs + pos * q.css + (n0 - hqd);
#pragma unroll
    for (int j = 0; j < 32; j += 8)
      *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(out + j);
    return;
  }
  if (EPI == HX_EPI_SWIGLU) {
    // 16 up columns then 16 gate columns -> 16 outputs at column n0/2.
    T* out = reinterpret_cast<T*>(a.C) + (int64_t)m * a.ldc + n0 / 2;
    if (n0 >= a.N) return;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float u = round_to<T>(v[j]);
      const float g = round_to<T>(v[16 + j]);
      out[j] = DT<T>::from_f(u * round_to<T>(silu_f(g)));
    }
    return;
  }
  T* out = reinterpret_cast<T*>(a.C) + (int64_t)m * a.ldc + n0;
  const T* res = EPI == HX_EPI_RESIDUAL ? reinterpret_cast<const T*>(a.R) + (int64_t)m * a.ldr + n0
                                        : nullptr;
  const int valid = min(32, a.N - n0);
  if (valid == 32 && ((uintptr_t)out % 16 == 0) && (!res || (uintptr_t)res % 16 == 0)) {
    constexpr int P = 16 / sizeof(T);
#pragma unroll
    for (int c = 0; c < 32; c += P) {
      T pack[P];
      T rpack[P];
      if (EPI == HX_EPI_RESIDUAL) *reinterpret_cast<uint4*>(rpack) = *reinterpret_cast<const uint4*>(res + c);
#pragma unroll
      for (int j = 0; j < P; ++j) {
        float x = round_to<T>(v[c + j]);
        if (EPI == HX_EPI_RESIDUAL) x = x + DT<T>::to_f(rpack[j]);
        pack[j] = DT<T>::from_f(x);
      }
      *reinterpret_cast<uint4*>(out + c) = *reinterpret_cast<uint4*>(pack);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < valid) {
        float x = round_to<T>(v[j]);
        if (EPI == HX_EPI_RESIDUAL) x = x + DT<T>::to_f(res[j]);
        out[j] = DT<T>::from_f(x);
      }
    }
  }
}

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + C::kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smB + C::kStages * C::kBBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // MMA completion barrier used on exit
  uint32_t* counters = reinterpret_cast<uint32_t*>(drain + 1);  // [0] loads issued, [1] consumed
  uint32_t* tmem_slot = counters + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = a.m_tiles * a.n_tiles * a.k_splits;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    counters[0] = counters[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
        const int split = t % a.k_splits;
        const int mn = t / a.k_splits;
        const int m_blk = mn % a.m_tiles, n_blk = mn / a.m_tiles;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) goto producer_done;
          mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          tma_load_2d(smA + stage * C::kABytes, &tmA, &full[stage], kb * BK, m_blk * BM);
          tma_load_2d(smB + stage * C::kBBytes, &tmB, &full[stage], kb * BK, n_blk * BN);
          ++issued;
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      counters[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<T>(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      uint32_t consumed = 0;
      for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
        const int split = t % a.k_splits;
        const int kb0 = split * a.kb_per_split;
        const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase)) goto mma_done;
          ++consumed;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * C::kABytes);
          const uint32_t b_addr = smem_u32(smB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t da = sw128_kmajor_desc(a_addr + k * 32);
            const uint64_t db = sw128_kmajor_desc(b_addr + k * 32);
            tc_mma_f16(d_tmem, da, db, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        tc_commit(&tfull[acc]);
      }
    mma_done:
      // No MMA of this CTA may still be running when TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0);
      counters[1] = consumed;
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++local) {
      const int split = t % a.k_splits;
      const int mn = t / a.k_splits;
      const int m_blk = mn % a.m_tiles, n_blk = mn / a.m_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase)) break;
      tc_fence_after();
      const int m = m_blk * BM + row;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN + c * 32, r);
        tc_wait_ld();
        const int n0 = n_blk * BN + c * 32;
        if (n0 >= a.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if (a.k_splits > 1) {
          if (m < a.M) {
            float* dst = a.ws + ((int64_t)split * a.M + m) * a.N + n0;
            const int valid = min(32, a.N - n0);
            if (valid == 32 && (a.N % 4 == 0)) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (j < valid) dst[j] = v[j];
            }
          }
        } else {
          epilogue_store<T, EPI>(a, m, n0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  // After an aborted wait, loads may have been issued that nobody consumed: let them land
  // (bounded) before the CTA's shared memory goes away.
  if (threadIdx.x == 0) {
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1)) break;
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

// ------------------------------------------------------------------------------------------
// Decode-shaped GEMM (M = batch <= 64): operands swapped + stream-K.
//   MMA A = weight rows (128 per tile, K-major), MMA B = the batch rows (N = 16/32/64), so no
//   tensor-core work or shared-memory bandwidth goes to padding rows. The (tile, k-block) units
//   of the whole problem are divided evenly between ~2 CTAs per SM: every CTA streams the same
//   number of weight bytes, with no wave tail. A CTA's range may start or end inside a tile; each
//   tile part ("segment") is written as f32 to partial slot (cta, segment), and
//   streamk_reduce_kernel sums the parts of each tile in CTA order and applies the epilogue.
// ------------------------------------------------------------------------------------------
HX_DEVICE int64_t sk_unit_begin(int c, int64_t units, int ctas) { return (int64_t)c * units / ctas; }

// One output element of the swapped layout (feature n, batch row b), called by all 32 lanes
// of a warp with a warp-uniform b (the epilogues exchange partners with shuffles).
template <typename T, int EPI>
HX_DEVICE void sk_store(const GemmArgs& a, int b, int n, int lane, float v) {
  if (EPI == HX_EPI_SWIGLU) {
    // Rows [32k, 32k+16) of a tile are up, [32k+16, 32k+32) the matching gates.
    const float gate = __shfl_xor_sync(0xffffffffu, v, 16);
    if (lane < 16 && b < a.M && n < a.N) {
      const float u = round_to<T>(v), g = round_to<T>(gate);
      reinterpret_cast<T*>(a.C)[(int64_t)b * a.ldc + (n >> 5) * 16 + lane] =
          DT<T>::from_f(u * round_to<T>(silu_f(g)));
    }
  } else if (EPI == HX_EPI_QKV_ROTARY) {
    const float other = __shfl_xor_sync(0xffffffffu, v, 1);
    if ((lane & 1) == 0) qkv_store_pair<T>(a, b, n, v, other);
  } else if (b < a.M && n < a.N) {
    float x = round_to<T>(v);
    if (EPI == HX_EPI_RESIDUAL)
      x += DT<T>::to_f(reinterpret_cast<const T*>(a.R)[(int64_t)b * a.ldr + n]);
    reinterpret_cast<T*>(a.C)[(int64_t)b * a.ldc + n] = DT<T>::from_f(x);
  }
}

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_streamk_kernel(const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmX, const GemmArgs a) {
  using C = Cfg<BN, true>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + C::kStages * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smB + C::kStages * C::kBBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* counters = reinterpret_cast<uint32_t*>(drain + 1);
  uint32_t* tmem_slot = counters + 2;
  volatile uint32_t* sk_last = tmem_slot + 1;                          // fixup decision
  int64_t* sk_off = reinterpret_cast<int64_t*>(tmem_slot + 2);        // [<= 24] part offsets

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = a.k_blocks;
  const int64_t units = (int64_t)a.m_tiles * kb;
  const int64_t u0 = sk_unit_begin(blockIdx.x, units, gridDim.x);
  const int64_t u1 = sk_unit_begin(blockIdx.x + 1, units, gridDim.x);

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    counters[0] = counters[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      for (int64_t u = u0; u < u1; ++u) {
        const int t = (int)(u / kb), kbi = (int)(u - (int64_t)t * kb);
        if (!mbar_wait(&empty[stage], phase ^ 1)) break;
        mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
        tma_load_2d(smA + stage * C::kABytes, &tmW, &full[stage], kbi * BK, t * BM);
        tma_load_2d(smB + stage * C::kBBytes, &tmX, &full[stage], kbi * BK, 0);
        ++issued;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      counters[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<T>(BM, BN);
      int stage = 0, seg = -1, cur = -1, acc = 0;
      uint32_t phase = 0, consumed = 0;
      bool first = false;
      for (int64_t u = u0; u < u1; ++u) {
        const int t = (int)(u / kb);
        if (t != cur) {  // a new tile segment starts: take the next accumulator buffer
          if (cur >= 0) tc_commit(&tfull[acc]);
          ++seg;
          acc = seg & 1;
          if (!mbar_wait(&tempty[acc], ((seg >> 1) & 1) ^ 1)) goto sk_mma_done;
          tc_fence_after();
          cur = t;
          first = true;
        }
        if (!mbar_wait(&full[stage], phase)) goto sk_mma_done;
        ++consumed;
        tc_fence_after();
        {
          const uint32_t a_addr = smem_u32(smA + stage * C::kABytes);
          const uint32_t b_addr = smem_u32(smB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_f16(tmem_base + acc * BN, sw128_kmajor_desc(a_addr + k * 32),
                       sw128_kmajor_desc(b_addr + k * 32), idesc, (first && k == 0) ? 0u : 1u);
        }
        first = false;
        tc_commit(&empty[stage]);
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (cur >= 0) tc_commit(&tfull[acc]);
    sk_mma_done:
      tc_commit(drain);
      mbar_wait(drain, 0);
      counters[1] = consumed;
    }
  } else if (u1 > u0) {
    // Epilogue warps 2..5 (named barrier 2). A tile this CTA owns alone is stored straight from
    // TMEM. Otherwise the part goes to partial slot (cta, segment); the CTA that completes a
    // tile's arrival count sums all parts of the tile in CTA order (deterministic), applies the
    // epilogue, and resets the counter for the next call.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int t_first = (int)(u0 / kb), t_last = (int)((u1 - 1) / kb);
    for (int t = t_first, seg = 0; t <= t_last; ++t, ++seg) {
      const int acc = seg & 1;
      if (!named_bar_and(2, 128, mbar_wait_warp(&tfull[acc], (seg >> 1) & 1))) break;
      tc_fence_after();
      const int64_t ua = (int64_t)t * kb, ub = (int64_t)(t + 1) * kb - 1;
      const int c0 = (int)(((ua + 1) * a.ctas - 1) / units);
      const int c1 = (int)(((ub + 1) * a.ctas - 1) / units);
      const int n = t * BM + r;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
      if (c0 == c1) {
#pragma unroll
        for (int c = 0; c < BN / 16; ++c) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(taddr + c * 16, v);
          tc_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) sk_store<T, EPI>(a, c * 16 + j, n, lane, __uint_as_float(v[j]));
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
      float* slot = a.ws + ((int64_t)blockIdx.x * a.segs + seg) * a.M * BM;
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(taddr + c * 16, v);
        tc_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int b = c * 16 + j;
          if (b < a.M) slot[(int64_t)b * BM + r] = __uint_as_float(v[j]);
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      __threadfence();
      named_bar_sync(2, 128);
      const int parts = c1 - c0 + 1;
      if (threadIdx.x == 64) {
        const uint32_t old = atomicAdd(&a.flags[t], 1u);
        *sk_last = (old == (uint32_t)(parts - 1)) ? 1u : 0u;
      }
      if (r < parts && r < 24) {  // offsets of the parts, contributor order
        const int c = c0 + r;
        const int seg_c = t - (int)(((int64_t)c * units / a.ctas) / kb);
        sk_off[r] = ((int64_t)c * a.segs + seg_c) * a.M * BM;
      }
      named_bar_sync(2, 128);
      if (*sk_last) {
        __threadfence();
        if (parts > 24) {
          if (r == 0) record_device_error(HX_DEVERR_BAD_ARGUMENT);
        } else {
          // All rows' loads are issued before any store, so the L2 round trips overlap.
          float sum[BN];
#pragma unroll
          for (int b = 0; b < BN; ++b) sum[b] = 0.f;
          for (int i = 0; i < parts; ++i) {
            const float* src = a.ws + sk_off[i] + r;
#pragma unroll
            for (int b = 0; b < BN; ++b)
              if (b < a.M) sum[b] += src[(int64_t)b * BM];
          }
#pragma unroll
          for (int b = 0; b < BN; ++b) sk_store<T, EPI>(a, b, n, lane, sum[b]);
        }
        if (threadIdx.x == 64) a.flags[t] = 0u;
      }
      named_bar_sync(2, 128);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait(&full[i % C::kStages], (i / C::kStages) & 1)) break;
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

// Split-K reduction in split order + epilogue. One thread per output element.
template <typename T, int EPI>
__global__ void splitk_reduce_kernel(const GemmArgs a) {
  const int64_t out_cols = (EPI == HX_EPI_SWIGLU || EPI == HX_EPI_QKV_ROTARY) ? a.N / 2 : a.N;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)a.M * out_cols) return;
  const int m = (int)(idx / out_cols);
  const int j = (int)(idx % out_cols);
  const int64_t plane = (int64_t)a.M * a.N;
  if (EPI == HX_EPI_QKV_ROTARY) {  // j indexes feature pairs
    float v0 = 0.f, v1 = 0.f;
    for (int s = 0; s < a.k_splits; ++s) {
      v0 += a.ws[s * plane + (int64_t)m * a.N + 2 * j];
      v1 += a.ws[s * plane + (int64_t)m * a.N + 2 * j + 1];
    }
    qkv_store_pair<T>(a, m, 2 * j, v0, v1);
    return;
  }
  if (EPI == HX_EPI_SWIGLU) {
    const int n_up = (j / 16) * 32 + (j % 16);
    float up = 0.f, gate = 0.f;
    for (int s = 0; s < a.k_splits; ++s) {
      up += a.ws[s * plane + (int64_t)m * a.N + n_up];
      gate += a.ws[s * plane + (int64_t)m * a.N + n_up + 16];
    }
    const float u = round_to<T>(up), g = round_to<T>(gate);
    reinterpret_cast<T*>(a.C)[(int64_t)m * a.ldc + j] = DT<T>::from_f(u * round_to<T>(silu_f(g)));
    return;
  }
  float acc = 0.f;
  for (int s = 0; s < a.k_splits; ++s) acc += a.ws[s * plane + (int64_t)m * a.N + j];
  float x = round_to<T>(acc);
  if (EPI == HX_EPI_RESIDUAL) x += DT<T>::to_f(reinterpret_cast<const T*>(a.R)[(int64_t)m * a.ldr + j]);
  reinterpret_cast<T*>(a.C)[(int64_t)m * a.ldc + j] = DT<T>::from_f(x);
}

// ---------------------------------------------------------------------------------------
// f32 CUDA-core GEMM: 64x64 tile, 16-deep K slices, 4x4 outputs per thread.
// ---------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ B,
                                                       GemmArgs a, int64_t lda, int64_t ldb) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < a.K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int r = i / 16, kk = i % 16;
      const int gm = m0 + r, gn = n0 + r, gk = k0 + kk;
      As[kk][r] = (gm < a.M && gk < a.K) ? A[(int64_t)gm * lda + gk] : 0.f;
      Bs[kk][r] = (gn < a.N && gk < a.K) ? B[(int64_t)gn * ldb + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        av[i] = As[kk][ty * 4 + i];
        bv[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
  float* C = reinterpret_cast<float*>(a.C);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= a.M) continue;
    if (EPI == HX_EPI_SWIGLU) {
      // Columns n0 + tx*4 .. +3 lie in one 32-column block: up part (<16) pairs with +16.
      // Handled by the dedicated swiglu pass below; store raw here.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n < a.N) a.ws[(int64_t)m * a.N + n] = acc[i][j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n >= a.N) continue;
        float x = acc[i][j];
        if (EPI == HX_EPI_RESIDUAL) x += reinterpret_cast<const float*>(a.R)[(int64_t)m * a.ldr + n];
        C[(int64_t)m * a.ldc + n] = x;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Host side: tensor maps, tile selection, launch.
// ---------------------------------------------------------------------------------------
// 2D K-major tensor map over a [rows, cols] matrix with leading dimension ld (elements),
// box [box_rows, 64], SWIZZLE_128B, zero fill out of bounds.
int make_map(CUtensorMap* out, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
             int box_rows, int dtype) {
  const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)rows};
  const uint64_t strides[1] = {(uint64_t)(ld * 2)};
  const uint32_t box[2] = {(uint32_t)BK, (uint32_t)box_rows};
  return make_tensor_map(out, ptr, 2, dims, strides, box, dtype);
}

int device_sms() { return device_sm_count(); }

struct Plan {
  int bn, m_tiles, n_tiles, k_splits, kb_per_split, k_blocks;
  bool swap;        // decode-shaped: operands swapped, stream-K
  int ctas, segs;   // stream-K CTAs and max tile segments per CTA
};

// Tile / split selection.
//  * Decode-shaped (M <= 64): operands swapped (128 weight rows per tile, N = batch rounded up
//    to 16/32/64) and stream-K over ~2 CTAs per SM.
//  * Otherwise: the widest tile that still fills the machine; split K if there are too few
//    tiles for the SMs.
Plan plan_gemm(int64_t M, int64_t N, int64_t K) {
  const int sms = device_sms();
  Plan p;
  p.k_blocks = ceil_div(K, BK);
  p.swap = M <= 64;
  p.ctas = p.segs = 0;
  int splits = 1;
  if (p.swap) {
    p.bn = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    p.m_tiles = ceil_div(N, BM);
    p.n_tiles = 1;
    const int64_t units = (int64_t)p.m_tiles * p.k_blocks;
    p.ctas = (int)std::min<int64_t>(units, 2 * (int64_t)sms);
    if ((units + 1) * (int64_t)p.ctas > INT32_MAX) p.swap = false;  // reduce uses 32-bit math
    int segs = 1;
    for (int c = 0; c < p.ctas; ++c) {
      const int64_t u0 = (int64_t)c * units / p.ctas, u1 = (int64_t)(c + 1) * units / p.ctas;
      segs = std::max(segs, (int)((u1 - 1) / p.k_blocks - u0 / p.k_blocks + 1));
    }
    p.segs = segs;
  } else {
    p.m_tiles = ceil_div(M, BM);
    const int64_t t256 = (int64_t)p.m_tiles * ceil_div(N, 256);
    const int64_t t128 = (int64_t)p.m_tiles * ceil_div(N, 128);
    if (t256 >= sms) p.bn = 256;
    else if (t128 >= sms) p.bn = 128;
    else p.bn = 64;
    p.n_tiles = ceil_div(N, p.bn);
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    if (tiles < sms && p.k_blocks >= 8) {
      splits = (int)std::min<int64_t>(ceil_div(sms, tiles), p.k_blocks / 4);
      splits = std::max(splits, 1);
    }
  }
  p.kb_per_split = ceil_div(p.k_blocks, splits);
  p.k_splits = ceil_div(p.k_blocks, p.kb_per_split);
  return p;
}

size_t plan_workspace(const Plan& p, int64_t M, int64_t N) {
  if (p.swap) return kFlagBytes + (size_t)p.ctas * p.segs * M * BM * sizeof(float);
  return p.k_splits > 1 ? kFlagBytes + (size_t)p.k_splits * M * N * sizeof(float) : 0;
}

template <typename T, int BN, int EPI>
int launch_streamk(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& a,
                   cudaStream_t stream) {
  using C = Cfg<BN, true>;
  auto kern = gemm_streamk_kernel<T, BN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)C::kSmemBytes),
                            "cudaFuncSetAttribute(gemm_streamk)");
    if (s) return s;
    attr_set[dev & 63] = true;
  }
  kern<<<a.ctas, kGemmThreads, C::kSmemBytes, stream>>>(mw, mx, a);
  HX_LAUNCH_CHECK("gemm_streamk_kernel");
  return HX_OK;
}

template <typename T, int BN, int EPI>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a,
              cudaStream_t stream) {
  using C = Cfg<BN>;
  auto kern = gemm_tcgen05_kernel<T, BN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)C::kSmemBytes),
                            "cudaFuncSetAttribute(gemm)");
    if (s) return s;
    attr_set[dev & 63] = true;
  }
  const int total = a.m_tiles * a.n_tiles * a.k_splits;
  const int grid = std::min(total, device_sms());
  kern<<<grid, kGemmThreads, C::kSmemBytes, stream>>>(ma, mb, a);
  HX_LAUNCH_CHECK("gemm_tcgen05_kernel");
  return HX_OK;
}

template <typename T, int EPI>
int gemm_half(const void* A, const void* B, void* Cp, int64_t M, int64_t N, int64_t K,
              int64_t lda, int64_t ldb, int64_t ldc, const void* R, int64_t ldr, void* ws,
              size_t ws_bytes, int dtype, cudaStream_t stream, const QkvArgs* qkv = nullptr) {
  const Plan p = plan_gemm(M, N, K);
  GemmArgs a;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.m_tiles = p.m_tiles;
  a.n_tiles = p.n_tiles;
  a.k_splits = p.k_splits;
  a.kb_per_split = p.kb_per_split;
  a.k_blocks = p.k_blocks;
  a.C = Cp;
  a.ldc = ldc;
  a.R = R;
  a.ldr = ldr;
  a.ws = nullptr;
  a.flags = nullptr;
  a.ctas = p.ctas;
  a.segs = p.segs;
  if (qkv) a.qkv = *qkv;
  const size_t need = plan_workspace(p, M, N);
  if (need) {
    HX_REQUIRE(ws && ws_bytes >= need, "hx_gemm: workspace too small (%zu < %zu)", ws_bytes, need);
    HX_REQUIRE((uintptr_t)ws % 16 == 0, "hx_gemm: workspace must be 16-byte aligned");
    a.flags = (uint32_t*)ws;
    a.ws = (float*)((uint8_t*)ws + kFlagBytes);
    HX_REQUIRE(!p.swap || p.m_tiles <= (int)(kFlagBytes / sizeof(uint32_t)),
               "hx_gemm: n too large for the tile counters");
  }
  CUtensorMap ma, mb;
  int s;
  if (p.swap) {
    // MMA A = weights (128-row boxes), MMA B = activations (bn-row box).
    s = make_map(&ma, B, N, K, ldb, BM, dtype);
    if (s) return s;
    s = make_map(&mb, A, M, K, lda, p.bn, dtype);
    if (s) return s;
    switch (p.bn) {
      case 16: return launch_streamk<T, 16, EPI>(ma, mb, a, stream);
      case 32: return launch_streamk<T, 32, EPI>(ma, mb, a, stream);
      default: return launch_streamk<T, 64, EPI>(ma, mb, a, stream);
    }
  } else {
    s = make_map(&ma, A, M, K, lda, BM, dtype);
    if (s) return s;
    s = make_map(&mb, B, N, K, ldb, p.bn, dtype);
    if (s) return s;
    switch (p.bn) {
      case 256: s = launch_tc<T, 256, EPI>(ma, mb, a, stream); break;
      case 128: s = launch_tc<T, 128, EPI>(ma, mb, a, stream); break;
      default: s = launch_tc<T, 64, EPI>(ma, mb, a, stream); break;
    }
  }
  if (s) return s;
  if (p.k_splits > 1) {
    const int64_t outs = M * ((EPI == HX_EPI_SWIGLU || EPI == HX_EPI_QKV_ROTARY) ? N / 2 : N);
    splitk_reduce_kernel<T, EPI><<<ceil_div(outs, 256), 256, 0, stream>>>(a);
    HX_LAUNCH_CHECK("splitk_reduce_kernel");
  }
  return HX_OK;
}

__global__ void swiglu_f32_kernel(const float* __restrict__ raw, int M, int N, float* __restrict__ C,
                                  int64_t ldc) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t outs = (int64_t)M * (N / 2);
  if (idx >= outs) return;
  const int m = (int)(idx / (N / 2)), j = (int)(idx % (N / 2));
  const int n_up = (j / 16) * 32 + (j % 16);
  const float u = raw[(int64_t)m * N + n_up], g = raw[(int64_t)m * N + n_up + 16];
  C[(int64_t)m * ldc + j] = u * silu_f(g);
}

int gemm_f32(const void* A, const void* B, void* Cp, int64_t M, int64_t N, int64_t K,
             int64_t lda, int64_t ldb, int64_t ldc, int epi, const void* R, int64_t ldr,
             void* ws, size_t ws_bytes, cudaStream_t stream) {
  GemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.C = Cp;
  a.ldc = ldc;
  a.R = R;
  a.ldr = ldr;
  dim3 grid(ceil_div(N, 64), ceil_div(M, 64));
  if (epi == HX_EPI_SWIGLU) {
    const size_t need = (size_t)M * N * sizeof(float);
    HX_REQUIRE(ws && ws_bytes >= need, "hx_gemm(f32 swiglu): workspace too small");
    a.ws = (float*)ws;
    gemm_f32_kernel<HX_EPI_SWIGLU><<<grid, 256, 0, stream>>>((const float*)A, (const float*)B, a, lda, ldb);
    HX_LAUNCH_CHECK("gemm_f32_kernel");
    swiglu_f32_kernel<<<ceil_div(M * (N / 2), 256), 256, 0, stream>>>(a.ws, (int)M, (int)N,
                                                                     (float*)Cp, ldc);
    HX_LAUNCH_CHECK("swiglu_f32_kernel");
  } else if (epi == HX_EPI_RESIDUAL) {
    gemm_f32_kernel<HX_EPI_RESIDUAL><<<grid, 256, 0, stream>>>((const float*)A, (const float*)B, a, lda, ldb);
    HX_LAUNCH_CHECK("gemm_f32_kernel");
  } else {
    gemm_f32_kernel<HX_EPI_NONE><<<grid, 256, 0, stream>>>((const float*)A, (const float*)B, a, lda, ldb);
    HX_LAUNCH_CHECK("gemm_f32_kernel");
  }
  return HX_OK;
}

}  // namespace

extern "C" {

size_t hx_gemm_workspace(int64_t m, int64_t n, int64_t k, int epilogue, int dtype) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  if (dtype == HX_F32) return epilogue == HX_EPI_SWIGLU ? (size_t)m * n * sizeof(float) : 0;
  return plan_workspace(plan_gemm(m, n, k), m, n);
}

int hx_gemm_qkv_rotary(const void* x, const void* w_qkv, int64_t m, int64_t k, int64_t ldx,
                       int64_t seqlen, int64_t n_heads, int64_t n_heads_kv, int64_t head_dim,
                       const int32_t* pos_start, const void* cos_table, const void* sin_table,
                       int64_t table_rows, void* q_out, void* cache, int64_t cache_batch_stride,
                       int64_t cache_seq_stride, int64_t cache_batch_offset,
                       int64_t cache_max_seq, void* workspace, size_t workspace_bytes, int dtype,
                       void* stream) {
  HX_REQUIRE(x && w_qkv && pos_start && cos_table && sin_table && q_out && cache,
             "hx_gemm_qkv_rotary: null pointer");
  HX_REQUIRE(dtype == HX_BF16 || dtype == HX_F16, "hx_gemm_qkv_rotary: f16/bf16 only");
  HX_REQUIRE(head_dim % 2 == 0 && n_heads > 0 && n_heads_kv > 0 && seqlen > 0 && m % seqlen == 0,
             "hx_gemm_qkv_rotary: bad shape");
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim && cache_seq_stride % 8 == 0 &&
                 cache_batch_stride % 8 == 0 && (uintptr_t)cache % 16 == 0 &&
                 (uintptr_t)q_out % 16 == 0 && (uintptr_t)cos_table % 16 == 0 &&
                 (uintptr_t)sin_table % 16 == 0,
             "hx_gemm_qkv_rotary: cache/q_out/tables must be 16-byte aligned (strides multiples of 8)");
  HX_REQUIRE((uintptr_t)x % 16 == 0 && (uintptr_t)w_qkv % 16 == 0 && ldx % 8 == 0 && k % 8 == 0,
             "hx_gemm_qkv_rotary: x/w must be 16-byte aligned with ldx, k multiples of 8");
  const int64_t n = (n_heads + 2 * n_heads_kv) * head_dim;
  if (m == 0) return HX_OK;
  QkvArgs q;
  q.q_out = q_out;
  q.cache = cache;
  q.cbs = cache_batch_stride;
  q.css = cache_seq_stride;
  q.cbo = cache_batch_offset;
  q.max_seq = cache_max_seq;
  q.table_rows = table_rows;
  q.pos_start = pos_start;
  q.cos = cos_table;
  q.sin = sin_table;
  q.n_heads = (int)n_heads;
  q.n_heads_kv = (int)n_heads_kv;
  q.head_dim = (int)head_dim;
  q.seqlen = (int)seqlen;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == HX_BF16)
    return gemm_half<__nv_bfloat16, HX_EPI_QKV_ROTARY>(x, w_qkv, nullptr, m, n, k, ldx, k, 0,
                                                       nullptr, 0, workspace, workspace_bytes,
                                                       dtype, s, &q);
  return gemm_half<__half, HX_EPI_QKV_ROTARY>(x, w_qkv, nullptr, m, n, k, ldx, k, 0, nullptr, 0,
                                              workspace, workspace_bytes, dtype, s, &q);
}

int hx_gemm(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
            int64_t lda, int64_t ldb, int64_t ldc, int epilogue, const void* residual,
            int64_t ld_residual, void* workspace, size_t workspace_bytes, int dtype,
            void* stream) {
  HX_REQUIRE(epilogue != HX_EPI_QKV_ROTARY, "hx_gemm: use hx_gemm_qkv_rotary for that epilogue");
  HX_REQUIRE(a && b && c && m >= 0 && n >= 0 && k > 0, "hx_gemm: bad arguments");
  HX_REQUIRE(lda >= k && ldb >= k, "hx_gemm: lda/ldb smaller than k");
  HX_REQUIRE(epilogue >= HX_EPI_NONE && epilogue <= HX_EPI_SWIGLU, "hx_gemm: bad epilogue");
  HX_REQUIRE(epilogue != HX_EPI_RESIDUAL || residual, "hx_gemm: residual epilogue needs residual");
  HX_REQUIRE(epilogue != HX_EPI_SWIGLU || n % 32 == 0,
             "hx_gemm: SwiGLU needs n divisible by 32 (interleaved [up16|gate16] rows)");
  HX_REQUIRE(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "hx_gemm: size too large");
  if (m == 0 || n == 0) return HX_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == HX_F32)
    return gemm_f32(a, b, c, m, n, k, lda, ldb, ldc, epilogue, residual, ld_residual, workspace,
                    workspace_bytes, s);
  HX_REQUIRE(dtype == HX_BF16 || dtype == HX_F16, "hx_gemm: unsupported dtype %d", dtype);
  HX_REQUIRE((uintptr_t)a % 16 == 0 && (uintptr_t)b % 16 == 0 && lda % 8 == 0 && ldb % 8 == 0,
             "hx_gemm: A/B must be 16-byte aligned with lda/ldb multiples of 8");
#define HX_GEMM_EPI(T)                                                                        \
  switch (epilogue) {                                                                         \
    case HX_EPI_NONE:                                                                         \
      return gemm_half<T, HX_EPI_NONE>(a, b, c, m, n, k, lda, ldb, ldc, residual, ld_residual, \
                                       workspace, workspace_bytes, dtype, s);                 \
    case HX_EPI_RESIDUAL:                                                                     \
      return gemm_half<T, HX_EPI_RESIDUAL>(a, b, c, m, n, k, lda, ldb, ldc, residual,         \
                                           ld_residual, workspace, workspace_bytes, dtype, s); \
    default:                                                                                  \
      return gemm_half<T, HX_EPI_SWIGLU>(a, b, c, m, n, k, lda, ldb, ldc, residual,           \
                                         ld_residual, workspace, workspace_bytes, dtype, s);  \
  }
  if (dtype == HX_BF16) {
    HX_GEMM_EPI(__nv_bfloat16)
  } else {
    HX_GEMM_EPI(__half)
  }
#undef HX_GEMM_EPI
  return HX_OK;
}

}  // extern "C"
