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
// Problems with M > 64 and too few tiles split K across CTAs; partial sums go to a
// caller-provided f32 workspace and a small kernel reduces them in split order.
// Decode-shaped problems (M <= 64) use gemm_decode_kernel: operands swapped and K split across
// the CTAs of a thread-block cluster, reduced through distributed shared memory (no workspace).
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

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
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
  // Packed prompts (seq_offsets != nullptr): prompt b owns rows [seq_offsets[b],
  // seq_offsets[b+1]) and cache row slots[b] (< cache_rows); seqlen and cbo are unused.
  const int32_t* seq_offsets;
  const int32_t* slots;
  int n_prompts;
  int64_t cache_rows;
};

// Prompt of output row m: m / seqlen for equal-length prompts, else the last b with
// seq_offsets[b] <= m (binary search; rows past the table's end fall into the last prompt and
// fail the position bound check).
HX_DEVICE int qkv_prompt(const QkvArgs& q, int m) {
  if (!q.seq_offsets) return m / q.seqlen;
  int lo = 0, hi = q.n_prompts - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (q.seq_offsets[mid] <= m) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}
// Cache position of row m of prompt b.
HX_DEVICE int64_t qkv_pos(const QkvArgs& q, int b, int m) {
  const int first = q.seq_offsets ? q.seq_offsets[b] : b * q.seqlen;
  return (int64_t)q.pos_start[b] + (m - first);
}
// Cache batch row of prompt b, or -1 when it lies outside the cache.
HX_DEVICE int64_t qkv_cache_row(const QkvArgs& q, int b) {
  const int64_t r = q.seq_offsets ? (int64_t)q.slots[b] : q.cbo + b;
  return r >= 0 && r < q.cache_rows ? r : -1;
}

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, k_splits, kb_per_split, k_blocks;
  void* C;
  int64_t ldc;
  const void* R;
  int64_t ldr;
  float* ws;        // split-K partials [k_splits][M][N] (M > 64 only)
  QkvArgs qkv;
};

HX_DEVICE float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Fused Wqkv epilogue for the feature pair (n, n+1), n even, of row m = row s of prompt b: the
// values are rounded like the reference's Linear output; q and k pairs are rotated (f32 math
// on the dtype-cached cos/sin, as flash_attn's rotary) and q goes to q_out, k and v to the cache
// row of position pos_start[b] + s (the packed [k; v] part of a row is exactly the cache's
// [2, hkv, d] row layout).
template <typename T>
HX_DEVICE void qkv_store_pair(const GemmArgs& a, int m, int n, float v0, float v1) {
  if (m >= a.M || n >= a.N) return;
  const QkvArgs& q = a.qkv;
  const int b = qkv_prompt(q, m);
  const int64_t pos = qkv_pos(q, b, m), row = qkv_cache_row(q, b);
  if (pos < 0 || pos >= q.max_seq || pos >= q.table_rows || row < 0) {
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
                   : reinterpret_cast<T*>(q.cache) + row * q.cbs + pos * q.css + (n - hqd);
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
    const int b = qkv_prompt(q, m);
    const int64_t pos = qkv_pos(q, b, m), row = qkv_cache_row(q, b);
    if (pos < 0 || pos >= q.max_seq || pos >= q.table_rows || row < 0) {
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
                      : reinterpret_cast<T*>(q.cache) + row * q.cbs + pos * q.css + (n0 - hqd);
#pragma unroll
    for (int j = 0; j < 32; j += 8)
      *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(out + j);
    return;
  }
  if (EPI == HX_EPI_SWIGLU) {
    // 16 up columns then 16 gate columns -> 16 outputs at column n0/2.
    T* out = reinterpret_cast<T*>(a.C) + (int64_t)m * a.ldc + n0 / 2;
    if (n0 >= a.N) return;
    alignas(16) T res16[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float u = round_to<T>(v[j]);
      const float g = round_to<T>(v[16 + j]);
      res16[j] = DT<T>::from_f(u * round_to<T>(silu_f(g)));
    }
    if (sizeof(T) == 2 && (uintptr_t)out % 16 == 0) {
      // 16 outputs = 32 bytes: two 16-byte stores instead of sixteen 2-byte ones.
      *reinterpret_cast<uint4*>(out) = *reinterpret_cast<const uint4*>(res16);
      *reinterpret_cast<uint4*>(out + 8) = *reinterpret_cast<const uint4*>(res16 + 8);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] = res16[j];
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
      if (!mbar_wait_drain(&full[i % C::kStages], (i / C::kStages) & 1)) break;
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

// ------------------------------------------------------------------------------------------
// Decode-shaped GEMM (M = batch <= 64): operands swapped, split-K inside a thread-block cluster.
//   MMA A = 128 weight rows (output features) per tile, K-major; MMA B = the batch rows
//   (N = 16/32/64, rows past M zero-filled by TMA), so no tensor-core work or shared-memory
//   bandwidth goes to padding rows. The K range of a tile is split across the S CTAs of one
//   cluster (S <= 8, chosen so that tiles x S fill ~2 CTAs per SM). Each CTA streams its slice
//   of the weight tile through a TMA ring into one TMEM accumulator, writes the f32 partial
//   [BN][128] into its own (now idle) ring, and after a cluster barrier CTA s sums batch rows
//   b = s, s + S, ... of all S partials through distributed shared memory, in rank order
//   (deterministic), and applies the epilogue. No global scratch, atomics or fences.
// ------------------------------------------------------------------------------------------
constexpr int kDecMaxStages = 16;

HX_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HX_DEVICE uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
HX_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// Address of the same shared variable in CTA `rank` of this cluster.
HX_DEVICE uint32_t dsmem_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
HX_DEVICE float dsmem_ld_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// Epilogue inputs of eight output rows (batch rows b[0..nr), feature n of this lane): the
// residual (RESIDUAL) or the rotary cos/sin at each row's position (QKV_ROTARY), read from
// global memory. Split from the store so the loads can be issued while the MMAs still run.
// pos_s[m] = position of batch row m (fused Wqkv epilogue only), in shared memory.
template <typename T, int EPI>
struct Epi8 {
  float x[8], y[8];
  int64_t pos[8];
};

template <typename T, int EPI>
HX_DEVICE void sk_load8(const GemmArgs& a, const int (&b)[8], int nr, int n, int lane,
                        const int* pos_s, Epi8<T, EPI>& e) {
  if (EPI == HX_EPI_QKV_ROTARY) {
    const QkvArgs& q = a.qkv;
    const bool rot = n < (q.n_heads + q.n_heads_kv) * q.head_dim;
    const int pair = (n % q.head_dim) >> 1;
    const T* cos_t = reinterpret_cast<const T*>(q.cos);
    const T* sin_t = reinterpret_cast<const T*>(q.sin);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      e.pos[i] = -1;
      e.x[i] = 1.f;
      e.y[i] = 0.f;
      if (i < nr && b[i] < a.M && !(lane & 1) && n < a.N) {
        e.pos[i] = pos_s[b[i]];
        if (rot && e.pos[i] >= 0 && e.pos[i] < q.table_rows) {
          e.x[i] = DT<T>::to_f(__ldg(cos_t + e.pos[i] * (q.head_dim / 2) + pair));
          e.y[i] = DT<T>::to_f(__ldg(sin_t + e.pos[i] * (q.head_dim / 2) + pair));
        }
      }
    }
  } else if (EPI == HX_EPI_RESIDUAL) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      e.x[i] = 0.f;
      if (i < nr && b[i] < a.M && n < a.N)
        e.x[i] = DT<T>::to_f(reinterpret_cast<const T*>(a.R)[(int64_t)b[i] * a.ldr + n]);
    }
  }
}

// Stores eight output rows (warp-uniform rows, one feature n per lane) from their f32
// accumulators and the inputs sk_load8 fetched.
template <typename T, int EPI>
HX_DEVICE void sk_store8(const GemmArgs& a, const int (&b)[8], int nr, int n, int lane,
                         const float (&v)[8], const Epi8<T, EPI>& e) {
  if (EPI == HX_EPI_SWIGLU) {
    float gate[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) gate[i] = __shfl_xor_sync(0xffffffffu, v[i], 16);
    if (lane < 16 && n < a.N) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < nr && b[i] < a.M) {
          const float u = round_to<T>(v[i]), g = round_to<T>(gate[i]);
          reinterpret_cast<T*>(a.C)[(int64_t)b[i] * a.ldc + (n >> 5) * 16 + lane] =
              DT<T>::from_f(u * round_to<T>(silu_f(g)));
        }
      }
    }
  } else if (EPI == HX_EPI_QKV_ROTARY) {
    float other[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) other[i] = __shfl_xor_sync(0xffffffffu, v[i], 1);
    if ((lane & 1) || n >= a.N) return;
    const QkvArgs& q = a.qkv;
    const int hqd = q.n_heads * q.head_dim;
    const bool rot = n < hqd + q.n_heads_kv * q.head_dim;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!(i < nr && b[i] < a.M)) continue;
      const int m = b[i];
      const int64_t pos = e.pos[i], row = qkv_cache_row(q, qkv_prompt(q, m));
      if (pos < 0 || pos >= q.max_seq || pos >= q.table_rows || row < 0) {
        record_device_error(HX_DEVERR_BAD_ARGUMENT);
        continue;
      }
      float x0 = round_to<T>(v[i]), x1 = round_to<T>(other[i]);
      if (rot) {
        const float c = e.x[i], sn = e.y[i];
        const float o0 = x0 * c - x1 * sn;
        const float o1 = x0 * sn + x1 * c;
        x0 = o0;
        x1 = o1;
      }
      T* dst = n < hqd ? reinterpret_cast<T*>(q.q_out) + (int64_t)m * hqd + n
                       : reinterpret_cast<T*>(q.cache) + row * q.cbs + pos * q.css + (n - hqd);
      T pr2[2] = {DT<T>::from_f(x0), DT<T>::from_f(x1)};
      *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(pr2);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < nr && b[i] < a.M && n < a.N) {
        float x = round_to<T>(v[i]);
        if (EPI == HX_EPI_RESIDUAL) x += e.x[i];
        reinterpret_cast<T*>(a.C)[(int64_t)b[i] * a.ldc + n] = DT<T>::from_f(x);
      }
    }
  }
}

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmX, const GemmArgs a, int stages) {
  constexpr int kWBytes = BM * BK * 2;
  constexpr int kXBytes = BN * BK * 2;
  constexpr int kStageBytes = kWBytes + kXBytes;
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + stages * kStageBytes);
  uint64_t* empty = full + kDecMaxStages;
  uint64_t* tfull = empty + kDecMaxStages;
  uint32_t* counters = reinterpret_cast<uint32_t*>(tfull + 1);  // [0] loads issued, [1] consumed
  uint32_t* tmem_slot = counters + 2;
  int* pos_s = reinterpret_cast<int*>(counters + 4);             // [BN] row positions (Wqkv)
  float* part = reinterpret_cast<float*>(ring);                  // [BN][BM] f32 after the loop

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.k_splits;
  const int split = S > 1 ? (int)cluster_ctarank() : 0;
  const int tile = S > 1 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(a.k_blocks, kb0 + a.kb_per_split);

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    counters[0] = counters[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (!(warp == 0 && lane == 0)) pdl_wait();  // the producer waits after its weight prefetch
  pdl_trigger();
  Epi8<T, EPI> pre;  // epilogue warps: inputs of the first eight rows they store

  if (warp == 0) {
    if (lane == 0) {
      // The weights are not produced by earlier kernels: the first ring's worth of weight
      // tiles is requested before waiting for the previous kernel (PDL), so the stream of
      // weight bytes starts while that kernel drains. Activation tiles follow the wait.
      const int npre = min(stages, kb1 - kb0);
      for (int i = 0; i < npre; ++i) {
        mbar_arrive_expect_tx(&full[i], kStageBytes);
        tma_load_2d(ring + i * kStageBytes, &tmW, &full[i], (kb0 + i) * BK, tile * BM);
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i)
        tma_load_2d(ring + i * kStageBytes + kWBytes, &tmX, &full[i], (kb0 + i) * BK, 0);
      int stage = npre == stages ? 0 : npre;
      uint32_t phase = npre == stages ? 1 : 0, issued = npre;
      for (int kb = kb0 + npre; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1)) break;
        mbar_arrive_expect_tx(&full[stage], kStageBytes);
        uint8_t* st = ring + stage * kStageBytes;
        tma_load_2d(st, &tmW, &full[stage], kb * BK, tile * BM);
        tma_load_2d(st + kWBytes, &tmX, &full[stage], kb * BK, 0);
        ++issued;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      counters[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<T>(BM, BN);
      int stage = 0;
      uint32_t phase = 0, consumed = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase)) break;
        ++consumed;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(ring + stage * kStageBytes);
        const uint32_t b_addr = a_addr + kWBytes;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          tc_mma_f16(tmem_base, sw128_kmajor_desc(a_addr + k * 32),
                     sw128_kmajor_desc(b_addr + k * 32), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == stages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // Completes once every MMA above has finished (also with none issued). After a timed-out
      // wait the accumulator is incomplete; the device error word already says so.
      tc_commit(tfull);
      counters[1] = consumed;
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4 = tile rows 32q..32q+31.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    if (EPI == HX_EPI_QKV_ROTARY) {
      // Row positions, loaded while the main loop runs.
      const QkvArgs& q = a.qkv;
      for (int m = threadIdx.x - 64; m < min(BN, a.M); m += 128)
        pos_s[m] = (int)qkv_pos(q, qkv_prompt(q, m), m);
      named_bar_sync(2, 128);
    }
    // The first eight rows this CTA stores: their epilogue inputs are fetched while the MMAs
    // still run.
    int rows0[8];
    const int rows_all = min(BN, a.M);
    const int nr0 = S == 1 ? min(8, rows_all) : min(8, max(0, (rows_all - split + S - 1) / S));
#pragma unroll
    for (int i = 0; i < 8; ++i) rows0[i] = S == 1 ? i : split + i * S;
    sk_load8<T, EPI>(a, rows0, nr0, tile * BM + r, lane, pos_s, pre);
    const bool ready = mbar_wait_warp(tfull, 0);
    tc_fence_after();
    const bool valid = ready && kb1 > kb0;
    const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16);
    if (S == 1) {
      if (valid) {
#pragma unroll
        for (int c = 0; c < BN / 16; ++c) {
          uint32_t v[16];
          tmem_ld_32x32b_x16(taddr + c * 16, v);
          tc_wait_ld();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            int rows[8];
            float vals[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              rows[j] = c * 16 + h * 8 + j;
              vals[j] = __uint_as_float(v[h * 8 + j]);
            }
            if (c == 0 && h == 0) {
              sk_store8<T, EPI>(a, rows, 8, tile * BM + r, lane, vals, pre);
            } else {
              Epi8<T, EPI> e;
              sk_load8<T, EPI>(a, rows, 8, tile * BM + r, lane, pos_s, e);
              sk_store8<T, EPI>(a, rows, 8, tile * BM + r, lane, vals, e);
            }
          }
        }
      }
    } else {
      // The ring is idle once every MMA has completed (all issued loads were consumed).
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        uint32_t v[16];
        if (valid) {
          tmem_ld_32x32b_x16(taddr + c * 16, v);
          tc_wait_ld();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) part[(c * 16 + j) * BM + r] = valid ? __uint_as_float(v[j]) : 0.f;
      }
    }
  }

  if (S > 1) {
    __syncwarp();
    cluster_sync_all();  // every partial of the cluster is in shared memory
    if (warp >= 2) {
      // CTA `split` owns batch rows split, split + S, ...; eight at a time, all S x 8 partial
      // loads in flight together, summed in rank order.
      const int r = (warp & 3) * 32 + lane;
      const int rows = min(BN, a.M);
      const uint32_t my = smem_u32(part + r);
      for (int b0 = split; b0 < rows; b0 += 8 * S) {
        int bs[8];
        float sums[8];
        const int nr = min(8, (rows - b0 + S - 1) / S);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          bs[i] = b0 + i * S;
          float v[8];
#pragma unroll
          for (int c = 0; c < 8; ++c)
            v[c] = (c < S && i < nr) ? dsmem_ld_f32(dsmem_map(my + (uint32_t)(bs[i] * BM * 4), (uint32_t)c)) : 0.f;
          float sum = 0.f;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c < S) sum += v[c];
          sums[i] = sum;
        }
        if (b0 == split) {
          sk_store8<T, EPI>(a, bs, nr, tile * BM + r, lane, sums, pre);
        } else {
          Epi8<T, EPI> e;
          sk_load8<T, EPI>(a, bs, nr, tile * BM + r, lane, pos_s, e);
          sk_store8<T, EPI>(a, bs, nr, tile * BM + r, lane, sums, e);
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // no CTA leaves while another still reads its partial
  }

  tc_fence_before();
  __syncthreads();
  // After an aborted wait, loads may have been issued that nobody consumed: let them land
  // (bounded) before the CTA's shared memory goes away.
  if (threadIdx.x == 0) {
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait_drain(&full[i % stages], (i / stages) & 1)) break;
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
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

// ------------------------------------------------------------------------------------------
// Prefill GEMM on CTA pairs (tcgen05 cta_group::2): one 256 x 256 output tile per pair of SMs.
//   The pair's MMA computes D[256 x 256] += A[256 x 16] B[256 x 16]^T per instruction; each CTA
//   holds its own 128 rows of A and its own 128 rows (output columns) of B in shared memory and
//   receives its 128 rows x 256 columns of D in its own TMEM. Per SM and k-block that is 32 KB
//   written by TMA and read by the tensor core for 4.2 MFLOP, half the shared-memory traffic of
//   a single-SM 128 x 256 tile, which is what bounds the single-SM kernel.
//   Roles per CTA: warp 0 TMA producer (both CTAs), warp 1 MMA issuer (even CTA only) and TMEM
//   owner, warps 2-5 epilogue (both CTAs).
//   Signals: the even CTA arms its stage barrier with both CTAs' bytes and both CTAs' TMA loads
//   complete on it; the MMA commits to the even CTA's barriers, whose observers relay them to
//   the odd CTA with a remote mbarrier arrive (stage free: the even producer; accumulator full:
//   an even epilogue thread); both epilogues release an accumulator on the even CTA's barrier.
//   Persistent over (row pair, column tile) work items; two TMEM accumulators so the epilogue
//   of one item overlaps the main loop of the next.
// ------------------------------------------------------------------------------------------
constexpr int kPairStages = 7;
constexpr int kPairTileBytes = 128 * BK * 2;                 // 128 rows x 64 k of A or of B
constexpr int kPairStageBytes = 2 * kPairTileBytes;
constexpr size_t kPairSmem = (size_t)kPairStages * kPairStageBytes + 1024 + 512;

HX_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HX_DEVICE void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
HX_DEVICE void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
HX_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D(tmem, both CTAs) (+)= A * B^T over the pair; issued by the even CTA with its own smem
// descriptors (the odd CTA's operands sit at the same offsets). No output lanes are disabled.
HX_DEVICE void tc_mma_pair(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                           uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
      ::"r"(tmem_d), "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}
// Arrive on a barrier of this CTA once all earlier pair MMAs issued by this thread complete.
HX_DEVICE void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// Tiled 2D TMA load into this CTA's shared memory whose completion is counted on an mbarrier
// that may live in the peer CTA of the pair (cluster address).
HX_DEVICE void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster,
                                int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
// Arrive on an mbarrier given by cluster address (this CTA's or the peer's), with the default
// CTA-scope release: the signals relayed with it carry no data of the arriving thread (what they
// order is the MMA's completion, established by tcgen05.commit and the tcgen05 fences), and a
// cluster-scope release would stall the thread until its earlier global stores are acknowledged.
HX_DEVICE void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

template <typename T, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
  constexpr int BNP = 256;  // output columns per pair tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + kPairStages * kPairTileBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty = full + kPairStages;
  uint64_t* tfull = empty + kPairStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* counters = reinterpret_cast<uint32_t*>(drain + 1);  // [0] loads issued, [1] consumed
  uint32_t* tmem_slot = counters + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0 = even CTA (issues the MMAs), 1 = odd
  const bool even = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int pm_tiles = (a.M + 2 * BM - 1) / (2 * BM);
  const int total = pm_tiles * a.n_tiles;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    counters[0] = counters[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BNP);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote arrive or load
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // A (activations) and the epilogue inputs come from earlier kernels

  // Cluster addresses of the even CTA's barriers / the odd CTA's relay targets.
  const uint32_t full_even = dsmem_map(smem_u32(full), 0);
  const uint32_t tempty_even = dsmem_map(smem_u32(tempty), 0);

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t empty_odd = dsmem_map(smem_u32(empty), 1);
      int stage = 0;
      uint32_t phase = 0, issued = 0;
      for (int t = pair; t < total; t += n_pairs) {
        const int pm = t % pm_tiles, nb = t / pm_tiles;
        const int row_a = pm * 2 * BM + (int)rank * BM;
        const int row_b = nb * BNP + (int)rank * BM;
        for (int kb = 0; kb < a.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) goto producer_done;
          // The even CTA saw the MMAs release this stage: pass it on to the odd CTA (from the
          // second round on; the first round of every stage starts free in both CTAs).
          if (even && issued >= (uint32_t)kPairStages) mbar_arrive_remote(empty_odd + stage * 8);
          if (even) mbar_arrive_expect_tx(&full[stage], kPairStageBytes * 2);
          tma_load_2d_pair(smA + stage * kPairTileBytes, &tmA, full_even + stage * 8, kb * BK, row_a);
          tma_load_2d_pair(smB + stage * kPairTileBytes, &tmB, full_even + stage * 8, kb * BK, row_b);
          ++issued;
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:
      counters[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0 && even) {
      constexpr uint32_t idesc = make_idesc_f16<T>(2 * BM, BNP);
      int stage = 0;
      uint32_t phase = 0, consumed = 0;
      int local = 0;
      for (int t = pair; t < total; t += n_pairs, ++local) {
        const int acc = local & 1;
        if (!mbar_wait(&tempty[acc], ((local >> 1) & 1) ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BNP;
        for (int kb = 0; kb < a.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase)) goto mma_done;
          ++consumed;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * kPairTileBytes);
          const uint32_t b_addr = smem_u32(smB + stage * kPairTileBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            tc_mma_pair(d_tmem, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32),
                        idesc, (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit_pair(&empty[stage]);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        tc_commit_pair(&tfull[acc]);
      }
    mma_done:
      tc_commit_pair(drain);
      mbar_wait(drain, 0);
      counters[1] = consumed;
    }
  } else {
    // Epilogue warps 2..5 of both CTAs: TMEM lane quarter = warp % 4, this CTA's 128 rows.
    const int quarter = warp & 3;
    const uint32_t tfull_odd = dsmem_map(smem_u32(tfull), 1);
    int local = 0;
    for (int t = pair; t < total; t += n_pairs, ++local) {
      const int pm = t % pm_tiles, nb = t / pm_tiles;
      const int acc = local & 1;
      if (!mbar_wait_warp(&tfull[acc], (local >> 1) & 1)) break;
      // Relay "accumulator ready" to the odd CTA (its MMAs completed with the same commit).
      if (even && warp == 2 && lane == 0) mbar_arrive_remote(tfull_odd + acc * 8);
      tc_fence_after();
      const int m = pm * 2 * BM + (int)rank * BM + quarter * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < BNP / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BNP + c * 32, r);
        tc_wait_ld();
        const int n0 = nb * BNP + c * 32;
        if (n0 >= a.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        epilogue_store<T, EPI>(a, m, n0, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_even + acc * 8);
    }
  }

  tc_fence_before();
  __syncthreads();
  // After an aborted wait, let issued-but-unconsumed loads land (bounded) before shared
  // memory goes away; they all complete on the even CTA's barriers.
  if (threadIdx.x == 0 && even) {
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait_drain(&full[i % kPairStages], (i / kPairStages) & 1)) break;
  }
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal or read it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, 2 * BNP);
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
  bool swap;    // decode-shaped: operands swapped, split-K inside a cluster (chosen at launch)
  bool pair;    // 256 x 256 tiles on CTA pairs (gemm_pair_kernel)
};

// Work items of the CTA-pair kernel: (256-row block, 256-column block).
int64_t pair_items(int64_t M, int64_t N) { return (int64_t)ceil_div(M, 2 * BM) * ceil_div(N, 256); }

// Tile / split selection.
//  * Decode-shaped (M <= 64): operands swapped (128 weight rows per tile, N = batch rounded up
//    to 16/32/64); the K split across a cluster is chosen by launch_decode.
//  * Otherwise: the widest tile that still fills the machine; split K if there are too few
//    tiles for the SMs (partials reduced by a second kernel in split order).
Plan plan_gemm(int64_t M, int64_t N, int64_t K) {
  const int sms = device_sms();
  Plan p;
  p.k_blocks = ceil_div(K, BK);
  p.swap = M <= 64;
  // CTA pairs when there are rows for both halves and at least ~3/7 of the pairs get an item:
  // a pair moves half the shared-memory bytes per FLOP of a single-SM tile, so even a partly
  // filled wave of pairs beats two waves of shared-memory-bound single-SM tiles (measured at
  // 900 rows: 64 items on 74 pairs 34 us vs 2 x 148 single-SM 128 x 128 tiles). Below that
  // (M <= 256, or narrow N), single-SM tiles with a K split.
  p.pair = !p.swap && M > BM && N >= 256 && pair_items(M, N) * 7 >= (int64_t)(sms / 2) * 3;
  int splits = 1;
  if (p.pair) {
    p.bn = 256;
    p.m_tiles = ceil_div(M, BM);
    p.n_tiles = ceil_div(N, 256);
  } else if (p.swap) {
    p.bn = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
    p.m_tiles = ceil_div(N, BM);
    p.n_tiles = 1;
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
  p.k_splits = ceil_div(p.k_blocks, p.kb_per_split);  // every split non-empty
  return p;
}

size_t plan_workspace(const Plan& p, int64_t M, int64_t N) {
  if (p.swap || p.pair) return 0;
  return p.k_splits > 1 ? (size_t)p.k_splits * M * N * sizeof(float) : 0;
}

// Decode GEMM launch. The K split S (= cluster size) is the largest S <= 8 with
// tiles x S <= 1.6 x SMs and at least two k-blocks per split: enough CTAs to keep every SM
// streaming weights, few enough that the clusters are co-resident (measured on B200: 3-CTA
// clusters x 96 tiles = 288 CTAs ran ~40% slower than 2 x 96, and 8 x 32 tiles was the best
// split for 32-tile shapes). The ring takes ~200 KB per CTA when the CTAs do not outnumber
// the SMs, ~100 KB when two share an SM.
template <typename T, int BN, int EPI>
int launch_decode(const CUtensorMap& mw, const CUtensorMap& mx, const GemmArgs& a0,
                  cudaStream_t stream) {
  auto kern = gemm_decode_kernel<T, BN, EPI>;
  constexpr int stage_bytes = BM * BK * 2 + BN * BK * 2;
  constexpr size_t smem_fixed = 1024 + 2 * kDecMaxStages * 8 + 64 + 64 * sizeof(int);
  const size_t smem_max = smem_fixed + (size_t)kDecMaxStages * stage_bytes;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)std::min<size_t>(smem_max, 227 * 1024)),
                            "cudaFuncSetAttribute(gemm_decode)");
    if (s) return s;
    attr_set[dev & 63] = true;
  }
  const int sms = device_sms();
  GemmArgs a = a0;
  const int64_t max_ctas = (int64_t)sms * 8 / 5;
  int split = (int)std::max<int64_t>(1, std::min<int64_t>({8, max_ctas / a.m_tiles, a.k_blocks / 2}));
  split = ceil_div(a.k_blocks, ceil_div(a.k_blocks, split));  // every split owns k-blocks
  const int kbs = ceil_div(a.k_blocks, split);
  const int64_t ctas = (int64_t)a.m_tiles * split;
  const int budget = ctas <= sms ? 200 * 1024 : 100 * 1024;
  const int stages = std::min(std::max(2, std::min(kDecMaxStages, budget / stage_bytes)),
                              std::max(2, kbs));
  a.k_splits = split;
  a.kb_per_split = ceil_div(a.k_blocks, split);
  const size_t smem = smem_fixed + (size_t)stages * stage_bytes;
  int s = hx::cuda_status(launch_ex(kern, dim3((unsigned)(a.m_tiles * split)), dim3(kGemmThreads),
                                    smem, stream, split, mw, mx, a, stages),
                          "gemm_decode_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("gemm_decode_kernel");
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
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& a,
                cudaStream_t stream) {
  auto kern = gemm_pair_kernel<T, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)kPairSmem),
                            "cudaFuncSetAttribute(gemm_pair)");
    if (s) return s;
    attr_set[dev & 63] = true;
  }
  const int64_t items = pair_items(a.M, a.N);
  const int pairs = (int)std::min<int64_t>(items, device_sms() / 2);
  int s = hx::cuda_status(launch_ex(kern, dim3((unsigned)(2 * pairs)), dim3(kGemmThreads),
                                    kPairSmem, stream, 2, ma, mb, a),
                          "gemm_pair_kernel launch");
  if (s) return s;
  HX_LAUNCH_CHECK("gemm_pair_kernel");
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
  if (qkv) a.qkv = *qkv;
  const size_t need = plan_workspace(p, M, N);
  if (need) {
    HX_REQUIRE(ws && ws_bytes >= need, "hx_gemm: workspace too small (%zu < %zu)", ws_bytes, need);
    HX_REQUIRE((uintptr_t)ws % 16 == 0, "hx_gemm: workspace must be 16-byte aligned");
    a.ws = (float*)ws;
  }
  CUtensorMap ma, mb;
  int s;
  if (p.pair) {
    // Each CTA of a pair loads 128 rows of A and 128 rows (output columns) of B per k-block.
    s = make_map(&ma, A, M, K, lda, BM, dtype);
    if (s) return s;
    s = make_map(&mb, B, N, K, ldb, BM, dtype);
    if (s) return s;
    return launch_pair<T, EPI>(ma, mb, a, stream);
  }
  if (p.swap) {
    // MMA A = weights (128-row boxes), MMA B = activations (bn-row box).
    s = make_map(&ma, B, N, K, ldb, BM, dtype);
    if (s) return s;
    s = make_map(&mb, A, M, K, lda, p.bn, dtype);
    if (s) return s;
    switch (p.bn) {
      case 16: return launch_decode<T, 16, EPI>(ma, mb, a, stream);
      case 32: return launch_decode<T, 32, EPI>(ma, mb, a, stream);
      default: return launch_decode<T, 64, EPI>(ma, mb, a, stream);
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

int hx_gemm_kernel_kind(int64_t m, int64_t n, int64_t k, int dtype) {
  if (m <= 0 || n <= 0 || k <= 0) return -1;
  if (dtype == HX_F32) return 0;
  const Plan p = plan_gemm(m, n, k);
  return p.swap ? 3 : (p.pair ? 2 : 1);
}

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
  q.seq_offsets = nullptr;
  q.slots = nullptr;
  q.n_prompts = (int)(m / seqlen);
  q.cache_rows = INT64_MAX;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == HX_BF16)
    return gemm_half<__nv_bfloat16, HX_EPI_QKV_ROTARY>(x, w_qkv, nullptr, m, n, k, ldx, k, 0,
                                                       nullptr, 0, workspace, workspace_bytes,
                                                       dtype, s, &q);
  return gemm_half<__half, HX_EPI_QKV_ROTARY>(x, w_qkv, nullptr, m, n, k, ldx, k, 0, nullptr, 0,
                                              workspace, workspace_bytes, dtype, s, &q);
}

int hx_gemm_qkv_rotary_varlen(const void* x, const void* w_qkv, int64_t m, int64_t k,
                              int64_t ldx, const int32_t* seq_offsets, const int32_t* slots,
                              const int32_t* pos_start, int64_t n_prompts, int64_t n_heads,
                              int64_t n_heads_kv, int64_t head_dim, const void* cos_table,
                              const void* sin_table, int64_t table_rows, void* q_out, void* cache,
                              int64_t cache_batch_stride, int64_t cache_seq_stride,
                              int64_t cache_rows, int64_t cache_max_seq, void* workspace,
                              size_t workspace_bytes, int dtype, void* stream) {
  HX_REQUIRE(x && w_qkv && seq_offsets && slots && pos_start && cos_table && sin_table &&
                 q_out && cache,
             "hx_gemm_qkv_rotary_varlen: null pointer");
  HX_REQUIRE(dtype == HX_BF16 || dtype == HX_F16, "hx_gemm_qkv_rotary_varlen: f16/bf16 only");
  HX_REQUIRE(head_dim % 2 == 0 && n_heads > 0 && n_heads_kv > 0 && n_prompts > 0 &&
                 n_prompts <= m && m <= INT32_MAX && cache_rows > 0,
             "hx_gemm_qkv_rotary_varlen: bad shape");
  HX_REQUIRE(cache_seq_stride >= 2 * n_heads_kv * head_dim && cache_seq_stride % 8 == 0 &&
                 cache_batch_stride % 8 == 0 && (uintptr_t)cache % 16 == 0 &&
                 (uintptr_t)q_out % 16 == 0 && (uintptr_t)cos_table % 16 == 0 &&
                 (uintptr_t)sin_table % 16 == 0,
             "hx_gemm_qkv_rotary_varlen: cache/q_out/tables must be 16-byte aligned (strides "
             "multiples of 8)");
  HX_REQUIRE((uintptr_t)x % 16 == 0 && (uintptr_t)w_qkv % 16 == 0 && ldx % 8 == 0 && k % 8 == 0,
             "hx_gemm_qkv_rotary_varlen: x/w must be 16-byte aligned with ldx, k multiples of 8");
  const int64_t n = (n_heads + 2 * n_heads_kv) * head_dim;
  QkvArgs q;
  q.q_out = q_out;
  q.cache = cache;
  q.cbs = cache_batch_stride;
  q.css = cache_seq_stride;
  q.cbo = 0;
  q.max_seq = cache_max_seq;
  q.table_rows = table_rows;
  q.pos_start = pos_start;
  q.cos = cos_table;
  q.sin = sin_table;
  q.n_heads = (int)n_heads;
  q.n_heads_kv = (int)n_heads_kv;
  q.head_dim = (int)head_dim;
  q.seqlen = 1;
  q.seq_offsets = seq_offsets;
  q.slots = slots;
  q.n_prompts = (int)n_prompts;
  q.cache_rows = cache_rows;
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
