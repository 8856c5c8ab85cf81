// K4 (tensor-core path): causal prefill attention on tcgen05 / TMEM, fed by TMA.
//
// Semantics are those of attn_prefill.cu (flash_attn_kvpacked_func as called at
// hexgen/hexgen_core/modules/mha.py:566-569, FlashAttention-2 numerics): f32 scores, f32 online
// softmax in base 2, probabilities rounded to the activation dtype before P.V, f32
// accumulation, bottom-right causal alignment (or no mask when causal == 0).
//
// One CTA = 128 queries of one head (f16/bf16, head_dim 64 or 128). Warp roles:
//   warp 0      TMA: the Q tile once, then K/V tiles of 128 keys straight out of the KV cache
//               ([B, max_seq, 2, hkv, d], a 4D tensor map) into a 2-stage ring.
//   warp 1      MMA (one thread): S_j = Q K_j^T into a double-buffered TMEM score tile
//               (M=128, N=128, K=d); O += P_j V_j into one TMEM output tile (M=128, N=d,
//               K=128, V read MN-major). S_{j+1} is issued before P_j V_j, so QK^T overlaps
//               the softmax.
//   warps 2-5   softmax + epilogue: thread = query row. The score row is read from TMEM once
//               (tiles below the causal diagonal skip the mask), P written to a double-buffered
//               shared-memory tile in the SW128 K-major layout the MMA reads. O never leaves
//               TMEM until the epilogue: the reference max of a row only moves when a tile's
//               max exceeds it by more than 2^8 (conditional rescaling, FlashAttention-4), and
//               only then is O rescaled in place (tcgen05.ld / st), so P stays below 256.
// Cache rows past the live range may hold stale bits; their scores are masked to -inf and
// their V rows are zeroed in shared memory before P.V so 0 * stale never reaches the MMA.
#include "common.cuh"

namespace {

constexpr int kRows = 128;       // queries per CTA, keys per tile
constexpr int kChunkBytes = kRows * 128;  // one [128 rows x 64 elements] swizzled chunk
constexpr int kThreads = 192;

template <int D>
struct Lay {
  static constexpr int kChunks = D / 64;
  static constexpr int kQ = 0;
  static constexpr int kK0 = kChunks * kChunkBytes;
  static constexpr int kKV = 2 * kChunks * kChunkBytes;  // K + V of one stage
  static constexpr int kP = kK0 + 2 * kKV;
  static constexpr int kPBytes = 2 * kChunkBytes;         // one [128 x 128 keys] P tile
  static constexpr int kBar = kP + 2 * kPBytes;           // P[2]
  static constexpr size_t kSmem = kBar + 256 + 1024;
  static constexpr uint32_t kTmemCols = 512;  // S[2] (256) + O (d), rounded to a power of 2
  static constexpr uint32_t kOCol = 256;
};

struct PAArgs {
  int seqlen_q, n_heads, n_heads_kv, causal;
  float scale_log2;
  void* out;
  const int32_t* pos_start;
  int64_t cache_batch_offset;
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                           const __grid_constant__ CUtensorMap tmKV, const PAArgs a) {
  using L = Lay<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBar);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;   // [2]
  uint64_t* o_full = bars + 11;  // [2]: P_j V_j complete, committed to o_full[j & 1]
  uint64_t* drain = bars + 15;  // MMA completion barrier used on exit
  uint32_t* counters = reinterpret_cast<uint32_t*>(bars + 16);  // [0] kv issued [1] kv consumed [2] q consumed
  uint32_t* tmem_slot = counters + 3;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heads vary fastest and query blocks run last-to-first, so under a causal mask the CTAs with
  // the most key tiles start in the first wave and the light ones fill the tail.
  const int h = blockIdx.x, qblk = gridDim.y - 1 - blockIdx.y, b = blockIdx.z;
  const int S = a.seqlen_q;
  const int q0 = qblk * kRows;
  const int nq = min(kRows, S - q0);
  const int p0 = a.pos_start[b];
  const int key_end = a.causal ? p0 + q0 + nq : p0 + S;
  const int n_tiles = (key_end + kRows - 1) / kRows;
  const int hk = h / (a.n_heads / a.n_heads_kv);

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmKV);
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    counters[0] = counters[1] = counters[2] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, L::kChunks * kChunkBytes);
      for (int c = 0; c < L::kChunks; ++c)
        tma_load_3d(sm + L::kQ + c * kChunkBytes, &tmQ, q_full, c * 64, h, b * S + q0);
      const int bb = (int)(a.cache_batch_offset + b);
      uint32_t issued = 0;
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1)) break;
        mbar_arrive_expect_tx(&kv_full[st], L::kKV);
        uint8_t* kb = sm + L::kK0 + st * L::kKV;
        uint8_t* vb = kb + L::kChunks * kChunkBytes;
        for (int c = 0; c < L::kChunks; ++c) {
          tma_load_4d(kb + c * kChunkBytes, &tmKV, &kv_full[st], c * 64, hk, j * kRows, bb);
          tma_load_4d(vb + c * kChunkBytes, &tmKV, &kv_full[st], c * 64, a.n_heads_kv + hk,
                      j * kRows, bb);
        }
        ++issued;
      }
      counters[0] = issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16<T>(128, 128);
      constexpr uint32_t idesc_o = make_idesc_f16<T>(128, D, 0, 1);
      bool ok = mbar_wait(q_full, 0);
      counters[2] = ok ? 1u : 0u;
      uint32_t consumed = 0;
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, sb = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1)) return false;
        ++consumed;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sm + L::kQ);
        const uint32_t ka = smem_u32(sm + L::kK0 + st * L::kKV);
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f16(tmem + sb * 128, sw128_kmajor_desc(qa + c * kChunkBytes + k * 32),
                       sw128_kmajor_desc(ka + c * kChunkBytes + k * 32), idesc_s,
                       (c | k) ? 1u : 0u);
        tc_commit(&s_full[sb]);
        return true;
      };
      if (ok && n_tiles > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1)) break;
        tc_fence_after();
        const int st = j & 1;
        const uint32_t pa = smem_u32(sm + L::kP + (j & 1) * L::kPBytes);
        const uint32_t va = smem_u32(sm + L::kK0 + st * L::kKV + L::kChunks * kChunkBytes);
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int key = kc * 64 + k * 16;
            tc_mma_f16(tmem + L::kOCol, sw128_kmajor_desc(pa + kc * kChunkBytes + k * 32),
                       sw128_mnmajor_desc(va + key * 128, kChunkBytes, 1024), idesc_o,
                       (j | kc | k) ? 1u : 0u);
          }
        tc_commit(&o_full[j & 1]);
        tc_commit(&kv_empty[st]);
      }
      // No MMA of this CTA may still be running when TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0);
      counters[1] = consumed;
    }
  } else {
    // Softmax / epilogue warps: row r of the tile, TMEM lane quarter = warp % 4.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const int qpos = p0 + q0 + r;
    // m_ref: the row's reference max (log2 units) that P is taken against; l_run: sum of P.
    float m_ref = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Ordering facts used below: S_j is issued after P_{j-2} V_{j-2}, and a tcgen05.commit
    // covers every earlier MMA of the issuing thread, so once S_j is complete at most one P.V
    // (P_{j-1} V_{j-1}) is still running, and each o_full[x] has at most one phase pending.
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int sb = j & 1;
      uint8_t* pbase = sm + L::kP + (j & 1) * L::kPBytes;
      if (!mbar_wait_warp(&s_full[sb], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      uint32_t v[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(lane_addr + sb * 128 + c * 32, v[c]);
      tc_wait_ld();
      // The score tile is in registers: hand its TMEM buffer back for S_{j+2}.
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      const int key0 = j * kRows;
      // Tiles wholly inside the live range and below the causal diagonal of every row of this
      // CTA need no mask (all but the last tile or two of a row block).
      const bool full = key0 + kRows <= key_end && (!a.causal || key0 + kRows - 1 <= p0 + q0);
      if (!full) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = key0 + c * 32 + i;
            const bool valid = key < key_end && (!a.causal || key <= qpos);
            if (!valid) v[c][i] = 0xff800000u;  // -inf: exp2 gives 0
          }
      }
      // Row max: eight independent 16-deep chains, then a tree.
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = __uint_as_float(v[0][k]);
#pragma unroll
      for (int idx = 8; idx < 128; idx += 8)
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], __uint_as_float(v[idx >> 5][(idx & 31) + k]));
#pragma unroll
      for (int k = 0; k < 4; ++k) m8[k] = fmaxf(m8[k], m8[k + 4]);
      // scale > 0, so max(s) * scale = max(s * scale); -inf stays -inf.
      const float tmax = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])) * a.scale_log2;
      // Conditional rescale. tcgen05.ld/st are warp-collective, so the warp decides together;
      // every row of a rescaling warp moves its reference to its running max.
      if (__any_sync(0xffffffffu, tmax > m_ref + 8.f)) {
        const float m_new = fmaxf(m_ref, tmax);
        const float alpha = m_ref == -INFINITY ? 0.f : ex2_approx(m_ref - m_new);
        l_run *= alpha;
        m_ref = m_new;
        if (j > 0) {
          // O holds P_0 V_0 .. P_{j-1} V_{j-1}; wait for the last of them, scale in place.
          if (!mbar_wait_warp(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(lane_addr + L::kOCol + c * 32, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(lane_addr + L::kOCol + c * 32, o);
          }
          tc_wait_st();
          tc_fence_before();
        }
      }
      // m_ref is finite from the first tile on (key 0 is valid for every row).
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      // P = exp2(s * scale - m_ref) -> swizzled K-major smem, and the row sum (eight
      // independent partial sums).
      float ps[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps[i] = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // 4 groups of 8 keys = 16 bytes of P
          float pf[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            pf[i] = ex2_approx(fmaf(__uint_as_float(v[c][g * 8 + i]), a.scale_log2, -mu));
            ps[i] += pf[i];
          }
          uint4 packed;
          packed.x = pack2<T>(pf[0], pf[1]);
          packed.y = pack2<T>(pf[2], pf[3]);
          packed.z = pack2<T>(pf[4], pf[5]);
          packed.w = pack2<T>(pf[6], pf[7]);
          const int col0 = c * 32 + g * 8;
          const int kc = col0 >> 6, unit = (col0 & 63) >> 3;
          uint8_t* dst = pbase + kc * kChunkBytes + r * 128 + ((unit ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = packed;
        }
      }
      // Last tile: zero V rows past the live keys (their cache rows may be stale).
      if (j == n_tiles - 1) {
        const int valid_rows = key_end - key0;
        if (r >= valid_rows) {
          uint8_t* vrow = sm + L::kK0 + (j & 1) * L::kKV + L::kChunks * kChunkBytes + r * 128;
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<uint4*>(vrow + c * kChunkBytes + u * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[j & 1]);
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
    }
    // Epilogue: the last P.V also completes every earlier one.
    const int jl = n_tiles - 1;
    if (ok && n_tiles > 0 && !mbar_wait_warp(&o_full[jl & 1], (jl >> 1) & 1)) ok = false;
    if (ok && n_tiles > 0) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + (((int64_t)b * S + q0 + r) * a.n_heads + h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lane_addr + L::kOCol + c * 32, o);
        tc_wait_ld();
        if (r < nq) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 pk;
            pk.x = pack2<T>(__uint_as_float(o[e + 0]) * inv, __uint_as_float(o[e + 1]) * inv);
            pk.y = pack2<T>(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            pk.z = pack2<T>(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            pk.w = pack2<T>(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = pk;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // After an aborted wait, let issued-but-unconsumed TMA loads land (bounded) before exit.
  if (threadIdx.x == 0) {
    if (!counters[2]) mbar_wait(q_full, 0);
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait(&kv_full[i & 1], (i >> 1) & 1)) break;
  }
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, L::kTmemCols);
}

template <typename T, int D>
int launch_tc(const void* q, const void* cache, int64_t cbs, int64_t css, int64_t cbo,
              const int32_t* pos_start, int64_t B, int64_t S, int64_t hq, int64_t hk,
              int causal, float scale, void* out, int dtype, cudaStream_t stream) {
  using L = Lay<D>;
  CUtensorMap mq, mkv;
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)hq, (uint64_t)(B * S)};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)hq * D * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)kRows};
    int s = make_tensor_map(&mq, q, 3, dims, strides, box, dtype);
    if (s) return s;
  }
  {
    // Cache [B_cap, max_seq, 2, hkv, d] addressed as (d, 2*hkv, position, batch); the batch
    // extent only needs to cover the rows this launch touches.
    const int64_t max_seq = css > 0 ? cbs / css : 0;
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(2 * hk), (uint64_t)max_seq,
                              (uint64_t)(cbo + B)};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)css * 2, (uint64_t)cbs * 2};
    const uint32_t box[4] = {64, 1, (uint32_t)kRows, 1};
    int s = make_tensor_map(&mkv, cache, 4, dims, strides, box, dtype);
    if (s) return s;
  }
  auto kern = prefill_attn_tc_kernel<T, D>;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    int s = hx::cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)L::kSmem),
                            "cudaFuncSetAttribute(prefill_attn_tc)");
    if (s) return s;
    attr[dev & 63] = true;
  }
  PAArgs args{(int)S, (int)hq, (int)hk, causal, scale * 1.4426950408889634f, out, pos_start, cbo};
  dim3 grid((unsigned)hq, ceil_div(S, kRows), (unsigned)B);
  kern<<<grid, kThreads, L::kSmem, stream>>>(mq, mkv, args);
  HX_LAUNCH_CHECK("prefill_attn_tc_kernel");
  return HX_OK;
}

}  // namespace

// Tensor-core prefill attention; returns HX_ERR_UNSUPPORTED for shapes it does not cover so
// the caller can use the CUDA-core kernel (f32, head_dim 32, unaligned strides).
int prefill_attention_tc(const void* q, const void* cache, int64_t cbs, int64_t css, int64_t cbo,
                         const int32_t* pos_start, int64_t B, int64_t S, int64_t hq, int64_t hk,
                         int64_t d, int causal, float scale, void* out, int dtype,
                         cudaStream_t stream) {
  if ((dtype != HX_BF16 && dtype != HX_F16) || (d != 64 && d != 128)) return HX_ERR_UNSUPPORTED;
  if (css % 8 || cbs % css || ((uintptr_t)q % 16) || ((uintptr_t)cache % 16) || B * S > INT32_MAX)
    return HX_ERR_UNSUPPORTED;
  if (dtype == HX_BF16) {
    if (d == 128)
      return launch_tc<__nv_bfloat16, 128>(q, cache, cbs, css, cbo, pos_start, B, S, hq, hk, causal, scale, out, dtype, stream);
    return launch_tc<__nv_bfloat16, 64>(q, cache, cbs, css, cbo, pos_start, B, S, hq, hk, causal, scale, out, dtype, stream);
  }
  if (d == 128)
    return launch_tc<__half, 128>(q, cache, cbs, css, cbo, pos_start, B, S, hq, hk, causal, scale, out, dtype, stream);
  return launch_tc<__half, 64>(q, cache, cbs, css, cbo, pos_start, B, S, hq, hk, causal, scale, out, dtype, stream);
}
