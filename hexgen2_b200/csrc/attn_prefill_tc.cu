// K4 (tensor-core path): causal prefill attention on tcgen05 / TMEM, fed by TMA.
//
// Semantics are those of attn_prefill.cu (flash_attn_kvpacked_func as called at
// hexgen/hexgen_core/modules/mha.py:566-569, FlashAttention-2 numerics): f32 scores, f32 online
// softmax in base 2, probabilities rounded to the activation dtype before P.V, f32
// accumulation, bottom-right causal alignment (or no mask when causal == 0).
//
// One CTA = 128 queries of one head (f16/bf16, head_dim 64 or 128). Warp roles:
//   warp 0      TMA: the Q tile once, then K and V tiles of 128 keys straight out of the KV
//               cache ([B, max_seq, 2, hkv, d], a 4D tensor map) into separate 2-stage K and V
//               rings, in the order the MMAs consume them (K0, K1, V0, K2, V1, ...). A K stage
//               is free as soon as its QK^T completes, so K_{j+2} streams in while tile j's
//               softmax and P.V still hold V_j.
//   warp 1      MMA (one thread): S_j = Q K_j^T into a double-buffered TMEM score tile
//               (M=128, N=128, K=d); O += P_j V_j into one TMEM output tile (M=128, N=d,
//               K=128, V read MN-major). S_{j+1} is issued before P_j V_j, so QK^T overlaps
//               the softmax.
//   warps 2-9   softmax + epilogue: two threads per query row, one in each of two
//               warpgroups, each owning 64 of the tile's 128 key columns and half of the O
//               columns. The score half-row is read from TMEM once (tiles below the causal
//               diagonal skip the mask); the pair exchanges its partial row max through shared
//               memory under a 64-thread named barrier; P is computed into registers and
//               then stored, once the previous P.V has finished reading it, into a shared-memory
//               tile in the SW128 K-major layout the MMA reads. O never leaves
//               TMEM until the epilogue: the reference max of a row only moves when a tile's
//               max exceeds it by more than 2^8 (conditional rescaling, FlashAttention-4), and
//               only then is O rescaled in place (tcgen05.ld / st), so P stays below 256.
// Cache rows past the live range may hold stale bits; their scores are masked to -inf and
// their V rows are zeroed in shared memory before P.V so 0 * stale never reaches the MMA.
#include "common.cuh"

namespace {

constexpr int kRows = 128;       // queries per CTA, keys per tile
constexpr int kChunkBytes = kRows * 128;  // one [128 rows x 64 elements] swizzled chunk
constexpr int kThreads = 320;    // TMA warp, MMA warp, 2 softmax warpgroups

template <int D>
struct Lay {
  static constexpr int kChunks = D / 64;
  static constexpr int kQ = 0;
  static constexpr int kTile = kChunks * kChunkBytes;    // one [128 keys x d] K or V tile
  static constexpr int kK0 = kTile;                       // K ring [2]
  static constexpr int kV0 = kK0 + 2 * kTile;             // V ring [2]
  static constexpr int kP = kV0 + 2 * kTile;
  static constexpr int kPBytes = 2 * kChunkBytes;         // one [128 x 128 keys] P tile
  static constexpr int kRed = kP + kPBytes;               // one P tile
  // Max exchange: float [2 tiles][2 halves][128 rows]; the epilogue reuses it for row sums.
  static constexpr int kBar = kRed + 2 * 2 * kRows * 4;
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
  // Variable-length launches (items != nullptr): the queries of n_prompts prompts are packed
  // row after row; prompt b owns q/out rows [seq_off[b], seq_off[b + 1]) and cache row
  // slots[b]; grid.y enumerates work items (prompt, query block), heaviest first.
  const int2* items;
  const int32_t* seq_off;
  const int32_t* slots;
  int n_prompts;
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
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;   // [2] (by tile parity; one P tile)
  uint64_t* o_full = bars + 11;  // [2]: P_j V_j complete, committed to o_full[j & 1]
  uint64_t* v_full = bars + 13;   // [2]
  uint64_t* drain = bars + 15;  // MMA completion barrier used on exit
  uint64_t* v_empty = bars + 16;  // [2]
  // [0] K issued [1] K consumed [2] q consumed [3] V issued [4] V consumed
  uint32_t* counters = reinterpret_cast<uint32_t*>(bars + 18);
  uint32_t* tmem_slot = counters + 5;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Heads vary fastest and query blocks run last-to-first, so under a causal mask the CTAs with
  // the most key tiles start in the first wave and the light ones fill the tail.
  const int h = blockIdx.x;
  int qblk, b, S;
  int64_t row0, bb;
  if (a.items) {
    const int2 it = a.items[blockIdx.y];
    b = it.x;
    qblk = it.y;
    if (b < 0 || b >= a.n_prompts) {  // the whole CTA leaves before any barrier or allocation
      if (threadIdx.x == 0) record_device_error(HX_DEVERR_BAD_ARGUMENT);
      return;
    }
    row0 = a.seq_off[b];
    S = a.seq_off[b + 1] - a.seq_off[b];
    bb = a.slots[b];
    if (qblk < 0 || qblk * kRows >= S) {
      if (threadIdx.x == 0) record_device_error(HX_DEVERR_BAD_ARGUMENT);
      return;
    }
  } else {
    qblk = gridDim.y - 1 - blockIdx.y;
    b = blockIdx.z;
    S = a.seqlen_q;
    row0 = (int64_t)b * S;
    bb = a.cache_batch_offset + b;
  }
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
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 256);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    counters[0] = counters[1] = counters[2] = counters[3] = counters[4] = 0;
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
        tma_load_3d(sm + L::kQ + c * kChunkBytes, &tmQ, q_full, c * 64, h, (int)(row0 + q0));
      uint32_t k_issued = 0, v_issued = 0;
      // Step i loads K_i, then V_{i-1}: the MMA thread's order is S_0, S_1, PV_0, S_2, PV_1, ...
      for (int i = 0; i <= n_tiles; ++i) {
        if (i < n_tiles) {
          const int st = i & 1;
          if (!mbar_wait(&k_empty[st], ((i >> 1) & 1) ^ 1)) break;
          mbar_arrive_expect_tx(&k_full[st], L::kTile);
          uint8_t* kb = sm + L::kK0 + st * L::kTile;
          for (int c = 0; c < L::kChunks; ++c)
            tma_load_4d(kb + c * kChunkBytes, &tmKV, &k_full[st], c * 64, hk, i * kRows, (int)bb);
          ++k_issued;
        }
        if (i >= 1) {
          const int t = i - 1, st = t & 1;
          if (!mbar_wait(&v_empty[st], ((t >> 1) & 1) ^ 1)) break;
          mbar_arrive_expect_tx(&v_full[st], L::kTile);
          uint8_t* vb = sm + L::kV0 + st * L::kTile;
          for (int c = 0; c < L::kChunks; ++c)
            tma_load_4d(vb + c * kChunkBytes, &tmKV, &v_full[st], c * 64, a.n_heads_kv + hk,
                        t * kRows, (int)bb);
          ++v_issued;
        }
      }
      counters[0] = k_issued;
      counters[3] = v_issued;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16<T>(128, 128);
      constexpr uint32_t idesc_o = make_idesc_f16<T>(128, D, 0, 1);
      bool ok = mbar_wait(q_full, 0);
      counters[2] = ok ? 1u : 0u;
      uint32_t k_consumed = 0, v_consumed = 0;
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1, sb = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1)) return false;
        ++k_consumed;
        if (!mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sm + L::kQ);
        const uint32_t ka = smem_u32(sm + L::kK0 + st * L::kTile);
#pragma unroll
        for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f16(tmem + sb * 128, sw128_kmajor_desc(qa + c * kChunkBytes + k * 32),
                       sw128_kmajor_desc(ka + c * kChunkBytes + k * 32), idesc_s,
                       (c | k) ? 1u : 0u);
        tc_commit(&s_full[sb]);
        tc_commit(&k_empty[st]);
        return true;
      };
      if (ok && n_tiles > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        const int st = j & 1;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1)) break;
        ++v_consumed;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sm + L::kP);
        const uint32_t va = smem_u32(sm + L::kV0 + st * L::kTile);
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
        tc_commit(&v_empty[st]);
      }
      // No MMA of this CTA may still be running when TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0);
      counters[1] = k_consumed;
      counters[4] = v_consumed;
    }
  } else {
    // Softmax / epilogue warps: row r of the tile (TMEM lane quarter = warp % 4); warpgroup
    // `half` owns key columns [64 half, 64 half + 64) and O columns [half D/2, half D/2 + D/2).
    // The two warps of a row quarter meet at named barrier 1 + quarter (64 threads).
    constexpr int kOHalf = D / 2;
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    const int qpos = p0 + q0 + r;
    float* red = reinterpret_cast<float*>(sm + L::kRed);  // [2][2][128], then [2][128]
    const int bar_id = 1 + quarter;
    // m_ref: the row's reference max (log2 units) that P is taken against; l_run: this half's
    // sum of P.
    float m_ref = -INFINITY, l_run = 0.f;
    bool ok = true;
    // Ordering facts used below: S_j is issued after P_{j-2} V_{j-2}, and a tcgen05.commit
    // covers every earlier MMA of the issuing thread, so once S_j is complete at most one P.V
    // (P_{j-1} V_{j-1}) is still running, and each o_full[x] has at most one phase pending.
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      const bool got = ok && mbar_wait_warp(&s_full[sb], (j >> 1) & 1);
      uint32_t v[2][32];
      float hmax = -INFINITY;
      const int key0 = j * kRows + half * 64;
      if (got) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) tmem_ld_32x32b_x32(lane_addr + sb * 128 + half * 64 + c * 32, v[c]);
        tc_wait_ld();
        // The score tile is in registers: hand its TMEM buffer back for S_{j+2}.
        tc_fence_before();
        mbar_arrive(&s_empty[sb]);
        // Tiles wholly inside the live range and below the causal diagonal of every row of
        // this CTA need no mask (all but the last tile or two of a row block).
        const bool full = j * kRows + kRows <= key_end && (!a.causal || j * kRows + kRows - 1 <= p0 + q0);
        if (!full) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int key = key0 + c * 32 + i;
              const bool valid = key < key_end && (!a.causal || key <= qpos);
              if (!valid) v[c][i] = 0xff800000u;  // -inf: exp2 gives 0
            }
        }
        // Half-row max: eight independent 8-deep chains, then a tree.
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = __uint_as_float(v[0][k]);
#pragma unroll
        for (int idx = 8; idx < 64; idx += 8)
#pragma unroll
          for (int k = 0; k < 8; ++k) m8[k] = fmaxf(m8[k], __uint_as_float(v[idx >> 5][(idx & 31) + k]));
#pragma unroll
        for (int k = 0; k < 4; ++k) m8[k] = fmaxf(m8[k], m8[k + 4]);
        hmax = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
      }
      // Exchange with the partner half. Slot j & 1: a slot is rewritten two tiles later, after
      // the partner has passed the barrier of the tile in between, i.e. after it read this
      // value. The barrier also carries the pair's common go / abort decision.
      red[((j & 1) * 2 + half) * kRows + r] = hmax;
      ok = named_bar_and(bar_id, 64, got);
      if (!ok) break;
      const float pmax = red[((j & 1) * 2 + (half ^ 1)) * kRows + r];
      // scale > 0, so max(s) * scale = max(s * scale); -inf stays -inf. fmaxf is commutative,
      // so both halves of a row hold the same value and take the same decisions below.
      const float tmax = fmaxf(hmax, pmax) * a.scale_log2;
      // Conditional rescale. tcgen05.ld/st are warp-collective, so the warp decides together;
      // every row of a rescaling warp moves its reference to its running max.
      if (__any_sync(0xffffffffu, tmax > m_ref + 8.f)) {
        const float m_new = fmaxf(m_ref, tmax);
        const float alpha = m_ref == -INFINITY ? 0.f : ex2_approx(m_ref - m_new);
        l_run *= alpha;
        m_ref = m_new;
        if (j > 0) {
          // O holds P_0 V_0 .. P_{j-1} V_{j-1}; wait for the last of them, scale this half in
          // place. A timed-out wait skips the scaling (the result is then discarded).
          if (!mbar_wait_warp(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
            ok = false;
          } else {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < kOHalf / 32; ++c) {
              uint32_t o[32];
              tmem_ld_32x32b_x32(lane_addr + L::kOCol + half * kOHalf + c * 32, o);
              tc_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st_32x32b_x32(lane_addr + L::kOCol + half * kOHalf + c * 32, o);
            }
            tc_wait_st();
            tc_fence_before();
          }
        }
      }
      // m_ref is finite from the first tile on (key 0 is valid for every row).
      const float mu = m_ref == -INFINITY ? 0.f : m_ref;
      // P = exp2(s * scale - m_ref) into registers, and this half's row sum (eight
      // independent partial sums).
      float ps[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ps[i] = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int u = 0; u < 8; ++u) {  // 8 groups of 8 keys = 16 bytes of P each
        float pf[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          pf[i] = ex2_approx(fmaf(__uint_as_float(v[u >> 2][(u & 3) * 8 + i]), a.scale_log2, -mu));
          ps[i] += pf[i];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) pk[u * 4 + i] = pack2<T>(pf[2 * i], pf[2 * i + 1]);
      }
      // The P tile is single-buffered: P_{j-1} V_{j-1} must be done reading it. S_j complete
      // implies P_{j-2} V_{j-2} complete, so o_full[(j-1) & 1] has one phase pending at most.
      if (j > 0 && !mbar_wait(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1)) ok = false;
      // Chunk `half` of the swizzled K-major P tile.
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        uint8_t* dst = sm + L::kP + half * kChunkBytes + r * 128 + ((u ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[u * 4], pk[u * 4 + 1], pk[u * 4 + 2], pk[u * 4 + 3]);
      }
      // Last tile: zero V rows past the live keys (their cache rows may be stale); each half
      // clears every other 16-byte unit of the row.
      // V_j lands on its own barrier: wait for it (V_{j-2}, the barrier's previous phase, has
      // been consumed by P_{j-2} V_{j-2}, so the parity is unambiguous).
      if (j == n_tiles - 1 && r >= key_end - j * kRows) {
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1)) {
          ok = false;
        } else {
          uint8_t* vrow = sm + L::kV0 + (j & 1) * L::kTile + r * 128;
#pragma unroll
          for (int c = 0; c < L::kChunks; ++c)
#pragma unroll
            for (int u = half; u < 8; u += 2)
              *reinterpret_cast<uint4*>(vrow + c * kChunkBytes + u * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&p_full[j & 1]);
      l_run += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
    }
    // Epilogue: the last P.V also completes every earlier one. The pair adds its row sums.
    const int jl = n_tiles - 1;
    if (ok && n_tiles > 0 && !mbar_wait_warp(&o_full[jl & 1], (jl >> 1) & 1)) ok = false;
    ok = named_bar_and(bar_id, 64, ok);
    if (ok && n_tiles > 0) {
      // (The partner read its last max before arriving at the barrier above.)
      red[half * kRows + r] = l_run;
      named_bar_sync(bar_id, 64);
      const float l_tot = l_run + red[(half ^ 1) * kRows + r];
      tc_fence_after();
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + ((row0 + q0 + r) * a.n_heads + h) * D + half * kOHalf;
#pragma unroll 1
      for (int c = 0; c < kOHalf / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(lane_addr + L::kOCol + half * kOHalf + c * 32, o);
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
    if (!counters[2]) mbar_wait_drain(q_full, 0);
    for (uint32_t i = counters[1]; i < counters[0]; ++i)
      if (!mbar_wait_drain(&k_full[i & 1], (i >> 1) & 1)) break;
    for (uint32_t i = counters[4]; i < counters[3]; ++i)
      if (!mbar_wait_drain(&v_full[i & 1], (i >> 1) & 1)) break;
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
  PAArgs args{(int)S, (int)hq, (int)hk, causal, scale * 1.4426950408889634f, out, pos_start, cbo,
              nullptr, nullptr, nullptr, 0};
  dim3 grid((unsigned)hq, ceil_div(S, kRows), (unsigned)B);
  kern<<<grid, kThreads, L::kSmem, stream>>>(mq, mkv, args);
  HX_LAUNCH_CHECK("prefill_attn_tc_kernel");
  return HX_OK;
}

// Variable-length launch: one grid over (head, work item) for all prompts of a packed pass.
template <typename T, int D>
int launch_tc_varlen(const void* q, const void* cache, int64_t cbs, int64_t css,
                     int64_t cache_rows, const int32_t* seq_off, const int32_t* slots,
                     const int32_t* pos_start, const int32_t* items, int64_t n_prompts,
                     int64_t n_items, int64_t total_rows, int64_t hq, int64_t hk, int causal,
                     float scale, void* out, int dtype, cudaStream_t stream) {
  using L = Lay<D>;
  CUtensorMap mq, mkv;
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)hq, (uint64_t)total_rows};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)hq * D * 2};
    const uint32_t box[3] = {64, 1, (uint32_t)kRows};
    int s = make_tensor_map(&mq, q, 3, dims, strides, box, dtype);
    if (s) return s;
  }
  {
    const int64_t max_seq = cbs / css;
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(2 * hk), (uint64_t)max_seq,
                              (uint64_t)cache_rows};
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
  PAArgs args{0, (int)hq, (int)hk, causal, scale * 1.4426950408889634f, out, pos_start, 0,
              reinterpret_cast<const int2*>(items), seq_off, slots, (int)n_prompts};
  dim3 grid((unsigned)hq, (unsigned)n_items, 1);
  kern<<<grid, kThreads, L::kSmem, stream>>>(mq, mkv, args);
  HX_LAUNCH_CHECK("prefill_attn_tc_kernel (varlen)");
  return HX_OK;
}

}  // namespace

// Variable-length tensor-core prefill attention (bf16/f16, head_dim 64/128); returns
// HX_ERR_UNSUPPORTED for other shapes so the caller can attend prompt by prompt.
int prefill_attention_tc_varlen(const void* q, const void* cache, int64_t cbs, int64_t css,
                                int64_t cache_rows, const int32_t* seq_off, const int32_t* slots,
                                const int32_t* pos_start, const int32_t* items,
                                int64_t n_prompts, int64_t n_items, int64_t total_rows,
                                int64_t hq, int64_t hk, int64_t d, int causal, float scale,
                                void* out, int dtype, cudaStream_t stream) {
  if ((dtype != HX_BF16 && dtype != HX_F16) || (d != 64 && d != 128)) return HX_ERR_UNSUPPORTED;
  if (css % 8 || css <= 0 || cbs % css || ((uintptr_t)q % 16) || ((uintptr_t)cache % 16) ||
      total_rows > INT32_MAX || n_items > 65535)
    return HX_ERR_UNSUPPORTED;
#define HX_PA_VARLEN(TT, DD)                                                                  \
  return launch_tc_varlen<TT, DD>(q, cache, cbs, css, cache_rows, seq_off, slots, pos_start,   \
                                  items, n_prompts, n_items, total_rows, hq, hk, causal, scale, \
                                  out, dtype, stream)
  if (dtype == HX_BF16) {
    if (d == 128) HX_PA_VARLEN(__nv_bfloat16, 128);
    HX_PA_VARLEN(__nv_bfloat16, 64);
  }
  if (d == 128) HX_PA_VARLEN(__half, 128);
  HX_PA_VARLEN(__half, 64);
#undef HX_PA_VARLEN
}

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
