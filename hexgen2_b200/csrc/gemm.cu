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

template <int BN>
struct Cfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = 2 * BN;  // two accumulators (power of two >= 32)
  static constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + 1024 /*align*/ + 256;
};

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, k_splits, kb_per_split, k_blocks;
  void* C;
  int64_t ldc;
  const void* R;
  int64_t ldr;
  float* ws;  // split-K partials [k_splits][M][N]
};

HX_DEVICE float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Applies the epilogue to 32 accumulator columns [n0, n0+32) of row m and stores them.
template <typename T, int EPI>
HX_DEVICE void epilogue_store(const GemmArgs& a, int m, int n0, const float* v) {
  if (m >= a.M) return;
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

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
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16<T>(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
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
    mma_done:;
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
      if (!mbar_wait(&tfull[acc], acc_phase)) break;
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
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::kTmemCols);
}

// Split-K reduction in split order + epilogue. One thread per output element.
template <typename T, int EPI>
__global__ void splitk_reduce_kernel(const GemmArgs a) {
  const int64_t out_cols = EPI == HX_EPI_SWIGLU ? a.N / 2 : a.N;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)a.M * out_cols) return;
  const int m = (int)(idx / out_cols);
  const int j = (int)(idx % out_cols);
  const int64_t plane = (int64_t)a.M * a.N;
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
};

// Tile / split-K selection. Prefill-shaped problems use the widest tile that still fills the
// machine; decode-shaped ones (one M tile) use BN=64 and split K so ~1-2 CTAs run per SM.
Plan plan_gemm(int64_t M, int64_t N, int64_t K) {
  const int sms = device_sms();
  Plan p;
  p.m_tiles = ceil_div(M, BM);
  p.k_blocks = ceil_div(K, BK);
  const int64_t t256 = (int64_t)p.m_tiles * ceil_div(N, 256);
  const int64_t t128 = (int64_t)p.m_tiles * ceil_div(N, 128);
  if (t256 >= sms) p.bn = 256;
  else if (t128 >= sms) p.bn = 128;
  else p.bn = 64;
  p.n_tiles = ceil_div(N, p.bn);
  const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
  int splits = 1;
  if (tiles < sms && p.k_blocks >= 8) {
    splits = (int)std::min<int64_t>(ceil_div(sms, tiles), p.k_blocks / 4);
    splits = std::max(splits, 1);
  }
  p.kb_per_split = ceil_div(p.k_blocks, splits);
  p.k_splits = ceil_div(p.k_blocks, p.kb_per_split);
  return p;
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
              size_t ws_bytes, int dtype, cudaStream_t stream) {
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
  if (p.k_splits > 1) {
    const size_t need = (size_t)p.k_splits * M * N * sizeof(float);
    HX_REQUIRE(ws && ws_bytes >= need, "hx_gemm: workspace too small (%zu < %zu)", ws_bytes, need);
    a.ws = (float*)ws;
  }
  CUtensorMap ma, mb;
  int s = make_map(&ma, A, M, K, lda, BM, dtype);
  if (s) return s;
  s = make_map(&mb, B, N, K, ldb, p.bn, dtype);
  if (s) return s;
  switch (p.bn) {
    case 256: s = launch_tc<T, 256, EPI>(ma, mb, a, stream); break;
    case 128: s = launch_tc<T, 128, EPI>(ma, mb, a, stream); break;
    default: s = launch_tc<T, 64, EPI>(ma, mb, a, stream); break;
  }
  if (s) return s;
  if (p.k_splits > 1) {
    const int64_t outs = M * (EPI == HX_EPI_SWIGLU ? N / 2 : N);
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
  const Plan p = plan_gemm(m, n, k);
  return p.k_splits > 1 ? (size_t)p.k_splits * m * n * sizeof(float) : 0;
}

int hx_gemm(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
            int64_t lda, int64_t ldb, int64_t ldc, int epilogue, const void* residual,
            int64_t ld_residual, void* workspace, size_t workspace_bytes, int dtype,
            void* stream) {
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
