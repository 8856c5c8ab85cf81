// Shared device/host helpers for the hexgen2_b200 kernels (sm_100a only).
//
// Everything here is plumbing: dtype conversion, launch-error bookkeeping, and thin
// inline-PTX wrappers for the Blackwell async machinery (mbarrier, TMA, tcgen05/TMEM).
// Every spin-wait is bounded: after HX_WAIT_LIMIT_NS of %globaltimer time it records an
// error code in g_hx_device_error and returns false so the kernel can unwind instead of
// hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <type_traits>
#include <utility>

#include "../../include/hexgen2_b200.h"

#define HX_DEVICE __device__ __forceinline__

// ---------------------------------------------------------------------------------------
// Host-side error reporting (thread-local message, returned through hx_last_error()).
// ---------------------------------------------------------------------------------------
namespace hx {
void set_error(const char* fmt, ...);
int cuda_status(cudaError_t e, const char* what);
}  // namespace hx

#define HX_REQUIRE(cond, ...)                 \
  do {                                        \
    if (!(cond)) {                            \
      hx::set_error(__VA_ARGS__);             \
      return HX_ERR_INVALID;                  \
    }                                         \
  } while (0)

// Host: cached cuTensorMapEncodeTiled for a `rank`-D tensor (dims innermost first, strides in
// bytes for dims 1..rank-1), SWIZZLE_128B, zero fill out of bounds. dtype is an hx_dtype.
int make_tensor_map(CUtensorMap* out, const void* ptr, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int dtype);
int device_sm_count();

#define HX_LAUNCH_CHECK(what) \
  do { int _s = hx::cuda_status(cudaGetLastError(), what); if (_s) return _s; } while (0)

// Device-side error word. Kernels write a nonzero code here when a bounded wait gives up
// or a device-side check fails; the host reads and clears it through hx_device_error().
extern __device__ int g_hx_device_error;

enum : int {
  HX_DEVERR_NONE = 0,
  HX_DEVERR_WAIT_TIMEOUT = 1,     // an mbarrier/flag wait exceeded its time budget
  HX_DEVERR_BAD_ARGUMENT = 2,     // a device-side argument check failed
};

static constexpr unsigned long long HX_WAIT_LIMIT_NS = 2000000000ull;  // 2 s per wait

// ---------------------------------------------------------------------------------------
// dtype helpers
// ---------------------------------------------------------------------------------------
template <typename T> struct DT;
template <> struct DT<float> {
  static HX_DEVICE float to_f(float x) { return x; }
  static HX_DEVICE float from_f(float x) { return x; }
};
template <> struct DT<__nv_bfloat16> {
  static HX_DEVICE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static HX_DEVICE __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct DT<__half> {
  static HX_DEVICE float to_f(__half x) { return __half2float(x); }
  static HX_DEVICE __half from_f(float x) { return __float2half_rn(x); }
};

// Round a float through the storage type T (identity for float).
template <typename T> HX_DEVICE float round_to(float x) { return DT<T>::to_f(DT<T>::from_f(x)); }

HX_DEVICE unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HX_DEVICE void record_device_error(int code) { atomicCAS(&g_hx_device_error, 0, code); }

// ---------------------------------------------------------------------------------------
// Shared-memory address / mbarrier wrappers
// ---------------------------------------------------------------------------------------
HX_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

HX_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

HX_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

HX_DEVICE void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

HX_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

HX_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

HX_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the mbarrier phase with the given parity to complete. Returns false (and
// records HX_DEVERR_WAIT_TIMEOUT) if the budget runs out; callers then unwind.
HX_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > HX_WAIT_LIMIT_NS) {
      record_device_error(HX_DEVERR_WAIT_TIMEOUT);
      return false;
    }
    // A device-wide error (another CTA gave up) also ends this wait early.
    if (*((volatile int*)&g_hx_device_error) != 0) return false;
  }
}

// Wait used when a CTA is about to exit after an aborted wait: lets TMA loads that were issued
// but never consumed land before the CTA's shared memory is released. Unlike mbar_wait it does
// not give up when another CTA has recorded an error (that is exactly when it runs), only after
// HX_DRAIN_LIMIT_NS.
static constexpr unsigned long long HX_DRAIN_LIMIT_NS = 200000000ull;  // 200 ms
HX_DEVICE bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < HX_DRAIN_LIMIT_NS)
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Bounded wait by a whole warp with a warp-uniform result, for code that follows the wait with
// warp-collective instructions (tcgen05.ld, shuffles): every lane leaves together.
HX_DEVICE bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

// AND-reduction of a predicate over the `count` threads of named barrier `id` (warp-aligned).
// Lets a group of warps take a common decision (e.g. all abort after a timed-out wait) so that
// no warp is left waiting at a later named barrier.
HX_DEVICE bool named_bar_and(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
HX_DEVICE void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) — tiled 2D/3D loads into this CTA's shared memory.
// Every tensor load here fills only the issuing CTA's own shared memory (one CTA per copy).
// ---------------------------------------------------------------------------------------
HX_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                           int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

HX_DEVICE void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                           int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

HX_DEVICE void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                           int32_t y, int32_t z, int32_t w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

HX_DEVICE void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05 / TMEM wrappers (cta_group::1 only).
// ---------------------------------------------------------------------------------------
HX_DEVICE void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
HX_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HX_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
HX_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
HX_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (bf16/f16 inputs, f32 accumulate).
HX_DEVICE void tc_mma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
HX_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
HX_DEVICE void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 32 consecutive columns per thread.
HX_DEVICE void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// Store of 32 lanes x 32 bit, 32 consecutive columns per thread; tc_wait_st() before the
// values are consumed by another thread or an MMA.
HX_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
HX_DEVICE void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
HX_DEVICE void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA with
// SWIZZLE_128B: rows of 128 bytes, 8-row (1024 B) swizzle atoms stacked along M/N.
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45 stride-dimension byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout type (2 = SWIZZLE_128B)
HX_DEVICE uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Shared-memory descriptor for an MN-major operand tile written by TMA with SWIZZLE_128B
// (used for V in P*V: V is [keys, head_dim] with head_dim contiguous, i.e. N-major for B).
//   Canonical MN-major SW128 layout: atoms of 64 (bf16) MN-elements x 8 K-rows (1024 B).
//   LBO = byte distance between atoms adjacent in MN, SBO = between atoms adjacent in K.
HX_DEVICE uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 with f32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 = f16, 1 = bf16),
//   bit 15 A major, bit 16 B major (0 = K-major, 1 = MN-major), 17-22 N>>3, 24-28 M>>4.
template <typename T>
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int a_mn_major = 0,
                                                      int b_mn_major = 0) {
  uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Kernels launched with launch_ex() may start while the
// previous kernel on the stream is still running: every thread calls pdl_wait() before it
// reads or writes memory that an earlier kernel produces or consumes (it returns once all
// prerequisite grids have completed and their memory is visible; without PDL it returns at
// once). pdl_trigger() lets the next kernel be scheduled as soon as every CTA of this grid
// has issued it, so its prologue overlaps this kernel's tail.
// ---------------------------------------------------------------------------------------
HX_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HX_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: cudaLaunchKernelEx with programmatic stream serialization and an optional 1-D cluster.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------------------------------
// Small math helpers
// ---------------------------------------------------------------------------------------
HX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
HX_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 2^x with the SFU's approximate exp2 (flush-to-zero): the instruction FlashAttention-2's
// softmax compiles to. For softmax arguments (x <= 0) the result is within 2 ulp of 2^x.
HX_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats rounded to nearest into one packed 32-bit pair of T (bf16 or f16), low half first.
template <typename T> HX_DEVICE uint32_t pack2(float lo, float hi);
template <> HX_DEVICE uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <> HX_DEVICE uint32_t pack2<__half>(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// The host picks the dtype-specialised kernel with this switch.
#define HX_DISPATCH_DTYPE(dtype, T, ...)                                  \
  switch (dtype) {                                                        \
    case HX_F32: { using T = float; __VA_ARGS__; break; }                 \
    case HX_F16: { using T = __half; __VA_ARGS__; break; }                \
    case HX_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }        \
    default: hx::set_error("unsupported dtype %d", (int)dtype); return HX_ERR_UNSUPPORTED; \
  }

#define HX_DISPATCH_HALF(dtype, T, ...)                                   \
  switch (dtype) {                                                        \
    case HX_F16: { using T = __half; __VA_ARGS__; break; }                \
    case HX_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }        \
    default: hx::set_error("dtype %d not supported here (f16/bf16 only)", (int)dtype); \
             return HX_ERR_UNSUPPORTED;                                   \
  }
