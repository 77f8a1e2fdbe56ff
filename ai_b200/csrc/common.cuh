// Shared device/host helpers for the ai_b200 sm_100a kernels.
//
// * status word: kernels never trap; a failed bounded wait or a bad device-side argument records a code in
//   `g_aib_status` (first writer wins) and the kernel returns. The host reads it with aib_status_read().
// * PDL: kernels are launched with programmatic stream serialization when enabled; each kernel calls
//   pdl_wait() before touching data produced or consumed by earlier kernels, and pdl_trigger() early so
//   the next kernel's CTAs can start streaming their (independent) weights.
// * mbarrier / TMA wrappers (inline PTX). Every wait is bounded.
#pragma once
#include <cstdint>
#include <utility>
#include <cuda_runtime.h>
#include <cuda.h>
#include <map>
#include <mutex>
#include <tuple>
#include "../../include/ai_b200.h"

#define AIB_DEV __device__ __forceinline__

namespace aib {

// ------------------------------------------------------------------------------------------ status
// The library is one translation unit (lib.cu), so the status word is defined here once.
__device__ int g_aib_status = 0;

AIB_DEV void set_status(int code) { atomicCAS(&g_aib_status, 0, code); }

// spin limit for bounded waits: 4M tries of a try_wait that suspends up to the hardware's limit -- tens of
// milliseconds to a few seconds in all, far longer than any legitimate wait in these kernels (the longest is a
// launch's early CTAs waiting out a millisecond-long previous kernel).
constexpr uint32_t kSpinLimit = 1u << 22;
// Test knobs (aib_debug_knob): a smaller spin limit, so a test can make a wait run out in milliseconds, and a
// switch under which the wide GEMV's producer issues no copies (its stages never fill). Zero = off.
__device__ uint32_t g_aib_spin_override = 0;
__device__ int g_aib_withhold_copies = 0;
AIB_DEV uint32_t spin_limit() {
  const uint32_t o = g_aib_spin_override;  // written by the host between launches only
  return o ? o : kSpinLimit;
}

// ------------------------------------------------------------------------------------------- PDL
AIB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
AIB_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------------------- mbarrier
AIB_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

AIB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
AIB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
AIB_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

AIB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
AIB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// A waiting thread may be suspended (taking no issue slots) until the phase completes or a time limit elapses:
// kSuspendNs when non-zero, else the hardware's own limit. The hardware's limit measured 0.5 % faster on the
// decode step than a 1 us hint (313.2 vs 314.8 tok/s).
#ifndef AIB_SUSPEND_NS
#define AIB_SUSPEND_NS 0
#endif
constexpr uint32_t kSuspendNs = AIB_SUSPEND_NS;
AIB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if (kSuspendNs) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}
// Bounded wait: returns false (and records `code`) if the phase did not complete in time.
// Non-blocking probe of a phase (never suspends): for a thread that polls several barriers in turn.
AIB_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

AIB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint32_t lim = spin_limit();
  for (uint32_t i = 0; i < lim; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  set_status(code);
  return false;
}

// ------------------------------------------------------------------------------------------- TMA
// 3-D tiled bulk tensor load (no multicast) into shared memory, completion on an mbarrier.
AIB_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// The same copy with an L2 cache policy (l2_evict_first: a stream read once, which should not push out what
// later kernels reuse -- activations, the KV cache, kernel code).
AIB_DEV void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}
// Flags between CTAs of one grid (GPU scope): a release store after the data it publishes, an acquire load
// before the data it guards.
AIB_DEV void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
AIB_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
AIB_DEV uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
AIB_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// named barrier among `threads` threads (multiple of 32)
AIB_DEV void named_sync(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// ------------------------------------------------------------------------------------ arithmetic
// D += A * B, m16n8k16, bf16 inputs, fp32 accumulators (A row-major 16x16, B col-major 16x8).
AIB_DEV void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

AIB_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
// d = a * b + c on two fp32 lanes (sm_100 packed FMA)
AIB_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t A, B, Cc, D;
  asm("mov.b64 %0, {%1,%2};" : "=l"(A) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1,%2};" : "=l"(B) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1,%2};" : "=l"(Cc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(D) : "l"(A), "l"(B), "l"(Cc));
  float2 d;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(D));
  return d;
}
AIB_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }
// round-to-nearest-even fp32 -> bf16 bits (NaN -> canonical 0x7FC0)
AIB_DEV uint16_t f32_to_bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0x7FC0;
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}
// The same rounding as one conversion instruction (cvt.rn, subnormals kept; a NaN becomes the hardware's
// canonical NaN): two floats packed as bf16x2 (lo in bits 0-15), or one.
AIB_DEV uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
AIB_DEV uint16_t bf16_rn(float f) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
  return r;
}

AIB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace aib

// --------------------------------------------------------------------------------------- host side
namespace aib {
int fail(int code, const char* fmt, ...);  // records the thread-local message, returns code
bool pdl_enabled();
int sm_count(int device = -1);
int launch_check(const char* what);  // maps cudaGetLastError to AIB_ECUDA
// Encodes a 3-D tiled tensor map (uint8 elements, no swizzle, no interleave).
int make_map_3d_u8(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1_bytes,
                   uint64_t s2_bytes, uint32_t b0, uint32_t b1, uint32_t b2);
// General tiled tensor map: `rank` dims (innermost first), rank-1 byte strides, box, swizzle mode.
int make_map(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, int rank, const void* base,
             const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Raise a kernel's dynamic shared-memory limit to the sm_100 per-block maximum (232448 bytes, static +
// dynamic), once per (kernel, device). A failure is reported and clears the runtime's sticky error.
bool smem_raised(const void* kernel, int device, bool record);  // true if already recorded
template <typename K>
int allow_smem(K kernel, size_t bytes) {
  constexpr size_t kMaxBlock = 232448;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(AIB_ECUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
  }
  if (bytes + fa.sharedSizeBytes > kMaxBlock)
    return fail(AIB_ENOTSUP, "kernel needs %zu + %zu bytes of shared memory", bytes, (size_t)fa.sharedSizeBytes);
  if (smem_raised(reinterpret_cast<const void*>(kernel), dev, false)) return AIB_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kMaxBlock - fa.sharedSizeBytes));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(AIB_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  smem_raised(reinterpret_cast<const void*>(kernel), dev, true);
  return AIB_OK;
}

// Launch with the PDL attribute (when enabled) on `stream`; cluster_x > 1: thread-block clusters of cluster_x
// CTAs along x (grid.x a multiple of it).
template <typename... KArgs, typename... Args>
int launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
              int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(AIB_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return AIB_OK;
}
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* what,
           Args&&... args) {
  return launch_ex(kernel, grid, block, smem, stream, what, 1, std::forward<Args>(args)...);
}

// Whether `need` clusters of cluster_x CTAs of `kernel` (dynamic shared memory `smem`, already allowed) can be
// resident at once on this device. Cached per (kernel, cluster size, shared memory).
template <typename... KArgs>
bool clusters_fit(void (*kernel)(KArgs...), dim3 block, size_t smem, int cluster_x, int need) {
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t>, int> cache;
  const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), cluster_x, smem);
  int n = -1;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) n = it->second;
  }
  if (n < 0) {
    n = 0;
    bool ok = true;
    if (cluster_x > 8 && cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
      ok = false;
    if (ok) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cluster_x);
      cfg.blockDim = block;
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = cluster_x;
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = 1;
      cfg.attrs = a;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = n;
  }
  return n >= need;
}
}  // namespace aib
