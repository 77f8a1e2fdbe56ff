// Prefill GEMM on the 5th-generation tensor cores: Y (+)= X W^T with W in the 12-bit codec, decoded on the fly.
//
// Replaces the reference's blocked prefill matrix product (`ramvi/engine/ramvi_engine/kernels/prefill.py:66-78`
// `matrix`, `prefill_kernels.py:8-27` `mm_k`, fed by the fp32 row blocks of `dequant_k` + `exceptions_k`,
// prefill_kernels.py:59-110): there every 512-row weight block is decoded to fp32 in HBM and multiplied with
// fp32 CUDA-core dots; here the codec planes are decoded straight into the tensor cores' shared-memory operand.
//
// Tile: 128 weight rows (the UMMA M) x TN prompt tokens (the UMMA N, <= 256), accumulator in TMEM (TN fp32
// columns x 128 lanes). K advances 64 columns per stage. Warp roles (224 threads, one CTA per SM):
//   warp 0      TMA of the codec planes: m8 and e4 tiles [128 rows x 64 bytes], 64-byte swizzled, NW-deep ring
//               (the e4 bytes of a 64-column block hold its codes in the low or the high nibble);
//   warp 2      TMA of the activation tiles [TN tokens x 64 columns] bf16 (one per precision part), 128-byte
//               swizzled -- the canonical K-major UMMA layout -- into the operand ring (NO deep);
//   warps 3..6  decoders: thread t owns weight row t of the tile; it turns its 64 codec bytes + 64 code nibbles
//               into bf16 pairs (byte permute + integer multiply-add + one LOP3 per pair, the decode of the
//               codec GEMV), writes them 128-byte swizzled into the operand ring's A tile, patches its row's
//               exceptions (code 15) with their exact bf16 values from the CSR, and fences the generic-proxy
//               stores for the async proxy before arriving on the stage barrier. After the K loop the same
//               warps are the epilogue: tcgen05.ld of their TMEM lane quarter, store / add / gated store;
//   warp 1      allocates TMEM and issues tcgen05.mma (kind::f16, bf16 x bf16 -> fp32, K = 16 per
//               instruction) from one thread; tcgen05.commit releases each operand stage and finally signals
//               the accumulator.
// Precision: `parts` = 1 multiplies bf16(x) (one MMA per K step); `parts` = 3 splits x into three bf16 parts
// (x = p1 + p2 + p3 to ~2^-24, the reference's bf16x3 idea, wcomp.py:129-140) and accumulates all three
// products: every product w * p_i is exact in fp32, so the result matches fp32 dots to accumulation rounding,
// like the reference's fp32 IEEE `mm_k`.
// Tiles are rastered token-tile first, so the CTAs that share a weight tile run together and the weights
// cross HBM about once. Every wait is bounded (status word + abort flag); TMEM is always released.
#include <algorithm>
#include <climits>
#include "common.cuh"

namespace aib {
namespace gemm {

constexpr int BM = 128;                // weight rows per tile
constexpr int BK = 64;                 // K columns per stage
constexpr int kWarps = 7;
constexpr int kThreads = kWarps * 32;
constexpr int kPlane = BM * 64;        // one staged plane tile: 128 rows x 64 bytes
constexpr int kWStage = 2 * kPlane;    // m8 + e4
constexpr int kATile = BM * BK * 2;    // decoded bf16 tile, 128 rows x 128 bytes
constexpr int kHeader = 1024;
constexpr int kMaxNW = 8, kMaxNO = 4;

struct Params {
  const int32_t* rp;
  const int32_t* ec;
  const float* ev;
  float* y;
  int ldy, ymode;  // 0: Y = XW^T; 1: Y += XW^T; 3: rows (2i, 2i+1) -> Y[:, i] = silu(gate) * up
  int N, K, M;
  int base;
  int TN, NW, NO, nkb;
  uint32_t idesc;
  uint32_t tmem_cols;
  int w_off, o_off, o_stage;
  uint32_t k128, k8;
  int ks, kb_per;  // split-K: blockIdx.z takes k-blocks [z * kb_per, (z + 1) * kb_per) of nkb
  float* part;     // ks > 1: [tile][split][BM rows][TN] fp32 partial tiles
  int* tick;       // ks > 1: one arrival counter per (token tile, weight tile), zero before the launch
};

// ----------------------------------------------------------------------------------- tcgen05 wrappers
AIB_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
AIB_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
AIB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
AIB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
AIB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
AIB_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
AIB_DEV void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
AIB_DEV void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
AIB_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory descriptor of a K-major operand tile with 128-byte swizzle: rows of 128 bytes (64 bf16),
// 8-row atoms of 1024 bytes (stride-dimension offset), version 1, layout type 2 (SWIZZLE_128B). The
// leading-dimension offset is unused for this layout (1). Advancing K by 16 elements adds 32 bytes to the
// start address; the hardware applies the swizzle to the absolute address, as the TMA and the decoders wrote it.
AIB_DEV uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}

AIB_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

AIB_DEV uint32_t merge_sm_e(uint32_t a, uint32_t b) {  // (a & 0x807F807F) | (b & ~0x807F807F)
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(a), "r"(b), "r"(0x807F807Fu));
  return r;
}

// Bounded wait on a barrier phase; gives up early once another thread has aborted.
AIB_DEV bool wait_b(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case reads no limit
  for (uint32_t i = 0, lim = spin_limit(); i < lim; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort_flag) return false;
  }
  set_status(code);
  *abort_flag = 1;
  return false;
}

// ------------------------------------------------------------------------------------------ kernel
template <int PARTS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_c12_kernel(const __grid_constant__ CUtensorMap tm8, const __grid_constant__ CUtensorMap tme4,
                    const __grid_constant__ CUtensorMap tmx, Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem);
  uint64_t* wempty = wfull + kMaxNW;
  uint64_t* ofull = wempty + kMaxNW;
  uint64_t* oempty = ofull + kMaxNO;
  uint64_t* accfull = oempty + kMaxNO;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 260);
  uint8_t* wring = smem + p.w_off;
  uint8_t* oring = smem + p.o_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * p.TN, n0 = blockIdx.y * BM;
  const int NW = p.NW, NO = p.NO;
  const int kb_begin = static_cast<int>(blockIdx.z) * p.kb_per;
  const int nk = max(0, min(p.nkb, kb_begin + p.kb_per) - kb_begin);  // k-blocks of this split

  if (threadIdx.x == 0) {
    for (int s = 0; s < NW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 4);
    }
    for (int s = 0; s < NO; ++s) {
      mbar_init(&ofull[s], 5);  // four decoder warps + the activation TMA's expect_tx arrival
      mbar_init(&oempty[s], 1);
    }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {  // ------------------------------------------------------- codec planes
    if (lane == 0) {
      prefetch_tensormap(&tm8);
      prefetch_tensormap(&tme4);
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % NW;
        if (i >= NW && !wait_b(&wempty[s], ((i / NW) - 1) & 1, abort_flag, AIB_DEV_TIMEOUT_EMPTY)) break;
        if (*abort_flag) break;
        uint8_t* st = wring + s * kWStage;
        const int kc = (kb_begin + i) * BK;
        mbar_arrive_expect_tx(&wfull[s], kWStage);
        tma_load_2d(st, &tm8, &wfull[s], kc, n0);
        tma_load_2d(st + kPlane, &tme4, &wfull[s], (kc >> 8) * 128 + (kc & 127), n0);
        issued = i + 1;
      }
      if (*abort_flag)  // never leave with copies in flight
        for (int it = (issued > NW ? issued - NW : 0); it < issued; ++it)
          mbar_wait(&wfull[it % NW], (it / NW) & 1, AIB_DEV_TIMEOUT_FULL);
    }
    pdl_trigger();
  } else if (warp == 2) {  // ----------------------------------------------- activations
    pdl_wait();
    if (lane == 0) {
      prefetch_tensormap(&tmx);
      int issued = 0;
      const uint32_t bytes = static_cast<uint32_t>(PARTS * p.TN * 128);
      for (int i = 0; i < nk; ++i) {
        const int s = i % NO;
        if (i >= NO && !wait_b(&oempty[s], ((i / NO) - 1) & 1, abort_flag, AIB_DEV_TIMEOUT_EMPTY)) break;
        if (*abort_flag) break;
        uint8_t* st = oring + s * p.o_stage + kATile;
        mbar_arrive_expect_tx(&ofull[s], bytes);
#pragma unroll
        for (int q = 0; q < PARTS; ++q)
          tma_load_3d(st + q * p.TN * 128, &tmx, &ofull[s], (kb_begin + i) * BK, m0, q);
        issued = i + 1;
      }
      if (*abort_flag)
        for (int it = (issued > NO ? issued - NO : 0); it < issued; ++it)
          mbar_wait(&ofull[it % NO], (it / NO) & 1, AIB_DEV_TIMEOUT_FULL);
    }
    pdl_trigger();
  } else if (warp == 1) {  // ----------------------------------------------- MMA issue
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % NO;
        if (!wait_b(&ofull[s], (i / NO) & 1, abort_flag, AIB_DEV_TIMEOUT_FULL)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(oring + s * p.o_stage), b0 = a0 + kATile;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
#pragma unroll
          for (int q = 0; q < PARTS; ++q)
            tc_mma(tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + q * p.TN * 128 + k * 32), p.idesc,
                   (i | k | q) != 0);
        tc_commit(&oempty[s]);
      }
      tc_commit(accfull);  // arrives once every MMA issued above has completed (also after an abort)
    }
    pdl_trigger();
  } else {  // --------------------------------------------------------------- decoders, then epilogue
    const int t = (warp - 3) * 32 + lane;  // weight row of the tile this thread decodes
    const int n = n0 + t;
    int xp = 0, xe = 0, xc = INT_MAX;
    float xv = 0.0f;
    if (n < p.N) {
      xp = p.rp[n];
      xe = p.rp[n + 1];
      while (xp < xe && p.ec[xp] < kb_begin * BK) ++xp;  // exceptions of earlier splits
      if (xp < xe) {
        xc = p.ec[xp];
        xv = p.ev[xp];
      }
    }
    const uint32_t base7 = (static_cast<uint32_t>(p.base) << 7) | (static_cast<uint32_t>(p.base) << 23);
    const uint32_t k128 = p.k128, k8 = p.k8;
    const int sx = (t >> 1) & 3, ax = t & 7;
    bool aborted = false;
    for (int i = 0; i < nk; ++i) {
      const int sw = i % NW, so = i % NO;
      bool ok = wait_b(&wfull[sw], (i / NW) & 1, abort_flag, AIB_DEV_TIMEOUT_FULL);
      if (ok && i >= NO) ok = wait_b(&oempty[so], ((i / NO) - 1) & 1, abort_flag, AIB_DEV_TIMEOUT_EMPTY);
      if (!__all_sync(0xffffffffu, ok)) {
        aborted = true;
        break;
      }
      const uint8_t* pm = wring + sw * kWStage + t * 64;
      const uint8_t* pe = pm + kPlane;
      uint8_t* pa = oring + so * p.o_stage + t * 128;
      const int kc = (kb_begin + i) * BK;
      const bool hi = (kc & 255) >= 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 mm = *reinterpret_cast<const uint4*>(pm + ((c ^ sx) << 4));
        const uint4 ee = *reinterpret_cast<const uint4*>(pe + ((c ^ sx) << 4));
        const uint32_t L[4] = {mm.x, mm.y, mm.z, mm.w}, E[4] = {ee.x, ee.y, ee.z, ee.w};
        uint32_t pr[8];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const uint32_t x01 = prmt(E[w], 0u, 0x4140u), x23 = prmt(E[w], 0u, 0x4342u);
          const uint32_t t01 = hi ? x01 * k8 + base7 : x01 * k128 + base7 - (x01 & 0x00F000F0u) * k128;
          const uint32_t t23 = hi ? x23 * k8 + base7 : x23 * k128 + base7 - (x23 & 0x00F000F0u) * k128;
          pr[2 * w] = merge_sm_e(prmt(L[w], 0u, 0x9180u), t01);
          pr[2 * w + 1] = merge_sm_e(prmt(L[w], 0u, 0xB3A2u), t23);
        }
        *reinterpret_cast<uint4*>(pa + (((2 * c) ^ ax) << 4)) = make_uint4(pr[0], pr[1], pr[2], pr[3]);
        *reinterpret_cast<uint4*>(pa + (((2 * c + 1) ^ ax) << 4)) = make_uint4(pr[4], pr[5], pr[6], pr[7]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[sw]);
      while (xc < kc + BK) {  // exceptions of this row in the block: exact bf16 values over the stand-ins
        const int j = xc - kc;
        *reinterpret_cast<uint16_t*>(pa + (((j >> 3) ^ ax) << 4) + (j & 7) * 2) =
            static_cast<uint16_t>(__float_as_uint(xv) >> 16);
        ++xp;
        xc = xp < xe ? p.ec[xp] : INT_MAX;
        xv = xp < xe ? p.ev[xp] : 0.0f;
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ofull[so]);
    }
    // ---- epilogue: this warp's TMEM lane quarter holds weight rows 32q .. 32q+31 of the tile
    pdl_wait();
    const bool acc_ok = wait_b(accfull, 0, abort_flag, AIB_DEV_TIMEOUT_FULL);
    aborted = !__all_sync(0xffffffffu, acc_ok && !aborted && !*abort_flag);
    pdl_trigger();
    tc_fence_after();
    const int q = warp & 3, row = 32 * q + lane, nn = n0 + row;
    if (p.ks > 1) {
      // split-K: this split's partial tile to the workspace; the last split of the tile to arrive adds the
      // splits in split order (deterministic) and applies the output mode
      const int tile = static_cast<int>(blockIdx.y * gridDim.x + blockIdx.x), ks = p.ks;
      float* mine = p.part + ((static_cast<size_t>(tile) * ks + blockIdx.z) * BM + row) * p.TN;
      for (int c0 = 0; c0 < p.TN; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), v);
        tmem_wait_ld();
        if (!aborted)
#pragma unroll
          for (int j = 0; j < 16; ++j) mine[c0 + j] = __uint_as_float(v[j]);
      }
      __threadfence();
      named_sync(1, 128);  // the four epilogue warps
      if (threadIdx.x == 96) *reinterpret_cast<volatile int*>(smem + 264) = atomicAdd(&p.tick[tile], 1) == ks - 1;
      named_sync(1, 128);
      if (*reinterpret_cast<volatile int*>(smem + 264) && !aborted) {
        __threadfence();
        const float* base = p.part + (static_cast<size_t>(tile) * ks * BM + row) * p.TN;
        for (int c = 0; c < p.TN; ++c) {
          const int m = m0 + c;
          if (m >= p.M) break;  // uniform across the warp
          float val = 0.0f;
          for (int z = 0; z < ks; ++z) val += __ldcg(base + static_cast<size_t>(z) * BM * p.TN + c);
          float* yr = p.y + static_cast<size_t>(m) * p.ldy;
          if (p.ymode == 3) {
            const float u = __shfl_down_sync(0xffffffffu, val, 1);
            if (!(lane & 1) && nn < p.N) yr[nn >> 1] = val / (1.0f + expf(-val)) * u;
          } else if (nn < p.N) {
            if (p.ymode == 1)
              yr[nn] += val;
            else
              yr[nn] = val;
          }
        }
        if (threadIdx.x == 96) p.tick[tile] = 0;
      }
    } else
    for (int c0 = 0; c0 < p.TN; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), v);
      tmem_wait_ld();
      if (aborted) continue;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = m0 + c0 + j;
        if (m >= p.M) break;  // uniform across the warp
        const float val = __uint_as_float(v[j]);
        float* yr = p.y + static_cast<size_t>(m) * p.ldy;
        if (p.ymode == 3) {
          const float u = __shfl_down_sync(0xffffffffu, val, 1);
          if (!(lane & 1) && nn < p.N) yr[nn >> 1] = val / (1.0f + expf(-val)) * u;
        } else if (nn < p.N) {
          if (p.ymode == 1)
            yr[nn] += val;
          else
            yr[nn] = val;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, p.tmem_cols);
  }
}

// ------------------------------------------------------------------------------------ activation prep
// xp[q][m][k] = bf16 part q of xin(X)[m][k]: xin = X (xmode 0) or silu(X[:, :K]) * X[:, K:2K] (xmode 2), then
// the optional RMSNorm lnw * (xin * rsqrt(mean(X[:, :K]^2) + eps)) (the gemvc1_k prologue, wcomp.py:75-86).
// parts = 1: bf16(xin); parts = 3: x1 = bf16(x), x2 = bf16(x - x1), x3 = bf16(x - x1 - x2), round to nearest.
__global__ void __launch_bounds__(256) prep_kernel(const float* __restrict__ x, int ldx, int M, int K, int xmode,
                                                   const uint16_t* __restrict__ lnw, float eps, int parts,
                                                   uint16_t* __restrict__ xp, int* tick, int ntick) {
  pdl_wait();
  const int m = blockIdx.x;
  if (m == 0)  // the split-K counters of the GEMM that follows (the previous GEMM is complete by now)
    for (int i = threadIdx.x; i < ntick; i += 256) tick[i] = 0;
  const float* xr = x + static_cast<size_t>(m) * ldx;
  float rs = 1.0f;
  if (lnw) {
    __shared__ float red[8];
    float ss = 0.0f;
#pragma unroll 8  // eight loads in flight per thread (a row is 16-48 KB: one round trip per eight)
    for (int k = threadIdx.x; k < K; k += 256) ss += xr[k] * xr[k];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    rs = rsqrtf(tot / static_cast<float>(K) + eps);
  }
  const size_t plane = static_cast<size_t>(M) * K;
  uint16_t* o = xp + static_cast<size_t>(m) * K;
#pragma unroll 8
  for (int k = threadIdx.x; k < K; k += 256) {
    float v = xr[k];
    if (xmode == 2) {
      const float u = xr[K + k];
      v = v / (1.0f + expf(-v)) * u;
    }
    if (lnw) v = bf16_to_f32(lnw[k]) * (v * rs);
    for (int q = 0; q < parts; ++q) {
      const uint16_t b = bf16_rn(v);
      o[q * plane + k] = b;
      v -= bf16_to_f32(b);
    }
  }
  pdl_trigger();
}

static int pick_tn(int M, int parts) {
  const int cap = parts == 3 ? 128 : 256;
  const int m16 = ((M + 15) / 16) * 16;
  if (m16 >= cap) return cap;
  return m16;
}

static uint32_t tmem_cols_for(int TN) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(TN)) c <<= 1;
  return c;
}

constexpr size_t kSmemMax = 227 * 1024;

// Split-K for few tokens (M <= 16: one token tile): the weight tiles alone would leave most SMs idle (N = 4096
// gives 32 tiles), so every tile's K range is split over up to 8 CTAs, at least 4 k-blocks each, about one CTA
// per SM in total. Workspace past the activation parts: [256-aligned] counters, partial tiles.
constexpr int kMaxTicks = 1024;
static int split_k(int M, int N, int K) {
  if (M > 16) return 1;
  const int tiles = (N + BM - 1) / BM, nkb = K / BK;
  int ks = std::max(1, std::min(8, sm_count() / std::max(1, tiles)));
  ks = std::min(ks, std::max(1, nkb / 4));
  if (tiles > kMaxTicks) ks = 1;
  const int per = (nkb + ks - 1) / ks;
  return (nkb + per - 1) / per;
}
static size_t split_bytes(int M) {  // counters + partial tiles (tiles * ks <= SMs; TN = 16)
  if (M > 16) return 0;
  return 256 + kMaxTicks * sizeof(int) + static_cast<size_t>(sm_count()) * BM * 16 * sizeof(float);
}
static size_t prep_bytes(int M, int K, int parts) {
  return ((static_cast<size_t>(parts) * M * K * sizeof(uint16_t) + 255) / 256) * 256;
}

template <int PARTS>
static int launch_gemm(const aib_c12* W, const uint16_t* xp, int M, float* y, int ldy, int ymode, cudaStream_t s,
                       int* tick, float* part) {
  const int N = W->N, K = W->K;
  const int TN = pick_tn(M, PARTS);
  const int o_stage = kATile + PARTS * TN * 128;
  int NW = 4;
  const size_t w_bytes = static_cast<size_t>(NW) * kWStage;
  int NO = static_cast<int>(std::min<size_t>(kMaxNO, (kSmemMax - kHeader - w_bytes) / o_stage));
  if (NO < 2) return fail(AIB_ENOTSUP, "aib_gemm_c12: tile does not fit in shared memory");
  const size_t smem = kHeader + w_bytes + static_cast<size_t>(NO) * o_stage;
  CUtensorMap tm8, tme4, tmx;
  {
    const uint64_t d[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)}, st[1] = {static_cast<uint64_t>(K)};
    const uint32_t box[2] = {64, BM};
    int rc = make_map(&tm8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, W->m8, d, st, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    const uint64_t d2[2] = {static_cast<uint64_t>(K / 2), static_cast<uint64_t>(N)},
                   st2[1] = {static_cast<uint64_t>(K / 2)};
    rc = make_map(&tme4, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, W->e4, d2, st2, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    const uint64_t d3[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint64_t>(PARTS)};
    const uint64_t st3[2] = {static_cast<uint64_t>(K) * 2, static_cast<uint64_t>(M) * K * 2};
    const uint32_t box3[3] = {64, static_cast<uint32_t>(TN), 1};
    rc = make_map(&tmx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, xp, d3, st3, box3, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Params p{};
  p.rp = W->rp;
  p.ec = W->ec;
  p.ev = W->ev;
  p.y = y;
  p.ldy = ldy;
  p.ymode = ymode;
  p.N = N;
  p.K = K;
  p.M = M;
  p.base = W->base;
  p.TN = TN;
  p.NW = NW;
  p.NO = NO;
  p.nkb = K / BK;
  // kind::f16 instruction descriptor: D fp32 (bits 4-5 = 1), A and B bf16 (bits 7-9, 10-12 = 1), both K-major,
  // N >> 3 at bits 17-22, M >> 4 at bits 24-28
  p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(TN >> 3) << 17) |
            (static_cast<uint32_t>(BM >> 4) << 24);
  p.tmem_cols = tmem_cols_for(TN);
  p.w_off = kHeader;
  p.o_off = kHeader + static_cast<int>(w_bytes);
  p.o_stage = o_stage;
  p.k128 = 128u;
  p.k8 = 8u;
  p.ks = split_k(M, N, K);
  p.kb_per = (p.nkb + p.ks - 1) / p.ks;
  p.part = part;
  p.tick = tick;
  const int rc = allow_smem(gemm_c12_kernel<PARTS>, smem);
  if (rc) return rc;
  const dim3 grid((M + TN - 1) / TN, (N + BM - 1) / BM, p.ks);
  return launch(gemm_c12_kernel<PARTS>, grid, dim3(kThreads), smem, s, "aib_gemm_c12", tm8, tme4, tmx, p);
}

}  // namespace gemm
}  // namespace aib

using namespace aib;

extern "C" {

size_t aib_gemm_c12_workspace(int M, int K, int precision) {
  if (M <= 0 || K <= 0 || (precision != 1 && precision != 3)) return 0;
  return gemm::prep_bytes(M, K, precision) + gemm::split_bytes(M);
}

int aib_gemm_c12(const aib_c12* W, const float* X, int M, int ldx, int xmode, const uint16_t* lnw, float eps, float* Y,
                 int ldy, int ymode, int precision, void* ws, size_t ws_bytes, void* stream) {
  if (!W || !X || !Y || !W->m8 || !W->e4 || !W->rp || (W->n_exc > 0 && (!W->ec || !W->ev)))
    return fail(AIB_EINVAL, "aib_gemm_c12: null pointer");
  if (M <= 0 || W->N <= 0 || W->K <= 0 || W->K % 256 || W->CH != 256)
    return fail(AIB_EINVAL, "aib_gemm_c12: bad shape (M=%d N=%d K=%d)", M, W->N, W->K);
  if (xmode != 0 && xmode != 2) return fail(AIB_EINVAL, "aib_gemm_c12: xmode must be 0 or 2");
  if (ymode != 0 && ymode != 1 && ymode != 3) return fail(AIB_EINVAL, "aib_gemm_c12: ymode must be 0, 1 or 3");
  if (ymode == 3 && (W->N & 1)) return fail(AIB_EINVAL, "aib_gemm_c12: ymode 3 needs an even N");
  if (precision != 1 && precision != 3) return fail(AIB_EINVAL, "aib_gemm_c12: precision must be 1 or 3");
  if (ldx < (xmode == 2 ? 2 * W->K : W->K) || ldy < (ymode == 3 ? W->N / 2 : W->N))
    return fail(AIB_EINVAL, "aib_gemm_c12: row strides too small");
  if (W->base < 0 || W->base > 241) return fail(AIB_EINVAL, "aib_gemm_c12: base %d out of range", W->base);
  if ((reinterpret_cast<uintptr_t>(W->m8) & 15) || (reinterpret_cast<uintptr_t>(W->e4) & 15))
    return fail(AIB_EINVAL, "aib_gemm_c12: m8/e4 must be 16-byte aligned");
  if (!ws || ws_bytes < aib_gemm_c12_workspace(M, W->K, precision) || (reinterpret_cast<uintptr_t>(ws) & 15))
    return fail(AIB_EWORKSPACE, "aib_gemm_c12: workspace %zu < %zu bytes", ws_bytes,
                aib_gemm_c12_workspace(M, W->K, precision));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint16_t* xp = static_cast<uint16_t*>(ws);
  uint8_t* sk = static_cast<uint8_t*>(ws) + gemm::prep_bytes(M, W->K, precision);
  int* tick = M <= 16 ? reinterpret_cast<int*>(sk + 256) : nullptr;
  float* part = M <= 16 ? reinterpret_cast<float*>(sk + 256 + gemm::kMaxTicks * sizeof(int)) : nullptr;
  int rc = launch(gemm::prep_kernel, dim3(M), dim3(256), 0, s, "aib_gemm_c12 (prep)", X, ldx, M, W->K, xmode, lnw,
                  eps, precision, xp, tick, tick ? gemm::kMaxTicks : 0);
  if (rc) return rc;
  return precision == 3 ? gemm::launch_gemm<3>(W, xp, M, Y, ldy, ymode, s, tick, part)
                        : gemm::launch_gemm<1>(W, xp, M, Y, ldy, ymode, s, tick, part);
}

}  // extern "C"
