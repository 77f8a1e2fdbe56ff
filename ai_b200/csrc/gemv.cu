// Codec GEMV: y (+)= W x with W in the 12-bit codec, decoded on the fly (sm_100a).
//
// Replaces the reference's gemvc1_k (T = 1, `ramvi/engine/ramvi_engine/kernels/wcomp.py:67-112`) and
// gemvc_tc_k (1 < T <= 16, wcomp.py:155-219). Same modes: 0: y = Wx; 1: y += Wx; 2: input silu(x[:K]) *
// x[K:2K], y += Wx; optional RMSNorm prologue for T = 1.
//
// Design (HBM-bound: 1.5 bytes/weight + exceptions):
//  * Weight stream: a dedicated producer warp issues 3-D TMA tile loads of the m8 and e4 planes (viewed as
//    [N][K/256][256] and [N][K/256][128]) into a ring of shared-memory stages, one mbarrier pair per stage.
//    A stage is RT rows x CW 256-column chunks (RT*CW = 32): 8 KB of m8 + 4 KB of e4. The producer never
//    waits on the previous kernel (PDL), so the ring fills with this kernel's weights while the previous
//    kernel drains.
//  * 256 consumer threads: thread t owns unit j = t%8 (columns 16j..16j+15 and 128+16j..128+16j+15 of a
//    chunk: one 16-byte e4 vector carries both nibble halves), chunk slot cc and row slot r. Each unit is
//    decoded with byte permutes into packed bf16 pairs (bf16 = sign<<15 | (code+base)<<7 | mantissa), split
//    into fp32 and accumulated with packed fp32 FMA (fma.rn.f32x2): exact bf16 weights times fp32 x, fp32
//    accumulation, like the reference.
//  * x (after the RMS / SiLU prologue) lives in shared memory in a permuted order so every 16-byte read of a
//    warp is bank-conflict free; for T > 1 the x columns of each stage are staged per stage.
//  * Exceptions: a unit that contains a code-15 element (found from the CSR, never by scanning the data) is
//    decoded by a slow path that zeroes those elements and adds their fp32 values times x in place.
//  * Per row tile the partial sums are reduced in a fixed order (shuffles, then chunk slots), so the result
//    is deterministic run to run.
//  * Every wait is bounded. On a timeout each consumer keeps walking the same sequence of named barriers
//    (skipping its work), so no thread is ever left at a barrier the others do not reach.
#include <algorithm>
#include <climits>
#include "common.cuh"

#ifndef AIB_GEMV_EARLY
#define AIB_GEMV_EARLY 1  // issue the ring's first stages before the CTA's shared prologue
#endif
#ifndef AIB_GEMV_LOWNIB2
#define AIB_GEMV_LOWNIB2 0  // low-nibble codes with one mask and one multiply-add (instead of two multiply-adds)
#endif
#ifndef AIB_GEMV_EVICT_FIRST
#define AIB_GEMV_EVICT_FIRST 1  // weight copies with an L2 evict-first policy
#endif
#ifndef AIB_GEMV_ACC
#define AIB_GEMV_ACC 2  // accumulator chains per consumer warp in the tensor-core T = 1 kernel (2 or 4)
#endif

namespace aib {
namespace gemv {

constexpr int kConsumers = 256;            // 8 consumer warps
constexpr int kThreads = kConsumers + 32;  // + 1 producer warp
constexpr int kStageM8 = 32 * 256;         // bytes of m8 per stage (RT*CW*256)
constexpr int kStageE4 = 32 * 128;
constexpr int kStageBytes = kStageM8 + kStageE4;
constexpr int kHeader = 1024;  // barriers, flags, reduction buffers

struct Params {
  const int32_t* rp;
  const int32_t* ec;
  const float* ev;
  const float* x;
  float* y;
  const uint16_t* lnw;
  float eps;
  int base, N, K, nch;
  int RT, CW, KS, tiles;
  int NS;
  int T, x_stride, y_stride;
  int xs_floats;
  int meta_rows;  // rows per CTA covered by the shared row-metadata arrays (tensor-core kernel)
  int ring_off;   // byte offset of the stage ring in shared memory (tensor-core kernel)
};

// permuted index of column k in the shared x buffer (see file comment)
AIB_DEV int xperm(int k) {
  const int c = k >> 8, hf = (k >> 7) & 1, jj = (k >> 4) & 7, q = (k >> 2) & 3, e = k & 3;
  return ((c * 2 + hf) * 4 + q) * 32 + jj * 4 + e;
}

AIB_DEV float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// What the wide kernels' decode makes of an exception (exponent code 15): sign and mantissa from its m8
// byte, exponent field (base + 15) mod 256 (the select-merge below drops the carry). Finite for base < 240.
AIB_DEV float exc_garbage(uint32_t m, int base) {
  return __uint_as_float((((m & 0x80u) << 8) | (((static_cast<uint32_t>(base) + 15u) & 0xFFu) << 7) | (m & 0x7Fu)) << 16);
}

// (a & 0x807F807F) | (b & 0x7F807F80) in one LOP3: sign and mantissa bits from a, exponent field from b
AIB_DEV uint32_t merge_sm_e(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(a), "r"(b), "r"(0x807F807Fu));
  return r;
}


// Decode one 32-element unit (fast path: no code-15 element) and accumulate w * x.
AIB_DEV void unit_fast(const uint4& ml, const uint4& mh, const uint4& ee, const float4* xl, const float4* xh,
                       uint32_t base7, float2& acc) {
  const uint32_t E[4] = {ee.x, ee.y, ee.z, ee.w};
  const uint32_t L[4] = {ml.x, ml.y, ml.z, ml.w};
  const uint32_t Hh[4] = {mh.x, mh.y, mh.z, mh.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t x01 = prmt(E[q], 0u, 0x4140u);  // [0, b1, 0, b0]
    const uint32_t x23 = prmt(E[q], 0u, 0x4342u);  // [0, b3, 0, b2]
    const uint32_t plo01 = ((x01 & 0x000F000Fu) << 7) + base7;
    const uint32_t phi01 = ((x01 & 0x00F000F0u) << 3) + base7;
    const uint32_t plo23 = ((x23 & 0x000F000Fu) << 7) + base7;
    const uint32_t phi23 = ((x23 & 0x00F000F0u) << 3) + base7;
    // [sign-rep(m1), m1, sign-rep(m0), m0] -> keep bit 15 and bits 0..6 of each half
    const uint32_t zlo01 = (prmt(L[q], 0u, 0x9180u) & 0x807F807Fu) | plo01;
    const uint32_t zlo23 = (prmt(L[q], 0u, 0xB3A2u) & 0x807F807Fu) | plo23;
    const uint32_t zhi01 = (prmt(Hh[q], 0u, 0x9180u) & 0x807F807Fu) | phi01;
    const uint32_t zhi23 = (prmt(Hh[q], 0u, 0xB3A2u) & 0x807F807Fu) | phi23;
    acc = ffma2(make_float2(__uint_as_float(zlo01 << 16), __uint_as_float(zlo01 & 0xFFFF0000u)),
                make_float2(xl[q].x, xl[q].y), acc);
    acc = ffma2(make_float2(__uint_as_float(zlo23 << 16), __uint_as_float(zlo23 & 0xFFFF0000u)),
                make_float2(xl[q].z, xl[q].w), acc);
    acc = ffma2(make_float2(__uint_as_float(zhi01 << 16), __uint_as_float(zhi01 & 0xFFFF0000u)),
                make_float2(xh[q].x, xh[q].y), acc);
    acc = ffma2(make_float2(__uint_as_float(zhi23 << 16), __uint_as_float(zhi23 & 0xFFFF0000u)),
                make_float2(xh[q].z, xh[q].w), acc);
  }
}

// Same decode, accumulated with scalar FMAs into four independent chains (shorter dependency chains and no
// register-pair packing; the four partial sums are added at the end of the row).
AIB_DEV void unit_fast4(const uint4& ml, const uint4& mh, const uint4& ee, const float4* xl, const float4* xh,
                        uint32_t base7, float4& a) {
  const uint32_t E[4] = {ee.x, ee.y, ee.z, ee.w};
  const uint32_t L[4] = {ml.x, ml.y, ml.z, ml.w};
  const uint32_t Hh[4] = {mh.x, mh.y, mh.z, mh.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t x01 = prmt(E[q], 0u, 0x4140u);
    const uint32_t x23 = prmt(E[q], 0u, 0x4342u);
    const uint32_t zlo01 = (prmt(L[q], 0u, 0x9180u) & 0x807F807Fu) | (((x01 & 0x000F000Fu) << 7) + base7);
    const uint32_t zlo23 = (prmt(L[q], 0u, 0xB3A2u) & 0x807F807Fu) | (((x23 & 0x000F000Fu) << 7) + base7);
    const uint32_t zhi01 = (prmt(Hh[q], 0u, 0x9180u) & 0x807F807Fu) | (((x01 & 0x00F000F0u) << 3) + base7);
    const uint32_t zhi23 = (prmt(Hh[q], 0u, 0xB3A2u) & 0x807F807Fu) | (((x23 & 0x00F000F0u) << 3) + base7);
    a.x = fmaf(__uint_as_float(zlo01 << 16), xl[q].x, a.x);
    a.y = fmaf(__uint_as_float(zlo01 & 0xFFFF0000u), xl[q].y, a.y);
    a.z = fmaf(__uint_as_float(zlo23 << 16), xl[q].z, a.z);
    a.w = fmaf(__uint_as_float(zlo23 & 0xFFFF0000u), xl[q].w, a.w);
    a.x = fmaf(__uint_as_float(zhi01 << 16), xh[q].x, a.x);
    a.y = fmaf(__uint_as_float(zhi01 & 0xFFFF0000u), xh[q].y, a.y);
    a.z = fmaf(__uint_as_float(zhi23 << 16), xh[q].z, a.z);
    a.w = fmaf(__uint_as_float(zhi23 & 0xFFFF0000u), xh[q].w, a.w);
  }
}

AIB_DEV float dec1(uint32_t m, uint32_t code, uint32_t base) {
  if (code == 15u) return 0.0f;
  return __uint_as_float(((m & 0x80u) << 24) | ((code + base) << 23) | ((m & 0x7Fu) << 16));
}

// Bounded consumer wait on a full-stage barrier; gives up early once another thread has aborted.
AIB_DEV bool wait_full(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case reads no limit
  for (uint32_t i = 0, lim = spin_limit(); i < lim; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && *abort_flag) return false;
  }
  set_status(AIB_DEV_TIMEOUT_FULL);
  *abort_flag = 1;
  return false;
}

// Does the 32-element unit (row's CSR slice, chunk starting at column c0) hold an exception?
// ex_p / ex_col track the first exception of the row at or after the current chunk.
AIB_DEV bool unit_has_exc(const int32_t* ec, int& ex_p, int ex_e, int& ex_col, int c0, uint32_t j) {
  while (ex_col < c0) {
    ++ex_p;
    ex_col = ex_p < ex_e ? ec[ex_p] : INT_MAX;
  }
  for (int q = ex_p; q < ex_e; ++q) {
    const int col = (q == ex_p) ? ex_col : ec[q];
    if (col >= c0 + 256) break;
    const uint32_t o = static_cast<uint32_t>(col - c0);
    if (col >= c0 && ((o & 127u) >> 4) == j) return true;
  }
  return false;
}

// ------------------------------------------------------------------------------ shared producer
// One elected thread streams the CTA's (tile, stage) sequence through the ring.
AIB_DEV void produce(const CUtensorMap* tm8, const CUtensorMap* tme4, uint8_t* ring, uint64_t* full, uint64_t* empty,
                     volatile int* abort_flag, int tb, int n_it, int KS, int RT, int CW, int NS) {
  prefetch_tensormap(tm8);
  prefetch_tensormap(tme4);
  int issued = 0;
  for (int it = 0; it < n_it; ++it) {
    const int s = it % NS;
    if (it >= NS) {
      bool ok = false;
      for (uint32_t i = 0, lim = spin_limit(); i < lim && !ok; ++i) {
        ok = mbar_try_wait(&empty[s], ((it / NS) - 1) & 1);
        if (!ok && *abort_flag) break;
      }
      if (!ok) {
        if (!*abort_flag) set_status(AIB_DEV_TIMEOUT_EMPTY);
        *abort_flag = 1;
        break;
      }
    }
    const int tile = tb + it / KS, ks = it % KS;
    uint8_t* st = ring + static_cast<size_t>(s) * kStageBytes;
    mbar_arrive_expect_tx(&full[s], kStageBytes);
    tma_load_3d(st, tm8, &full[s], 0, ks * CW, tile * RT);
    tma_load_3d(st + kStageM8, tme4, &full[s], 0, ks * CW, tile * RT);
    issued = it + 1;
  }
  // Never leave with copies in flight: on the abort path wait (bounded) for the stages this thread issued
  // that the consumers may not have observed. In the normal path all of them were consumed.
  if (*abort_flag) {
    for (int it = (issued > NS ? issued - NS : 0); it < issued; ++it)
      mbar_wait(&full[it % NS], (it / NS) & 1, AIB_DEV_TIMEOUT_FULL);
  }
}

AIB_DEV void init_barriers(uint64_t* full, uint64_t* empty, volatile int* abort_flag, int NS) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers / 32);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------ T = 1 kernel
// 16 consumer warps in two groups of 8; group g consumes the CTA's tiles g, g+2, g+4, ... (the producer
// interleaves the two groups' stages in the ring). Within a stage a warp owns whole row(s): lane = (row r,
// chunk slot cc, unit j) with the CW chunk slots of a row in the same warp, so a row reduces with shuffles
// and no CTA-wide barrier runs in the main loop.
constexpr int kT1Consumers = 512;
constexpr int kT1Threads = kT1Consumers + 32;

AIB_DEV void produce_pairs(const CUtensorMap* tm8, const CUtensorMap* tme4, uint8_t* ring, uint64_t* full,
                           uint64_t* empty, volatile int* abort_flag, int tb, int ntiles, int KS, int RT, int CW,
                           int NS, uint32_t stage_bytes, uint32_t e4_off) {
  // Half h owns ring slots h, h+2, h+4, ...; its j-th stage (tile 2*(j/KS)+h, chunk group j%KS) goes to slot
  // h + 2*(j % (NS/2)), use j / (NS/2). The two halves are served in whatever order their slots free up, so
  // a lagging half never starves the other.
  prefetch_tensormap(tm8);
  prefetch_tensormap(tme4);
  const int per = NS / 2;
  int n[2] = {((ntiles + 1) / 2) * KS, (ntiles / 2) * KS};
  int j[2] = {0, 0};
  uint32_t idle = 0;
  while ((j[0] < n[0] || j[1] < n[1]) && !*abort_flag) {
    bool progressed = false;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (j[h] >= n[h]) continue;
      const int s = h + 2 * (j[h] % per), use = j[h] / per;
      if (use > 0 && !mbar_test_wait(&empty[s], (use - 1) & 1)) continue;
      const int tile = tb + 2 * (j[h] / KS) + h, ks = j[h] % KS;
      uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_3d(st, tm8, &full[s], 0, ks * CW, tile * RT);
      tma_load_3d(st + e4_off, tme4, &full[s], 0, ks * CW, tile * RT);
      ++j[h];
      progressed = true;
    }
    idle = progressed ? 0 : idle + 1;
    if (!progressed) __nanosleep(64);  // both halves full: back off instead of taking issue slots from them
    if (idle > spin_limit()) {
      set_status(AIB_DEV_TIMEOUT_EMPTY);
      *abort_flag = 1;
    }
  }
  // Never leave with copies in flight: on the abort path wait (bounded) for the last issued use of every slot.
  if (*abort_flag) {
    for (int h = 0; h < 2; ++h)
      for (int k = (j[h] > per ? j[h] - per : 0); k < j[h]; ++k)
        mbar_wait(&full[h + 2 * (k % per)], (k / per) & 1, AIB_DEV_TIMEOUT_FULL);
  }
}

template <int MODE, bool RMS>
__global__ void __launch_bounds__(kT1Threads, 1)
    gemv_t1_kernel(const __grid_constant__ CUtensorMap tm8, const __grid_constant__ CUtensorMap tme4, Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 16;  // up to 16 ring slots
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 256);
  float* red = reinterpret_cast<float*>(smem + 512);  // RMS partials
  float* xs = reinterpret_cast<float*>(smem + kHeader);
  uint8_t* ring = smem + kHeader + ((p.xs_floats * 4 + 1023) / 1024) * 1024;

  const int tid = threadIdx.x;
  const int tb = static_cast<int>((static_cast<long long>(blockIdx.x) * p.tiles) / gridDim.x);
  const int te = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * p.tiles) / gridDim.x);
  const int ntiles = te - tb;

  if (tid == 0) {
    for (int s = 0; s < p.NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 8);  // the 8 warps of the consuming group
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();

  if (tid >= kT1Consumers) {  // producer warp
    if (tid == kT1Consumers)
      produce_pairs(&tm8, &tme4, ring, full, empty, abort_flag, tb, ntiles, p.KS, p.RT, p.CW, p.NS, kStageBytes,
                    kStageM8);
    return;
  }

  // -------- consumers: x prologue shared by both groups
  pdl_wait();  // x / y are produced / consumed by neighbouring kernels
  const int K = p.K;
  float rs = 1.0f;
  if (RMS) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += kT1Consumers) {
      const float v = p.x[k];
      ss += v * v;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    named_sync(1, kT1Consumers);
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kT1Consumers / 32; ++w) tot += red[w];
    rs = rsqrtf(tot / static_cast<float>(K) + p.eps);
  }
  for (int k = tid; k < K; k += kT1Consumers) {
    float v = (MODE == 2) ? silu_mul(p.x[k], p.x[K + k]) : p.x[k];
    if (RMS) v = bf16_to_f32(p.lnw[k]) * (v * rs);
    xs[xperm(k)] = v;
  }
  named_sync(1, kT1Consumers);

  const int grp = tid >> 8, gt = tid & 255;  // group, thread within group
  const int j = gt & 7, slot = gt >> 3;      // slot = r * CW + cc
  const int CW = p.CW, cc = slot % CW, r = slot / CW;
  const uint32_t base7 = (static_cast<uint32_t>(p.base) << 7) | (static_cast<uint32_t>(p.base) << 23);
  const int my_tiles = grp == 0 ? (ntiles + 1) / 2 : ntiles / 2;
  const int m8_off = slot * 256 + 16 * j, e4_off = kStageM8 + slot * 128 + 16 * j;
  bool aborted = false;

  for (int ti = 0; ti < my_tiles; ++ti) {
    const int tile = tb + 2 * ti + grp;
    const int row = tile * p.RT + r;
    int ex_p = 0, ex_e = 0;
    if (row < p.N) {
      ex_p = p.rp[row];
      ex_e = p.rp[row + 1];
    }
    int ex_col = ex_p < ex_e ? p.ec[ex_p] : INT_MAX;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (int ks = 0; ks < p.KS; ++ks) {
      const int it = 2 * (ti * p.KS + ks) + grp;
      const int s = it % p.NS;
      const bool ok = !aborted && wait_full(&full[s], (it / p.NS) & 1, abort_flag);
      if (!ok) aborted = true;
      const int gc = ks * CW + cc;
      if (ok && row < p.N && gc < p.nch) {
        const uint8_t* st = ring + static_cast<size_t>(s) * kStageBytes;
        const uint4 ml = *reinterpret_cast<const uint4*>(st + m8_off);
        const uint4 mh = *reinterpret_cast<const uint4*>(st + m8_off + 128);
        const uint4 ee = *reinterpret_cast<const uint4*>(st + e4_off);
        const float4* xb = reinterpret_cast<const float4*>(xs) + gc * 64;
        float4 xl[4], xh[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          xl[q] = xb[q * 8 + j];
          xh[q] = xb[32 + q * 8 + j];
        }
        const int c0 = gc * 256;
        if (!unit_has_exc(p.ec, ex_p, ex_e, ex_col, c0, j)) {
          unit_fast4(ml, mh, ee, xl, xh, base7, acc);
        } else {
          const uint32_t E[4] = {ee.x, ee.y, ee.z, ee.w}, L[4] = {ml.x, ml.y, ml.z, ml.w},
                         Hh[4] = {mh.x, mh.y, mh.z, mh.w};
          const float* xlf = reinterpret_cast<const float*>(xl);
          const float* xhf = reinterpret_cast<const float*>(xh);
          float sacc = 0.0f;
          for (int q = 0; q < 4; ++q)
            for (int b = 0; b < 4; ++b) {
              const uint32_t eb = (E[q] >> (8 * b)) & 0xFFu;
              sacc += dec1((L[q] >> (8 * b)) & 0xFFu, eb & 15u, p.base) * xlf[q * 4 + b];
              sacc += dec1((Hh[q] >> (8 * b)) & 0xFFu, eb >> 4, p.base) * xhf[q * 4 + b];
            }
          for (int q = ex_p; q < ex_e; ++q) {
            const int col = p.ec[q];
            if (col >= c0 + 256) break;
            const uint32_t o = static_cast<uint32_t>(col - c0);
            if (col >= c0 && ((o & 127u) >> 4) == static_cast<uint32_t>(j)) sacc += p.ev[q] * xs[xperm(col)];
          }
          acc.x += sacc;
        }
      }
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(&empty[s]);
    }
    // row complete: fixed-order reduction inside the warp (units, then chunk slots)
    float v = (acc.x + acc.y) + (acc.z + acc.w);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    for (int o = 8; o < 8 * CW; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (j == 0 && cc == 0 && row < p.N && !aborted) {
      if (MODE == 0)
        p.y[row] = v;
      else
        p.y[row] += v;
    }
  }
}

// ------------------------------------------- the tensor-core wide-stage kernel's exception table
struct ExcTab {  // the CTA's exceptions: CSR slice in shared memory (columns + corrections) or in global memory
  const int* rps;   // row pointers of the CTA's rows (shared)
  const int* ecs;   // staged columns (shared), valid when staged
  const float* evs; // staged corrections v - G (shared), valid when staged
  bool staged;
  int e0, row0;
  const int32_t* ec;
  const float* ev;
  const uint8_t* m8;
  int K, base;
};
// ------------------------------------------- producer and finisher warps of the tensor-core wide-stage kernel
// The producer only streams: one thread issues stage i (two 3-D TMA copies, m8 and e4, no multicast) as soon as
// its slot's previous stage has been consumed; a slot's full barrier completes on that one arrival plus the
// copied bytes. Stages below `first` were issued before the CTA's prologue. A wait that runs out raises the
// abort flag and, before returning, waits (bounded) for the copies still in flight.
// Bounded wait until the copies into the last min(NS, n) issued stages (launch-wide indices < n) have landed, so
// no copy is in flight into shared memory when the CTA exits after an abort.
AIB_DEV void drain_ring(uint64_t* full, int n, int NS) {
  for (int k = max(0, n - NS); k < n; ++k) mbar_wait(&full[k % NS], (k / NS) & 1, AIB_DEV_TIMEOUT_FULL);
}

// i0: stages this ring streamed before (slots and phases follow the stage index i0 + i). Stops issuing when any
// role has raised the abort flag, and then waits for the copies in flight. False when aborted.
AIB_DEV bool issue_stages(const CUtensorMap* tm8, const CUtensorMap* tme4, uint8_t* ring, uint64_t* full,
                          uint64_t* empty, volatile int* abort_flag, int tb, int ks0, int n_st, int first, int R,
                          int CW, int KS, int NS, uint32_t stage_bytes, int i0 = 0) {
  if (g_aib_withhold_copies) return true;
  const uint32_t m8_bytes = static_cast<uint32_t>(R * CW * 256);
  const uint64_t pol = l2_evict_first();
  int ks = ks0 + first, tile = tb;
  tile += ks / KS;
  ks %= KS;
  for (int i = first; i < n_st; ++i) {
    const int gi = i0 + i, s = gi % NS;
    bool ok = true;
    if (gi >= NS) {
      const uint32_t par = ((gi / NS) - 1) & 1;
      ok = mbar_try_wait(&empty[s], par);
      for (uint32_t k = 0, lim = ok ? 0u : spin_limit(); k < lim && !ok; ++k) {
        ok = mbar_try_wait(&empty[s], par);
        if (!ok && (k & 63) == 63 && *abort_flag) break;
      }
      if (!ok && !*abort_flag) set_status(AIB_DEV_TIMEOUT_EMPTY);
    }
    // checked after the wait: aborted consumers release slots without waiting for their copies, so a slot freed
    // after an abort may still be filling and must not be reused
    if (ok && *abort_flag) ok = false;
    if (!ok) {
      *abort_flag = 1;
      drain_ring(full, gi, NS);
      return false;
    }
    uint8_t* st = ring + static_cast<size_t>(s) * stage_bytes;
    mbar_arrive_expect_tx(&full[s], stage_bytes);
    if (AIB_GEMV_EVICT_FIRST) {
      tma_load_3d_hint(st, tm8, &full[s], 0, ks * CW, tile * R, pol);
      tma_load_3d_hint(st + m8_bytes, tme4, &full[s], 0, ks * CW, tile * R, pol);
    } else {
      tma_load_3d(st, tm8, &full[s], 0, ks * CW, tile * R);
      tma_load_3d(st + m8_bytes, tme4, &full[s], 0, ks * CW, tile * R);
    }
    if (++ks == KS) ks = 0, ++tile;
  }
  return true;
}

// Byte offset of the x record (8 bytes: low pair, high pair) for chunk gc, MMA i, lane quad t, column block
// blk and part sp. Parts 0 and 1 of all (blk, t) form one 128-byte line per (gc, i) and part 2 a 64-byte line
// in a second region (nch*8*128 bytes further), so each half-warp's 8-byte loads hit 16 distinct bank pairs.
AIB_DEV int tc_xrec(int nch, int gc, int i, int blk, int t, int sp) {
  const int gi = gc * 8 + i;
  return sp < 2 ? gi * 128 + (blk * 2 + sp) * 32 + t * 8 : nch * 1024 + gi * 64 + blk * 32 + t * 8;
}
// Column (chunk * 256 + c, c < 128; the record also holds c + 1, 128 + c, 129 + c) of prologue record pr. Within a
// chunk's 64 records the order is (i, blk, t) from slow to fast, so the 16 lanes of a half-warp building
// consecutive records store to 16 distinct 8-byte slots of the record lines (no shared-memory bank conflicts).
AIB_DEV int tc_rec_col(int pr) {
  const int l6 = pr & 63;
  return (pr >> 6) * 256 + ((l6 >> 2) & 1) * 64 + (l6 & 3) * 16 + (l6 >> 3) * 2;
}
// Exact value of x[col] from its three bf16 parts in the records.
AIB_DEV float tc_xval(const uint8_t* xr, int nch, int col) {
  const int gc = col >> 8, cc = col & 255, hf = cc >> 7, c = cc & 127;
  const int b2 = c >> 6, t2 = (c >> 4) & 3, i2 = (c & 15) >> 1, sh = (c & 1) * 16;
  float parts[3];
#pragma unroll
  for (int s2 = 0; s2 < 3; ++s2) {
    const uint32_t wv = *reinterpret_cast<const uint32_t*>(xr + tc_xrec(nch, gc, i2, b2, t2, s2) + hf * 4);
    parts[s2] = bf16_to_f32(static_cast<uint16_t>(wv >> sh));
  }
  return (parts[0] + parts[1]) + parts[2];
}

struct TcXval {  // x[col] of the tensor-core kernel's three-part records
  const uint8_t* xr;
  int nch;
  AIB_DEV float operator()(int col) const { return tc_xval(xr, nch, col); }
};

// Exception correction of tile-local row lr over the columns [lo, hi): sum_e (v_e - G_e) * x[c_e] in column order
// (the consumers decode every element, exceptions included, as a finite stand-in G_e -- see exc_garbage).
AIB_DEV float row_correction(const ExcTab& et, TcXval xval, int lr, int row, int lo, int hi) {
  const int qa = et.rps[lr] - et.e0, qb = et.rps[lr + 1] - et.e0;
  float corr = 0.0f;
  for (int q = qa; q < qb; ++q) {
    const int col = et.staged ? et.ecs[q] : et.ec[et.e0 + q];
    if (col >= hi) break;
    if (col < lo) continue;
    const float d = et.staged ? et.evs[q]
                              : et.ev[et.e0 + q] - exc_garbage(et.m8[static_cast<size_t>(row) * et.K + col], et.base);
    corr = fmaf(d, xval(col), corr);
  }
  return corr;
}

// Writes finished row values (lane r < R: row `row`): mode 0 stores, modes 1 / 2 add to y (yold: y[row] read
// ahead, when use_yold), mode 3 stores silu(gate) * up of the lane pairs (2i, 2i + 1). Warp-wide.
template <int MODE>
AIB_DEV void store_rows(float v, float yold, bool use_yold, int row, int R, int N, float* y) {
  const int lane = threadIdx.x & 31;
  if (MODE == 3) {
    const float vu = __shfl_down_sync(0xffffffffu, v, 1);
    if (lane < R && !(lane & 1) && row + 1 < N) y[row >> 1] = silu_mul(v, vu);
  } else if (lane < R && row < N) {
    if (MODE == 0)
      y[row] = v;
    else
      y[row] = (use_yold ? yold : y[row]) + v;
  }
}

// The finisher warp stages the CTA's slice of the exception CSR (weights only, so before the grid-dependency
// wait, and off the consumers' path): the row pointers, then each exception's column and correction v - G (G:
// what the decode makes of the element, from its m8 byte). Every batch issues all its loads (8 per lane) before
// using any, so it costs one memory round trip. False when the exceptions do not fit (ecap): the finish then
// reads them from global memory.
AIB_DEV bool stage_csr_warp(int* rps, int* ecs, float* evs, int ecap, int nrows, int row0, const int32_t* rp,
                            const int32_t* ec, const float* ev, const uint8_t* m8, int K, int base) {
  const int lane = threadIdx.x & 31;
  for (int b0 = 0; b0 <= nrows; b0 += 256) {
    int v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = b0 + lane + 32 * u;
      v[u] = i <= nrows ? rp[row0 + i] : 0;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = b0 + lane + 32 * u;
      if (i <= nrows) rps[i] = v[u];
    }
  }
  __syncwarp();
  const int e0 = rps[0], n_exc = rps[nrows] - e0;
  if (n_exc > ecap) return false;
  for (int b0 = 0; b0 < n_exc; b0 += 256) {
    int col[8], lr[8];
    float val[8];
    uint32_t mb[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = b0 + lane + 32 * u;
      col[u] = 0;
      val[u] = 0.0f;
      if (q < n_exc) {
        col[u] = ec[e0 + q];
        val[u] = ev[e0 + q];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {  // the exception's row: the last one whose CSR range starts at or before q
      const int q = b0 + lane + 32 * u;
      int lo = 0, hi = nrows - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (rps[mid] - e0 <= q)
          lo = mid;
        else
          hi = mid - 1;
      }
      lr[u] = lo;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = b0 + lane + 32 * u;
      mb[u] = q < n_exc ? m8[static_cast<size_t>(row0 + lr[u]) * K + col[u]] : 0u;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = b0 + lane + 32 * u;
      if (q < n_exc) {
        ecs[q] = col[u];
        evs[q] = val[u] - exc_garbage(mb[u], base);
      }
    }
  }
  __syncwarp();
  return true;
}

// The finisher warp walks the consumers' segments (maximal runs of one tile's stages). At the j-th segment end
// the consumer warps have left one partial per (row, warp) in buffer j & 1 (float [R][pw]) and arrived on
// ready[j & 1]; the finisher adds each row's pw partials in warp order, releases the buffer (free[j & 1]: the
// consumers reuse it at segment end j + 2), adds the exception correction and writes y. A whole tile's
// correction and (modes 1, 2) the y it adds to are computed / read before the wait, once the consumers have
// published the x records (xready), so that only the partial sums and the store follow the consumers' last
// stage. Two buffers: the consumers wait only when the finisher is two segments behind.
//
// Stream-K (a workspace: the grid splits the tiles * KS stages evenly, so a tile may be split between
// neighbouring CTAs bf..bl): CTA bf holds the tile's head as the last segment of its range and finishes the tile;
// each other part (CTAs bf+1..bl: the tile is the first segment of their ranges, so they publish it early) goes,
// exception corrections of its columns included, to the workspace slot [tile][b - bf - 1] with a release flag.
// CTA bf reads those parts while its own last stages are still in flight (they are normally published by then),
// adds them after its own part in CTA order (deterministic), resets the flags for the next launch and writes y.
// A CTA only ever waits for higher-numbered CTAs, and only for work they do first.
// j: segment ends finished before (updated), xpar: the xready parity. False when the work was abandoned (a wait
// ran out or another role aborted).
template <int MODE>
AIB_DEV bool finish_segments(const float* pbuf, int pstride, uint64_t* ready, uint64_t* free_, uint64_t* xready,
                             volatile int* abort_flag, const ExcTab& et, TcXval xval, float* y, int N, int tb, int ks0,
                             int n_st, int R, int CW, int KS, int nrows, int pw, float* wsp, int* wsc, int maxp,
                             int tiles, int& j, uint32_t xpar = 0) {
  const int lane = threadIdx.x & 31;
  pdl_wait();  // y is read (modes 1, 2) and written after the previous kernel's
  // bounded wait on a barrier that lane 0 polls; false (abort raised) when it runs out or another role aborted
  auto wait_bar = [&](uint64_t* bar, uint32_t par) -> bool {
    int ok = 1;
    if (lane == 0) {
      ok = mbar_try_wait(bar, par);
      for (uint32_t k = 0, lim = ok ? 0u : spin_limit(); k < lim && !ok; ++k) {
        ok = mbar_try_wait(bar, par);
        if (!ok && (k & 63) == 63 && *abort_flag) break;
      }
      if (!ok) {
        if (!*abort_flag) set_status(AIB_DEV_TIMEOUT_FULL);
        *abort_flag = 1;
      }
      if (*abort_flag) ok = 0;
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
  };
  if (!wait_bar(xready, xpar)) return false;
  const long long nall = static_cast<long long>(tiles) * KS, G = gridDim.x;
  const int b = static_cast<int>(blockIdx.x);
  int ks = ks0, tile = tb;
  for (int i = 0; i < n_st;) {
    const int len = min(KS - ks, n_st - i), fks = ks + len - 1;
    const bool whole = ks == 0 && fks == KS - 1;
    const int pb = j & 1, lr = (tile - tb) * R + lane, row = tile * R + lane;
    const bool has_row = lane < R && lr < nrows;
    float corr = 0.0f;
    if (has_row) corr = row_correction(et, xval, lr, row, ks * CW * 256, (fks + 1) * CW * 256);
    const bool use_yold = (MODE == 1 || MODE == 2) && (whole || ks == 0);
    const float yold = use_yold && lane < R && row < N ? __ldcg(y + row) : 0.0f;
    // a split tile's head (ks == 0): this CTA finishes it; the other parts are read before its own partial
    float other = 0.0f;
    if (!whole && ks == 0) {
      const long long st0 = static_cast<long long>(tile) * KS;
      const int np = static_cast<int>(((st0 + KS) * G + nall - 1) / nall - 1) - b;  // parts of CTAs b+1..bl
      const int* flags = wsc + static_cast<size_t>(tile) * maxp;
      bool ok = true;
      for (int pi = 0; pi < np && ok; ++pi) {  // all lanes poll (acquire for each lane's reads below)
        ok = ld_acquire_gpu(flags + pi) == 1;
        for (uint32_t k = 0, lim = ok ? 0u : spin_limit(); k < lim && !ok; ++k) {
          ok = ld_acquire_gpu(flags + pi) == 1;
          if (!ok && (k & 63) == 63 && *abort_flag) break;
        }
      }
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) {
          if (!*abort_flag) set_status(AIB_DEV_TIMEOUT_FULL);
          *abort_flag = 1;
        }
        return false;
      }
      const float* parts = wsp + static_cast<size_t>(tile) * maxp * R;
      if (lane < R)
        for (int pi = 0; pi < np; ++pi) other += __ldcg(parts + pi * R + lane);
      __syncwarp();
      for (int pi = lane; pi < np; pi += 32) wsc[static_cast<size_t>(tile) * maxp + pi] = 0;  // next launch
    }
    if (!wait_bar(&ready[pb], (j >> 1) & 1)) return false;
    float v = 0.0f;
    if (lane < R) {
      const float* pp = pbuf + pb * pstride + lane * pw;
      v = pp[0];
      for (int w = 1; w < pw; ++w) v += pp[w];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&free_[pb]);
    if (has_row) v += corr;
    if (whole || ks == 0) {
      store_rows<MODE>(v + other, yold, use_yold, row, R, N, y);
    } else {  // a later part of a tile whose head a lower-numbered CTA holds
      const long long st0 = static_cast<long long>(tile) * KS;
      const int bf = static_cast<int>(((st0 + 1) * G + nall - 1) / nall - 1);
      const int pi = b - bf - 1;
      if (lane < R) wsp[(static_cast<size_t>(tile) * maxp + pi) * R + lane] = v;
      __threadfence();
      __syncwarp();
      if (lane == 0) st_release_gpu(wsc + static_cast<size_t>(tile) * maxp + pi, 1);
    }
    i += len;
    ks = 0;
    ++tile;
    ++j;
  }
  return true;
}

// --------------------------------------------------------------------- T = 1 wide-stage kernel
// Shared parameters of the wide-stage launches: the matrix, x / y, the stage geometry (R rows x CW chunks per
// stage, KS stages per row tile, NS ring slots), the shared-memory offsets and the stream-K workspace.
struct RowsParams {
  const uint8_t* m8;  // the code planes (exception stand-ins are read from m8 when not staged)
  const int32_t* rp;
  const int32_t* ec;
  const float* ev;
  const float* x;
  float* y;
  const uint16_t* lnw;
  float eps;
  int base, N, K, nch;
  int R, CW, KS, tiles, NS;
  int xs_off, rps_off, ecs_off, ecap, ring_off;
  uint32_t k128, k8, k65536;  // 128, 8, 65536: decode multipliers passed as values, so they stay on the FMA pipe
  float* wsp;                 // stream-K partials [tiles][maxp][R] (null: whole row tiles per CTA)
  int* wsc;                   // stream-K tickets [tiles], zero between launches
  int maxp;                   // partial slots per tile
};

// The CTA's share of the (tile, chunk group) stages. Without a workspace every CTA takes whole row tiles;
// with one (stream-K) the tiles * KS stages are split evenly, so a tile may be shared by neighbouring CTAs.
struct WideShare {
  int g0, n_st, tb, ks0, row0, nrows;
};
AIB_DEV WideShare wide_share(const RowsParams& p) {
  WideShare w;
  const long long b = blockIdx.x, G = gridDim.x;
  if (p.wsp) {
    const long long n = static_cast<long long>(p.tiles) * p.KS;
    const long long g0 = b * n / G, g1 = (b + 1) * n / G;
    w.g0 = static_cast<int>(g0);
    w.n_st = static_cast<int>(g1 - g0);
    w.tb = static_cast<int>(g0 / p.KS);
    w.ks0 = static_cast<int>(g0 % p.KS);
    const int tl = w.n_st > 0 ? static_cast<int>((g1 - 1) / p.KS) : w.tb;
    w.row0 = w.tb * p.R;
    w.nrows = max(0, min((tl - w.tb + 1) * p.R, p.N - w.row0));
  } else {
    const int tb = static_cast<int>(b * p.tiles / G), te = static_cast<int>((b + 1) * p.tiles / G);
    w.g0 = tb * p.KS;
    w.n_st = (te - tb) * p.KS;
    w.tb = tb;
    w.ks0 = 0;
    w.row0 = tb * p.R;
    w.nrows = max(0, min((te - tb) * p.R, p.N - w.row0));
  }
  return w;
}

// ----------------------------------------------------------- T = 1 wide-stage tensor-core kernel
// Same 48 KB stages and producer bookkeeping as gemv_rows_kernel, but the decoded bf16 pairs are fed to
// mma.sync.m16n8k16 (bf16 x bf16 -> fp32) as A fragments, so neither an fp32 split nor an FMA per weight is
// needed. x is stored once in shared memory as three bf16 parts (x = x0 + x1 + x2 exactly, the reference's
// `_x3` split, wcomp.py:130-140) placed in different B columns: one MMA per 8 weights and lane.
//
// Stage = R rows (RG = R/16 row groups of 16) x CW chunks; 16 warps = RG x CW x 2. Warp (rg, q, hh) handles
// chunk q of row group rg: lane (g, t) holds rows g and g+8 and, for parity par = g & 1, the 16 low columns
// blk*64 + 16t + [0, 16) with blk = hh ^ par, plus the 16 high columns 128 + those -- exactly one codec unit
// (chunk q, 16-column group 4*blk + t) per row. MMA i (0..7) takes low columns 2i, 2i+1 and high columns
// 128 + 2i, 129 + 2i of that range. Even and odd rows of the warp use different column blocks, which keeps
// the 16-byte shared loads of a quarter-warp on distinct banks; B column n = 2*sp + par carries x part sp in
// the column order of parity par, and a row reads its result from the columns of its own parity.
#ifndef AIB_REC_UNROLL
#define AIB_REC_UNROLL 8
#endif
constexpr int kTcPrologueRecords = 8;
constexpr int kRecUnroll = AIB_REC_UNROLL;  // x records per consumer thread per prologue batch (K <= 16384: one batch)

// NCW consumer warps: 16 with 48 KB stages (R * CW = 128, one CTA per SM), or 8 with 24 KB stages (R * CW = 64,
// <= 113 KB of shared memory and 288 threads, so two CTAs share an SM: two of the same launch, or the tail of one
// launch and the head of the next, whose producer then streams its weights while the previous CTA drains).
// SPL = 2 splits each (row group, chunk slot, half) unit's eight MMA steps between two warps (four each), so 16
// consumer warps share a 24 KB stage and two 544-thread CTAs fit an SM: 32 consumer warps per SM to hide the
// decode's dependency chains.
// Consumer warps of the tensor-core wide-stage kernel for one matrix pass ("phase"): the x prologue (three-part
// B records of xin(x), the RMSNorm folded in; after the grid-dependency wait when wait_pdl), then the stages of
// the CTA's share `sh`. The ring position (s, ph), the segment-end count jc and the abort state carry over from one
// phase to the next when several matrices stream through one ring.
template <int MODE, bool RMS, int NCW, int SPL>
AIB_DEV void tc_consume(const RowsParams& p, const WideShare& sh_, uint8_t* xr, float* rms_red, uint8_t* ring,
                        uint64_t* full, uint64_t* empty, float* pbuf, uint64_t* pready, uint64_t* pfree,
                        uint64_t* xready, volatile int* abort_flag, bool wait_pdl, int& s, int& ph, int& jc,
                        bool& aborted) {
  constexpr int kTcConsumers = NCW * 32;
  constexpr int kStage = NCW * 2048 * 3 / 2 / SPL;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tb = sh_.tb, ks0 = sh_.ks0, n_st = sh_.n_st;
  const int R = p.R, CW = p.CW, KS = p.KS, NS = p.NS;
  const int PW = 2 * CW * SPL;
  // x prologue into the three-part B records
  // Record pr holds columns (c, c+1) and (128+c, 129+c) of chunk gc = pr / 64 (c from tc_rec_col). Consumer
  // thread tid owns records tid + 512 j. All of a batch's loads are issued before any is used (one memory
  // round trip per batch; one batch up to K = 16384), the RMS sum reuses the loaded values, and the norm
  // weights -- constant inputs -- are read before the grid dependency resolves.
  const int K = p.K, npr = K / 4;
  constexpr int kBatch = kTcPrologueRecords * kTcConsumers;
  uint32_t lwa[kTcPrologueRecords], lwb[kTcPrologueRecords];
  if (RMS) {
#pragma unroll
    for (int j = 0; j < kTcPrologueRecords; ++j) {
      const int pr = tid + j * kTcConsumers;
      const int k0 = tc_rec_col(pr);
      lwa[j] = pr < npr ? *reinterpret_cast<const uint32_t*>(p.lnw + k0) : 0u;
      lwb[j] = pr < npr ? *reinterpret_cast<const uint32_t*>(p.lnw + k0 + 128) : 0u;
    }
  }
  if (wait_pdl) pdl_wait();
  float rs = 1.0f;
  if (RMS && npr > kBatch) {  // several batches: the sum of squares first
    const float4* xg = reinterpret_cast<const float4*>(p.x);
    float ss = 0.0f;
    for (int k = tid; k < K / 4; k += kTcConsumers) {
      const float4 v = xg[k];
      ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    }
    ss = warp_sum(ss);
    if (lane == 0) rms_red[tid >> 5] = ss;
    named_sync(1, kTcConsumers);
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kTcConsumers / 32; ++w) tot += rms_red[w];
    rs = rsqrtf(tot / static_cast<float>(K) + p.eps);
  }
  for (int b0 = 0; b0 < npr; b0 += kBatch) {
    float4 xv[kTcPrologueRecords];  // x at (c, c+1, 128+c, 129+c) of the record's chunk
#pragma unroll
    for (int j = 0; j < kTcPrologueRecords; ++j) {
      const int pr = b0 + tid + j * kTcConsumers;
      const int k0 = tc_rec_col(pr);
      float2 lo = make_float2(0.0f, 0.0f), hi = lo;
      if (pr < npr) {
        lo = *reinterpret_cast<const float2*>(p.x + k0);
        hi = *reinterpret_cast<const float2*>(p.x + k0 + 128);
      }
      xv[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    if (MODE == 2) {  // input silu(x[k]) * x[K + k]
#pragma unroll
      for (int j = 0; j < kTcPrologueRecords; ++j) {
        const int pr = b0 + tid + j * kTcConsumers;
        const int k0 = tc_rec_col(pr);
        if (pr < npr) {
          const float2 lo = *reinterpret_cast<const float2*>(p.x + K + k0);
          const float2 hi = *reinterpret_cast<const float2*>(p.x + K + k0 + 128);
          xv[j] = make_float4(silu_mul(xv[j].x, lo.x), silu_mul(xv[j].y, lo.y), silu_mul(xv[j].z, hi.x),
                              silu_mul(xv[j].w, hi.y));
        }
      }
    }
    if (RMS && npr <= kBatch) {  // one batch: the sum of squares from the loaded values (zeros past K)
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < kTcPrologueRecords; ++j)
        ss += (xv[j].x * xv[j].x + xv[j].y * xv[j].y) + (xv[j].z * xv[j].z + xv[j].w * xv[j].w);
      ss = warp_sum(ss);
      if (lane == 0) rms_red[tid >> 5] = ss;
      named_sync(1, kTcConsumers);
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kTcConsumers / 32; ++w) tot += rms_red[w];
      rs = rsqrtf(tot / static_cast<float>(K) + p.eps);
    }
#pragma unroll kRecUnroll
    for (int j = 0; j < kTcPrologueRecords; ++j) {
      const int pr = b0 + tid + j * kTcConsumers;
      if (pr >= npr) continue;
      const int gc = pr >> 6, c = tc_rec_col(pr) & 255;
      float v[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
      if (RMS) {
        uint32_t wa = lwa[j], wb = lwb[j];
        if (b0 > 0) {  // later batches read their weights here
          const int k0 = gc * 256 + c;
          wa = *reinterpret_cast<const uint32_t*>(p.lnw + k0);
          wb = *reinterpret_cast<const uint32_t*>(p.lnw + k0 + 128);
        }
        v[0] = __uint_as_float(wa << 16) * (v[0] * rs);
        v[1] = __uint_as_float(wa & 0xFFFF0000u) * (v[1] * rs);
        v[2] = __uint_as_float(wb << 16) * (v[2] * rs);
        v[3] = __uint_as_float(wb & 0xFFFF0000u) * (v[3] * rs);
      }
      uint32_t w[3][2];  // parts: one conversion instruction per pair (this loop bounds the prologue)
#pragma unroll
      for (int sp = 0; sp < 3; ++sp) {
        w[sp][0] = bf16x2_rn(v[0], v[1]);
        w[sp][1] = bf16x2_rn(v[2], v[3]);
        v[0] -= __uint_as_float(w[sp][0] << 16);
        v[1] -= __uint_as_float(w[sp][0] & 0xFFFF0000u);
        v[2] -= __uint_as_float(w[sp][1] << 16);
        v[3] -= __uint_as_float(w[sp][1] & 0xFFFF0000u);
      }
      const int blk = c >> 6, t = (c >> 4) & 3, i = (c & 15) >> 1;
      // parts 0 and 1 share a 128-byte line per (chunk, i): lanes of odd i store part 1 first, so each store
      // instruction of a half-warp covers 16 distinct bank pairs
      const int o0 = tc_xrec(p.nch, gc, i, blk, t, 0), sw = i & 1;
      *reinterpret_cast<uint2*>(xr + o0 + sw * 32) = sw ? make_uint2(w[1][0], w[1][1]) : make_uint2(w[0][0], w[0][1]);
      *reinterpret_cast<uint2*>(xr + o0 + (sw ^ 1) * 32) =
          sw ? make_uint2(w[0][0], w[0][1]) : make_uint2(w[1][0], w[1][1]);
      *reinterpret_cast<uint2*>(xr + tc_xrec(p.nch, gc, i, blk, t, 2)) = make_uint2(w[2][0], w[2][1]);
    }
  }
  named_sync(1, kTcConsumers);
  if (tid == 0) mbar_arrive(xready);  // the finisher reads x records for the exception corrections

  const int warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int half = SPL == 2 ? (warp & 1) : 0, wu = SPL == 2 ? (warp >> 1) : warp;  // wu: the warp's unit
  const int hh = wu & 1, q = (wu >> 1) % CW, rg = (wu >> 1) / CW;
  const int par = g & 1, blk = hh ^ par;
  const int rA = rg * 16 + g, rB = rA + 8;
  const uint32_t colo = static_cast<uint32_t>(q * 256 + blk * 64 + 16 * t);
  const uint32_t m8A = static_cast<uint32_t>(rA * CW * 256) + colo, m8B = static_cast<uint32_t>(rB * CW * 256) + colo;
  const uint32_t e4o = static_cast<uint32_t>(R * CW * 256 + q * 128 + blk * 64 + 16 * t);
  const uint32_t e4A = e4o + static_cast<uint32_t>(rA * CW * 128), e4B = e4o + static_cast<uint32_t>(rB * CW * 128);
  const bool bl = g < 6;  // lanes supplying a B column (parts 0..2 x 2 parities); columns 6, 7 stay zero
  const int sp = g >> 1;
  const uint32_t base7 = (static_cast<uint32_t>(p.base) << 7) | (static_cast<uint32_t>(p.base) << 23);
  const uint32_t k128 = p.k128, k8 = p.k8;

  constexpr int NACC = AIB_GEMV_ACC;  // independent accumulator chains (MMA i feeds chain i % NACC)
  float acc[NACC][4];
#pragma unroll
  for (int a = 0; a < NACC; ++a) acc[a][0] = acc[a][1] = acc[a][2] = acc[a][3] = 0.0f;
  int ks = ks0, tile = tb;
  for (int it = 0; it < n_st; ++it) {
    // warp-uniform: the MMAs below must run with all 32 lanes converged
    const bool ok = __all_sync(0xffffffffu, !aborted && wait_full(&full[s], ph, abort_flag));
    if (!ok) aborted = true;
    const int gc = ks * CW + q;
    if (ok && gc < p.nch) {
      const uint8_t* st = ring + static_cast<size_t>(s) * kStage;
      uint32_t la[4], ha[4], ea[4], lb[4], hb[4], eb[4];  // the lane's 16 columns (SPL 2: its half, words 0-1)
      if (SPL == 1) {
        const uint4 LA = *reinterpret_cast<const uint4*>(st + m8A);
        const uint4 HA = *reinterpret_cast<const uint4*>(st + m8A + 128);
        const uint4 EA = *reinterpret_cast<const uint4*>(st + e4A);
        const uint4 LB = *reinterpret_cast<const uint4*>(st + m8B);
        const uint4 HB = *reinterpret_cast<const uint4*>(st + m8B + 128);
        const uint4 EB = *reinterpret_cast<const uint4*>(st + e4B);
        la[0] = LA.x, la[1] = LA.y, la[2] = LA.z, la[3] = LA.w;
        ha[0] = HA.x, ha[1] = HA.y, ha[2] = HA.z, ha[3] = HA.w;
        ea[0] = EA.x, ea[1] = EA.y, ea[2] = EA.z, ea[3] = EA.w;
        lb[0] = LB.x, lb[1] = LB.y, lb[2] = LB.z, lb[3] = LB.w;
        hb[0] = HB.x, hb[1] = HB.y, hb[2] = HB.z, hb[3] = HB.w;
        eb[0] = EB.x, eb[1] = EB.y, eb[2] = EB.z, eb[3] = EB.w;
      } else {
        const uint32_t ho = static_cast<uint32_t>(half * 8);
        const uint2 LA = *reinterpret_cast<const uint2*>(st + m8A + ho);
        const uint2 HA = *reinterpret_cast<const uint2*>(st + m8A + 128 + ho);
        const uint2 EA = *reinterpret_cast<const uint2*>(st + e4A + ho);
        const uint2 LB = *reinterpret_cast<const uint2*>(st + m8B + ho);
        const uint2 HB = *reinterpret_cast<const uint2*>(st + m8B + 128 + ho);
        const uint2 EB = *reinterpret_cast<const uint2*>(st + e4B + ho);
        la[0] = LA.x, la[1] = LA.y, ha[0] = HA.x, ha[1] = HA.y, ea[0] = EA.x, ea[1] = EA.y;
        lb[0] = LB.x, lb[1] = LB.y, hb[0] = HB.x, hb[1] = HB.y, eb[0] = EB.x, eb[1] = EB.y;
        la[2] = la[3] = ha[2] = ha[3] = ea[2] = ea[3] = lb[2] = lb[3] = hb[2] = hb[3] = eb[2] = eb[3] = 0u;
      }
      // this lane's B records for MMA i: xg + i * (128 or 64)
      const uint8_t* xg = sp < 2 ? xr + (gc * 8) * 128 + (blk * 2 + sp) * 32 + t * 8
                                 : xr + p.nch * 1024 + (gc * 8) * 64 + blk * 32 + t * 8;
      const int xstep = sp < 2 ? 128 : 64;
      {  // exceptions decode to their stand-ins; the producer adds the corrections
#pragma unroll
        for (int ii = 0; ii < 8 / SPL; ++ii) {
          const int i = ii + half * (8 / SPL);  // MMA step within the unit (its K slice)
          // x2 = [0, e1, 0, e0] (two code bytes: low nibble = low-half column, high nibble = high-half column).
          // High codes: x2*8 + base7 puts the high nibbles in the exponent fields and the low nibbles in
          // mantissa bits that the merge discards (no carry reaches the exponent). Low codes: x2*128 + base7
          // minus the high nibbles times 128 -- exact integer arithmetic, multiplies on the FMA pipe.
          const int wd = ii >> 1;
          const uint32_t sel = (i & 1) ? 0xB3A2u : 0x9180u, esel = (i & 1) ? 0x4342u : 0x4140u;
          const uint32_t xa2 = prmt(ea[wd], 0u, esel), xb2 = prmt(eb[wd], 0u, esel);
#if AIB_GEMV_LOWNIB2
          const uint32_t tA = (xa2 & 0x000F000Fu) * k128 + base7;
          const uint32_t tB = (xb2 & 0x000F000Fu) * k128 + base7;
#else
          const uint32_t tA = xa2 * k128 + base7 - (xa2 & 0x00F000F0u) * k128;
          const uint32_t tB = xb2 * k128 + base7 - (xb2 & 0x00F000F0u) * k128;
#endif
          const uint32_t a0 = merge_sm_e(prmt(la[wd], 0u, sel), tA);
          const uint32_t a1 = merge_sm_e(prmt(lb[wd], 0u, sel), tB);
          const uint32_t a2 = merge_sm_e(prmt(ha[wd], 0u, sel), xa2 * k8 + base7);
          const uint32_t a3 = merge_sm_e(prmt(hb[wd], 0u, sel), xb2 * k8 + base7);
          uint2 bb = make_uint2(0u, 0u);
          if (bl) bb = *reinterpret_cast<const uint2*>(xg + i * xstep);
          mma_bf16(acc[i % NACC], a0, a1, a2, a3, bb.x, bb.y);
        }
      }
    }
    __syncwarp();  // the stage's shared loads are done (their values fed the MMAs): release the slot
    if (lane == 0) mbar_arrive(&empty[s]);
    if (ks == KS - 1 || it == n_st - 1) {  // segment end: row g takes the columns of its parity (quads t = 0..2)
      float vA = par ? (acc[0][1] + acc[1][1]) : (acc[0][0] + acc[1][0]);
      float vB = par ? (acc[0][3] + acc[1][3]) : (acc[0][2] + acc[1][2]);
      if (NACC == 4) {
        vA += par ? (acc[2][1] + acc[3][1]) : (acc[2][0] + acc[3][0]);
        vB += par ? (acc[2][3] + acc[3][3]) : (acc[2][2] + acc[3][2]);
      }
      if (t == 3) vA = vB = 0.0f;
      vA += __shfl_xor_sync(0xffffffffu, vA, 1);
      vB += __shfl_xor_sync(0xffffffffu, vB, 1);
      vA += __shfl_xor_sync(0xffffffffu, vA, 2);
      vB += __shfl_xor_sync(0xffffffffu, vB, 2);
      // partial buffer jc & 1: wait until the finisher has read its previous contents (segment end jc - 2)
      const int b = jc & 1;
      if (jc >= 2 && !aborted) {
        int fr = 1;
        if (lane == 0) {
          const uint32_t fpar = ((jc >> 1) - 1) & 1;
          fr = mbar_try_wait(&pfree[b], fpar);
          for (uint32_t k = 0, lim = fr ? 0u : spin_limit(); k < lim && !fr; ++k) {
            fr = mbar_try_wait(&pfree[b], fpar);
            if (!fr && (k & 63) == 63 && *abort_flag) break;
          }
          if (!fr) {
            if (!*abort_flag) set_status(AIB_DEV_TIMEOUT_EMPTY);
            *abort_flag = 1;
          }
        }
        if (!__shfl_sync(0xffffffffu, fr, 0)) aborted = true;
      }
      if (t == 0 && !aborted) {
        float* part = pbuf + b * 256;
        const int wi = (q * 2 + hh) * SPL + half;
        part[rA * PW + wi] = vA;
        part[rB * PW + wi] = vB;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pready[b]);
      ++jc;
#pragma unroll
      for (int a = 0; a < NACC; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = 0.0f;
    }
    if (++ks == KS) ks = 0, ++tile;
    if (++s == NS) s = 0, ph ^= 1;
  }
}

template <int MODE, bool RMS, int NCW, int SPL = 1>
__global__ void __launch_bounds__(NCW * 32 + 64, (NCW == 16 && SPL == 1) ? 1 : 2)
    gemv_tc_kernel(const __grid_constant__ CUtensorMap tm8, const __grid_constant__ CUtensorMap tme4, RowsParams p) {
  constexpr int kTcConsumers = NCW * 32;
  constexpr int kTcThreads = kTcConsumers + 64;  // + producer warp + finisher warp
  constexpr int kStage = NCW * 2048 * 3 / 2 / SPL;  // bytes per ring slot: 2048 / SPL weights per consumer warp
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 16;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 256);
  uint64_t* pready = reinterpret_cast<uint64_t*>(smem + 384);  // partial buffers: consumers -> finisher
  uint64_t* pfree = pready + 2;                                // finisher -> consumers
  uint64_t* xready = pready + 4;                               // consumers -> finisher: x records built
  float* rms_red = reinterpret_cast<float*>(smem + 512);
  float* pbuf = reinterpret_cast<float*>(smem + 1024);  // two partial buffers, float [R][PW] each (<= 1 KB)
  uint8_t* xr = smem + p.xs_off;
  int* rps = reinterpret_cast<int*>(smem + p.rps_off);
  int* ecs = reinterpret_cast<int*>(smem + p.ecs_off);
  uint8_t* ring = smem + p.ring_off;

  const int tid = threadIdx.x, lane = tid & 31;
  const WideShare sh_ = wide_share(p);
  const int tb = sh_.tb, ks0 = sh_.ks0;
  const int R = p.R, CW = p.CW, KS = p.KS, NS = p.NS;
  const int PW = 2 * CW * SPL;  // partials per row (warps per row group)
  const int n_st = sh_.n_st;
  const int row0 = sh_.row0;
  const int nrows = sh_.nrows;
  // The producer thread initialises the barriers and issues the ring's first stages, so the weights start
  // streaming at once (they do not depend on the previous kernel).
  const int first = AIB_GEMV_EARLY ? min(NS, n_st) : 0;
  if (tid == kTcConsumers) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);  // the TMA arrival (with the stage's bytes)
      mbar_init(&empty[s], kTcConsumers / 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pready[b], kTcConsumers / 32);
      mbar_init(&pfree[b], 1);
    }
    mbar_init(xready, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (!g_aib_withhold_copies) {
      prefetch_tensormap(&tm8);
      prefetch_tensormap(&tme4);
      const uint32_t m8_bytes = static_cast<uint32_t>(R * CW * 256);
      const uint64_t pol = l2_evict_first();
      int ks = ks0, tile = tb;
      for (int i = 0; i < first; ++i) {
        uint8_t* st = ring + static_cast<size_t>(i) * kStage;
        mbar_arrive_expect_tx(&full[i], kStage);
        if (AIB_GEMV_EVICT_FIRST) {
          tma_load_3d_hint(st, &tm8, &full[i], 0, ks * CW, tile * R, pol);
          tma_load_3d_hint(st + m8_bytes, &tme4, &full[i], 0, ks * CW, tile * R, pol);
        } else {
          tma_load_3d(st, &tm8, &full[i], 0, ks * CW, tile * R);
          tma_load_3d(st + m8_bytes, &tme4, &full[i], 0, ks * CW, tile * R);
        }
        if (++ks == KS) ks = 0, ++tile;
      }
    }
  }
  __syncthreads();
  pdl_trigger();

  if (tid >= kTcConsumers + 32) {  // ---------------- finisher warp: the CSR slice, then the segments
    float* evs = reinterpret_cast<float*>(ecs + p.ecap);
    const bool staged = stage_csr_warp(rps, ecs, evs, p.ecap, nrows, row0, p.rp, p.ec, p.ev, p.m8, p.K, p.base);
    const ExcTab et{rps, ecs, evs, staged, rps[0], row0, p.ec, p.ev, p.m8, p.K, p.base};
    int j = 0;
    finish_segments<MODE>(pbuf, 256, pready, pfree, xready, abort_flag, et, TcXval{xr, p.nch}, p.y, p.N, tb, ks0, n_st,
                          R, CW, KS, nrows, PW, p.wsp, p.wsc, p.maxp, p.tiles, j);
    return;
  }
  if (tid >= kTcConsumers) {  // ---------------- producer warp: one thread streams the stages
    // after the last copy, wait for the ring's copies to land: the CTA must not exit with copies in flight if
    // another role aborts and the consumers stop waiting for the stages
    if (tid == kTcConsumers &&
        issue_stages(&tm8, &tme4, ring, full, empty, abort_flag, tb, ks0, n_st, first, R, CW, KS, NS, kStage) &&
        !g_aib_withhold_copies)
      drain_ring(full, n_st, NS);
    return;
  }

  int s_ = 0, ph_ = 0, jc_ = 0;
  bool aborted_ = false;
  tc_consume<MODE, RMS, NCW, SPL>(p, sh_, xr, rms_red, ring, full, empty, pbuf, pready, pfree, xready, abort_flag, true,
                                  s_, ph_, jc_, aborted_);
}

// ------------------------------------------------------------------------------- batched kernel
// T <= TMAX tokens, RT = 32 rows x CW = 1 chunk per stage; the x columns of each stage (T x 256 floats,
// SiLU-gated for mode 2) are staged in shared memory by the consumers.
template <int MODE, int TMAX>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tn_kernel(const __grid_constant__ CUtensorMap tm8, const __grid_constant__ CUtensorMap tme4, Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + 16;  // up to 16 ring slots
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 256);
  float* xs = reinterpret_cast<float*>(smem + kHeader);  // [TMAX][256] (permuted)
  uint8_t* ring = smem + kHeader + ((TMAX * 256 * 4 + 1023) / 1024) * 1024;

  const int tid = threadIdx.x;
  const int tb = static_cast<int>((static_cast<long long>(blockIdx.x) * p.tiles) / gridDim.x);
  const int te = static_cast<int>((static_cast<long long>(blockIdx.x + 1) * p.tiles) / gridDim.x);
  const int n_it = (te - tb) * p.KS;
  init_barriers(full, empty, abort_flag, p.NS);
  pdl_trigger();
  if (tid >= kConsumers) {
    if (tid == kConsumers) produce(&tm8, &tme4, ring, full, empty, abort_flag, tb, n_it, p.KS, 32, 1, p.NS);
    return;
  }
  pdl_wait();
  const int K = p.K, T = p.T;
  const int j = tid & 7, r = tid >> 3;
  const uint32_t base7 = (static_cast<uint32_t>(p.base) << 7) | (static_cast<uint32_t>(p.base) << 23);
  float2 acc[TMAX];
  int row = 0, ex_p = 0, ex_e = 0, ex_col = INT_MAX;
  bool aborted = false;
  for (int it = 0; it < n_it; ++it) {
    const int s = it % p.NS;
    const int tile = tb + it / p.KS, ks = it % p.KS;
    if (ks == 0) {
      row = tile * 32 + r;
#pragma unroll
      for (int t = 0; t < TMAX; ++t) acc[t] = make_float2(0.0f, 0.0f);
      ex_p = 0;
      ex_e = 0;
      if (row < p.N) {
        ex_p = p.rp[row];
        ex_e = p.rp[row + 1];
      }
      ex_col = ex_p < ex_e ? p.ec[ex_p] : INT_MAX;
    }
    // stage the x columns of chunk ks for all tokens
    named_sync(1, kConsumers);  // previous chunk fully consumed
    for (int i = tid; i < T * 256; i += kConsumers) {
      const int t = i >> 8, k = ks * 256 + (i & 255);
      const float* xr = p.x + static_cast<size_t>(t) * p.x_stride;
      xs[t * 256 + xperm(i & 255)] = (MODE == 2) ? silu_mul(xr[k], xr[K + k]) : xr[k];
    }
    named_sync(1, kConsumers);
    const bool ok = !aborted && wait_full(&full[s], (it / p.NS) & 1, abort_flag);
    if (!ok) aborted = true;  // keep walking the barrier sequence, skip the work
    if (ok && row < p.N) {
      const uint8_t* st = ring + static_cast<size_t>(s) * kStageBytes;
      const uint4 ml = *reinterpret_cast<const uint4*>(st + r * 256 + 16 * j);
      const uint4 mh = *reinterpret_cast<const uint4*>(st + r * 256 + 128 + 16 * j);
      const uint4 ee = *reinterpret_cast<const uint4*>(st + kStageM8 + r * 128 + 16 * j);
      const int c0 = ks * 256;
      if (!unit_has_exc(p.ec, ex_p, ex_e, ex_col, c0, j)) {
#pragma unroll
        for (int t = 0; t < TMAX; ++t) {
          if (t < T) {
            const float4* xb = reinterpret_cast<const float4*>(xs + t * 256);
            float4 xl[4], xh[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              xl[q] = xb[q * 8 + j];
              xh[q] = xb[32 + q * 8 + j];
            }
            unit_fast(ml, mh, ee, xl, xh, base7, acc[t]);
          }
        }
      } else {
        const uint32_t E[4] = {ee.x, ee.y, ee.z, ee.w}, L[4] = {ml.x, ml.y, ml.z, ml.w},
                       Hh[4] = {mh.x, mh.y, mh.z, mh.w};
        for (int t = 0; t < T; ++t) {
          const float* xt = xs + t * 256;
          float sacc = 0.0f;
          for (int q = 0; q < 4; ++q)
            for (int b = 0; b < 4; ++b) {
              const uint32_t eb = (E[q] >> (8 * b)) & 0xFFu;
              const int kl = 16 * j + 4 * q + b, kh = 128 + kl;
              sacc += dec1((L[q] >> (8 * b)) & 0xFFu, eb & 15u, p.base) * xt[xperm(kl)];
              sacc += dec1((Hh[q] >> (8 * b)) & 0xFFu, eb >> 4, p.base) * xt[xperm(kh)];
            }
          for (int q = ex_p; q < ex_e; ++q) {
            const int col = p.ec[q];
            if (col >= c0 + 256) break;
            const uint32_t o = static_cast<uint32_t>(col - c0);
            if (col >= c0 && ((o & 127u) >> 4) == static_cast<uint32_t>(j)) sacc += p.ev[q] * xt[xperm(col - c0)];
          }
#pragma unroll
          for (int tt = 0; tt < TMAX; ++tt)
            if (tt == t) acc[tt].x += sacc;
        }
      }
    }
    __syncwarp();
    if ((tid & 31) == 0) mbar_arrive(&empty[s]);
    if (ks == p.KS - 1) {
#pragma unroll
      for (int t = 0; t < TMAX; ++t) {
        float v = acc[t].x + acc[t].y;
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (MODE == 3) {  // rows r = tid/8: (2i, 2i+1) = (gate_i, up_i) are 8 lanes apart
          const float vu = __shfl_down_sync(0xffffffffu, v, 8);
          if (j == 0 && !(r & 1) && t < T && row + 1 < p.N && !aborted)
            p.y[static_cast<size_t>(t) * p.y_stride + (row >> 1)] = silu_mul(v, vu);
        } else if (j == 0 && t < T && row < p.N && !aborted) {
          float* yr = p.y + static_cast<size_t>(t) * p.y_stride + row;
          if (MODE == 0)
            *yr = v;
          else
            *yr += v;
        }
      }
    }
  }
}

// ----------------------------------------------------------------------------------- host side
struct Geometry {
  int RT, CW, KS, tiles, grid;
};

// Row-tile shape for the T = 1 kernel: a warp holds 4 (row, chunk) pairs, so CW <= 4 keeps every row inside
// one warp; the widest CW the row length allows gives the smallest tiles (RT = 32 / CW) and the best balance.
static Geometry pick_geometry(int N, int nch, int sms) {
  const int CW = nch >= 4 ? 4 : (nch >= 2 ? 2 : 1);
  const int RT = 32 / CW;
  const int tiles = (N + RT - 1) / RT;
  return {RT, CW, (nch + CW - 1) / CW, tiles, std::min(tiles, sms)};
}

static int make_maps(const aib_c12* c, int RT, int CW, CUtensorMap* tm8, CUtensorMap* tme4) {
  const uint64_t N = c->N, nch = c->K / 256;
  int rc = make_map_3d_u8(tm8, c->m8, 256, nch, N, 256, static_cast<uint64_t>(c->K), 256, CW, RT);
  if (rc) return rc;
  return make_map_3d_u8(tme4, c->e4, 128, nch, N, 128, static_cast<uint64_t>(c->K) / 2, 128, CW, RT);
}

constexpr size_t kSmemTarget = 112 * 1024;  // leaves room for a neighbouring kernel's CTA (PDL overlap)
constexpr size_t kSmemMax = 227 * 1024;

// Stream-K split of `tiles * KS` stages over `grid` CTAs: the most CTAs that share one tile.
static int streamk_max_parts(int tiles, int KS, int grid) {
  const long long n = static_cast<long long>(tiles) * KS, G = grid;
  int mp = 1;
  for (int t = 0; t < tiles; ++t) {
    const long long st0 = static_cast<long long>(t) * KS;
    const long long bf = ((st0 + 1) * G + n - 1) / n - 1, bl = ((st0 + KS) * G + n - 1) / n - 1;
    mp = std::max(mp, static_cast<int>(bl - bf + 1));
  }
  return mp;
}
// Workspace of a wide-stage launch (zero before the first launch; every launch leaves it zero):
// [ints: tiles x maxp (16-byte padded)][partials: tiles x maxp x R floats]. The tensor-core kernel keeps one
// ready flag per (tile, part) in the ints, the CUDA-core kernel one ticket per tile (the first `tiles` ints).
struct StreamK {
  int grid, maxp;
  size_t flag_bytes, bytes;
};
static StreamK streamk_plan(int tiles, int KS, int R, int max_grid) {
  StreamK k;
  const long long n = static_cast<long long>(tiles) * KS;
  k.grid = static_cast<int>(std::min<long long>(max_grid, n));
  k.maxp = streamk_max_parts(tiles, KS, k.grid);
  k.flag_bytes = ((static_cast<size_t>(tiles) * k.maxp * 4 + 15) / 16) * 16;
  k.bytes = k.flag_bytes + static_cast<size_t>(tiles) * k.maxp * R * 4;
  return k;
}

// Kernel choice for T = 1 (test knob 4, aib_debug_knob): 3 (default) the tensor-core wide-stage kernel -- two
// CTAs per SM with 24 KB stages where the shape fits, else one with 48 KB stages; 4 the one-CTA geometry only;
// 1 the CUDA-core 12 KB-stage kernel for every shape it takes. Shapes the tensor-core kernel cannot take (K not a
// multiple of 1024, x records too large for shared memory, base >= 240) always use the CUDA-core kernel.
int g_variant = 3;
constexpr size_t kSmemPair = 113 * 1024;  // two CTAs per SM (228 KB per SM, 1 KB reserved per CTA)

template <int NCW, int SPL = 1>
static int run_tc_var(const aib_c12* c, const float* x, float* y, int mode, const uint16_t* lnw, float eps, void* ws,
                      size_t ws_bytes, cudaStream_t s) {
  constexpr int kThreadsV = NCW * 32 + 64;
  constexpr size_t kStage = static_cast<size_t>(NCW) * 2048 * 3 / 2 / SPL;
  constexpr bool kPair = !(NCW == 16 && SPL == 1);  // two CTAs per SM
  const size_t smem_max = kPair ? kSmemPair : kSmemMax;
  const int nch = c->K / 256;
  const int CW = kStage == 49152 ? (nch % 8 == 0 ? 8 : 4) : 4;
  const int R = static_cast<int>(kStage / 384) / CW, KS = nch / CW;
  if (R * 2 * CW * SPL > 256) return fail(AIB_ENOTSUP, "aib_gemv_c12: partial buffer too small");
  const int tiles = (c->N + R - 1) / R;
  const int max_grid = kPair ? 2 * sm_count() : sm_count();
  // stream-K (with a workspace) when an even split of the stages shortens the longest CTA's share
  const StreamK sk = streamk_plan(tiles, KS, R, max_grid);
  const int whole_grid = std::min(tiles, max_grid);
  const long long whole_max = static_cast<long long>((tiles + whole_grid - 1) / whole_grid) * KS;
  const long long sk_max = (static_cast<long long>(tiles) * KS + sk.grid - 1) / sk.grid;
  const bool use_sk = ws && ws_bytes >= sk.bytes && !(reinterpret_cast<uintptr_t>(ws) & 15) && sk_max < whole_max;
  const int grid = use_sk ? sk.grid : whole_grid;
  const int per = static_cast<int>((static_cast<long long>(tiles) * KS + grid - 1) / grid);
  const int rows_max = use_sk ? ((per + KS - 1) / KS + 1) * R : ((tiles + grid - 1) / grid) * R;
  // layout: header, two partial buffers, x records (6 bytes per column), row pointers, staged exception
  // columns, ring; the deepest ring that fits
  int NS = 8;
  size_t xs_off = 0, rps_off = 0, ecs_off = 0;
  for (; NS >= 2; --NS) {
    xs_off = 1024 + 2 * 1024;
    rps_off = xs_off + static_cast<size_t>(nch) * 1536;
    ecs_off = rps_off + ((static_cast<size_t>(rows_max + 1) * 4 + 127) / 128) * 128;
    const size_t ring_need = ((ecs_off + 1023) / 1024) * 1024;  // staged exception columns take what is left
    if (ring_need + static_cast<size_t>(NS) * kStage <= smem_max) break;
  }
  if (NS < 2) return fail(AIB_ENOTSUP, "aib_gemv_c12: K=%d too large for the tensor-core kernel", c->K);
  const size_t ring_off = ((smem_max - static_cast<size_t>(NS) * kStage) / 1024) * 1024;
  const int ecap = static_cast<int>((ring_off - ecs_off) / 8);  // column + correction per staged exception
  const size_t smem = ring_off + static_cast<size_t>(NS) * kStage;
  CUtensorMap tm8, tme4;
  int rc = make_maps(c, R, CW, &tm8, &tme4);
  if (rc) return rc;
  RowsParams p{static_cast<const uint8_t*>(c->m8), c->rp, c->ec, c->ev, x, y, lnw, eps, c->base, c->N, c->K, nch, R, CW, KS, tiles, NS,
               static_cast<int>(xs_off), static_cast<int>(rps_off), static_cast<int>(ecs_off), ecap,
               static_cast<int>(ring_off), 128u, 8u, 65536u,
               use_sk ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + sk.flag_bytes) : nullptr,
               use_sk ? static_cast<int*>(ws) : nullptr, sk.maxp};
  auto go = [&](auto kernel) -> int {
    const int r2 = allow_smem(kernel, smem);
    if (r2) return r2;
    return launch(kernel, dim3(grid), dim3(kThreadsV), smem, s, "aib_gemv_c12(T=1, tensor)", tm8, tme4, p);
  };
  if (lnw) {
    if (mode == 0) return go(gemv_tc_kernel<0, true, NCW, SPL>);
    if (mode == 1) return go(gemv_tc_kernel<1, true, NCW, SPL>);
    if (mode == 3) return go(gemv_tc_kernel<3, true, NCW, SPL>);
    return go(gemv_tc_kernel<2, true, NCW, SPL>);
  }
  if (mode == 0) return go(gemv_tc_kernel<0, false, NCW, SPL>);
  if (mode == 1) return go(gemv_tc_kernel<1, false, NCW, SPL>);
  if (mode == 3) return go(gemv_tc_kernel<3, false, NCW, SPL>);
  return go(gemv_tc_kernel<2, false, NCW, SPL>);
}

// Wide-stage tensor-core kernel: K a multiple of 1024; ENOTSUP when x's three-part records do not fit.
static int run_tc(const aib_c12* c, const float* x, float* y, int mode, const uint16_t* lnw, float eps, void* ws,
                  size_t ws_bytes, cudaStream_t s) {
  const int nch = c->K / 256;
  if (nch % 4) return fail(AIB_ENOTSUP, "aib_gemv_c12: K=%d is not a multiple of 1024", c->K);
  if (c->base >= 240)  // the exception stand-in (exponent base + 15) would not be finite
    return fail(AIB_ENOTSUP, "aib_gemv_c12: base %d: exceptions need the exact-path kernel", c->base);
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(lnw) & 7))
    return fail(AIB_ENOTSUP, "aib_gemv_c12: x / lnw not aligned for vector loads");
  if (g_variant == 3) {
    const int rc = run_tc_var<8>(c, x, y, mode, lnw, eps, ws, ws_bytes, s);
    if (rc != AIB_ENOTSUP) return rc;
  }
  return run_tc_var<16>(c, x, y, mode, lnw, eps, ws, ws_bytes, s);
}

static int run_t1(const aib_c12* c, const float* x, float* y, int mode, const uint16_t* lnw, float eps, void* ws,
                  size_t ws_bytes, cudaStream_t s) {
  if (mode == 3) {  // gated output: the wide kernel only (its finisher pairs the rows)
    const int rc = run_tc(c, x, y, mode, lnw, eps, ws, ws_bytes, s);
    if (rc != AIB_ENOTSUP) return rc;
    return fail(AIB_ENOTSUP, "aib_gemv_c12: mode 3 with T == 1 needs K a multiple of 1024, base < 240 and x "
                             "within shared memory (K=%d, base %d)", c->K, c->base);
  }
  if (g_variant != 1) {
    const int rc = run_tc(c, x, y, mode, lnw, eps, ws, ws_bytes, s);
    if (rc != AIB_ENOTSUP) return rc;  // other shapes use the 12 KB-stage kernel
  }
  const int nch = c->K / 256;
  const Geometry g = pick_geometry(c->N, nch, sm_count());
  CUtensorMap tm8, tme4;
  int rc = make_maps(c, g.RT, g.CW, &tm8, &tme4);
  if (rc) return rc;
  const size_t xs_bytes = ((static_cast<size_t>(c->K) * 4 + 1023) / 1024) * 1024;
  if (kHeader + xs_bytes + 2 * kStageBytes > kSmemMax)
    return fail(AIB_ENOTSUP, "aib_gemv_c12: K=%d too large for the shared x buffer", c->K);
  int NS = static_cast<int>((kSmemMax - kHeader - xs_bytes) / kStageBytes);
  NS = std::max(2, std::min(NS, 16)) & ~1;  // even: the two consumer groups own alternate ring slots
  const size_t smem = kHeader + xs_bytes + static_cast<size_t>(NS) * kStageBytes;
  Params p{c->rp, c->ec, c->ev, x, y, lnw, eps, c->base, c->N, c->K, nch, g.RT, g.CW, g.KS, g.tiles, NS, 1, 0, 0,
           c->K, 0, 0};
  auto go = [&](auto kernel) -> int {
    const int r2 = allow_smem(kernel, smem);
    if (r2) return r2;
    return launch(kernel, dim3(g.grid), dim3(kT1Threads), smem, s, "aib_gemv_c12(T=1)", tm8, tme4, p);
  };
  if (lnw) {
    if (mode == 0) return go(gemv_t1_kernel<0, true>);
    if (mode == 1) return go(gemv_t1_kernel<1, true>);
    return go(gemv_t1_kernel<2, true>);
  }
  if (mode == 0) return go(gemv_t1_kernel<0, false>);
  if (mode == 1) return go(gemv_t1_kernel<1, false>);
  return go(gemv_t1_kernel<2, false>);
}

template <int MODE, int TMAX>
static int run_tn_t(const aib_c12* c, const float* x, float* y, int T, int xs_, int ys_, cudaStream_t s) {
  const int nch = c->K / 256;
  const int tiles = (c->N + 31) / 32;
  const int grid = std::min(tiles, sm_count());
  CUtensorMap tm8, tme4;
  int rc = make_maps(c, 32, 1, &tm8, &tme4);
  if (rc) return rc;
  const size_t xs_bytes = ((TMAX * 256 * 4 + 1023) / 1024) * 1024;
  int NS = static_cast<int>((kSmemTarget - kHeader - xs_bytes) / kStageBytes);
  NS = std::max(2, std::min(NS, 8));
  const size_t smem = kHeader + xs_bytes + static_cast<size_t>(NS) * kStageBytes;
  Params p{c->rp, c->ec, c->ev, x, y, nullptr, 0.0f, c->base, c->N, c->K, nch, 32, 1, nch, tiles, NS, T, xs_, ys_, 0, 0,
           0};
  rc = allow_smem(gemv_tn_kernel<MODE, TMAX>, smem);
  if (rc) return rc;
  return launch(gemv_tn_kernel<MODE, TMAX>, dim3(grid), dim3(kThreads), smem, s, "aib_gemv_c12(T>1)", tm8, tme4, p);
}

template <int TMAX>
static int run_tn_mode(const aib_c12* c, const float* x, float* y, int T, int xs_, int ys_, int mode, cudaStream_t s) {
  if (mode == 0) return run_tn_t<0, TMAX>(c, x, y, T, xs_, ys_, s);
  if (mode == 1) return run_tn_t<1, TMAX>(c, x, y, T, xs_, ys_, s);
  if (mode == 3) return run_tn_t<3, TMAX>(c, x, y, T, xs_, ys_, s);
  return run_tn_t<2, TMAX>(c, x, y, T, xs_, ys_, s);
}

}  // namespace gemv
}  // namespace aib

using namespace aib;

extern "C" {


size_t aib_gemv_c12_workspace(const aib_c12* c, int T) {
  if (!c || T != 1 || c->N <= 0 || c->K <= 0 || c->K % 1024) return 0;
  const int nch = c->K / 256;
  size_t need = 0;
  const int sms = aib::sm_count();
  // the wide-stage geometries: tensor-core 48 KB stages (one CTA per SM), tensor-core 24 KB stages (two per
  // SM), CUDA-core 48 KB stages
  const int cws[3] = {nch % 8 == 0 ? 8 : 4, 4, nch % 16 == 0 ? 16 : (nch % 8 == 0 ? 8 : 4)};
  const int rws[3] = {128 / cws[0], 16, 128 / cws[2]};
  const int grids[3] = {sms, 2 * sms, sms};
  for (int g = 0; g < 3; ++g) {
    const int tiles = (c->N + rws[g] - 1) / rws[g];
    need = std::max(need, gemv::streamk_plan(tiles, nch / cws[g], rws[g], grids[g]).bytes);
  }
  return need;
}

int aib_gemv_c12(const aib_c12* c, const float* x, float* y, int T, int x_stride, int y_stride, int mode,
                 const uint16_t* lnw, float eps, void* ws, size_t ws_bytes, void* stream) {
  if (!c || !x || !y || !c->m8 || !c->e4 || !c->rp || (c->n_exc > 0 && (!c->ec || !c->ev)))
    return fail(AIB_EINVAL, "aib_gemv_c12: null pointer");
  if (c->N <= 0 || c->K <= 0 || c->K % 256 || c->CH != 256)
    return fail(AIB_EINVAL, "aib_gemv_c12: K must be a positive multiple of 256 (N=%d K=%d CH=%d)", c->N, c->K, c->CH);
  if (mode < 0 || mode > 3) return fail(AIB_EINVAL, "aib_gemv_c12: mode must be 0, 1, 2 or 3");
  if (mode == 3 && (c->N & 1)) return fail(AIB_EINVAL, "aib_gemv_c12: mode 3 needs an even N (gate/up row pairs)");
  if (c->base < 0 || c->base > 241) return fail(AIB_EINVAL, "aib_gemv_c12: base %d out of range", c->base);
  if (T < 1 || T > 16) return fail(AIB_EINVAL, "aib_gemv_c12: T must be in 1..16");
  if ((reinterpret_cast<uintptr_t>(c->m8) & 15) || (reinterpret_cast<uintptr_t>(c->e4) & 15))
    return fail(AIB_EINVAL, "aib_gemv_c12: m8/e4 must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (T == 1) return gemv::run_t1(c, x, y, mode, lnw, eps, ws, ws_bytes, s);
  if (lnw) return fail(AIB_EINVAL, "aib_gemv_c12: the RMS prologue is only available for T == 1");
  const int xin = mode == 2 ? 2 * c->K : c->K;
  if (x_stride < xin || y_stride < (mode == 3 ? c->N / 2 : c->N))
    return fail(AIB_EINVAL, "aib_gemv_c12: row strides too small");
  if (T <= 2) return gemv::run_tn_mode<2>(c, x, y, T, x_stride, y_stride, mode, s);
  if (T <= 4) return gemv::run_tn_mode<4>(c, x, y, T, x_stride, y_stride, mode, s);
  if (T <= 8) return gemv::run_tn_mode<8>(c, x, y, T, x_stride, y_stride, mode, s);
  return gemv::run_tn_mode<16>(c, x, y, T, x_stride, y_stride, mode, s);
}

}  // extern "C"
