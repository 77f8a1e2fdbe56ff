// Exact vocabulary logits from the 12-bit head (sm_100a).
//
// Replaces the full-vocabulary `exact_rows` call that the reference's Head.pick makes for sampling
// (`ramvi/engine/ramvi_engine/generation/head.py:19-26` and :62-71, temperature > 0): for every vocabulary row
// v and token row t,  out[t, v] = (...((0 + fl(w[v,0] h[t,0])) + fl(w[v,1] h[t,1])) + ...) + fl(w[v,D-1] h[t,D-1]),
// each product rounded to fp32 and the sum taken sequentially in column order in fp32 -- the same bits as the
// reference's Numba loop (fastmath off, so no contraction). The reference computes these on the CPU after a
// device-to-host copy; here they stay on the device and feed the sampler directly.
//
// B200 design (HBM-bound: 1.5 bytes per weight of codec planes):
//  * Lane per vocabulary row: a warp owns 32 consecutive rows and walks their 256-column chunks in order, so
//    every lane's sum is sequential with no cross-lane reduction (the reference's order by construction).
//  * Each warp stages its rows' chunk (32 x 256 bytes of m8 + 32 x 128 bytes of e4) with 16-byte cp.async
//    copies into a private slot (see AIB_EXACT_SLOTS for why one slot and 16 warps). Rows are stored
//    with their 16-byte pieces XOR-swizzled by (row & 7), so the lanes' 16-byte reads of 32 different rows
//    hit every bank group evenly (four wavefronts per LDS.128, the minimum).
//  * Decode: byte permutes put sign and mantissa of two columns in a bf16 pair, the exponent codes (plus the
//    matrix's base) come from integer multiply-adds, one LOP3 merges them (the codec GEMV's decode); the pair
//    splits into two exact fp32 weights. Products use packed fp32 multiplies (two IEEE round-to-nearest
//    products per instruction), the sum scalar adds.
//  * Exceptions (code 15, ~0.015 % of weights) are patched in the weight registers of the 16-column group that
//    holds them, from the row's CSR slice walked in column order, before the group's products are formed.
//  * h (T rows of fp32) is staged once per CTA in shared memory; reads are warp-wide broadcasts.
#include <algorithm>
#include <climits>
#include "common.cuh"

namespace aib {
namespace exact {

// Ring slots per warp: 1 (default) -- each warp waits for its chunk, sums it and only then fetches the next,
// and the shared memory saved doubles the warps per SM (16), which hides the sequential add chains and the
// copy latency better than double buffering with 8 warps (Qwen3-8B head: 251 vs 275 us); 2 double-buffers.
#ifndef AIB_EXACT_SLOTS
#define AIB_EXACT_SLOTS 1
#endif
constexpr int kSlotM8 = 32 * 256;
constexpr int kSlotE4 = 32 * 128;
constexpr int kSlot = kSlotM8 + kSlotE4;  // 12 KB per ring slot
constexpr int kMaxWarps = AIB_EXACT_SLOTS == 1 ? 16 : 8;

AIB_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
AIB_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
AIB_DEV void cp_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
AIB_DEV void cp_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Two IEEE round-to-nearest fp32 products in one instruction.
AIB_DEV float2 fmul2(float2 a, float2 b) {
  uint64_t A, B, D;
  asm("mov.b64 %0, {%1,%2};" : "=l"(A) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1,%2};" : "=l"(B) : "f"(b.x), "f"(b.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(D) : "l"(A), "l"(B));
  float2 d;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(D));
  return d;
}

AIB_DEV uint32_t merge_sm_e(uint32_t a, uint32_t b) {  // (a & 0x807F807F) | (b & ~0x807F807F)
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;" : "=r"(r) : "r"(a), "r"(b), "r"(0x807F807Fu));
  return r;
}

struct Args {
  const float* h;
  int ldh, T;
  aib_c12 W;
  float* out;
  int ldo;
  int nwarps;          // warps per CTA (the ring holds two slots per warp)
  int h_off;           // byte offset of h in shared memory
  uint32_t k128, k8;   // runtime constants (keep the multiplies on the FMA pipe)
};

// Issue the copies of chunk c of the 32-row group starting at v0 into slot `sl` (rows past V are skipped).
AIB_DEV void stage_chunk(const Args& a, uint8_t* sl, int v0, int c, int lane) {
  const int V = a.W.N, K = a.W.K;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int p = lane + 32 * i, row = p >> 4, j = p & 15;
    if (v0 + row < V)
      cp_async16(sl + row * 256 + ((j ^ (row & 7)) << 4),
                 a.W.m8 + static_cast<size_t>(v0 + row) * K + c * 256 + j * 16);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int p = lane + 32 * i, row = p >> 3, j = p & 7;
    if (v0 + row < V)
      cp_async16(sl + kSlotM8 + row * 128 + ((j ^ (row & 7)) << 4),
                 a.W.e4 + static_cast<size_t>(v0 + row) * (K / 2) + c * 128 + j * 16);
  }
}

template <int TT>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) exact_logits_kernel(Args a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int V = a.W.N, K = a.W.K, nch = K / 256;
  const int groups = (V + 31) / 32;
  const int gw = gridDim.x * a.nwarps;  // warps in the grid
  const int g0 = blockIdx.x * a.nwarps + warp;
  uint8_t* ring = smem + static_cast<size_t>(warp) * AIB_EXACT_SLOTS * kSlot;
  float* hs = reinterpret_cast<float*>(smem + a.h_off);
  const int n_groups = g0 < groups ? (groups - 1 - g0) / gw + 1 : 0;
  const int n_it = n_groups * nch;

  // the weights do not depend on the previous kernel: start streaming before the grid dependency resolves
  if (n_it > 0) stage_chunk(a, ring, g0 * 32, 0, lane);
  cp_commit();
  pdl_trigger();
  pdl_wait();
  for (int i = threadIdx.x; i < a.T * K; i += blockDim.x) {
    const int t = i / K, d = i - t * K;
    hs[i] = a.h[static_cast<size_t>(t) * a.ldh + d];
  }
  __syncthreads();

  const uint32_t base7 = (static_cast<uint32_t>(a.W.base) << 7) | (static_cast<uint32_t>(a.W.base) << 23);
  const uint32_t k128 = a.k128, k8 = a.k8;
  const int r = lane, rx = lane & 7;
  float s[TT];
  int xp = 0, xe = 0, xc = INT_MAX;
  for (int it = 0; it < n_it; ++it) {
    const int gi = it / nch, c = it - gi * nch;
    const int v0 = (g0 + gi * gw) * 32, v = v0 + r;
    if (c == 0) {  // a new row group: reset the sums, find the row's first exception
#pragma unroll
      for (int t = 0; t < TT; ++t) s[t] = 0.0f;
      xp = v < V ? a.W.rp[v] : 0;
      xe = v < V ? a.W.rp[v + 1] : 0;
      xc = xp < xe ? a.W.ec[xp] : INT_MAX;
    }
    // prefetch the next chunk (or the next group's first) into the other slot, then wait for this one
#if AIB_EXACT_SLOTS == 2
    if (it + 1 < n_it) {
      const int gn = (it + 1) / nch, cn = (it + 1) - gn * nch;
      stage_chunk(a, ring + ((it + 1) & 1) * kSlot, (g0 + gn * gw) * 32, cn, lane);
    }
    cp_commit();
    cp_wait1();
    const int cur = it & 1;
#else
    cp_wait0();
    const int cur = 0;
#endif
    __syncwarp();
    const uint8_t* sm8 = ring + cur * kSlot + r * 256;
    const uint8_t* se4 = ring + cur * kSlot + kSlotM8 + r * 128;
#pragma unroll 1
    for (int hf = 0; hf < 2; ++hf) {
#pragma unroll 2
      for (int q = 0; q < 8; ++q) {
        const uint4 mm = *reinterpret_cast<const uint4*>(sm8 + (((hf * 8 + q) ^ rx) << 4));
        const uint4 ee = *reinterpret_cast<const uint4*>(se4 + ((q ^ rx) << 4));
        const uint32_t L[4] = {mm.x, mm.y, mm.z, mm.w}, E[4] = {ee.x, ee.y, ee.z, ee.w};
        float w[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t x01 = prmt(E[k], 0u, 0x4140u), x23 = prmt(E[k], 0u, 0x4342u);
          uint32_t t01, t23;
          if (hf == 0) {  // low nibbles: codes of columns 0..127 of the chunk
            t01 = x01 * k128 + base7 - (x01 & 0x00F000F0u) * k128;
            t23 = x23 * k128 + base7 - (x23 & 0x00F000F0u) * k128;
          } else {        // high nibbles: columns 128..255
            t01 = x01 * k8 + base7;
            t23 = x23 * k8 + base7;
          }
          const uint32_t z01 = merge_sm_e(prmt(L[k], 0u, 0x9180u), t01);
          const uint32_t z23 = merge_sm_e(prmt(L[k], 0u, 0xB3A2u), t23);
          w[4 * k + 0] = __uint_as_float(z01 << 16);
          w[4 * k + 1] = __uint_as_float(z01 & 0xFFFF0000u);
          w[4 * k + 2] = __uint_as_float(z23 << 16);
          w[4 * k + 3] = __uint_as_float(z23 & 0xFFFF0000u);
        }
        const int col0 = c * 256 + hf * 128 + q * 16;
        if (xc < col0 + 16) {  // rare: exact values of this group's exceptions (code 15) from the CSR
          do {
            const int j = xc - col0;
            const float ev = a.W.ev[xp];
#pragma unroll
            for (int k = 0; k < 16; ++k)
              if (k == j) w[k] = ev;
            ++xp;
            xc = xp < xe ? a.W.ec[xp] : INT_MAX;
          } while (xc < col0 + 16);
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
          const float4* hp = reinterpret_cast<const float4*>(hs + t * K + col0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float4 hv = hp[k];
            const float2 p01 = fmul2(make_float2(w[4 * k], w[4 * k + 1]), make_float2(hv.x, hv.y));
            const float2 p23 = fmul2(make_float2(w[4 * k + 2], w[4 * k + 3]), make_float2(hv.z, hv.w));
            s[t] = __fadd_rn(s[t], p01.x);
            s[t] = __fadd_rn(s[t], p01.y);
            s[t] = __fadd_rn(s[t], p23.x);
            s[t] = __fadd_rn(s[t], p23.y);
          }
        }
      }
    }
    __syncwarp();  // the slot is refilled two iterations from now (one, with a single slot: right here)
#if AIB_EXACT_SLOTS == 1
    if (it + 1 < n_it) {
      const int gn = (it + 1) / nch, cn = (it + 1) - gn * nch;
      stage_chunk(a, ring, (g0 + gn * gw) * 32, cn, lane);
    }
    cp_commit();
#endif
    if (c == nch - 1 && v < V) {
#pragma unroll
      for (int t = 0; t < TT; ++t)
        if (t < a.T) a.out[static_cast<size_t>(t) * a.ldo + v] = s[t];
    }
  }
  cp_wait0();
}

template <int TT>
static int launch_tt(Args a, cudaStream_t st) {
  const int K = a.W.K;
  const size_t h_bytes = static_cast<size_t>(TT) * K * sizeof(float);
  constexpr size_t kMax = 227 * 1024;
  if (h_bytes + AIB_EXACT_SLOTS * kSlot > kMax) return fail(AIB_ENOTSUP, "aib_head_exact_logits: K=%d too large", K);
  a.nwarps = static_cast<int>(std::min<size_t>(kMaxWarps, (kMax - h_bytes) / (AIB_EXACT_SLOTS * kSlot)));
  a.h_off = a.nwarps * AIB_EXACT_SLOTS * kSlot;
  const size_t smem = a.h_off + h_bytes;
  const int rc = allow_smem(exact_logits_kernel<TT>, smem);
  if (rc) return rc;
  const int groups = (a.W.N + 31) / 32;
  const int grid = std::max(1, std::min(sm_count(), (groups + a.nwarps - 1) / a.nwarps));
  return launch(exact_logits_kernel<TT>, dim3(grid), dim3(a.nwarps * 32), smem, st, "aib_head_exact_logits", a);
}

}  // namespace exact
}  // namespace aib

using namespace aib;

extern "C" {

int aib_head_exact_logits(const float* h, int T, int ldh, const aib_c12* W, float* out, int ldo, void* stream) {
  if (!h || !W || !out || !W->m8 || !W->e4 || !W->rp || (W->n_exc > 0 && (!W->ec || !W->ev)))
    return fail(AIB_EINVAL, "aib_head_exact_logits: null pointer");
  if (T < 1 || T > 16 || W->N <= 0 || W->K <= 0 || W->K % 256 || W->CH != 256 || ldh < W->K || ldo < W->N)
    return fail(AIB_EINVAL, "aib_head_exact_logits: bad shape (T=%d N=%d K=%d ldh=%d ldo=%d)", T, W->N, W->K, ldh,
                ldo);
  if (W->base < 0 || W->base > 241) return fail(AIB_EINVAL, "aib_head_exact_logits: base %d out of range", W->base);
  if ((reinterpret_cast<uintptr_t>(W->m8) & 15) || (reinterpret_cast<uintptr_t>(W->e4) & 15))
    return fail(AIB_EINVAL, "aib_head_exact_logits: m8/e4 must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int t0 = 0; t0 < T; t0 += 8) {
    const int tt = std::min(8, T - t0);
    exact::Args a{h + static_cast<size_t>(t0) * ldh, ldh, tt, *W, out + static_cast<size_t>(t0) * ldo, ldo, 0, 0,
                  128u, 8u};
    const int rc = tt == 1 ? exact::launch_tt<1>(a, s)
                   : tt == 2 ? exact::launch_tt<2>(a, s)
                   : tt <= 4 ? exact::launch_tt<4>(a, s)
                             : exact::launch_tt<8>(a, s);
    if (rc) return rc;
  }
  return AIB_OK;
}

}  // extern "C"
