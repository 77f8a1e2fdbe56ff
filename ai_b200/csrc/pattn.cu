// Causal prefill attention over the bf16 KV cache on the tensor cores (sm_100a).
//
// Replaces the reference's blocked prefill attention att_k (`ramvi/engine/ramvi_engine/kernels/prefill_kernels.py:
// 30-56`): prompt row i (position start + i) of query head h attends cache positions 0 .. start + i of KV group
// h / G with an online softmax, scores = (q . k) * HD^-0.5, fp32 throughout.
//
// B200 design (flash-attention style, one CTA per (query tile, KV group)):
//  * A tile is 64 query rows = the G heads of the group x 64/G consecutive prompt positions, so every K/V row
//    staged in shared memory serves all G heads (GQA reuse). Four warps, 16 rows each.
//  * K and V blocks of 32 positions are double-buffered with 16-byte cp.async copies into padded rows (row
//    stride HD*2 + 16 bytes: the 8 row addresses of an ldmatrix land in 8 different bank groups).
//  * S = Q K^T and O += P V run as mma.sync m16n8k16 with bf16 operands: K and V are exact bf16 cache rows;
//    q and the probabilities enter as three bf16 parts each (x = p1 + p2 + p3 to ~2^-24), so every product is
//    exact and accumulation is fp32 -- the accuracy of the reference's fp32 IEEE dots. The probabilities are
//    reused from the score accumulators in registers (the m16n8 accumulator layout is the m16k16 operand
//    layout).
//  * Tiles are scheduled longest first (the last prompt positions see the most keys).
#include "common.cuh"

namespace aib {
namespace pattn {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 64;  // query rows per CTA
constexpr int kBlk = 32;   // key positions per block

template <int HD>
__host__ __device__ constexpr int rstride() {
  return HD * 2 + 16;
}
template <int HD>
__host__ __device__ constexpr size_t smem_bytes() {
  return static_cast<size_t>(3 * kRows + 4 * kBlk) * rstride<HD>();
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads)
    prefill_attn_kernel(const float* __restrict__ q, const uint16_t* __restrict__ kc, const uint16_t* __restrict__ vc,
                        float* __restrict__ out, int n, int start, int H, int maxt, float scale) {
  constexpr int BQ = kRows / G;
  constexpr int RS = rstride<HD>();
  constexpr int NT = HD / 8;  // 8-column tiles of the output
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* qs = sm;                      // [3 parts][kRows][RS]
  uint8_t* ks = sm + 3 * kRows * RS;     // [2][kBlk][RS]
  uint8_t* vs = ks + 2 * kBlk * RS;      // [2][kBlk][RS]
  const int qt = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // longest tiles first
  const int g = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint16_t* kg = kc + static_cast<size_t>(g) * maxt * HD;
  const uint16_t* vg = vc + static_cast<size_t>(g) * maxt * HD;
  const int i_hi = min(n, (qt + 1) * BQ) - 1;  // last prompt row of the tile
  const int kend = start + i_hi + 1;           // keys [0, kend) are visible to some row of the tile
  const int nblk = (kend + kBlk - 1) / kBlk;

  auto stage = [&](int b, int buf) {
    for (int idx = tid; idx < kBlk * (HD / 8); idx += kThreads) {
      const int r = idx / (HD / 8), c = idx % (HD / 8), j = b * kBlk + r;
      uint8_t* dk = ks + (buf * kBlk + r) * RS + c * 16;
      uint8_t* dv = vs + (buf * kBlk + r) * RS + c * 16;
      if (j < kend) {
        attn::cp16(dk, kg + static_cast<size_t>(j) * HD + c * 8);
        attn::cp16(dv, vg + static_cast<size_t>(j) * HD + c * 8);
      } else {  // past the visible keys: zero rows (their probabilities are 0; 0 * garbage could be NaN)
        *reinterpret_cast<uint4*>(dk) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(dv) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  };

  pdl_wait();
  stage(0, 0);
  attn::cp_commit();
  // q rows of the tile as three bf16 parts (rows past the prompt are zero)
  for (int idx = tid; idx < kRows * HD / 2; idx += kThreads) {
    const int r = idx / (HD / 2), c2 = idx % (HD / 2);
    const int hh = r / BQ, i = qt * BQ + r % BQ;
    float lo = 0.0f, hi = 0.0f;
    if (i < n) {
      const float* qr = q + static_cast<size_t>(i) * H * HD + static_cast<size_t>(g * G + hh) * HD;
      lo = qr[2 * c2];
      hi = qr[2 * c2 + 1];
    }
    uint32_t w[3];
    attn::split3_pair(lo, hi, w);
#pragma unroll
    for (int p = 0; p < 3; ++p) *reinterpret_cast<uint32_t*>(qs + (p * kRows + r) * RS + c2 * 4) = w[p];
  }

  const int rA = warp * 16 + (lane >> 2), rB = rA + 8;
  const int iA = qt * BQ + rA % BQ, iB = qt * BQ + rB % BQ;
  const int limA = start + iA, limB = start + iB;  // last key each row may see
  const int t4 = lane & 3;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;
  float o[NT][4];
#pragma unroll
  for (int d = 0; d < NT; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.0f;

  for (int b = 0; b < nblk; ++b) {
    if (b + 1 < nblk) stage(b + 1, (b + 1) & 1);
    attn::cp_commit();
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    const uint8_t* kb = ks + (b & 1) * kBlk * RS;
    const uint8_t* vb = vs + (b & 1) * kBlk * RS;
    // ---- S = Q K^T (16 rows x 32 keys per warp)
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t a[3][4];
#pragma unroll
      for (int p = 0; p < 3; ++p)
        attn::ldsm_x4(smem_u32(qs + (p * kRows + warp * 16 + (lane & 15)) * RS + kk * 32 + (lane >> 4) * 16), a[p][0],
                      a[p][1], a[p][2], a[p][3]);
#pragma unroll
      for (int n2 = 0; n2 < 2; ++n2) {
        uint32_t b0, b1, b2, b3;
        attn::ldsm_x4(smem_u32(kb + (n2 * 16 + (lane & 7) + ((lane >> 4) << 3)) * RS + kk * 32 + ((lane >> 3) & 1) * 16),
                      b0, b1, b2, b3);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          mma_bf16(s[2 * n2], a[p][0], a[p][1], a[p][2], a[p][3], b0, b1);
          mma_bf16(s[2 * n2 + 1], a[p][0], a[p][1], a[p][2], a[p][3], b2, b3);
        }
      }
    }
    // ---- scale, causal mask, online softmax (per row; a row's 32 keys are spread over the 4 lanes of a quad)
    float xA = mA, xB = mB;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = b * kBlk + nt * 8 + 2 * t4 + e;
        const float sa = (j <= limA && j < kend) ? s[nt][e] * scale : -INFINITY;
        const float sb = (j <= limB && j < kend) ? s[nt][2 + e] * scale : -INFINITY;
        s[nt][e] = sa;
        s[nt][2 + e] = sb;
        xA = fmaxf(xA, sa);
        xB = fmaxf(xB, sb);
      }
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 1));
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 2));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 1));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 2));
    // key 0 is visible to every row, so the running maxima are finite from the first block on
    const float alA = expf(mA - xA), alB = expf(mB - xB);
    mA = xA;
    mB = xB;
    float sumA = 0.0f, sumB = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[nt][e] = expf(s[nt][e] - xA);
        s[nt][2 + e] = expf(s[nt][2 + e] - xB);
        sumA += s[nt][e];
        sumB += s[nt][2 + e];
      }
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
#pragma unroll
    for (int d = 0; d < NT; ++d) {
      o[d][0] *= alA;
      o[d][1] *= alA;
      o[d][2] *= alB;
      o[d][3] *= alB;
    }
    // ---- O += P V: the score accumulators of key tiles (2k, 2k+1) are the k-th 16-key operand
#pragma unroll
    for (int k2 = 0; k2 < kBlk / 16; ++k2) {
      uint32_t a[4][3];  // [operand register][part]
      attn::split3_pair(s[2 * k2][0], s[2 * k2][1], a[0]);
      attn::split3_pair(s[2 * k2][2], s[2 * k2][3], a[1]);
      attn::split3_pair(s[2 * k2 + 1][0], s[2 * k2 + 1][1], a[2]);
      attn::split3_pair(s[2 * k2 + 1][2], s[2 * k2 + 1][3], a[3]);
#pragma unroll
      for (int d2 = 0; d2 < HD / 16; ++d2) {
        uint32_t b0, b1, b2, b3;
        attn::ldsm_x4_t(
            smem_u32(vb + (k2 * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * RS + d2 * 32 + (lane >> 4) * 16), b0, b1,
            b2, b3);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          mma_bf16(o[2 * d2], a[0][p], a[1][p], a[2][p], a[3][p], b0, b1);
          mma_bf16(o[2 * d2 + 1], a[0][p], a[1][p], a[2][p], a[3][p], b2, b3);
        }
      }
    }
    __syncthreads();  // the buffer read here is refilled by the next iteration's copies
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  const int hA = g * G + rA / BQ, hB = g * G + rB / BQ;
#pragma unroll
  for (int d = 0; d < NT; ++d) {
    const int col = d * 8 + 2 * t4;
    if (iA < n) {
      float* oa = out + static_cast<size_t>(iA) * H * HD + static_cast<size_t>(hA) * HD + col;
      oa[0] = o[d][0] / lA;
      oa[1] = o[d][1] / lA;
    }
    if (iB < n) {
      float* ob = out + static_cast<size_t>(iB) * H * HD + static_cast<size_t>(hB) * HD + col;
      ob[0] = o[d][2] / lB;
      ob[1] = o[d][3] / lB;
    }
  }
  pdl_trigger();
}

template <int HD, int G>
static int launch_hg(const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int n, int start, int H,
                     int KV, int maxt, float scale, cudaStream_t s) {
  constexpr size_t smem = smem_bytes<HD>();
  const int rc = allow_smem(prefill_attn_kernel<HD, G>, smem);
  if (rc) return rc;
  const int BQ = kRows / G;
  return launch(prefill_attn_kernel<HD, G>, dim3((n + BQ - 1) / BQ, KV), dim3(kThreads), smem, s, "aib_attn_prefill",
                q, kc, vc, out, n, start, H, maxt, scale);
}

template <int HD>
static int launch_h(int G, const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int n, int start, int H,
                    int KV, int maxt, float scale, cudaStream_t s) {
  switch (G) {
    case 1: return launch_hg<HD, 1>(q, kc, vc, out, n, start, H, KV, maxt, scale, s);
    case 2: return launch_hg<HD, 2>(q, kc, vc, out, n, start, H, KV, maxt, scale, s);
    case 4: return launch_hg<HD, 4>(q, kc, vc, out, n, start, H, KV, maxt, scale, s);
    case 8: return launch_hg<HD, 8>(q, kc, vc, out, n, start, H, KV, maxt, scale, s);
    default: return fail(AIB_ENOTSUP, "aib_attn_prefill: H/KV = %d (1, 2, 4 or 8 supported)", G);
  }
}

}  // namespace pattn
}  // namespace aib

using namespace aib;

extern "C" {

int aib_attn_prefill(const float* q, const uint16_t* kc, const uint16_t* vc, float* out, int n, int start, int H, int KV,
                     int HD, int maxt, float scale, void* stream) {
  if (!q || !kc || !vc || !out || n <= 0 || start < 0 || H <= 0 || KV <= 0 || H % KV || maxt <= 0 ||
      static_cast<long long>(start) + n > maxt)
    return fail(AIB_EINVAL, "aib_attn_prefill: bad arguments (n=%d start=%d maxt=%d)", n, start, maxt);
  if (HD != 64 && HD != 128) return fail(AIB_EINVAL, "aib_attn_prefill: head_dim must be 64 or 128");
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return fail(AIB_EINVAL, "aib_attn_prefill: KV caches must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int G = H / KV;
  return HD == 128 ? pattn::launch_h<128>(G, q, kc, vc, out, n, start, H, KV, maxt, scale, s)
                   : pattn::launch_h<64>(G, q, kc, vc, out, n, start, H, KV, maxt, scale, s);
}

}  // extern "C"
