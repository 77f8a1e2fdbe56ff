// Int8 vocabulary head: quantised copy, per-token logit bounds, exact greedy pick (sm_100a).
//
// Replaces, for the greedy path of the reference's vocabulary head:
//   * Head.__init__ (`ramvi/engine/ramvi_engine/generation/head.py:29-50`): per vocabulary row v,
//     s_v = float(max|e_v| / 127) (1 when that is 0), q_v = round_half_even(e_v / s_v) clamped to +-127, and
//     the error bounds C1 = max|d_v| (1 + 1e-6), C2 = ||d_v||_2 (1 + 1e-6), AM = max|e_v| with
//     d_v = e_v - s_v q_v, all in float64 -> aib_head8_tables;
//   * vocab_a_k (`kernels/vocab8.py:19-44`): a_v = s_v q_v.h, B_v = min(C2 ||h||_2, C1 ||h||_1) +
//     2e-4 AM ||h||_1, HI_v = a_v + B_v and LO = max_v (a_v - B_v) -> aib_head8_bounds;
//   * Head.pick with temperature 0 (head.py:59-88) / vocab_b_k + vocab_c_k (vocab8.py:46-77): exact fp32
//     logits (each product rounded to fp32, summed in column order, head.py:19-26) of the candidates
//     HI_v >= LO, argmax with the smallest id on ties -> aib_head8_greedy. The exact rows are decoded from
//     the lossless 12-bit head, so the bf16 head need not stay in memory.
//
// B200 design. Tables: one warp per row, float64 as the reference. Bounds: an HBM-bound pass over the int8
// copy (V x D bytes): every warp streams one row at a time with all of the row's 16-byte loads in flight,
// h (up to 8 tokens) sits in shared memory in a lane-interleaved order (conflict-free float4 reads), int8
// values become floats with a byte permute into the mantissa of 2^23 and one subtraction (exact), fp32
// FMAs accumulate; LO is an exact max, reduced per CTA and then by the last CTA in a fixed order (ticket,
// no waiting). Greedy: one thread per (token, candidate row) runs the reference's sequential fp32 sum over
// the row decoded from the codec planes (exceptions walked in column order from the CSR), and a 64-bit
// ordered key (logit order, then smaller id) picks the winner with one atomicMax; the last CTA writes the ids
// and clears the keys.
#include <algorithm>
#include "common.cuh"

namespace aib {
namespace head8 {

constexpr float kSlack = 2e-4f;  // vocab8.py:14
constexpr int kThreads = 256;
constexpr int kTokPass = 8;      // tokens per bounds pass (their h in shared memory)
constexpr int kChunk = 512;      // int8 columns per warp load step (16 per lane)
constexpr int kMaxGrid = 1024;

// ------------------------------------------------------------------------------------------ tables
__global__ void __launch_bounds__(kThreads) tables_kernel(const uint16_t* __restrict__ w, int V, int D,
                                                          int8_t* __restrict__ Q, float* __restrict__ S,
                                                          float* __restrict__ C1, float* __restrict__ C2,
                                                          float* __restrict__ AM) {
  const int lane = threadIdx.x & 31;
  const long long v = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  if (v >= V) return;
  const uint16_t* row = w + v * D;
  double am = 0.0;
  for (int d = lane; d < D; d += 32) am = fmax(am, fabs(static_cast<double>(bf16_to_f32(row[d]))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = fmax(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float sf = __double2float_rn(am / 127.0);
  const double s = sf == 0.0f ? 1.0 : static_cast<double>(sf);
  double mx = 0.0, ss = 0.0;
  int8_t* qrow = Q + v * D;
  for (int d = lane; d < D; d += 32) {
    const double e = static_cast<double>(bf16_to_f32(row[d]));
    const double q = fmin(fmax(rint(e / s), -127.0), 127.0);  // rint: half to even, like torch.round
    qrow[d] = static_cast<int8_t>(q);
    const double dd = e - q * s;
    mx = fmax(mx, fabs(dd));
    ss += dd * dd;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  if (lane == 0) {
    S[v] = static_cast<float>(s);
    C1[v] = __double2float_rn(mx * (1.0 + 1e-6));
    C2[v] = __double2float_rn(sqrt(ss) * (1.0 + 1e-6));
    AM[v] = __double2float_rn(am);
  }
}

// ------------------------------------------------------------------------------------------ bounds
// Shared-memory position of h column d (per token, padded to whole 512-column chunks): lane L of a warp
// reads columns [16 L, 16 L + 16) of a chunk as four float4 that sit 512 bytes apart.
AIB_DEV int hpos(int d) {
  const int c = d >> 9, L = (d & 511) >> 4, j = (d & 15) >> 2, e = d & 3;
  return (((c * 4 + j) * 32 + L) << 2) + e;
}

// Four int8 in a word -> four exact floats: byte k (sign flipped) in the low mantissa byte of 2^23, minus
// 2^23 + 128.
AIB_DEV void i8x4(uint32_t w, float* f) {
  const uint32_t u = w ^ 0x80808080u;
#pragma unroll
  for (int k = 0; k < 4; ++k) f[k] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650u + k)) - 8388736.0f;
}

struct BoundsArgs {
  const float* h;
  int ldh, T;  // tokens of this pass (<= kTokPass)
  const int8_t* Q;
  const float *S, *C1, *C2, *AM;
  int V, D, nch;
  float* HI;
  int ldhi;
  float* LO;
  float* part;  // [kTokPass][gridDim.x] CTA maxima of a - B
  int* ticket;
  int kk;       // LO = a lower bound of the kk-th largest exact logit (1: the largest lower bound)
};

// TT: tokens handled per pass, rounded up to 1, 2, 4 or 8 (loops over t < a.T inside). Each warp walks its
// rows as units of up to 8 chunks (one unit per row when D <= 4096) and keeps two units of loads in
// flight: the next unit's loads are issued before the current unit's math.
template <int TT>
__global__ void __launch_bounds__(kThreads, 2) bounds_kernel(BoundsArgs a) {
  extern __shared__ __align__(16) float hs[];  // [T][nch * 512] permuted, then n1[kTokPass], n2[kTokPass]
  __shared__ float wlo[kThreads / 32][kTokPass];
  __shared__ int last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = a.T, D = a.D, nch = a.nch, hstride = nch * kChunk;
  float* n1s = hs + T * hstride;
  float* n2s = n1s + kTokPass;
  pdl_wait();
  for (int i = tid; i < T * hstride; i += kThreads) {
    const int t = i / hstride, d = i % hstride;
    hs[t * hstride + hpos(d)] = d < D ? a.h[static_cast<size_t>(t) * a.ldh + d] : 0.0f;
  }
  if (warp < T) {  // ||h||_1 and ||h||_2 of token `warp`, fixed order
    float s1 = 0.0f, s2 = 0.0f;
    for (int d = lane; d < D; d += 32) {
      const float x = a.h[static_cast<size_t>(warp) * a.ldh + d];
      s1 += fabsf(x);
      s2 = fmaf(x, x, s2);
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      n1s[warp] = s1;
      n2s[warp] = sqrtf(s2);
    }
  }
  __syncthreads();
  pdl_trigger();
  // lo[t]: lane j holds the warp's (j+1)-th largest lower bound a - B so far (descending across lanes)
  float lo[TT], acc[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) lo[t] = -INFINITY, acc[t] = 0.0f;
  const int ngr = (nch + 7) >> 3;
  const long long nw = static_cast<long long>(gridDim.x) * (kThreads / 32);
  long long v = static_cast<long long>(blockIdx.x) * (kThreads / 32) + warp;
  int gi = 0;
  auto load = [&](long long vv, int g, uint4 (&q)[8]) {
    const uint4* qrow = reinterpret_cast<const uint4*>(a.Q + vv * D);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = g * 8 + k, col = c * kChunk + lane * 16;
      q[k] = c < nch && col < D ? __ldg(qrow + (col >> 4)) : make_uint4(0u, 0u, 0u, 0u);  // zeros: q = 0
    }
  };
  // math of unit (v, gi) from q, then the row epilogue after its last unit; false once the warp is done
  auto step = [&](uint4 (&q)[8], uint4 (&qn)[8]) -> bool {
    long long vn = v;
    int gn = gi + 1;
    if (gn == ngr) gn = 0, vn = v + nw;
    if (vn < a.V) load(vn, gn, qn);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = gi * 8 + k;
      if (c < nch) {
        const float* hb = hs + ((c * 4 * 32 + lane) << 2);
        const uint32_t wd[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[4];
          i8x4(wd[j], f);
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            if (t < T) {
              const float4 x = *reinterpret_cast<const float4*>(hb + t * hstride + j * 128);
              acc[t] = fmaf(f[0], x.x, acc[t]);
              acc[t] = fmaf(f[1], x.y, acc[t]);
              acc[t] = fmaf(f[2], x.z, acc[t]);
              acc[t] = fmaf(f[3], x.w, acc[t]);
            }
          }
        }
      }
    }
    if (gi == ngr - 1) {  // row v complete
      const float s = a.S[v], c1 = a.C1[v], c2 = a.C2[v], am = a.AM[v];
#pragma unroll
      for (int t = 0; t < TT; ++t) {
        if (t < T) {
          const float dot = warp_sum(acc[t]);
          const float av = s * dot;
          const float b = fminf(c2 * n2s[t], c1 * n1s[t]) + kSlack * am * n1s[t];
          if (lane == 0) a.HI[static_cast<size_t>(t) * a.ldhi + v] = av + b;
          // insert av - b (the same value in every lane) into the warp's sorted list
          const float x = av - b, prev = __shfl_up_sync(0xffffffffu, lo[t], 1);
          if (x > lo[t]) lo[t] = (lane == 0 || x <= prev) ? x : prev;
        }
        acc[t] = 0.0f;
      }
    }
    v = vn;
    gi = gn;
    return v < a.V;
  };
  uint4 qa[8], qb[8];
  if (v < a.V) {
    load(v, 0, qa);
    while (step(qa, qb) && step(qb, qa)) {
    }
  }
  // the warp's kk-th largest lower bound: at most the grid's kk-th largest, so the maximum over the warps is a
  // lower bound of the kk-th largest exact logit (every warp's kk values are distinct rows)
#pragma unroll
  for (int t = 0; t < kTokPass; ++t) {
    const float w = t < TT ? __shfl_sync(0xffffffffu, lo[t < TT ? t : 0], a.kk - 1) : -INFINITY;
    if (lane == 0) wlo[warp][t] = w;
  }
  __syncthreads();
  if (tid < T) {
    float m = -INFINITY;
    for (int w = 0; w < kThreads / 32; ++w) m = fmaxf(m, wlo[w][tid]);
    a.part[tid * gridDim.x + blockIdx.x] = m;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(a.ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last) {  // the maxima of every CTA are visible: reduce them (a max is exact in any order)
    __threadfence();
    if (warp < T) {
      float m = -INFINITY;
      for (int b = lane; b < static_cast<int>(gridDim.x); b += 32) m = fmaxf(m, __ldcg(a.part + warp * gridDim.x + b));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) a.LO[warp] = m;
    }
    if (tid == 0) *a.ticket = 0;
  }
}

// ------------------------------------------------------------------------------------------ greedy
// 64-bit key: the fp32 logit in an order-preserving unsigned form, then 0xFFFFFFFF - v (a larger key is a
// larger logit, or the same logit at a smaller id). 0 is below every key. -0.0 and +0.0 compare equal, as in
// the reference's `l == l.max()`, so both map to the key of +0.0.
AIB_DEV unsigned long long pick_key(float x, int v) {
  const uint32_t b = x == 0.0f ? 0u : __float_as_uint(x);
  const uint32_t u = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(v));
}

// Candidates (t, v) with HI[t, v] >= LO[t], appended as t << 24 | v; with `fill`, every other (t, v) gets
// fill[t * ldf + v] = -inf (the candidates' exact logits are written there afterwards).
__global__ void __launch_bounds__(kThreads) cand_kernel(const float* __restrict__ HI, int ldhi,
                                                        const float* __restrict__ LO, int T, int V, int* list,
                                                        int* count, float* fill, int ldf) {
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x;
  if (i < static_cast<long long>(V) * T) {
    const int t = static_cast<int>(i / V), v = static_cast<int>(i % V);
    if (HI[static_cast<size_t>(t) * ldhi + v] >= LO[t])
      list[atomicAdd(count, 1)] = (t << 24) | v;
    else if (fill)
      fill[static_cast<size_t>(t) * ldf + v] = -INFINITY;
  }
  pdl_trigger();
}

constexpr int kXWarps = 4;  // candidates in flight per CTA (each warp: the row's fp32 products in shared memory)

struct GreedyArgs {
  const float* h;
  int ldh;
  aib_c12 W;
  const int* list;
  int* count;
  int T;
  int64_t* out;
  unsigned long long* best;  // [16], zero between calls
  int* ticket;
  float* logits;  // non-null: write every candidate's exact logit to logits[t * ldl + v] instead of picking
  int ldl;
};

// Exact logit of every listed candidate: the warp decodes row v from the codec planes (4 columns per lane
// per step, exceptions patched from the CSR afterwards) into products w_d * h_d rounded to fp32, then lane 0
// adds them in column order (head.py:19-26); atomicMax of the 64-bit key picks the winner. The last CTA
// writes the ids and clears the keys and the candidate count.
__global__ void __launch_bounds__(kXWarps * 32) exact_kernel(GreedyArgs a) {
  extern __shared__ __align__(16) float prod[];  // [kXWarps][D]
  __shared__ int last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, D = a.W.K;
  pdl_wait();
  const int n = *a.count;
  float* p = prod + warp * D;
  const uint32_t base = static_cast<uint32_t>(a.W.base);
  for (int i = blockIdx.x * kXWarps + warp; i < n; i += gridDim.x * kXWarps) {
    const int e = a.list[i], t = e >> 24, v = e & 0xFFFFFF;
    const uint8_t* m8 = a.W.m8 + static_cast<size_t>(v) * D;
    const uint8_t* e4 = a.W.e4 + static_cast<size_t>(v) * (D / 2);
    const float* h = a.h + static_cast<size_t>(t) * a.ldh;
    for (int d0 = lane * 4; d0 < D; d0 += 128) {
      const uint32_t mw = *reinterpret_cast<const uint32_t*>(m8 + d0);
      const int i0 = d0 & 255;
      const uint32_t ew = *reinterpret_cast<const uint32_t*>(e4 + (d0 >> 8) * 128 + (i0 & 127)) >> ((i0 & 128) ? 4 : 0);
      const float4 x = *reinterpret_cast<const float4*>(h + d0);
      const float xs[4] = {x.x, x.y, x.z, x.w};
      float4 o;
      float* op = &o.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t m = (mw >> (8 * k)) & 0xFFu, code = (ew >> (8 * k)) & 15u;
        const float w = __uint_as_float(((m & 0x80u) << 24) | (((code + base) & 0xFFu) << 23) | ((m & 0x7Fu) << 16));
        op[k] = __fmul_rn(w, xs[k]);  // code-15 elements are replaced below
      }
      *reinterpret_cast<float4*>(p + d0) = o;
    }
    __syncwarp();
    for (int q = a.W.rp[v] + lane; q < a.W.rp[v + 1]; q += 32) {
      const int col = a.W.ec[q];
      p[col] = __fmul_rn(a.W.ev[q], h[col]);
    }
    __syncwarp();
    if (lane == 0) {
      float sum = 0.0f;
      for (int d = 0; d < D; d += 4) {
        const float4 y = *reinterpret_cast<const float4*>(p + d);
        sum = __fadd_rn(sum, y.x);
        sum = __fadd_rn(sum, y.y);
        sum = __fadd_rn(sum, y.z);
        sum = __fadd_rn(sum, y.w);
      }
      if (a.logits)
        a.logits[static_cast<size_t>(t) * a.ldl + v] = sum;
      else
        atomicMax(a.best + t, pick_key(sum, v));
    }
    __syncwarp();  // the products are rewritten by the next candidate
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(a.ticket, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (last) {
    __threadfence();
    for (int t = threadIdx.x; t < a.T && !a.logits; t += kXWarps * 32) {
      const unsigned long long k = atomicExch(a.best + t, 0ull);
      a.out[t] = k ? static_cast<int64_t>(0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull)) : -1;
    }
    if (threadIdx.x == 0) {
      *a.count = 0;
      *a.ticket = 0;
    }
  }
  pdl_trigger();
}

template <typename K>
static int resident_grid(K kernel, int threads, size_t smem, int cap) {
  int per = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kernel, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    per = 1;
  }
  return std::max(1, std::min(kMaxGrid, sm_count() * std::max(1, std::min(per, cap))));
}

// Workspace layout: [0, 256) bounds ticket; CTA maxima [kTokPass][kMaxGrid] floats; greedy block of 256
// bytes (ticket, candidate count); keys [16] u64; candidate list [16][V] ints.
constexpr size_t kPartOff = 256;
constexpr size_t kGreedyOff = kPartOff + static_cast<size_t>(kTokPass) * kMaxGrid * sizeof(float);
constexpr size_t kBestOff = kGreedyOff + 256;
constexpr size_t kListOff = kBestOff + 16 * 8;

template <int TT>
static int launch_bounds_tt(const BoundsArgs& a, size_t smem, cudaStream_t s) {
  const int rc = allow_smem(bounds_kernel<TT>, smem);
  if (rc) return rc;
  const int grid = resident_grid(bounds_kernel<TT>, kThreads, smem, 4);
  return launch(bounds_kernel<TT>, dim3(grid), dim3(kThreads), smem, s, "aib_head8_bounds", a);
}

}  // namespace head8
}  // namespace aib

using namespace aib;

extern "C" {

int aib_head8_tables(const uint16_t* w, int V, int D, int8_t* Q, float* S, float* C1, float* C2, float* AM,
                     void* stream) {
  if (!w || !Q || !S || !C1 || !C2 || !AM || V <= 0 || D <= 0)
    return fail(AIB_EINVAL, "aib_head8_tables: bad arguments");
  const long long threads = static_cast<long long>(V) * 32;
  const int grid = static_cast<int>((threads + head8::kThreads - 1) / head8::kThreads);
  return launch(head8::tables_kernel, dim3(grid), dim3(head8::kThreads), 0, static_cast<cudaStream_t>(stream),
                "aib_head8_tables", w, V, D, Q, S, C1, C2, AM);
}

size_t aib_head8_workspace(int V, int D, int T) {
  (void)D;
  (void)T;
  if (V <= 0) return 0;
  return head8::kListOff + static_cast<size_t>(16) * V * sizeof(int);
}

int aib_head8_bounds_topk(const float* h, int T, int ldh, const int8_t* Q, const float* S, const float* C1,
                          const float* C2, const float* AM, int V, int D, float* HI, int ldhi, float* LO, int k,
                          void* ws, size_t ws_bytes, void* stream) {
  if (!h || !Q || !S || !C1 || !C2 || !AM || !HI || !LO || V <= 0 || D <= 0 || T < 1 || T > 16 || ldh < D ||
      ldhi < V || V >= (1 << 24) || k < 1 || k > 32)
    return fail(AIB_EINVAL, "aib_head8_bounds: bad arguments");
  if (D % 16 || (reinterpret_cast<uintptr_t>(Q) & 15))
    return fail(AIB_EINVAL, "aib_head8_bounds: D must be a multiple of 16 and Q 16-byte aligned (D=%d)", D);
  if (!ws || ws_bytes < aib_head8_workspace(V, D, T) || (reinterpret_cast<uintptr_t>(ws) & 15))
    return fail(AIB_EWORKSPACE, "aib_head8_bounds: workspace %zu < %zu bytes", ws_bytes,
                aib_head8_workspace(V, D, T));
  const int nch = (D + head8::kChunk - 1) / head8::kChunk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int t0 = 0; t0 < T; t0 += head8::kTokPass) {
    const int tt = std::min(head8::kTokPass, T - t0);
    const size_t smem = (static_cast<size_t>(tt) * nch * head8::kChunk + 2 * head8::kTokPass) * sizeof(float);
    head8::BoundsArgs a{h + static_cast<size_t>(t0) * ldh, ldh, tt, Q, S, C1, C2, AM, V, D, nch,
                        HI + static_cast<size_t>(t0) * ldhi, ldhi, LO + t0,
                        reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + head8::kPartOff), static_cast<int*>(ws),
                        k};
    const int rc = tt == 1   ? head8::launch_bounds_tt<1>(a, smem, s)
                   : tt == 2 ? head8::launch_bounds_tt<2>(a, smem, s)
                   : tt <= 4 ? head8::launch_bounds_tt<4>(a, smem, s)
                             : head8::launch_bounds_tt<8>(a, smem, s);
    if (rc) return rc;
  }
  return AIB_OK;
}

int aib_head8_bounds(const float* h, int T, int ldh, const int8_t* Q, const float* S, const float* C1,
                     const float* C2, const float* AM, int V, int D, float* HI, int ldhi, float* LO, void* ws,
                     size_t ws_bytes, void* stream) {
  return aib_head8_bounds_topk(h, T, ldh, Q, S, C1, C2, AM, V, D, HI, ldhi, LO, 1, ws, ws_bytes, stream);
}

// Candidates HI >= LO, then their exact logits: the greedy pick (out) or, with `logits`, the logits row itself
// (-inf outside the candidates).
static int head8_candidates(const float* h, int T, int ldh, const aib_c12* W, const float* HI, int ldhi,
                            const float* LO, int64_t* out, float* logits, int ldl, void* ws, size_t ws_bytes,
                            void* stream) {
  if (!h || !W || !W->m8 || !W->e4 || !W->rp || (W->n_exc > 0 && (!W->ec || !W->ev)) || !HI || !LO ||
      (!out && !logits) || T < 1 || T > 16 || W->N <= 0 || W->K <= 0 || W->K % 256 || ldh < W->K || ldhi < W->N ||
      W->N >= (1 << 24) || (logits && ldl < W->N))
    return fail(AIB_EINVAL, "aib_head8_greedy: bad arguments");
  if ((ldh & 3) || (reinterpret_cast<uintptr_t>(h) & 15) || (reinterpret_cast<uintptr_t>(W->m8) & 15) ||
      (reinterpret_cast<uintptr_t>(W->e4) & 15))
    return fail(AIB_EINVAL, "aib_head8_greedy: h rows, m8 and e4 must be 16-byte aligned");
  if (!ws || ws_bytes < aib_head8_workspace(W->N, W->K, T) || (reinterpret_cast<uintptr_t>(ws) & 15))
    return fail(AIB_EWORKSPACE, "aib_head8_greedy: workspace %zu < %zu bytes", ws_bytes,
                aib_head8_workspace(W->N, W->K, T));
  const size_t smem = static_cast<size_t>(head8::kXWarps) * W->K * sizeof(float);
  int rc = allow_smem(head8::exact_kernel, smem);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* w8 = static_cast<uint8_t*>(ws);
  int* ticket = reinterpret_cast<int*>(w8 + head8::kGreedyOff);
  int* count = ticket + 1;
  int* list = reinterpret_cast<int*>(w8 + head8::kListOff);
  const long long n = static_cast<long long>(W->N) * T;
  rc = launch(head8::cand_kernel, dim3(static_cast<int>((n + head8::kThreads - 1) / head8::kThreads)),
              dim3(head8::kThreads), 0, s, "aib_head8_greedy (candidates)", HI, ldhi, LO, T, W->N, list, count,
              logits, ldl);
  if (rc) return rc;
  head8::GreedyArgs a{h, ldh, *W, list, count, T, out,
                      reinterpret_cast<unsigned long long*>(w8 + head8::kBestOff), ticket, logits, ldl};
  const int grid = head8::resident_grid(head8::exact_kernel, head8::kXWarps * 32, smem, 4);
  return launch(head8::exact_kernel, dim3(grid), dim3(head8::kXWarps * 32), smem, s, "aib_head8_greedy", a);
}

int aib_head8_greedy(const float* h, int T, int ldh, const aib_c12* W, const float* HI, int ldhi, const float* LO,
                     int64_t* out, void* ws, size_t ws_bytes, void* stream) {
  if (!out) return fail(AIB_EINVAL, "aib_head8_greedy: out is NULL");
  return head8_candidates(h, T, ldh, W, HI, ldhi, LO, out, nullptr, 0, ws, ws_bytes, stream);
}

int aib_head8_candidate_logits(const float* h, int T, int ldh, const aib_c12* W, const float* HI, int ldhi,
                               const float* LO, float* logits, int ldl, void* ws, size_t ws_bytes, void* stream) {
  if (!logits) return fail(AIB_EINVAL, "aib_head8_candidate_logits: logits is NULL");
  return head8_candidates(h, T, ldh, W, HI, ldhi, LO, nullptr, logits, ldl, ws, ws_bytes, stream);
}

}  // extern "C"
