// Decode attention over a bf16 KV cache (sm_100a).
//
// aib_rope_attn_decode replaces the reference's fused T=1 step rope_attn_k
// (`ramvi/engine/ramvi_engine/kernels/tkernels.py:164-213`): QK-RMSNorm + half-split RoPE of the q heads of
// a KV group and of the group's k, bf16 rounding of the current k/v (tkernels.py:187-190), cache write at
// pos, and online-softmax attention over positions 0..pos-1 from the cache plus the current token.
// aib_qk_rope_cache / aib_attn_cached replace the batched pair qk_rope_cache_k / attn_k (:82-150).
//
// B200 design: flash-decoding. The grid is (S splits, KV groups[, T tokens]); each CTA serves all G = H/KV
// query heads of its group, so every K/V row is read from HBM once per group. Each CTA writes a partial
// (m, l, acc) to the workspace; the last CTA of a group (atomic ticket, no waiting) merges the partials in
// split order -- starting, like the reference, from the current token -- so results are deterministic. The
// ticket counters return to zero.
// Data movement: before the grid-dependency wait a CTA asks L2 to prefetch its K/V rows (bulk L2 prefetch
// of two contiguous ranges, addressed from a possibly stale read of pos: a hint only, always in bounds).
// After the wait every warp starts asynchronous 16-byte copies (cp.async, coalesced 512 bytes per warp
// instruction) of its first block of 32 K rows and 32 V rows into its own shared-memory slot, and only then
// runs the q/k norm + RoPE prologue, so the HBM latency overlaps the prologue. K rows land with a 16-byte
// pad per row so that lane = position reads are bank-conflict free. Each warp pipelines K and V through
// its one slot: scores on K(i) -> copy K(i+1) -> softmax -> P.V on V(i) -> copy V(i+1).
// Compute: lane = position for the scores (q broadcast from shared memory, no reduction across lanes); the
// block's softmax and P.V run warp-wide with the lane owning HD/32 dimensions. The warps' states are
// combined once, at the end. The merge loads every split's partial in parallel (weights exp(m_s - M) first,
// then the sums).
#include <algorithm>
#include "common.cuh"

namespace aib {
namespace attn {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int GMAX = 8;

constexpr int kBlk = 32;  // positions per warp block (lane = position)
constexpr int kMaxSplits = 32;

// Per-warp K/V slot: kBlk K rows then kBlk V rows, each at a padded stride (HD + 8 bf16: consecutive rows
// start 16 bytes apart modulo 128, so the 8 row addresses of an ldmatrix hit 8 different bank groups).
template <int HD>
__host__ __device__ constexpr int k_stride() {
  return (HD + 8) * 2;
}
template <int HD>
__host__ __device__ constexpr size_t slot_bytes() {
  return static_cast<size_t>(kBlk) * 2 * k_stride<HD>();  // K rows, then V rows, both padded
}
__host__ __device__ constexpr size_t cmax(size_t a, size_t b) { return a > b ? a : b; }
// Dynamic shared memory: the warps' K/V slots; afterwards reused for the warps' final states
// [kWarps][GMAX][HD + 2] and by the merge to stage the splits' partials (kMaxSplits x GMAX x (HD + 2) floats).
template <int HD>
__host__ __device__ constexpr size_t ring_bytes() {
  return cmax(kWarps * slot_bytes<HD>(),
              static_cast<size_t>(kMaxSplits > kWarps ? kMaxSplits : kWarps) * GMAX * (HD + 2) * sizeof(float));
}

// 16-byte asynchronous global -> shared copy (L2 only), and its group bookkeeping.
AIB_DEV void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
AIB_DEV void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
AIB_DEV void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Hint L2 to fetch [p, p + bytes) (bytes a multiple of 16, p 16-byte aligned).
AIB_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Distributed shared memory: the generic address of the same shared-memory location in cluster CTA `rank`,
// and a full cluster barrier (release / acquire: shared-memory writes to peers before it are visible after it).
AIB_DEV float* cluster_map(float* p, uint32_t rank) {
  uint64_t r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<float*>(r);
}
AIB_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Warp-cooperative copy of `cnt` (<= kBlk) consecutive cache rows into a slot region with row stride STRIDE:
// 16-byte chunk c of the source goes to row c / (HD/8), chunk c % (HD/8); consecutive lanes take
// consecutive chunks (coalesced).
template <int HD, int STRIDE>
AIB_DEV void copy_rows(uint8_t* dst, const uint16_t* rows, int cnt) {
  constexpr int CPR = HD / 8;
  const int lane = threadIdx.x & 31;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(rows);
  for (int c = lane; c < cnt * CPR; c += 32) cp16(dst + (c / CPR) * STRIDE + (c % CPR) * 16, src + c * 16);
}

// This warp's share [w0, w1) of the CTA range [j0, j1).
AIB_DEV void warp_range(int j0, int j1, int* w0, int* w1) {
  const int warp = threadIdx.x >> 5;
  const int n = j1 - j0, per_warp = (n + kWarps - 1) / kWarps;
  *w0 = j0 + min(n, warp * per_warp);
  *w1 = j0 + min(n, (warp + 1) * per_warp);
}

// Start the copies of this warp's first block (two commit groups, K then V, possibly empty). Must be called
// by every thread of the CTA exactly once before attend_range.
template <int HD>
AIB_DEV void attend_start(uint8_t* ring, const uint16_t* kc, const uint16_t* vc, int j0, int j1) {
  int w0, w1;
  warp_range(j0, j1, &w0, &w1);
  uint8_t* kslot = ring + (threadIdx.x >> 5) * slot_bytes<HD>();
  const int cnt = min(kBlk, w1 - w0);
  if (cnt > 0) copy_rows<HD, k_stride<HD>()>(kslot, kc + static_cast<size_t>(w0) * HD, cnt);
  cp_commit();
  if (cnt > 0) copy_rows<HD, k_stride<HD>()>(kslot + kBlk * k_stride<HD>(), vc + static_cast<size_t>(w0) * HD, cnt);
  cp_commit();
}

// L2 prefetch of the K and V rows [j0, j1) of one group (one thread).
template <int HD>
AIB_DEV void prefetch_range(const uint16_t* kc, const uint16_t* vc, int j0, int j1) {
  if (j1 <= j0) return;
  const uint32_t bytes = static_cast<uint32_t>(j1 - j0) * HD * 2;
  prefetch_l2(kc + static_cast<size_t>(j0) * HD, bytes);
  prefetch_l2(vc + static_cast<size_t>(j0) * HD, bytes);
}

template <int HD>
struct Smem {
  float q[GMAX][HD];
  float kcur[HD];
  float vcur[HD];
  float cur_score[GMAX];
  float cs[HD / 2], sn[HD / 2];
  float raw[GMAX + 2][HD];       // the group's q rows, its k row and its v row as produced by the qkv GEMV
  uint16_t wq[HD], wk[HD];       // q / k norm weights (bf16 bits)
  float pw[kWarps][GMAX][kBlk];  // each warp's block probabilities
  float mw[kMaxSplits][GMAX];    // merge weights exp(m_s - M) per split
  float mM[GMAX], mL[GMAX], mc[GMAX], ones[GMAX];
  float cwt[kWarps][GMAX];  // the warps' weights exp(m_w - M) in the CTA's combine
  float cM[GMAX];
  long long pos_spec;  // pos as read before the grid dependency resolved (one read for the whole CTA)
  int last;
};

// RMSNorm (weight w) + RoPE of one head vector held by a warp: lane owns elements lane + 32*i.
template <int HD>
AIB_DEV void norm_rope(const float* v, const uint16_t* w, const float* cs, const float* sn, float eps, float* out) {
  constexpr int PER = HD / 32, HALF = HD / 2;
  const int lane = threadIdx.x & 31;
  float e[PER];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    e[i] = v[lane + 32 * i];
    ss += e[i] * e[i];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / static_cast<float>(HD) + eps);
#pragma unroll
  for (int i = 0; i < PER / 2; ++i) {
    const int r = lane + 32 * i;  // r < HALF, partner r + HALF
    const float a = bf16_to_f32(w[r]) * (e[i] * rs);
    const float b = bf16_to_f32(w[r + HALF]) * (e[i + PER / 2] * rs);
    out[r] = a * cs[r] - b * sn[r];
    out[r + HALF] = b * cs[r] + a * sn[r];
  }
}

// ldmatrix: four 8x8 b16 matrices, lane L gives the row address of matrix L / 8, row L % 8; with .trans each
// matrix arrives transposed.
AIB_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
AIB_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// x = p0 + p1 + p2 in bf16 parts (round to nearest even at each step): fp32-faithful products on bf16 MMAs
AIB_DEV void split3_pair(float lo, float hi, uint32_t* w) {  // w[part] = (hi part << 16) | lo part
#pragma unroll
  for (int k = 0; k < 3; ++k) {  // the same roundings, one conversion instruction per pair
    w[k] = bf16x2_rn(lo, hi);
    lo -= __uint_as_float(w[k] << 16);
    hi -= __uint_as_float(w[k] & 0xFFFF0000u);
  }
}

// Attention of the G query heads in sm.q over cache rows [j0, j1) of one group, on the tensor cores. Warp w
// takes a contiguous slice of the range in blocks of 32 positions, the block's K and V rows in the warp's
// slot (attend_start issued the first block's copies). mma.sync m16n8k16 with bf16 operands: the K and V
// rows are exact bf16, q and the probabilities enter as three bf16 parts each, so products and fp32
// accumulation are as accurate as fp32 FMAs.
//  1. wait for K(i); S = K q^T: A = K rows (ldmatrix), B = q (heads as the 8 columns), 2 position tiles x
//     HD/16 dimension steps x 3 parts; then start the copy of K(i+1) into the slot;
//  2. per head: block max and sum over the 32 positions (lanes holding the same head), p = exp(s - m'),
//     rescale alpha = exp(m - m'); p goes to shared memory to be re-read in the B layout;
//  3. wait for V(i); O^T += V^T P: A = V rows transposed (ldmatrix.trans), B = p (3 parts), HD/16 dimension
//     tiles x 2 position steps; then start the copy of V(i+1).
// Lane (g, t) accumulates O^T rows (dims) g and g + 8 of every 16-dim tile for heads 2t and 2t + 1. The
// warps' (m, l, acc) are combined in warp order at the end and written as the CTA partial to `part`.
template <int HD, int G>
AIB_DEV void attend_range(Smem<HD>& sm, uint8_t* ring, const uint16_t* kc, const uint16_t* vc, int j0, int j1,
                          float scale, float* part) {
  constexpr int KS = k_stride<HD>(), NT = HD / 16;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  int w0, w1;
  warp_range(j0, j1, &w0, &w1);
  uint8_t* kslot = ring + warp * slot_bytes<HD>();
  uint8_t* vslot = kslot + kBlk * KS;
  const uint32_t ks32 = smem_u32(kslot), vs32 = smem_u32(vslot);
  // B fragments of q (head g, dims 16 s + 2t, +1, +8, +9), three parts, for every dimension step
  uint32_t bq[NT][3][2];
#pragma unroll
  for (int st = 0; st < NT; ++st) {
    const float* q = sm.q[g];
    const bool hv = g < G;
    const int d = st * 16 + 2 * t;
    uint32_t w[3];
    split3_pair(hv ? q[d] : 0.0f, hv ? q[d + 1] : 0.0f, w);
    uint32_t w2[3];
    split3_pair(hv ? q[d + 8] : 0.0f, hv ? q[d + 9] : 0.0f, w2);
#pragma unroll
    for (int k = 0; k < 3; ++k) bq[st][k][0] = w[k], bq[st][k][1] = w2[k];
  }
  const int h0 = 2 * t, h1 = 2 * t + 1;  // this lane's heads in the accumulators
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  float acc[NT][4];
#pragma unroll
  for (int dt = 0; dt < NT; ++dt) acc[dt][0] = acc[dt][1] = acc[dt][2] = acc[dt][3] = 0.0f;
  float* pw = &sm.pw[warp][0][0];  // [GMAX][kBlk] probabilities of the block
  // ldmatrix row addresses: lane L -> matrix L / 8, row L % 8
  const int mr = (lane & 7) + ((lane >> 3) & 1) * 8, mc = (lane >> 4) * 8;  // A (non-transposed) tile
  const int vr = (lane & 7) + (lane >> 4) * 8, vcol = ((lane >> 3) & 1) * 8;  // V tile, transposed load
  for (int b0 = w0; b0 < w1; b0 += kBlk) {
    const int cnt = min(kBlk, w1 - b0);
    const int nb0 = b0 + kBlk, ncnt = max(0, min(kBlk, w1 - nb0));
    // 1. scores (K(i) is the older of the two pending groups)
    cp_wait<1>();
    __syncwarp();
    float sc[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.0f;
#pragma unroll
      for (int st = 0; st < NT; ++st) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(ks32 + (mt * 16 + mr) * KS + (st * 16 + mc) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int k = 0; k < 3; ++k) mma_bf16(sc[mt], a0, a1, a2, a3, bq[st][k][0], bq[st][k][1]);
      }
    }
    __syncwarp();  // every lane is done with the K rows
    if (ncnt > 0) copy_rows<HD, KS>(kslot, kc + static_cast<size_t>(nb0) * HD, ncnt);
    cp_commit();
    // 2. block softmax: sc[mt][0/1] position mt*16+g heads h0/h1, sc[mt][2/3] position mt*16+g+8
    float s0[4], s1[4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int pos = mt * 16 + g + hi * 8;
        const bool ok = pos < cnt;
        s0[mt * 2 + hi] = ok ? sc[mt][hi * 2] * scale : -INFINITY;
        s1[mt * 2 + hi] = ok ? sc[mt][hi * 2 + 1] * scale : -INFINITY;
      }
    float mb0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s0[2], s0[3]));
    float mb1 = fmaxf(fmaxf(s1[0], s1[1]), fmaxf(s1[2], s1[3]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mb0 = fmaxf(mb0, __shfl_xor_sync(0xffffffffu, mb0, o));
      mb1 = fmaxf(mb1, __shfl_xor_sync(0xffffffffu, mb1, o));
    }
    const float mn0 = fmaxf(m0, mb0), mn1 = fmaxf(m1, mb1);
    float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int pos = (i >> 1) * 16 + g + (i & 1) * 8;
      const float p0 = s0[i] == -INFINITY ? 0.0f : expf(s0[i] - mn0);
      const float p1 = s1[i] == -INFINITY ? 0.0f : expf(s1[i] - mn1);
      ps0 += p0;
      ps1 += p1;
      pw[h0 * kBlk + pos] = p0;  // h0, h1 < GMAX always; heads >= G carry zeros (q = 0) and are ignored
      pw[h1 * kBlk + pos] = p1;
    }
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, o);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, o);
    }
    const float al0 = m0 == -INFINITY ? 0.0f : expf(m0 - mn0), al1 = m1 == -INFINITY ? 0.0f : expf(m1 - mn1);
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
    m0 = mn0;
    m1 = mn1;
    // 3. P.V (V(i) is now the older pending group); rows past cnt hold stale bytes: zero them first
    cp_wait<1>();
    if (cnt < kBlk)
      for (int i = lane; i < (kBlk - cnt) * (HD / 8); i += 32)
        *reinterpret_cast<uint4*>(vslot + (cnt + i / (HD / 8)) * KS + (i % (HD / 8)) * 16) = make_uint4(0, 0, 0, 0);
    __syncwarp();
    // B fragments of p (positions 16 s + 2t, +1, +8, +9 for head g), three parts
    uint32_t bp[2][3][2];
#pragma unroll
    for (int ps = 0; ps < 2; ++ps) {
      const float* pr = pw + (g < GMAX ? g : 0) * kBlk + ps * 16 + 2 * t;
      const float2 lo = *reinterpret_cast<const float2*>(pr);
      const float2 hi = *reinterpret_cast<const float2*>(pr + 8);
      const bool hv = g < G;
      uint32_t w[3], w2[3];
      split3_pair(hv ? lo.x : 0.0f, hv ? lo.y : 0.0f, w);
      split3_pair(hv ? hi.x : 0.0f, hv ? hi.y : 0.0f, w2);
#pragma unroll
      for (int k = 0; k < 3; ++k) bp[ps][k][0] = w[k], bp[ps][k][1] = w2[k];
    }
#pragma unroll
    for (int dt = 0; dt < NT; ++dt) {
      acc[dt][0] *= al0;
      acc[dt][1] *= al1;
      acc[dt][2] *= al0;
      acc[dt][3] *= al1;
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(vs32 + (ps * 16 + vr) * KS + (dt * 16 + vcol) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int k = 0; k < 3; ++k) mma_bf16(acc[dt], a0, a1, a2, a3, bp[ps][k][0], bp[ps][k][1]);
      }
    }
    __syncwarp();  // pw and the V rows are rewritten next
    if (ncnt > 0) copy_rows<HD, KS>(vslot, vc + static_cast<size_t>(nb0) * HD, ncnt);
    cp_commit();
  }
  cp_wait<0>();     // nothing of this thread may land in the ring once it is reused below
  __syncthreads();  // every warp is done with its slot
  // this warp's state for its heads: m, l and O rows (dims dt*16 + g, + 8)
  float* wst = reinterpret_cast<float*>(ring);  // [kWarps][GMAX][HD + 2]
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int h = 2 * t + hh;
    if (h < G) {
      float* dst = wst + (static_cast<size_t>(warp) * GMAX + h) * (HD + 2);
#pragma unroll
      for (int dt = 0; dt < NT; ++dt) {
        dst[dt * 16 + g] = acc[dt][hh];
        dst[dt * 16 + g + 8] = acc[dt][2 + hh];
      }
      if (g == 0) {
        dst[HD] = hh ? m1 : m0;
        dst[HD + 1] = hh ? l1 : l0;
      }
    }
  }
  __syncthreads();
  // combine the warps in order: the weights exp(m_w - M) once per (warp, head) (0 for a warp without
  // positions), then fixed-order weighted sums
  if (threadIdx.x < G * kWarps) {
    const int h = threadIdx.x / kWarps, w = threadIdx.x % kWarps;
    float M = -INFINITY;
    for (int w2 = 0; w2 < kWarps; ++w2) M = fmaxf(M, wst[(w2 * GMAX + h) * (HD + 2) + HD]);
    const float mw = wst[(w * GMAX + h) * (HD + 2) + HD];
    sm.cwt[w][h] = (M == -INFINITY || mw == -INFINITY) ? 0.0f : expf(mw - M);
    if (w == 0) sm.cM[h] = M;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
    const int h = idx / HD, d = idx % HD;
    float A = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) A += wst[(w * GMAX + h) * (HD + 2) + d] * sm.cwt[w][h];
    float* ph = part + static_cast<size_t>(h) * (HD + 2);
    ph[d] = A;
    if (d == 0) {
      float L = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) L += wst[(w * GMAX + h) * (HD + 2) + HD + 1] * sm.cwt[w][h];
      ph[HD] = sm.cM[h];
      ph[HD + 1] = L;
    }
  }
  __syncthreads();  // the buffer is reused by the merge
}

// Merge S partials in split order on top of an initial state (m0, l0, acc0[d]; null = empty) and write out.
// The group's partial block (S x G x (HD+2) floats, contiguous) is first copied into shared memory (`stage`,
// the now idle K/V ring) with asynchronous 16-byte copies all in flight at once, then merged from there:
// weights exp(m_s - M) per split, fixed-order sums.
template <int HD>
AIB_DEV void merge_write(Smem<HD>& sm, float* stage, const float* parts, int S, int G, const float* m0,
                         const float* l0, const float* acc0, float* out) {
  const int nf = S * G * (HD + 2);
  const int n4 = nf / 4;
  if (parts == stage) {  // already in shared memory (cluster merge)
  } else if ((nf & 3) == 0 && (reinterpret_cast<uintptr_t>(parts) & 15) == 0) {
    // asynchronous 16-byte copies from L2 (every copy in flight at once), then one wait
    for (int i = threadIdx.x; i < n4; i += kThreads) cp16(stage + 4 * i, parts + 4 * i);
    cp_commit();
    cp_wait<0>();
  } else {
    for (int i = threadIdx.x; i < nf; i += kThreads) stage[i] = __ldcg(parts + i);
  }
  __syncthreads();
  {  // statistics: warp h for head h, lane s for split s (S <= 32), fixed-order sums
    const int lane = threadIdx.x & 31, h = threadIdx.x >> 5;
    if (h < G) {
      const float ms = lane < S ? stage[(lane * G + h) * (HD + 2) + HD] : -INFINITY;
      float M = m0 ? m0[h] : -INFINITY;
      float mm = ms;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, o));
      M = fmaxf(M, mm);
      const float w = (ms == -INFINITY || M == -INFINITY) ? 0.0f : expf(ms - M);
      if (lane < S) sm.mw[lane][h] = w;
      float lw = lane < S ? w * stage[(lane * G + h) * (HD + 2) + HD + 1] : 0.0f;
      // sum over the splits in a fixed butterfly order (deterministic; a serial chain of S shuffles was ~3 us)
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
      const float L = ((m0 && M != -INFINITY) ? l0[h] * expf(m0[h] - M) : 0.0f) + lw;
      if (lane == 0) {
        sm.mL[h] = L;
        sm.mc[h] = (m0 && M != -INFINITY) ? expf(m0[h] - M) : 0.0f;
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
    const int h = idx / HD, d = idx % HD;
    float a = acc0 ? sm.mc[h] * acc0[d] : 0.0f;
    for (int s = 0; s < S; ++s) a += sm.mw[s][h] * stage[(s * G + h) * (HD + 2) + d];
    out[h * HD + d] = sm.mL[h] > 0.0f ? a / sm.mL[h] : 0.0f;
  }
}

// ------------------------------------------------------------------------------ fused T = 1 step
// blockIdx.z = b selects one of B independent sequences (batched decode): its qkv row (qkv + b * qkv_ld), its
// position pos_p[b], its caches (kc / vc + b * kv_bstride elements) and its output row (out + b * out_ld); the
// split partials and tickets of (b, group) use slot b * KV + g of the workspace.
template <int HD, int G>
__global__ void __launch_bounds__(kThreads)
    rope_attn_kernel(const float* __restrict__ qkv, const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn,
                     const float* __restrict__ inv, const int64_t* __restrict__ pos_p, uint16_t* kc, uint16_t* vc,
                     float* __restrict__ out, int H, int KV, int maxt, float eps, float scale, float* ws_part,
                     int* ws_cnt, int qkv_ld, long long kv_bstride, int out_ld, int clustered) {
  __shared__ Smem<HD> sm;
  extern __shared__ __align__(128) uint8_t ring[];
  const int s = blockIdx.x, S = gridDim.x, g = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot = b * KV + g;
  qkv += static_cast<size_t>(b) * qkv_ld;
  pos_p += b;
  kc += static_cast<size_t>(b) * kv_bstride;
  vc += static_cast<size_t>(b) * kv_bstride;
  out += static_cast<size_t>(b) * out_ld;
  uint16_t* kg = kc + static_cast<size_t>(g) * maxt * HD;
  uint16_t* vg = vc + static_cast<size_t>(g) * maxt * HD;
  // Before the grid dependency resolves: the constant inputs (RoPE frequencies, q / k norm weights) and,
  // from a speculative read of pos, this split's first K/V rows. The cache rows below pos were written by
  // the attention of earlier steps, long complete (the kernels in flight at once are the few whose CTAs fit
  // the SMs together), and no kernel of this step writes them; the rows are re-fetched below if pos turns
  // out different.
  const float inv_r = threadIdx.x < HD / 2 ? inv[threadIdx.x] : 0.0f;
  for (int d = threadIdx.x; d < HD; d += kThreads) {
    sm.wq[d] = qn[d];
    sm.wk[d] = kn[d];
  }
  if (threadIdx.x == 0) sm.pos_spec = *reinterpret_cast<const volatile long long*>(pos_p);
  __syncthreads();
  const long long pos_spec = sm.pos_spec;
  const int n_spec = (pos_spec > 0 && pos_spec < maxt) ? static_cast<int>(pos_spec) : 0;
  const int chunk_spec = (n_spec + S - 1) / S;
  const int j0s = min(n_spec, s * chunk_spec), j1s = min(n_spec, j0s + chunk_spec);
  attend_start<HD>(ring, kg, vg, j0s, j1s);
  pdl_wait();
  // every CTA of this grid is resident by now: the next kernel may launch onto SMs as they free up (it waits
  // for this grid to complete before it reads anything written here)
  pdl_trigger();
  // pos and the group's q, k and v rows in one round trip
  const long long pos_ll = *pos_p;
  for (int i = threadIdx.x; i < (G + 2) * HD; i += kThreads) {
    const int r = i / HD, d = i % HD;
    const int row = r < G ? g * G + r : (r == G ? H + g : H + KV + g);
    sm.raw[r][d] = qkv[static_cast<size_t>(row) * HD + d];
  }
  const bool pos_ok = pos_ll >= 0 && pos_ll < maxt;
  if (!pos_ok && s == 0 && threadIdx.x == 0) set_status(AIB_DEV_BAD_POS);
  const int pos = pos_ok ? static_cast<int>(pos_ll) : 0;
  // this split's share of the past positions 0..pos-1; its first rows start streaming now
  const int n = pos_ok ? pos : 0;
  const int chunk = (n + S - 1) / S;
  const int j0 = min(n, s * chunk), j1 = min(n, j0 + chunk);
  if (j0 != j0s || j1 != j1s) {  // pos moved since the speculative read: drop those rows, fetch the right ones
    cp_wait<0>();
    __syncwarp();
    attend_start<HD>(ring, kg, vg, j0, j1);
  }
  if (threadIdx.x < HD / 2) {
    const float ang = static_cast<float>(pos) * inv_r;
    sm.cs[threadIdx.x] = cosf(ang);
    sm.sn[threadIdx.x] = sinf(ang);
  }
  __syncthreads();
  // warp per vector: the q heads of the group, the group's k (norm, RoPE, bf16 rounding, cache write) and
  // its v (bf16 rounding, cache write); lane owns elements lane + 32 i
  for (int t = warp; t < G + 2; t += kWarps) {
    if (t < G) {
      norm_rope<HD>(sm.raw[t], sm.wq, sm.cs, sm.sn, eps, sm.q[t]);
    } else {
      float* cur = t == G ? sm.kcur : sm.vcur;
      uint16_t* cache = t == G ? kg : vg;
      if (t == G) norm_rope<HD>(sm.raw[G], sm.wk, sm.cs, sm.sn, eps, sm.kcur);
      __syncwarp();
#pragma unroll
      for (int i = 0; i < HD / 32; ++i) {
        const int d = lane + 32 * i;
        const uint16_t b = f32_to_bf16_rne(t == G ? sm.kcur[d] : sm.raw[G + 1][d]);
        cur[d] = bf16_to_f32(b);
        if (s == 0 && pos_ok) cache[static_cast<size_t>(pos) * HD + d] = b;
      }
    }
  }
  __syncthreads();
  for (int h = warp; h < G; h += kWarps) {  // score of the current token
    float sc = 0.0f;
    for (int d = lane; d < HD; d += 32) sc += sm.q[h][d] * sm.kcur[d];
    sc = warp_sum(sc);
    if (lane == 0) sm.cur_score[h] = sc * scale;
  }
  if (clustered) {
    // the group's S splits form one cluster: every CTA writes its partial straight into the shared-memory
    // stage of split 0 (after the ring), one cluster barrier, and split 0 merges them in split order
    float* stage = reinterpret_cast<float*>(ring + ring_bytes<HD>());
    attend_range<HD, G>(sm, ring, kg, vg, j0, j1, scale, cluster_map(stage + s * G * (HD + 2), 0));
    cluster_sync_all();
    if (s == 0) {
      if (threadIdx.x < GMAX) sm.ones[threadIdx.x] = 1.0f;  // the current token enters with weight 1
      __syncthreads();
      merge_write<HD>(sm, stage, stage, S, G, sm.cur_score, sm.ones, sm.vcur, out + static_cast<size_t>(g) * G * HD);
    }
    return;
  }
  float* part = ws_part + (static_cast<size_t>(slot) * S + s) * G * (HD + 2);
  attend_range<HD, G>(sm, ring, kg, vg, j0, j1, scale, part);
  // ordered merge by the last CTA of the group
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&ws_cnt[slot], 1);
    sm.last = (old == S - 1);
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    if (threadIdx.x < GMAX) sm.ones[threadIdx.x] = 1.0f;  // the current token enters with weight 1
    __syncthreads();
    merge_write<HD>(sm, reinterpret_cast<float*>(ring), ws_part + static_cast<size_t>(slot) * S * G * (HD + 2), S, G,
                    sm.cur_score, sm.ones, sm.vcur, out + static_cast<size_t>(g) * G * HD);
    if (threadIdx.x == 0) ws_cnt[slot] = 0;
  }
}

// ------------------------------------------------------------------------------------ batched
template <int HD>
__global__ void qk_rope_cache_kernel(const float* __restrict__ qkv, const uint16_t* __restrict__ qn,
                                     const uint16_t* __restrict__ kn, const float* __restrict__ inv,
                                     const int64_t* __restrict__ pos_p, float* __restrict__ q, uint16_t* kc,
                                     uint16_t* vc, int H, int KV, int maxt, float eps) {
  __shared__ float cs[HD / 2], sn[HD / 2];
  __shared__ float tmp[HD];
  const int h = blockIdx.x, t = blockIdx.y;
  pdl_wait();
  const long long p = *pos_p + t;
  const bool ok = p >= 0 && p < maxt;
  if (!ok && h == 0 && threadIdx.x == 0) set_status(AIB_DEV_BAD_POS);
  const int pos = ok ? static_cast<int>(p) : 0;
  for (int r = threadIdx.x; r < HD / 2; r += blockDim.x) {
    const float ang = static_cast<float>(pos) * inv[r];
    cs[r] = cosf(ang);
    sn[r] = sinf(ang);
  }
  __syncthreads();
  const float* row = qkv + static_cast<size_t>(t) * (H + 2 * KV) * HD;
  if (h < H + KV) {
    if (threadIdx.x < 32) norm_rope<HD>(row + static_cast<size_t>(h) * HD, h < H ? qn : kn, cs, sn, eps, tmp);
    __syncthreads();
    if (h < H) {
      for (int d = threadIdx.x; d < HD; d += blockDim.x) q[(static_cast<size_t>(t) * H + h) * HD + d] = tmp[d];
    } else if (ok) {
      uint16_t* dst = kc + (static_cast<size_t>(h - H) * maxt + pos) * HD;
      for (int d = threadIdx.x; d < HD; d += blockDim.x) dst[d] = f32_to_bf16_rne(tmp[d]);
    }
  } else if (ok) {
    const int g = h - H - KV;
    uint16_t* dst = vc + (static_cast<size_t>(g) * maxt + pos) * HD;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) dst[d] = f32_to_bf16_rne(row[static_cast<size_t>(h) * HD + d]);
  }
  pdl_trigger();
}

template <int HD, int G>
__global__ void __launch_bounds__(kThreads)
    attn_cached_kernel(const float* __restrict__ q, const uint16_t* kc, const uint16_t* vc,
                       const int64_t* __restrict__ pos_p, float* __restrict__ out, int H, int KV, int maxt,
                       float scale, float* ws_part, int* ws_cnt) {
  __shared__ Smem<HD> sm;
  extern __shared__ __align__(128) uint8_t ring[];
  const int s = blockIdx.x, S = gridDim.x, g = blockIdx.y, t = blockIdx.z;
  const uint16_t* kg = kc + static_cast<size_t>(g) * maxt * HD;
  const uint16_t* vg = vc + static_cast<size_t>(g) * maxt * HD;
  if (threadIdx.x == 0) {  // L2 hint from a possibly stale pos: any value it reads gives in-bounds rows
    const long long ph = *reinterpret_cast<const volatile long long*>(pos_p) + t;
    const int n = (ph >= 0 && ph < maxt) ? static_cast<int>(ph) + 1 : 0;
    const int chunk = (n + S - 1) / S, a = min(n, s * chunk);
    prefetch_range<HD>(kg, vg, a, min(n, a + chunk));
  }
  pdl_wait();
  pdl_trigger();  // as in rope_attn_kernel
  const long long p = *pos_p + t;
  const bool ok = p >= 0 && p < maxt;
  const int n = ok ? static_cast<int>(p) + 1 : 0;
  const int chunk = (n + S - 1) / S;
  const int j0 = min(n, s * chunk), j1 = min(n, j0 + chunk);
  attend_start<HD>(ring, kg, vg, j0, j1);
  for (int idx = threadIdx.x; idx < G * HD; idx += kThreads)
    sm.q[idx / HD][idx % HD] = q[(static_cast<size_t>(t) * H + g * G) * HD + idx];
  __syncthreads();
  const size_t slot = static_cast<size_t>(t) * KV + g;
  float* part = ws_part + (slot * S + s) * G * (HD + 2);
  attend_range<HD, G>(sm, ring, kg, vg, j0, j1, scale, part);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&ws_cnt[slot], 1);
    sm.last = (old == S - 1);
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    merge_write<HD>(sm, reinterpret_cast<float*>(ring), ws_part + slot * S * G * (HD + 2), S, G, nullptr, nullptr,
                    nullptr, out + (static_cast<size_t>(t) * H + g * G) * HD);
    if (threadIdx.x == 0) ws_cnt[slot] = 0;
  }
}

// Splits per (group, token): about one CTA per SM in total, capped so that a group's partials
// (S x G x (HD+2) floats) fit the staging ring for the merge.
static int splits(int KV, int T, int G, int HD) {
  const int sms = sm_count();
  int S = std::max(1, sms / (KV * T));
  S = std::min(S, kMaxSplits);
  const size_t ring = HD == 128 ? ring_bytes<128>() : ring_bytes<64>();
  const int fit = static_cast<int>(ring / (static_cast<size_t>(G) * (HD + 2) * sizeof(float)));
  return std::max(1, std::min(S, fit));
}

// Cluster sizes tried for the cluster merge (largest first; 16 is the largest B200 schedules). Off by default
// (g_cluster_sizes = 0: the ticket merge): on this pool's B200s clusters of 16 do not all fit at once (7 of the 8
// groups' clusters) and clusters of 8 (64 CTAs) stream K/V slower than the ticket merge's 144 CTAs gain back. The
// debug knob 3 sets how many sizes are tried; the feasibility query it needs is not allowed inside a CUDA graph
// capture, so a process that turns it on must make its first launch of each shape outside a capture.
static const int kClusterSizes[2] = {16, 8};
int g_cluster_sizes = 0;

// Workspace layout: [ticket counters: kMaxSlots ints][partials]. The counters sit at a fixed offset for every
// T so they are never overwritten by another launch's partials (every launch leaves them at zero).
constexpr int kMaxSlots = 65536;  // KV * T
constexpr size_t kCntBytes = kMaxSlots * sizeof(int);

static size_t ws_bytes_for(int H, int KV, int HD, int T) {
  const int G = H / KV, S = splits(KV, T, G, HD);
  return kCntBytes + static_cast<size_t>(T) * KV * S * G * (HD + 2) * sizeof(float);
}

static int check_heads(int H, int KV, int HD) {
  if (H <= 0 || KV <= 0 || H % KV || H / KV > GMAX || (HD != 64 && HD != 128))
    return fail(AIB_ENOTSUP, "attention: need H %% KV == 0, H/KV <= %d and HD in {64,128} (H=%d KV=%d HD=%d)", GMAX, H,
                KV, HD);
  return AIB_OK;
}

// Instantiation for the group size G = H / KV (1..GMAX) and head dim HD.
template <template <int, int> class KSel, typename Go>
static int dispatch_g(int HD, int G, const char* what, Go go) {
  switch (HD * 16 + G) {
#define AIB_ATTN_CASE(hd, g) \
  case hd * 16 + g:          \
    return go(KSel<hd, g>::k);
    AIB_ATTN_CASE(128, 1) AIB_ATTN_CASE(128, 2) AIB_ATTN_CASE(128, 3) AIB_ATTN_CASE(128, 4)
    AIB_ATTN_CASE(128, 5) AIB_ATTN_CASE(128, 6) AIB_ATTN_CASE(128, 7) AIB_ATTN_CASE(128, 8)
    AIB_ATTN_CASE(64, 1) AIB_ATTN_CASE(64, 2) AIB_ATTN_CASE(64, 3) AIB_ATTN_CASE(64, 4)
    AIB_ATTN_CASE(64, 5) AIB_ATTN_CASE(64, 6) AIB_ATTN_CASE(64, 7) AIB_ATTN_CASE(64, 8)
#undef AIB_ATTN_CASE
    default:
      return fail(AIB_ENOTSUP, "%s: HD=%d G=%d", what, HD, G);
  }
}
// Launch a kernel template instantiated for the group size G = H / KV (1..GMAX) and head dim HD.
template <template <int, int> class KSel, typename... Args>
static int launch_g(int HD, int G, dim3 grid, size_t smem, cudaStream_t s, const char* what, Args... args) {
  auto go = [&](auto kernel) -> int {
    const int rc = allow_smem(kernel, smem);
    if (rc) return rc;
    return launch(kernel, grid, dim3(kThreads), smem, s, what, args...);
  };
  return dispatch_g<KSel>(HD, G, what, go);
}
// Same, for a kernel whose last argument selects the cluster merge: one cluster of cx CTAs (the group's
// splits) per (group, sequence) -- grid (cx, KV, B) -- for the first cx in `cxs` (descending, <= S) at which
// the device holds every cluster at once, else the ticket merge over S splits.
template <template <int, int> class KSel, typename... Args>
static int launch_g_cluster(int HD, int G, int S, int KV, int B, const int* cxs, int ncx, size_t smem, cudaStream_t s,
                            const char* what, Args... args) {
  auto go = [&](auto kernel) -> int {
    for (int i = 0; i < ncx; ++i) {
      const int cx = std::min(cxs[i], S);
      if (cx < 2) break;
      const size_t smem_cl = smem + static_cast<size_t>(cx) * G * (HD + 2) * sizeof(float);
      if (allow_smem(kernel, smem_cl) == AIB_OK && clusters_fit(kernel, dim3(kThreads), smem_cl, cx, KV * B))
        return launch_ex(kernel, dim3(cx, KV, B), dim3(kThreads), smem_cl, s, what, cx, args..., 1);
      cudaGetLastError();
    }
    const int rc = allow_smem(kernel, smem);
    if (rc) return rc;
    return launch(kernel, dim3(S, KV, B), dim3(kThreads), smem, s, what, args..., 0);
  };
  return dispatch_g<KSel>(HD, G, what, go);
}
template <int HD, int G>
struct RopeAttnSel {
  static constexpr auto k = rope_attn_kernel<HD, G>;
};
template <int HD, int G>
struct AttnCachedSel {
  static constexpr auto k = attn_cached_kernel<HD, G>;
};

}  // namespace attn
}  // namespace aib

using namespace aib;

extern "C" {

size_t aib_attn_workspace(int H, int KV, int HD, int maxt, int T) {
  (void)maxt;
  if (H <= 0 || KV <= 0 || T <= 0) return 0;
  return attn::ws_bytes_for(H, KV, HD, T);
}

int aib_rope_attn_decode(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv,
                         const int64_t* pos, uint16_t* kc, uint16_t* vc, float* out, int H, int KV, int HD, int maxt,
                         float eps, float scale, void* ws, size_t ws_bytes, void* stream) {
  int rc = attn::check_heads(H, KV, HD);
  if (rc) return rc;
  if (!qkv || !qn || !kn || !inv || !pos || !kc || !vc || !out || maxt <= 0)
    return fail(AIB_EINVAL, "aib_rope_attn_decode: bad arguments");
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return fail(AIB_EINVAL, "aib_rope_attn_decode: KV caches must be 16-byte aligned");
  const size_t need = attn::ws_bytes_for(H, KV, HD, 1);
  if (!ws || ws_bytes < need)
    return fail(AIB_EWORKSPACE, "aib_rope_attn_decode: workspace %zu < %zu bytes", ws_bytes, need);
  const int S = attn::splits(KV, 1, H / KV, HD);
  int* cnt = static_cast<int*>(ws);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + attn::kCntBytes);
  const size_t smem = HD == 128 ? attn::ring_bytes<128>() : attn::ring_bytes<64>();
  return attn::launch_g_cluster<attn::RopeAttnSel>(HD, H / KV, S, KV, 1, attn::kClusterSizes, attn::g_cluster_sizes, smem,
                                                   static_cast<cudaStream_t>(stream), "aib_rope_attn_decode", qkv, qn,
                                                   kn, inv, pos, kc, vc, out, H, KV, maxt, eps, scale, part, cnt,
                                                   (H + 2 * KV) * HD, 0LL, H * HD);
}

size_t aib_attn_batch_workspace(int H, int KV, int HD, int maxt, int B) {
  (void)maxt;
  if (H <= 0 || KV <= 0 || B <= 0) return 0;
  return attn::ws_bytes_for(H, KV, HD, B);
}

int aib_rope_attn_decode_batch(const float* qkv, int qkv_ld, const uint16_t* qn, const uint16_t* kn, const float* inv,
                               const int64_t* pos, uint16_t* kc, uint16_t* vc, long long kv_bstride, float* out,
                               int out_ld, int B, int H, int KV, int HD, int maxt, float eps, float scale, void* ws,
                               size_t ws_bytes, void* stream) {
  int rc = attn::check_heads(H, KV, HD);
  if (rc) return rc;
  if (!qkv || !qn || !kn || !inv || !pos || !kc || !vc || !out || maxt <= 0 || B < 1 ||
      static_cast<long long>(B) * KV > attn::kMaxSlots || qkv_ld < (H + 2 * KV) * HD || out_ld < H * HD ||
      (B > 1 && kv_bstride < static_cast<long long>(KV) * maxt * HD) || kv_bstride < 0)
    return fail(AIB_EINVAL, "aib_rope_attn_decode_batch: bad arguments");
  if (((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) || (kv_bstride * 2) % 16)
    return fail(AIB_EINVAL, "aib_rope_attn_decode_batch: KV caches must be 16-byte aligned");
  const size_t need = attn::ws_bytes_for(H, KV, HD, B);
  if (!ws || ws_bytes < need)
    return fail(AIB_EWORKSPACE, "aib_rope_attn_decode_batch: workspace %zu < %zu bytes", ws_bytes, need);
  const int S = attn::splits(KV, B, H / KV, HD);
  int* cnt = static_cast<int*>(ws);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + attn::kCntBytes);
  const size_t smem = HD == 128 ? attn::ring_bytes<128>() : attn::ring_bytes<64>();
  return attn::launch_g_cluster<attn::RopeAttnSel>(HD, H / KV, S, KV, B, attn::kClusterSizes, attn::g_cluster_sizes, smem,
                                                   static_cast<cudaStream_t>(stream), "aib_rope_attn_decode_batch", qkv,
                                                   qn, kn, inv, pos, kc, vc, out, H, KV, maxt, eps, scale, part, cnt,
                                                   qkv_ld, kv_bstride, out_ld);
}

int aib_qk_rope_cache(const float* qkv, const uint16_t* qn, const uint16_t* kn, const float* inv, const int64_t* pos,
                      float* q, uint16_t* kc, uint16_t* vc, int T, int H, int KV, int HD, int maxt, float eps,
                      void* stream) {
  int rc = attn::check_heads(H, KV, HD);
  if (rc) return rc;
  if (!qkv || !qn || !kn || !inv || !pos || !q || !kc || !vc || T <= 0 || T > 65535 || maxt <= 0)
    return fail(AIB_EINVAL, "aib_qk_rope_cache: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (HD == 128)
    return launch(attn::qk_rope_cache_kernel<128>, dim3(H + 2 * KV, T), dim3(128), 0, s, "aib_qk_rope_cache", qkv, qn,
                  kn, inv, pos, q, kc, vc, H, KV, maxt, eps);
  return launch(attn::qk_rope_cache_kernel<64>, dim3(H + 2 * KV, T), dim3(128), 0, s, "aib_qk_rope_cache", qkv, qn, kn,
                inv, pos, q, kc, vc, H, KV, maxt, eps);
}

int aib_attn_cached(const float* q, const uint16_t* kc, const uint16_t* vc, const int64_t* pos, float* out, int T,
                    int H, int KV, int HD, int maxt, float scale, void* ws, size_t ws_bytes, void* stream) {
  int rc = attn::check_heads(H, KV, HD);
  if (rc) return rc;
  if (!q || !kc || !vc || !pos || !out || T <= 0 || T > 65535 || maxt <= 0)
    return fail(AIB_EINVAL, "aib_attn_cached: bad arguments");
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return fail(AIB_EINVAL, "aib_attn_cached: KV caches must be 16-byte aligned");
  if (static_cast<long long>(T) * KV > attn::kMaxSlots)
    return fail(AIB_EINVAL, "aib_attn_cached: T * KV must be <= %d", attn::kMaxSlots);
  const size_t need = attn::ws_bytes_for(H, KV, HD, T);
  if (!ws || ws_bytes < need) return fail(AIB_EWORKSPACE, "aib_attn_cached: workspace %zu < %zu bytes", ws_bytes, need);
  const int S = attn::splits(KV, T, H / KV, HD);
  int* cnt = static_cast<int*>(ws);
  float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + attn::kCntBytes);
  const size_t smem = HD == 128 ? attn::ring_bytes<128>() : attn::ring_bytes<64>();
  return attn::launch_g<attn::AttnCachedSel>(HD, H / KV, dim3(S, KV, T), smem, static_cast<cudaStream_t>(stream),
                                             "aib_attn_cached", q, kc, vc, pos, out, H, KV, maxt, scale, part, cnt);
}

}  // extern "C"
