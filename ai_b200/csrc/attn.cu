// Decode attention over a bf16 KV cache (sm_100a).
//
// aib_rope_attn_decode replaces the reference's fused T=1 step rope_attn_k
// (`ramvi/engine/ramvi_engine/kernels/tkernels.py:164-213`): QK-RMSNorm + half-split RoPE of the q heads of
// a KV group and of the group's k, bf16 rounding of the current k/v (tkernels.py:187-190), cache write at
// pos, and online-softmax attention over positions 0..pos-1 from the cache plus the current token.
// aib_qk_rope_cache / aib_attn_cached replace the batched pair qk_rope_cache_k / attn_k (:82-150).
//
// B200 design: flash-decoding. The grid is (S splits, KV groups[, T tokens]); each CTA serves all G = H/KV
// query heads of its group, so every K/V row is read from HBM once per group, with coalesced loads (a
// warp covers one bf16 row). Each CTA writes a partial (m, l, acc) to the workspace; the last CTA of a
// group (atomic ticket, no waiting) merges the partials in split order -- starting, like the reference,
// from the current token -- so results are deterministic. The ticket counters return to zero.
// K/V rows of a CTA's range are staged into shared memory by bulk asynchronous copies (cp.async.bulk,
// no multicast) through a ring of 32-position sub-chunks, so the whole range is in flight at once; the
// merge loads every split's partial in parallel (weights exp(m_s - M) first, then the sums).
#include <algorithm>
#include "common.cuh"

namespace aib {
namespace attn {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int GMAX = 8;

AIB_DEV void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

constexpr int kSub = 32;   // positions per staged sub-chunk
constexpr int kMaxSplits = 32;
constexpr int kSlots = 4;  // ring depth

template <int HD>
constexpr size_t ring_bytes() {
  return static_cast<size_t>(kSlots) * kSub * HD * 2 * 2;
}

template <int HD>
struct Smem {
  float q[GMAX][HD];
  float kcur[HD];
  float vcur[HD];
  float cur_score[GMAX];
  float cs[HD / 2], sn[HD / 2];
  float wm[kWarps][GMAX], wl[kWarps][GMAX];
  float wacc[kWarps][GMAX][HD];
  float mw[kMaxSplits][GMAX];  // merge weights exp(m_s - M) per split
  float mM[GMAX], mL[GMAX], mc[GMAX];
  uint64_t bar[kSlots];
  int last;
  int abort;
  int issued;
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

// PER consecutive bf16 values of a row (lane's slice) as fp32
template <int PER>
AIB_DEV void load_row(const uint16_t* p, float* o) {
  if (PER == 4) {
    const uint2 r = *reinterpret_cast<const uint2*>(p);
    o[0] = __uint_as_float(r.x << 16);
    o[1] = __uint_as_float(r.x & 0xFFFF0000u);
    o[PER - 2] = __uint_as_float(r.y << 16);
    o[PER - 1] = __uint_as_float(r.y & 0xFFFF0000u);
  } else {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(p);
    o[0] = __uint_as_float(r << 16);
    o[PER - 1] = __uint_as_float(r & 0xFFFF0000u);
  }
}

// Attention of the G query heads in sm.q over cache rows [j0, j1) of one group. The rows are streamed into
// `ring` (dynamic shared memory) by bulk copies issued by thread 0, kSub positions per slot; every wait is
// bounded and, on a timeout, all threads keep the same barrier sequence and skip the math. Writes the CTA
// partial (acc[HD], m, l per head) to `part`.
template <int HD>
AIB_DEV void attend_range(Smem<HD>& sm, uint8_t* ring, const uint16_t* kc, const uint16_t* vc, int G, int j0, int j1,
                          float scale, float* part) {
  constexpr int PER = HD / 32;  // dims per lane: 4 (HD=128) or 2 (HD=64)
  constexpr uint32_t kRowBytes = HD * 2, kHalf = kSub * kRowBytes;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float q[GMAX][PER], acc[GMAX][PER], m[GMAX], l[GMAX];
#pragma unroll
  for (int h = 0; h < GMAX; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      acc[h][i] = 0.0f;
      q[h][i] = (h < G) ? sm.q[h][lane * PER + i] * scale : 0.0f;
    }
  }
  const int n = j1 - j0, nsub = (n + kSub - 1) / kSub;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&sm.bar[i], 1);
    sm.abort = 0;
    sm.issued = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_flag = &sm.abort;
  auto issue = [&](int i) {
    sm.issued = i + 1;
    const int p0 = j0 + i * kSub, cnt = min(kSub, j1 - p0);
    uint8_t* slot = ring + static_cast<size_t>(i % kSlots) * 2 * kHalf;
    mbar_arrive_expect_tx(&sm.bar[i % kSlots], 2 * cnt * kRowBytes);
    bulk_g2s(slot, kc + static_cast<size_t>(p0) * HD, cnt * kRowBytes, &sm.bar[i % kSlots]);
    bulk_g2s(slot + kHalf, vc + static_cast<size_t>(p0) * HD, cnt * kRowBytes, &sm.bar[i % kSlots]);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kSlots, nsub); ++i) issue(i);
  for (int i = 0; i < nsub; ++i) {
    bool ok = false;
    if (!*abort_flag) {
      for (uint32_t it = 0; it < kSpinLimit && !ok; ++it) {
        ok = mbar_try_wait(&sm.bar[i % kSlots], (i / kSlots) & 1);
        if (!ok && *abort_flag) break;
      }
      if (!ok && !*abort_flag) {
        set_status(AIB_DEV_TIMEOUT_FULL);
        *abort_flag = 1;
      }
    }
    if (ok) {
      const uint8_t* slot = ring + static_cast<size_t>(i % kSlots) * 2 * kHalf;
      const int cnt = min(kSub, j1 - (j0 + i * kSub));
      for (int pp = warp; pp < cnt; pp += kWarps) {
        float kv[PER], vv[PER];
        load_row<PER>(reinterpret_cast<const uint16_t*>(slot + pp * kRowBytes) + lane * PER, kv);
        load_row<PER>(reinterpret_cast<const uint16_t*>(slot + kHalf + pp * kRowBytes) + lane * PER, vv);
#pragma unroll
        for (int h = 0; h < GMAX; ++h) {
          if (h >= G) break;
          float sc = 0.0f;
#pragma unroll
          for (int d = 0; d < PER; ++d) sc += q[h][d] * kv[d];
          sc = warp_sum(sc);
          const float mn = fmaxf(m[h], sc);
          const float alpha = expf(m[h] - mn);
          const float pr = expf(sc - mn);
          l[h] = l[h] * alpha + pr;
#pragma unroll
          for (int d = 0; d < PER; ++d) acc[h][d] = acc[h][d] * alpha + pr * vv[d];
          m[h] = mn;
        }
      }
    }
    __syncthreads();  // every warp is done with this slot
    if (threadIdx.x == 0 && i + kSlots < nsub && !*abort_flag) {
      fence_proxy_async();
      issue(i + kSlots);
    }
  }
  if (*abort_flag && threadIdx.x == 0) {  // never leave with copies in flight
    const int last = sm.issued;
    for (int i = max(0, last - kSlots); i < last; ++i) mbar_wait(&sm.bar[i % kSlots], (i / kSlots) & 1, AIB_DEV_TIMEOUT_FULL);
  }
  // combine the warps in order
#pragma unroll
  for (int h = 0; h < GMAX; ++h) {
    if (h >= G) break;
    if (lane == 0) {
      sm.wm[warp][h] = m[h];
      sm.wl[warp][h] = l[h];
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) sm.wacc[warp][h][lane * PER + i] = acc[h][i];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
    const int h = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm.wm[w][h]);
    float L = 0.0f, A = 0.0f;
    if (M != -INFINITY) {
      for (int w = 0; w < kWarps; ++w) {
        const float f = expf(sm.wm[w][h] - M);
        L += sm.wl[w][h] * f;
        A += sm.wacc[w][h][d] * f;
      }
    }
    float* ph = part + static_cast<size_t>(h) * (HD + 2);
    ph[d] = A;
    if (d == 0) {
      ph[HD] = M;
      ph[HD + 1] = L;
    }
  }
}

// Merge S partials in split order on top of an initial state (m0, l0, acc0[d]; null = empty) and write out.
// The group's partial block (S x G x (HD+2) floats, contiguous) is first copied into shared memory (`stage`,
// the now idle K/V ring) with every thread issuing independent 16-byte loads, then merged from there:
// weights exp(m_s - M) per split, fixed-order sums.
template <int HD>
AIB_DEV void merge_write(Smem<HD>& sm, float* stage, const float* parts, int S, int G, const float* m0,
                         const float* l0, const float* acc0, float* out) {
  const int nf = S * G * (HD + 2);
  const int n4 = nf / 4;
  if ((nf & 3) == 0 && (reinterpret_cast<uintptr_t>(parts) & 15) == 0) {
    const float4* src = reinterpret_cast<const float4*>(parts);
    float4* dst = reinterpret_cast<float4*>(stage);
    for (int i = threadIdx.x; i < n4; i += kThreads) dst[i] = __ldcg(src + i);
  } else {
    for (int i = threadIdx.x; i < nf; i += kThreads) stage[i] = __ldcg(parts + i);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < G; h += kThreads) {
    float M = m0 ? m0[h] : -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, stage[(s * G + h) * (HD + 2) + HD]);
    float L = (m0 && M != -INFINITY) ? l0[h] * expf(m0[h] - M) : 0.0f;
    sm.mc[h] = (m0 && M != -INFINITY) ? expf(m0[h] - M) : 0.0f;
    for (int s = 0; s < S; ++s) {
      const float ms = stage[(s * G + h) * (HD + 2) + HD];
      const float w = (ms == -INFINITY || M == -INFINITY) ? 0.0f : expf(ms - M);
      sm.mw[s][h] = w;
      L += w * stage[(s * G + h) * (HD + 2) + HD + 1];
    }
    sm.mL[h] = L;
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
template <int HD>
__global__ void __launch_bounds__(kThreads)
    rope_attn_kernel(const float* __restrict__ qkv, const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn,
                     const float* __restrict__ inv, const int64_t* __restrict__ pos_p, uint16_t* kc, uint16_t* vc,
                     float* __restrict__ out, int H, int KV, int maxt, float eps, float scale, float* ws_part,
                     int* ws_cnt) {
  __shared__ Smem<HD> sm;
  extern __shared__ __align__(128) uint8_t ring[];
  const int s = blockIdx.x, S = gridDim.x, g = blockIdx.y;
  const int G = H / KV;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  const long long pos_ll = *pos_p;
  const bool pos_ok = pos_ll >= 0 && pos_ll < maxt;
  if (!pos_ok && s == 0 && threadIdx.x == 0) set_status(AIB_DEV_BAD_POS);
  const int pos = pos_ok ? static_cast<int>(pos_ll) : 0;
  for (int r = threadIdx.x; r < HD / 2; r += kThreads) {
    const float ang = static_cast<float>(pos) * inv[r];
    sm.cs[r] = cosf(ang);
    sm.sn[r] = sinf(ang);
  }
  __syncthreads();
  // q heads of the group + the group's k (warp per head vector)
  for (int t = warp; t <= G; t += kWarps) {
    if (t < G)
      norm_rope<HD>(qkv + static_cast<size_t>(g * G + t) * HD, qn, sm.cs, sm.sn, eps, sm.q[t]);
    else
      norm_rope<HD>(qkv + static_cast<size_t>(H + g) * HD, kn, sm.cs, sm.sn, eps, sm.kcur);
  }
  __syncthreads();
  uint16_t* kg = kc + static_cast<size_t>(g) * maxt * HD;
  uint16_t* vg = vc + static_cast<size_t>(g) * maxt * HD;
  for (int d = threadIdx.x; d < HD; d += kThreads) {
    const uint16_t kb = f32_to_bf16_rne(sm.kcur[d]);
    const uint16_t vb = f32_to_bf16_rne(qkv[static_cast<size_t>(H + KV + g) * HD + d]);
    sm.kcur[d] = bf16_to_f32(kb);
    sm.vcur[d] = bf16_to_f32(vb);
    if (s == 0 && pos_ok) {
      kg[static_cast<size_t>(pos) * HD + d] = kb;
      vg[static_cast<size_t>(pos) * HD + d] = vb;
    }
  }
  __syncthreads();
  for (int h = warp; h < G; h += kWarps) {  // score of the current token
    float sc = 0.0f;
    for (int d = lane; d < HD; d += 32) sc += sm.q[h][d] * sm.kcur[d];
    sc = warp_sum(sc);
    if (lane == 0) sm.cur_score[h] = sc * scale;
  }
  // this split's share of the past positions 0..pos-1
  const int n = pos_ok ? pos : 0;
  const int chunk = (n + S - 1) / S;
  const int j0 = min(n, s * chunk), j1 = min(n, j0 + chunk);
  float* part = ws_part + (static_cast<size_t>(g) * S + s) * G * (HD + 2);
  attend_range<HD>(sm, ring, kg, vg, G, j0, j1, scale, part);
  // ordered merge by the last CTA of the group
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&ws_cnt[g], 1);
    sm.last = (old == S - 1);
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    float l0[GMAX];
#pragma unroll
    for (int h = 0; h < GMAX; ++h) l0[h] = 1.0f;
    merge_write<HD>(sm, reinterpret_cast<float*>(ring), ws_part + static_cast<size_t>(g) * S * G * (HD + 2), S, G,
                    sm.cur_score, l0, sm.vcur, out + static_cast<size_t>(g) * G * HD);
    if (threadIdx.x == 0) ws_cnt[g] = 0;
  }
  pdl_trigger();
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

template <int HD>
__global__ void __launch_bounds__(kThreads)
    attn_cached_kernel(const float* __restrict__ q, const uint16_t* kc, const uint16_t* vc,
                       const int64_t* __restrict__ pos_p, float* __restrict__ out, int H, int KV, int maxt,
                       float scale, float* ws_part, int* ws_cnt) {
  __shared__ Smem<HD> sm;
  extern __shared__ __align__(128) uint8_t ring[];
  const int s = blockIdx.x, S = gridDim.x, g = blockIdx.y, t = blockIdx.z;
  const int G = H / KV;
  pdl_wait();
  const long long p = *pos_p + t;
  const bool ok = p >= 0 && p < maxt;
  const int n = ok ? static_cast<int>(p) + 1 : 0;
  for (int idx = threadIdx.x; idx < G * HD; idx += kThreads)
    sm.q[idx / HD][idx % HD] = q[(static_cast<size_t>(t) * H + g * G) * HD + idx];
  __syncthreads();
  const int chunk = (n + S - 1) / S;
  const int j0 = min(n, s * chunk), j1 = min(n, j0 + chunk);
  const size_t slot = static_cast<size_t>(t) * KV + g;
  float* part = ws_part + (slot * S + s) * G * (HD + 2);
  attend_range<HD>(sm, ring, kc + static_cast<size_t>(g) * maxt * HD, vc + static_cast<size_t>(g) * maxt * HD, G, j0,
                   j1, scale, part);
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
  pdl_trigger();
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (HD == 128) {
    rc = allow_smem(attn::rope_attn_kernel<128>, attn::ring_bytes<128>());
    if (rc) return rc;
    return launch(attn::rope_attn_kernel<128>, dim3(S, KV), dim3(attn::kThreads), attn::ring_bytes<128>(), s,
                  "aib_rope_attn_decode", qkv, qn, kn, inv, pos, kc, vc, out, H, KV, maxt, eps, scale, part, cnt);
  }
  rc = allow_smem(attn::rope_attn_kernel<64>, attn::ring_bytes<64>());
  if (rc) return rc;
  return launch(attn::rope_attn_kernel<64>, dim3(S, KV), dim3(attn::kThreads), attn::ring_bytes<64>(), s,
                "aib_rope_attn_decode", qkv, qn, kn, inv, pos, kc, vc, out, H, KV, maxt, eps, scale, part, cnt);
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (HD == 128) {
    rc = allow_smem(attn::attn_cached_kernel<128>, attn::ring_bytes<128>());
    if (rc) return rc;
    return launch(attn::attn_cached_kernel<128>, dim3(S, KV, T), dim3(attn::kThreads), attn::ring_bytes<128>(), s,
                  "aib_attn_cached", q, kc, vc, pos, out, H, KV, maxt, scale, part, cnt);
  }
  rc = allow_smem(attn::attn_cached_kernel<64>, attn::ring_bytes<64>());
  if (rc) return rc;
  return launch(attn::attn_cached_kernel<64>, dim3(S, KV, T), dim3(attn::kThreads), attn::ring_bytes<64>(), s,
                "aib_attn_cached", q, kc, vc, pos, out, H, KV, maxt, scale, part, cnt);
}

}  // extern "C"
